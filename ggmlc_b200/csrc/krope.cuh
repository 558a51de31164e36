// RoPE of one element with the reference's arithmetic (ggml-cpu/ops.cpp:5910-5923 table,
// :5998-6015 NEOX rotation) from the host-built (cos, sin) table of the executor; positions
// outside the table recompute theta with the same fp32 recurrence.
#pragma once

#include <cstdint>

#include "kernels.h"

namespace gb {
namespace {

__device__ __forceinline__ void rope_cs(const RopeTable& tab, int64_t p, int i, float& c, float& s) {
    if (tab.cs && p >= 0 && p < tab.n_pos) {
        const float2 v = tab.cs[p * (tab.n_dims / 2) + i];
        c = v.x;
        s = v.y;
    } else {
        float theta = (float)p;
        for (int k = 0; k < i; ++k) theta = __fmul_rn(theta, tab.theta_scale);
        c = (float)cos((double)theta);
        s = (float)sin((double)theta);
    }
}

// rotated value of element d (< hd) of a head vector src (f32, contiguous) at position p
__device__ __forceinline__ float rope_elem(const float* src, int d, int hd, const RopeTable& tab,
                                           int64_t p) {
    const int half = tab.n_dims / 2;
    if (d >= tab.n_dims) return src[d];
    const int i = d < half ? d : d - half;
    float c, s;
    rope_cs(tab, p, i, c, s);
    const float x0 = src[i], x1 = src[i + half];
    return d < half ? __fmaf_rn(x0, c, -__fmul_rn(x1, s)) : __fmaf_rn(x0, s, __fmul_rn(x1, c));
}

}  // namespace
}  // namespace gb
