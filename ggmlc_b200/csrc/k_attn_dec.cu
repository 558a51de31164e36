// Fused attention-side kernels over the F16 KV cache.
//
// k_rope_qkv (any s): RoPE of q and k read straight from the QKV projection output, rotated q to
//   an f32 buffer, rotated k and v rows to the F16 cache at rows pos..pos+s-1 (the reference's
//   ROPE x2 + SET_ROWS x2, executor.cpp:2132-2184, in one launch).
// k_attn_decode (s == 1): split-KV flash decoding.  grid = (splits, Hkv); each CTA rotates the q
//   heads of its GQA group itself, the CTA whose range holds the new position also rotates the
//   new k and writes k, v into the cache, then the CTA scores its positions (one warp per
//   position, lanes across head_dim), runs the softmax over its range and accumulates V.
//   Partials (m, l, acc) go to a workspace.
// k_attn_combine: merges the splits of each head and writes the head's output as f32 and/or as
//   Q8_0 blocks for the output projection (head_dim % 32 == 0, so blocks never straddle heads).
//
// RoPE arithmetic is the reference's (ops.cpp:5910-5923, 5998-6015) with the host cos/sin table;
// attention accumulates in fp32 (the CPU rounds its V accumulator to fp16 per position).
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

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

__global__ void k_rope_qkv(QkvRopeArgs a) {
    const int hd = a.hd;
    const int64_t base = (a.step ? a.step->pos : 0) + a.pos_off;
    const int64_t heads = (int64_t)a.Hq + 2 * a.Hkv;
    const int64_t total = (int64_t)a.s * heads * hd;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(idx % hd);
        const int64_t hh = (idx / hd) % heads;
        const int64_t t = idx / (hd * heads);
        const float* row = a.qkv + t * a.qkv_stride;
        const int64_t p = base + t;
        if (hh < a.Hq) {
            const float* src = row + a.q_off + hh * hd;
            a.q_out[(t * a.Hq + hh) * hd + d] = rope_elem(src, d, hd, a.tab, p);
        } else if (hh < a.Hq + a.Hkv) {
            const int64_t h = hh - a.Hq;
            const float* src = row + a.k_off + h * hd;
            a.kc[(h * a.ctx + p) * hd + d] = __float2half_rn(rope_elem(src, d, hd, a.tab, p));
        } else {
            const int64_t h = hh - a.Hq - a.Hkv;
            a.vc[(h * a.ctx + p) * hd + d] = __float2half_rn(row[a.v_off + h * hd + d]);
        }
    }
}

constexpr int kDecWarps = 4;
constexpr int kMaxRk = 8;     // q heads per KV head handled by one CTA
constexpr int kMaxSpan = 512; // positions per split staged in shared memory

__global__ void __launch_bounds__(kDecWarps * 32) k_attn_decode(AttnDecArgs a) {
    __shared__ float sq[kMaxRk * 256];          // rotated q (fp16-rounded) for the group
    __shared__ float ss[kMaxRk * kMaxSpan];     // scores / probabilities
    __shared__ float sred[kDecWarps * kMaxRk];
    __shared__ float sacc[kDecWarps * kMaxRk * 256 / 4];  // reused per 64-dim slab
    const int hd = a.hd;
    const int rk = a.Hq / a.Hkv;
    const int hk = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pos = (a.step ? a.step->pos : 0) + a.pos_off;  // position of the new token
    const int64_t nkv = pos + 1;
    const int64_t per = (nkv + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = (int64_t)blockIdx.x * per;
    const int64_t c1 = min(c0 + per, nkv);
    const float* row = a.qkv;
    // q heads of this group, rotated at pos and rounded to fp16 (q_to_vec_dot)
    for (int e = threadIdx.x; e < rk * hd; e += blockDim.x) {
        const int h = e / hd, d = e % hd;
        const float* src = row + a.q_off + (int64_t)(hk * rk + h) * hd;
        sq[h * hd + d] = __half2float(__float2half_rn(rope_elem(src, d, hd, a.tab, pos)));
    }
    // the split holding the new position writes its k, v rows into the cache
    if (c0 <= pos && pos < c1) {
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            const float* ks = row + a.k_off + (int64_t)hk * hd;
            a.kc[((int64_t)hk * a.ctx + pos) * hd + d] = __float2half_rn(rope_elem(ks, d, hd, a.tab, pos));
            a.vc[((int64_t)hk * a.ctx + pos) * hd + d] = __float2half_rn(row[a.v_off + (int64_t)hk * hd + d]);
        }
    }
    __syncthreads();
    float* part = a.part + ((int64_t)blockIdx.x * a.Hq + (int64_t)hk * rk) * (hd + 2);
    if (c0 >= c1) {
        for (int e = threadIdx.x; e < rk * (hd + 2); e += blockDim.x) {
            const int h = e / (hd + 2), k = e % (hd + 2);
            part[h * (hd + 2) + k] = k == 0 ? -INFINITY : 0.0f;
        }
        return;
    }
    const int64_t span = c1 - c0;
    const __half* kbase = a.kc + ((int64_t)hk * a.ctx) * hd;
    const __half* vbase = a.vc + ((int64_t)hk * a.ctx) * hd;
    const int per_lane = hd / 32;  // 2 (hd 64) or 4 (hd 128) or 8 (hd 256)
    // pass 1: scores, one warp per position
    for (int64_t c = c0 + warp; c < c1; c += kDecWarps) {
        float kv[8];
        const __half* kr = kbase + c * hd + lane * per_lane;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < per_lane) kv[j] = __half2float(kr[j]);
        for (int h = 0; h < rk; ++h) {
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < per_lane) dot = __fmaf_rn(kv[j], sq[h * hd + lane * per_lane + j], dot);
            dot = warp_sum(dot);
            if (lane == 0) ss[h * kMaxSpan + (c - c0)] = __fmul_rn(dot, a.scale);
        }
    }
    __syncthreads();
    // softmax statistics per head over this split (warp h handles head h, strided)
    for (int h = warp; h < rk; h += kDecWarps) {
        float mx = -INFINITY;
        for (int64_t c = lane; c < span; c += 32) mx = fmaxf(mx, ss[h * kMaxSpan + c]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int64_t c = lane; c < span; c += 32) {
            const float p = expf(ss[h * kMaxSpan + c] - mx);
            ss[h * kMaxSpan + c] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            part[h * (hd + 2) + 0] = mx;
            part[h * (hd + 2) + 1] = l;
        }
    }
    __syncthreads();
    // pass 2: V accumulation, one warp per position, lanes across head_dim
    float acc[kMaxRk][8];
#pragma unroll
    for (int h = 0; h < kMaxRk; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h][j] = 0.0f;
    for (int64_t c = c0 + warp; c < c1; c += kDecWarps) {
        float vv[8];
        const __half* vr = vbase + c * hd + lane * per_lane;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < per_lane) vv[j] = __half2float(vr[j]);
#pragma unroll
        for (int h = 0; h < kMaxRk; ++h) {
            if (h < rk) {
                const float p = ss[h * kMaxSpan + (c - c0)];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (j < per_lane) acc[h][j] = __fmaf_rn(p, vv[j], acc[h][j]);
            }
        }
    }
    // reduce across warps through shared memory, one head at a time
    for (int h = 0; h < rk; ++h) {
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < per_lane) sacc[warp * hd + lane * per_lane + j] = acc[h][j];
        __syncthreads();
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            float v = 0.0f;
            for (int w = 0; w < kDecWarps; ++w) v += sacc[w * hd + d];
            part[h * (hd + 2) + 2 + d] = v;
        }
    }
}

__global__ void k_attn_combine(AttnDecArgs a) {
    const int h = blockIdx.x;  // q head
    const int hd = a.hd;
    const int S = a.splits;
    float M = -INFINITY;
    for (int sp = 0; sp < S; ++sp) M = fmaxf(M, a.part[((int64_t)sp * a.Hq + h) * (hd + 2)]);
    float L = 0.0f;
    for (int sp = 0; sp < S; ++sp) {
        const float* pr = a.part + ((int64_t)sp * a.Hq + h) * (hd + 2);
        if (pr[0] != -INFINITY) L += pr[1] * expf(pr[0] - M);
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    const int lane = threadIdx.x & 31;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float v = 0.0f;
        for (int sp = 0; sp < S; ++sp) {
            const float* pr = a.part + ((int64_t)sp * a.Hq + h) * (hd + 2);
            if (pr[0] != -INFINITY) v += pr[2 + d] * expf(pr[0] - M);
        }
        v *= inv;
        if (a.o) a.o[(int64_t)h * hd + d] = v;
        if (a.oq) {  // blockDim.x == hd: warp w owns elements 32w..32w+31 of the head
            float d16, q;
            q8_block(v, lane, d16, q);
            a.oq[(int64_t)h * hd + d] = (int8_t)__float2int_rn(q);
            if (lane == 0) a.od[((int64_t)h * hd + d) / 32] = d16;
        }
    }
}

}  // namespace

void launch_rope_qkv(const QkvRopeArgs& a, cudaStream_t st) {
    const int64_t total = (int64_t)a.s * (a.Hq + 2 * a.Hkv) * a.hd;
    if (!total) return;
    GB_CHECK(a.tab.n_dims <= a.hd && a.tab.n_dims % 2 == 0, "rope_qkv: bad n_dims");
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_rope_qkv<<<(unsigned)blocks, 256, 0, st>>>(a);
    GB_CUDA(cudaGetLastError());
}

int attn_decode_splits(int64_t Hkv, int64_t max_kv) {
    // about two CTAs per SM, and at most kMaxSpan positions per split
    int64_t s = (296 + Hkv - 1) / Hkv;
    const int64_t need = (max_kv + kMaxSpan - 1) / kMaxSpan;
    if (s < need) s = need;
    if (s > 256) s = 256;
    return (int)(s < 1 ? 1 : s);
}

size_t attn_decode_workspace(int64_t Hq, int64_t hd, int splits) {
    return (size_t)splits * Hq * (hd + 2) * sizeof(float);
}

void launch_attn_decode(const AttnDecArgs& a, cudaStream_t st) {
    GB_CHECK(a.hd % 32 == 0 && a.hd <= 256, "attn_decode: head_dim must be a multiple of 32, <= 256");
    GB_CHECK(a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRk, "attn_decode: GQA group too large");
    GB_CHECK(a.splits >= 1 && a.splits * (int64_t)kMaxSpan >= a.max_kv,
             "attn_decode: too few splits for the context");
    dim3 grid((unsigned)a.splits, (unsigned)a.Hkv);
    k_attn_decode<<<grid, kDecWarps * 32, 0, st>>>(a);
    GB_CUDA(cudaGetLastError());
    k_attn_combine<<<(unsigned)a.Hq, (unsigned)a.hd, 0, st>>>(a);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
