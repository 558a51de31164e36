// Device helpers shared by the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "common.h"

#define GB_CUDA(expr)                                                                        \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess)                                                               \
            throw ::gb::Error(std::string("ggmlc_b200: CUDA error: ") +                      \
                              cudaGetErrorString(e_) + " at " + __FILE__ + ":" +             \
                              std::to_string(__LINE__));                                     \
    } while (0)

namespace gb {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q8_0 quantization of one 32-element block held one element per lane (full warp).
// Returns the fp16-rounded scale (as float) and the rounded quant (as float, RNE).
__device__ __forceinline__ void q8_block(float v, int lane, float& d16, float& q) {
    const float amax = warp_max(fabsf(v));
    const float d = __fdiv_rn(amax, 127.0f);
    d16 = __half2float(__float2half_rn(d));
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    q = rintf(__fmul_rn(v, id));
    (void)lane;
}

// Vector exp of the reference's AVX2+FMA CPU build (ggml-cpu/vec.h:1209-1253), the published
// Arm optimized-routines single-precision exp: x = n*ln2 + b with a two-part ln2, a degree-5
// polynomial in b, scaling by 2^n with a special path for |n| > 126.  Restated with explicit
// IEEE fma/mul/add so each value matches the CPU lane exactly.
__device__ __forceinline__ float ref_v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float n = __fsub_rn(z, r);
    const float b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, __fmaf_rn(-n, 0x1.62e4p-1f, x));
    const unsigned e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + __float_as_uint(1.0f));
    const bool c = fabsf(n) > 126.0f;
    const float u = __fmul_rn(b, b);
    const float j = __fmaf_rn(__fmaf_rn(__fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                                        __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                              u, __fmul_rn(0x1.ffffecp-1f, b));
    if (!c) return __fmaf_rn(j, k, k);
    const unsigned g = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(g + 0x7f000000u);
    const float s2 = __uint_as_float(e - g);
    if (fabsf(n) > 192.0f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}

// ggml_v_silu (vec.h:1255-1262): x / (1 + exp(-x)).
__device__ __forceinline__ float ref_v_silu(float x) {
    const float e = ref_v_expf(__fsub_rn(0.0f, x));
    return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

// Packed fp32 pairs (sm_100 f32x2 instructions, the CUDA builtins): elementwise IEEE
// round-to-nearest, the same results as two scalar operations in half the instructions.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    return __fadd2_rn(a, make_float2(-b.x, -b.y));
}

// Programmatic dependent launch.  A kernel launched with launch_pdl may start while the previous
// kernel on its stream is still running; it must call pdl_wait() before it reads anything that
// kernel writes and before it writes anything (the wait returns once the previous grid has
// completed and its memory is visible).  pdl_launch() lets the next launch start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// SM count of a device (cached per device).
int sm_count(int dev);

template <typename... P, typename... A>
void launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GB_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...));
}

}  // namespace gb
