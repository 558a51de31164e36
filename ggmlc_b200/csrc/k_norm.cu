// Row kernels: RMSNorm, LayerNorm, SwiGLU, bias+GELU, each optionally emitting the Q8_0
// activation rows its consumer matmul needs (fusing the activation quantization that the
// reference runs inside every MUL_MAT, ggml-cpu.c:1322-1356).
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kRowThreads = 256;

__device__ double block_sum_d(double v, double* sh) {
    v = warp_sum_d(v);
    const int w = threadIdx.x / 32, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) sh[0] = t;
    }
    __syncthreads();
    return sh[0];
}

// Store a finished row: f32 copy and/or Q8_0 blocks.  A warp quantizes four 32-element blocks
// at once (lane = element; the four amax butterflies interleaved), with q8_block's arithmetic.
__device__ void emit_row(const float* __restrict__ row_vals, int64_t D, float* y, int8_t* yq,
                         float* yd) {
    const int lane = threadIdx.x & 31, w = threadIdx.x / 32, nw = blockDim.x / 32;
    if (y)
        for (int64_t k = threadIdx.x; k < D; k += blockDim.x) y[k] = row_vals[k];
    if (yq) {
        const int64_t nbk = D / QK;
        for (int64_t b0 = (int64_t)w * 4; b0 < nbk; b0 += (int64_t)nw * 4) {  // warp-uniform
            float v[4], am[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[j] = b0 + j < nbk ? row_vals[(b0 + j) * QK + lane] : 0.0f;
                am[j] = fabsf(v[j]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int j = 0; j < 4; ++j) am[j] = fmaxf(am[j], __shfl_xor_sync(0xffffffffu, am[j], o));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (b0 + j >= nbk) break;
                const float d16 = __half2float(__float2half_rn(__fdiv_rn(am[j], 127.0f)));
                const float id = am[j] != 0.0f ? __fdiv_rn(127.0f, am[j]) : 0.0f;
                yq[(b0 + j) * QK + lane] = (int8_t)__float2int_rn(rintf(__fmul_rn(v[j], id)));
                if (lane == 0) yd[b0 + j] = d16;
            }
        }
    }
}

// rms_norm (ggml-cpu/ops.cpp:3859-3920): squares rounded to fp32 and summed in double,
// mean = (float)(sum / D), scale = 1/sqrtf(mean + eps), y = x*scale (* gamma).
__global__ void k_rms_norm(const float* __restrict__ x, int64_t x_stride, int64_t D, float eps,
                           const float* __restrict__ gamma, float* y, int64_t y_stride,
                           int8_t* yq, float* yd) {
    extern __shared__ float srow[];
    __shared__ double sh[32];
    const int64_t m = blockIdx.x;
    const float* xr = x + m * x_stride;
    // programmatic dependent launch: wait for the producer of x, then let the consumer start
    // (it prefetches its weights until its own wait)
    pdl_wait();
    pdl_launch();
    double s = 0.0;
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        const float v = xr[k];
        srow[k] = v;
        s += (double)__fmul_rn(v, v);
    }
    s = block_sum_d(s, sh);
    const float mean = (float)(s / (double)D);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        float t = __fmul_rn(srow[k], scale);
        if (gamma) t = __fmul_rn(t, gamma[k]);
        srow[k] = t;
    }
    __syncthreads();
    emit_row(srow, D, y ? y + m * y_stride : nullptr, yq ? yq + m * D : nullptr,
             yd ? yd + m * (D / QK) : nullptr);
}

// NORM on the x86 AVX2+FMA build (ggml-cpu/ops.cpp:3762-3805, vec.cpp:455-519
// ggml_vec_cvar_f32): mean = (float)(double sum) / D in fp32; centred squares reduced per
// 8-wide chunk as ((c0+c4)+(c2+c6))+((c1+c5)+(c3+c7)) in fp32 and accumulated in double;
// scale = 1/sqrtf(var + eps); y = (x-mean)*scale (* gamma) (+ beta).
__global__ void k_layer_norm(const float* __restrict__ x, int64_t x_stride, int64_t D, float eps,
                             const float* __restrict__ gamma, const float* __restrict__ beta,
                             float* y, int64_t y_stride, int8_t* yq, float* yd) {
    extern __shared__ float srow[];
    __shared__ double sh[32];
    const int64_t m = blockIdx.x;
    const float* xr = x + m * x_stride;
    double s = 0.0;
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        const float v = xr[k];
        srow[k] = v;
        s += (double)v;
    }
    s = block_sum_d(s, sh);
    const float mean = __fdiv_rn((float)s, (float)D);
    double v2 = 0.0;
    const int64_t nch = D / 8;
    for (int64_t c = threadIdx.x; c < nch; c += blockDim.x) {
        float q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float c0 = __fsub_rn(srow[c * 8 + j], mean);
            q[j] = __fmul_rn(c0, c0);
        }
        const float h = __fadd_rn(__fadd_rn(__fadd_rn(q[4], q[0]), __fadd_rn(q[6], q[2])),
                                  __fadd_rn(__fadd_rn(q[5], q[1]), __fadd_rn(q[7], q[3])));
        v2 += (double)h;
    }
    for (int64_t k = nch * 8 + threadIdx.x; k < D; k += blockDim.x) {
        const float c0 = __fsub_rn(srow[k], mean);
        v2 += (double)__fmul_rn(c0, c0);
    }
    v2 = block_sum_d(v2, sh);
    const float var = (float)(v2 / (double)D);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        float t = __fmul_rn(__fsub_rn(srow[k], mean), scale);
        if (gamma) t = __fmul_rn(t, gamma[k]);
        if (beta) t = __fadd_rn(t, beta[k]);
        srow[k] = t;
    }
    __syncthreads();
    emit_row(srow, D, y ? y + m * y_stride : nullptr, yq ? yq + m * D : nullptr,
             yd ? yd + m * (D / QK) : nullptr);
}

// ggml_vec_swiglu_f32 (vec.cpp:417-426): silu(gate) * up on 8-wide AVX2 vectors; a tail
// shorter than 8 uses scalar x/(1+expf(-x)).
__global__ void k_swiglu(const float* __restrict__ x, int64_t x_stride, int64_t F, int swapped,
                         float* y, int64_t y_stride, int8_t* yq, float* yd) {
    extern __shared__ float srow[];
    const int64_t m = blockIdx.x;
    const float* g = x + m * x_stride + (swapped ? F : 0);
    const float* u = x + m * x_stride + (swapped ? 0 : F);
    const int64_t nv = F & ~(int64_t)7;
    for (int64_t k = threadIdx.x; k < F; k += blockDim.x) {
        const float gv = g[k];
        const float sv = k < nv ? ref_v_silu(gv) : __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        srow[k] = __fmul_rn(sv, u[k]);
    }
    __syncthreads();
    emit_row(srow, F, y ? y + m * y_stride : nullptr, yq ? yq + m * F : nullptr,
             yd ? yd + m * (F / QK) : nullptr);
}

// fast_gelu_f32 of the CPU custom op (runtime/src/stdlib_kernels.cpp:9-19, :62-70), with the
// contraction x + A*x^3 -> fma that the reference's GNU build applies.
__global__ void k_bias_gelu(const float* __restrict__ x, int64_t x_stride,
                            const float* __restrict__ bias, int64_t F, float* y,
                            int64_t y_stride, int8_t* yq, float* yd) {
    extern __shared__ float srow[];
    const int64_t m = blockIdx.x;
    const float kS = 0.79788456080286535587989211986876f, kA = 0.044715f;
    for (int64_t k = threadIdx.x; k < F; k += blockDim.x) {
        float v = x[m * x_stride + k];
        if (bias) v = __fadd_rn(v, bias[k]);
        const float v3 = __fmul_rn(__fmul_rn(v, v), v);
        float inner = __fmul_rn(kS, __fmaf_rn(kA, v3, v));
        inner = fmaxf(-9.0f, fminf(9.0f, inner));
        // the CPU's libm expf is correctly rounded but for rare last-bit cases; exp in double
        // rounded once to float is correctly rounded
        const float e2 = (float)exp((double)__fmul_rn(2.0f, inner));
        const float th = __fdiv_rn(__fsub_rn(e2, 1.0f), __fadd_rn(e2, 1.0f));
        srow[k] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, th));
    }
    __syncthreads();
    emit_row(srow, F, y ? y + m * y_stride : nullptr, yq ? yq + m * F : nullptr,
             yd ? yd + m * (F / QK) : nullptr);
}

void check_row_smem(int64_t D) {
    GB_CHECK(D * 4 <= 200 * 1024, "row kernel: row longer than the shared-memory stage");
}

template <class K>
void set_smem(K kernel) {
    static bool done = false;
    if (!done) {
        GB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
        done = true;
    }
}

}  // namespace

void launch_rms_norm(const float* x, int64_t x_stride, int64_t M, int64_t D, float eps,
                     const float* gamma, float* y, int64_t y_stride, int8_t* yq, float* yd,
                     cudaStream_t st) {
    if (!M) return;
    check_row_smem(D);
    GB_CHECK(!yq || D % QK == 0, "rms_norm: quantized output needs D % 32 == 0");
    set_smem(k_rms_norm);
    // a batched decode step normalizes at most 16 rows: a wide CTA per row shortens the chain
    const unsigned threads = M <= kMaxRows ? 1024 : kRowThreads;
    launch_pdl(k_rms_norm, dim3((unsigned)M), dim3(threads), (size_t)(D * 4), st, x, x_stride, D,
               eps, gamma, y, y_stride, yq, yd);
}

void launch_layer_norm(const float* x, int64_t x_stride, int64_t M, int64_t D, float eps,
                       const float* gamma, const float* beta, float* y, int64_t y_stride,
                       int8_t* yq, float* yd, cudaStream_t st) {
    if (!M) return;
    check_row_smem(D);
    GB_CHECK(!yq || D % QK == 0, "layer_norm: quantized output needs D % 32 == 0");
    set_smem(k_layer_norm);
    k_layer_norm<<<(unsigned)M, kRowThreads, D * 4, st>>>(x, x_stride, D, eps, gamma, beta, y,
                                                          y_stride, yq, yd);
    GB_CUDA(cudaGetLastError());
}

void launch_swiglu(const float* x, int64_t x_stride, int64_t M, int64_t F, bool swapped,
                   float* y, int64_t y_stride, int8_t* yq, float* yd, cudaStream_t st) {
    if (!M) return;
    check_row_smem(F);
    GB_CHECK(!yq || F % QK == 0, "swiglu: quantized output needs F % 32 == 0");
    set_smem(k_swiglu);
    k_swiglu<<<(unsigned)M, kRowThreads, F * 4, st>>>(x, x_stride, F, swapped ? 1 : 0, y,
                                                      y_stride, yq, yd);
    GB_CUDA(cudaGetLastError());
}

void launch_bias_gelu(const float* x, int64_t x_stride, const float* bias, int64_t M, int64_t F,
                      float* y, int64_t y_stride, int8_t* yq, float* yd, cudaStream_t st) {
    if (!M) return;
    check_row_smem(F);
    GB_CHECK(!yq || F % QK == 0, "bias_gelu: quantized output needs F % 32 == 0");
    set_smem(k_bias_gelu);
    k_bias_gelu<<<(unsigned)M, kRowThreads, F * 4, st>>>(x, x_stride, bias, F, y, y_stride, yq,
                                                         yd);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
