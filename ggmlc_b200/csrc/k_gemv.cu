// Decode GEMV (M <= 8) over the group weight layout, bit-exact with the reference CPU kernels,
// with optional fused RMSNorm+quantize prologue and SwiGLU+quantize epilogue.
//
// Arithmetic order.  The reference's x86 kernels (ggml_vec_dot_q{8,4}_0_q8_0,
// arch/x86/quants.c:1308-1342 and :701; llamafile tinyBLAS_Q0_AVX, sgemm.cpp:1353) keep 8 fp32
// lanes per output: lane i accumulates, block after block, fma(d_w*d_x, float(int dot of
// elements 4i..4i+3), acc_i); the lanes are reduced ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)).  A
// quad of threads owns an output row; thread t carries lanes t and t+4.
//
// Throughput.  Weight words stream from HBM in 16-byte loads (one thread's words of 4 blocks)
// through an 8-group register ring, so ~200 bytes per thread are in flight.  Q4_0 nibbles are
// turned into int8 with a shift and two bitwise ops: (q<<4) ^ 0x80 read as int8 is 16*(q-8), so
// dp4a yields 16x the exact lane dot and an arithmetic shift by 4 recovers it.  Q8_0
// activations live in shared memory in the same group layout (16-byte shared loads).
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kDepth = 8;  // groups of 4 blocks prefetched per thread
constexpr size_t kSmemMax = 200 * 1024;

template <int WT>
struct Grp {
    uint4 a, b;  // Q8_0: a,b = (word t, word t+4) of blocks 0..3; Q4_0: a = word t of blocks 0..3
    uint2 d;     // 4 fp16 scales
};

template <int WT>
__device__ __forceinline__ void ld_grp(Grp<WT>& g, const uint8_t* __restrict__ wrow,
                                       const __half* __restrict__ drow, int gi, int t) {
    if (WT == T_Q8_0) {
        const uint4* p = (const uint4*)(wrow + gi * 128 + t * 32);
        g.a = __ldg(p);
        g.b = __ldg(p + 1);
    } else {
        g.a = __ldg((const uint4*)(wrow + gi * 64 + t * 16));
    }
    g.d = __ldg((const uint2*)(drow + gi * 4));
}

__device__ __forceinline__ float h2f_lo(unsigned v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(unsigned v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

template <int WT, int MAXM>
__device__ __forceinline__ void consume(const Grp<WT>& g, int gi, int nb, int t, int M,
                                        const uint8_t* sx, const float* sxd, int nbp,
                                        float (&acc0)[MAXM], float (&acc1)[MAXM]) {
    const float dwf[4] = {h2f_lo(g.d.x), h2f_hi(g.d.x), h2f_lo(g.d.y), h2f_hi(g.d.y)};
    int wl[4], wh[4];
    if (WT == T_Q8_0) {
        wl[0] = g.a.x; wh[0] = g.a.y; wl[1] = g.a.z; wh[1] = g.a.w;
        wl[2] = g.b.x; wh[2] = g.b.y; wl[3] = g.b.z; wh[3] = g.b.w;
    } else {
        const unsigned wv[4] = {g.a.x, g.a.y, g.a.z, g.a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wl[j] = (int)(((wv[j] << 4) & 0xF0F0F0F0u) ^ 0x80808080u);  // 16*(q_lo - 8)
            wh[j] = (int)((wv[j] & 0xF0F0F0F0u) ^ 0x80808080u);         // 16*(q_hi - 8)
        }
    }
    const int jmax = min(4, nb - gi * 4);
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
            const uint4* xs = (const uint4*)(sx + m * nbp * 32 + gi * 128 + t * 32);
            const uint4 xa = xs[0], xb = xs[1];
            const float4 dx = *(const float4*)(sxd + m * nbp + gi * 4);
            const int xl[4] = {(int)xa.x, (int)xa.z, (int)xb.x, (int)xb.z};
            const int xh[4] = {(int)xa.y, (int)xa.w, (int)xb.y, (int)xb.w};
            const float dxf[4] = {dx.x, dx.y, dx.z, dx.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < jmax) {
                    const float s = __fmul_rn(dwf[j], dxf[j]);
                    int p0 = __dp4a(wl[j], xl[j], 0);
                    int p1 = __dp4a(wh[j], xh[j], 0);
                    if (WT == T_Q4_0) {
                        p0 >>= 4;
                        p1 >>= 4;
                    }
                    acc0[m] = __fmaf_rn(s, __int2float_rn(p0), acc0[m]);
                    acc1[m] = __fmaf_rn(s, __int2float_rn(p1), acc1[m]);
                }
            }
        }
    }
}

__device__ double cta_sum_d(double v, double* sh) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += sh[i];
    return t;
}

// Shared-memory Q8_0 activations: [MAXM][nbp*32] quants in group layout, then [MAXM][nbp] fp32.
template <int MAXM, int IN>
__device__ void stage_inputs(const GemvArgs& a, int nb, int nbp, uint8_t* sx, float* sxd,
                             double* shd) {
    const int K = (int)a.w.K;
    if (IN == 0) {
        for (int idx = threadIdx.x; idx < a.M * nbp * 8; idx += blockDim.x) {
            const int m = idx / (nbp * 8), r = idx % (nbp * 8), b = r >> 3, w = r & 7;
            const int v = b < nb ? __ldg((const int*)(a.xq + (int64_t)m * K + b * 32) + w) : 0;
            *(int*)(sx + m * nbp * 32 + q8_word_off(b, w)) = v;
        }
        for (int idx = threadIdx.x; idx < a.M * nbp; idx += blockDim.x) {
            const int m = idx / nbp, b = idx % nbp;
            sxd[idx] = b < nb ? a.xd[(int64_t)m * nb + b] : 0.0f;
        }
    } else {
        // RMSNorm (ggml-cpu/ops.cpp:3859-3920) then Q8_0 (arch/x86/quants.c:302-392)
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
        for (int m = 0; m < a.M; ++m) {
            const float* xr = a.xf + (int64_t)m * a.xf_stride;
            double s = 0.0;
            for (int k = threadIdx.x; k < K; k += blockDim.x) {
                const float v = xr[k];
                s += (double)__fmul_rn(v, v);
            }
            s = cta_sum_d(s, shd);
            const float mean = (float)(s / (double)K);
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            for (int b = warp; b < nbp; b += nw) {
                float d16 = 0.0f, q = 0.0f;
                if (b < nb) {
                    float v = __fmul_rn(xr[b * 32 + lane], scale);
                    if (a.gamma) v = __fmul_rn(v, a.gamma[b * 32 + lane]);
                    q8_block(v, lane, d16, q);
                }
                sx[m * nbp * 32 + q8_word_off(b, lane >> 2) + (lane & 3)] =
                    (uint8_t)(int8_t)__float2int_rn(q);
                if (lane == 0) sxd[m * nbp + b] = d16;
            }
        }
    }
}

template <int WT, int MAXM, int IN, int SWI>
__global__ void __launch_bounds__(SWI ? 256 : 128) k_gemv_fused(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double shd[8];
    __shared__ float sres[SWI ? MAXM * 64 : 1];
    const int K = (int)a.w.K;
    const int nb = K / QK;
    const int nbp = (int)nb_padded(K);
    const int ng = nbp / 4;
    uint8_t* sx = smem;
    float* sxd = (float*)(smem + (size_t)MAXM * nbp * 32);
    stage_inputs<MAXM, IN>(a, nb, nbp, sx, sxd, shd);
    __syncthreads();

    const int t = threadIdx.x & 3;
    const int quad = threadIdx.x >> 2;
    const int64_t row_bytes = qrow_bytes(WT, K);
    const uint8_t* qs = (const uint8_t*)a.w.qs;
    const int N = (int)a.w.N;
    // plain: tile = 32 rows; SwiGLU: tile = 32 output columns = 32 gate rows + 32 up rows
    const int ntiles = SWI ? (int)(a.F / 32) : (N + 31) / 32;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        int row;
        if (SWI) row = quad < 32 ? tile * 32 + quad : (int)a.F + tile * 32 + (quad - 32);
        else row = tile * 32 + quad;
        const bool valid = row < N;
        const int r = valid ? row : N - 1;
        const uint8_t* wrow = qs + (int64_t)r * row_bytes;
        const __half* drow = a.w.d + (int64_t)r * nbp;
        float acc0[MAXM], acc1[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc0[m] = acc1[m] = 0.0f;
        Grp<WT> ring[kDepth];
#pragma unroll
        for (int i = 0; i < kDepth; ++i)
            if (i < ng) ld_grp<WT>(ring[i], wrow, drow, i, t);
        for (int g0 = 0; g0 < ng; g0 += kDepth) {
#pragma unroll
            for (int i = 0; i < kDepth; ++i) {
                const int gi = g0 + i;
                if (gi < ng) {
                    consume<WT, MAXM>(ring[i], gi, nb, t, a.M, sx, sxd, nbp, acc0, acc1);
                    if (gi + kDepth < ng) ld_grp<WT>(ring[i], wrow, drow, gi + kDepth, t);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < a.M) {
                const float tt = __fadd_rn(acc0[m], acc1[m]);  // a_t + a_{t+4}
                const float u = __fadd_rn(tt, __shfl_down_sync(0xffffffffu, tt, 2, 4));
                float res = __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 1, 4));
                if (t == 0) {
                    if (SWI) {
                        sres[m * 64 + quad] = res;
                    } else if (valid) {
                        if (a.bias) res = __fadd_rn(res, a.bias[row]);
                        if (a.residual) res = __fadd_rn(a.residual[(int64_t)m * a.res_stride + row], res);
                        a.y[(int64_t)m * a.y_stride + row] = res;
                    }
                }
            }
        }
        if (SWI) {
            __syncthreads();
            const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            for (int m = warp; m < a.M; m += (int)(blockDim.x >> 5)) {
                // ggml_vec_swiglu_f32 (vec.cpp:417-426): v_silu(gate) * up
                const float h = __fmul_rn(ref_v_silu(sres[m * 64 + lane]), sres[m * 64 + 32 + lane]);
                const int64_t col = (int64_t)tile * 32 + lane;
                if (a.y) a.y[(int64_t)m * a.y_stride + col] = h;
                if (a.yq) {
                    float d16, q;
                    q8_block(h, lane, d16, q);
                    a.yq[(int64_t)m * a.F + col] = (int8_t)__float2int_rn(q);
                    if (lane == 0) a.yd[(int64_t)m * (a.F / 32) + tile] = d16;
                }
            }
            __syncthreads();
        }
    }
}

size_t smem_bytes(int maxm, int64_t K) { return (size_t)maxm * nb_padded(K) * 36; }

template <int WT, int MAXM, int IN, int SWI>
void launch_t(const GemvArgs& a, cudaStream_t st) {
    const size_t smem = smem_bytes(MAXM, a.w.K);
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static unsigned configured = 0;
    if (!(configured & (1u << (dev & 31)))) {
        GB_CUDA(cudaFuncSetAttribute(k_gemv_fused<WT, MAXM, IN, SWI>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax));
        configured |= 1u << (dev & 31);
    }
    const int64_t tiles = SWI ? a.F / 32 : (a.w.N + 31) / 32;
    const int64_t blocks = tiles < 148 * 16 ? tiles : 148 * 16;
    k_gemv_fused<WT, MAXM, IN, SWI><<<(unsigned)blocks, SWI ? 256 : 128, smem, st>>>(a);
    GB_CUDA(cudaGetLastError());
}

template <int WT, int IN, int SWI>
void launch_m(const GemvArgs& a, cudaStream_t st) {
    if (a.M == 1) launch_t<WT, 1, IN, SWI>(a, st);
    else if (a.M <= 4) launch_t<WT, 4, IN, SWI>(a, st);
    else launch_t<WT, 8, IN, SWI>(a, st);
}

}  // namespace

bool gemv_fused_fits(int64_t K, int M) {
    const int maxm = M == 1 ? 1 : (M <= 4 ? 4 : 8);
    return M >= 1 && M <= 8 && smem_bytes(maxm, K) <= kSmemMax;
}

void launch_gemv_fused(const GemvArgs& a, cudaStream_t st) {
    GB_CHECK(a.w.type == T_Q8_0 || a.w.type == T_Q4_0, "gemv: quantized weights required");
    GB_CHECK(a.w.K % QK == 0 && a.w.K < (1LL << 30) && a.w.N < (1LL << 30), "gemv: bad shape");
    GB_CHECK(gemv_fused_fits(a.w.K, a.M), "gemv: M or K too large for the shared-memory stage");
    GB_CHECK(!a.swiglu || (a.w.N == 2 * a.F && a.F % 32 == 0), "gemv: SwiGLU needs N == 2F, F % 32 == 0");
    GB_CHECK(a.xf || (a.xq && a.xd), "gemv: no input");
    if (a.w.N == 0 || a.M == 0) return;
    const bool q8 = a.w.type == T_Q8_0;
    const int in = a.xf ? 1 : 0;
    if (q8) {
        if (in == 0 && !a.swiglu) launch_m<T_Q8_0, 0, 0>(a, st);
        else if (in == 0) launch_m<T_Q8_0, 0, 1>(a, st);
        else if (!a.swiglu) launch_m<T_Q8_0, 1, 0>(a, st);
        else launch_m<T_Q8_0, 1, 1>(a, st);
    } else {
        if (in == 0 && !a.swiglu) launch_m<T_Q4_0, 0, 0>(a, st);
        else if (in == 0) launch_m<T_Q4_0, 0, 1>(a, st);
        else if (!a.swiglu) launch_m<T_Q4_0, 1, 0>(a, st);
        else launch_m<T_Q4_0, 1, 1>(a, st);
    }
}

}  // namespace gb
