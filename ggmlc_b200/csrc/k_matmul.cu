// Quantized MUL_MAT kernels.
//
// gemv_exact (M <= 8, the decode path): one 8-lane group per output row.  Lane i owns fp32
// accumulator i and, block after block, adds fma(d_w*d_x, dp4a(w[4i..4i+3], x[4i..4i+3]), acc).
// That is the exact arithmetic order of the reference's x86 kernels (ggml_vec_dot_q{8,4}_0_q8_0,
// arch/x86/quants.c:1308-1342 and :701, and llamafile tinyBLAS_Q0_AVX sgemm.cpp:1353), so the
// fp32 outputs are bit-identical to the CPU's for identical inputs.  Weight quants stream from
// HBM as 32-bit words (a 32-byte Q8_0 block / 16-byte Q4_0 block per 8 lanes), the Q8_0
// activations sit in shared memory.
//
// gemm_block (M > 8, prefill): int8 tensor-core tiles (mma m16n8k32, one instruction per 32-K
// block) give the exact int32 block dot; the per-block scale product d_w*d_x is applied in fp32
// right after each block.  Integer block sums are exact, the fp32 summation order differs from
// the CPU's lane order.
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

__device__ __forceinline__ int load_w_word(const uint8_t* __restrict__ row, int wtype, int64_t b,
                                           int i) {
    if (wtype == T_Q8_0) {
        return __ldg((const int*)(row + b * 32 + 4 * i));
    }
    const unsigned w = (unsigned)__ldg((const int*)(row + b * 16 + 4 * (i & 3)));
    const unsigned v = (w >> (4 * (i >> 2))) & 0x0F0F0F0Fu;
    return (int)__vsub4(v, 0x08080808u);
}

template <int WT, int MAXM>
__global__ void __launch_bounds__(128) k_gemv_exact(const uint8_t* __restrict__ qs,
                                                    const __half* __restrict__ dw,
                                                    int64_t N, int64_t K,
                                                    const int8_t* __restrict__ xq,
                                                    const float* __restrict__ xd, int M,
                                                    float* __restrict__ y, int64_t y_stride,
                                                    MatmulEpilogue ep) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t nb = K / QK;
    int8_t* sx = (int8_t*)smem;
    float* sxd = (float*)(smem + (size_t)MAXM * K);
    // stage Q8_0 activations (M rows) in shared memory
    {
        const int64_t nw = (int64_t)M * K / 4;
        for (int64_t t = threadIdx.x; t < nw; t += blockDim.x)
            ((int*)sx)[t] = ((const int*)xq)[t];
        for (int64_t t = threadIdx.x; t < (int64_t)M * nb; t += blockDim.x) sxd[t] = xd[t];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int i = lane & 7;
    const int grp = lane >> 3;
    const int warps = blockDim.x / 32;
    const int64_t row_bytes = WT == T_Q8_0 ? K : K / 2;
    const unsigned gmask = 0xFFu << (grp * 8);
    for (int64_t base = ((int64_t)blockIdx.x * warps + threadIdx.x / 32) * 4; base < N;
         base += (int64_t)gridDim.x * warps * 4) {
        const int64_t n = base + grp;
        const bool valid = n < N;
        const int64_t nr = valid ? n : N - 1;
        const uint8_t* wrow = qs + nr * row_bytes;
        const __half* drow = dw + nr * nb;
        float acc[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
#pragma unroll 4
        for (int64_t b = 0; b < nb; ++b) {
            const int wv = load_w_word(wrow, WT, b, i);
            const float dwb = __half2float(drow[b]);
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    const int xv = *(const int*)(sx + (int64_t)m * K + b * 32 + 4 * i);
                    const int p = __dp4a(wv, xv, 0);
                    const float s = __fmul_rn(dwb, sxd[(int64_t)m * nb + b]);
                    acc[m] = __fmaf_rn(s, (float)p, acc[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                // ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7))  (hsum_float_8)
                float t = __fadd_rn(acc[m], __shfl_down_sync(gmask, acc[m], 4, 8));
                float u = __fadd_rn(t, __shfl_down_sync(gmask, t, 2, 8));
                float r = __fadd_rn(u, __shfl_down_sync(gmask, u, 1, 8));
                if (i == 0 && valid) {
                    if (ep.bias) r = __fadd_rn(r, ep.bias[n]);
                    if (ep.residual) r = __fadd_rn(ep.residual[(int64_t)m * ep.res_stride + n], r);
                    y[(int64_t)m * y_stride + n] = r;
                }
            }
        }
    }
}

// ---- block GEMM on int8 tensor cores (prefill) ----------------------------------------------
// CTA tile 64 (activation rows m) x 64 (weight rows n), 4 warps each 32 x 32, one mma.sync
// m16n8k32.s8 per 32-K block per 16x8 sub-tile; int32 block sums scaled into fp32 accumulators.
__device__ __forceinline__ void mma_s8(int (&c)[4], const int (&a)[4], const int (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int WT>
__global__ void __launch_bounds__(128) k_gemm_block(const uint8_t* __restrict__ qs,
                                                    const __half* __restrict__ dw, int64_t N,
                                                    int64_t K, const int8_t* __restrict__ xq,
                                                    const float* __restrict__ xd, int64_t M,
                                                    float* __restrict__ y, int64_t y_stride,
                                                    MatmulEpilogue ep) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int64_t m0 = (int64_t)blockIdx.y * 64 + (warp >> 1) * 32;
    const int64_t n0 = (int64_t)blockIdx.x * 64 + (warp & 1) * 32;
    const int64_t nb = K / QK;
    const int64_t wrow_bytes = WT == T_Q8_0 ? K : K / 2;
    float acc[2][4][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.0f;
    // clamp rows for loads; stores are masked
    int64_t arow[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
        arow[mt][0] = min(m0 + mt * 16 + g, M - 1);
        arow[mt][1] = min(m0 + mt * 16 + g + 8, M - 1);
    }
    int64_t brow[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) brow[nt] = min(n0 + nt * 8 + g, N - 1);

    for (int64_t kb = 0; kb < nb; ++kb) {
        int af[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            const int8_t* r0 = xq + arow[mt][0] * K + kb * 32;
            const int8_t* r1 = xq + arow[mt][1] * K + kb * 32;
            af[mt][0] = __ldg((const int*)(r0 + 4 * tg));
            af[mt][1] = __ldg((const int*)(r1 + 4 * tg));
            af[mt][2] = __ldg((const int*)(r0 + 16 + 4 * tg));
            af[mt][3] = __ldg((const int*)(r1 + 16 + 4 * tg));
        }
        int bf[4][2];
        float dwv[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const uint8_t* wr = qs + brow[nt] * wrow_bytes;
            if (WT == T_Q8_0) {
                bf[nt][0] = __ldg((const int*)(wr + kb * 32 + 4 * tg));
                bf[nt][1] = __ldg((const int*)(wr + kb * 32 + 16 + 4 * tg));
            } else {
                const unsigned w = (unsigned)__ldg((const int*)(wr + kb * 16 + 4 * tg));
                bf[nt][0] = (int)__vsub4(w & 0x0F0F0F0Fu, 0x08080808u);
                bf[nt][1] = (int)__vsub4((w >> 4) & 0x0F0F0F0Fu, 0x08080808u);
            }
            // scales of the two output columns this thread holds (n = n0+nt*8+2tg, +1)
            const int64_t c0 = min(n0 + nt * 8 + 2 * tg, N - 1);
            const int64_t c1 = min(n0 + nt * 8 + 2 * tg + 1, N - 1);
            dwv[nt][0] = __half2float(dw[c0 * nb + kb]);
            dwv[nt][1] = __half2float(dw[c1 * nb + kb]);
        }
        float dxv[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            dxv[mt][0] = xd[arow[mt][0] * nb + kb];
            dxv[mt][1] = xd[arow[mt][1] * nb + kb];
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                int c[4] = {0, 0, 0, 0};
                mma_s8(c, af[mt], bf[nt]);
                acc[mt][nt][0] = __fmaf_rn(__fmul_rn(dwv[nt][0], dxv[mt][0]), (float)c[0], acc[mt][nt][0]);
                acc[mt][nt][1] = __fmaf_rn(__fmul_rn(dwv[nt][1], dxv[mt][0]), (float)c[1], acc[mt][nt][1]);
                acc[mt][nt][2] = __fmaf_rn(__fmul_rn(dwv[nt][0], dxv[mt][1]), (float)c[2], acc[mt][nt][2]);
                acc[mt][nt][3] = __fmaf_rn(__fmul_rn(dwv[nt][1], dxv[mt][1]), (float)c[3], acc[mt][nt][3]);
            }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int64_t m = m0 + mt * 16 + g + (e >= 2 ? 8 : 0);
                const int64_t n = n0 + nt * 8 + 2 * tg + (e & 1);
                if (m < M && n < N) {
                    float r = acc[mt][nt][e];
                    if (ep.bias) r = __fadd_rn(r, ep.bias[n]);
                    if (ep.residual) r = __fadd_rn(ep.residual[m * ep.res_stride + n], r);
                    y[m * y_stride + n] = r;
                }
            }
}

// float-weight fallback (F32/F16 W): one warp per (row n, activation m)
__global__ void k_matmul_f(QWeight w, const float* __restrict__ x, int64_t x_stride, int64_t M,
                           float* __restrict__ y, int64_t y_stride, MatmulEpilogue ep) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int64_t m = blockIdx.y;
    if (n >= w.N || m >= M) return;
    float s = 0.0f;
    for (int64_t k = lane; k < w.K; k += 32) {
        const float wv = w.type == T_F16 ? __half2float(((const __half*)w.qs)[n * w.K + k])
                                         : ((const float*)w.qs)[n * w.K + k];
        s = __fmaf_rn(wv, x[m * x_stride + k], s);
    }
    s = warp_sum(s);
    if (lane == 0) {
        if (ep.bias) s = __fadd_rn(s, ep.bias[n]);
        if (ep.residual) s = __fadd_rn(ep.residual[m * ep.res_stride + n], s);
        y[m * y_stride + n] = s;
    }
}

template <int WT, int MAXM>
void gemv_launch(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                 int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    const size_t smem = (size_t)MAXM * w.K + (size_t)MAXM * (w.K / QK) * 4;
    static bool configured = false;
    if (!configured) {
        GB_CUDA(cudaFuncSetAttribute(k_gemv_exact<WT, MAXM>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        configured = true;
    }
    GB_CHECK(smem <= 200 * 1024, "gemv: activation rows do not fit in shared memory");
    const int threads = 128;
    const int64_t tasks = (w.N + 3) / 4;  // 4 rows per warp
    int64_t blocks = (tasks + threads / 32 - 1) / (threads / 32);
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_gemv_exact<WT, MAXM><<<(unsigned)blocks, threads, smem, st>>>(
        (const uint8_t*)w.qs, w.d, w.N, w.K, xq, xd, (int)M, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

}  // namespace

void launch_matmul_q_exact(const QWeight& w, const int8_t* xq, const float* xd, int64_t M,
                           float* y, int64_t y_stride, const MatmulEpilogue& ep,
                           cudaStream_t st) {
    GB_CHECK(w.K % QK == 0, "matmul: K must be a multiple of 32");
    if (M == 0 || w.N == 0) return;
    if (M <= 8) {
        const bool q8 = w.type == T_Q8_0;
        if (M == 1) {
            if (q8) gemv_launch<T_Q8_0, 1>(w, xq, xd, M, y, y_stride, ep, st);
            else gemv_launch<T_Q4_0, 1>(w, xq, xd, M, y, y_stride, ep, st);
        } else if (M <= 4) {
            if (q8) gemv_launch<T_Q8_0, 4>(w, xq, xd, M, y, y_stride, ep, st);
            else gemv_launch<T_Q4_0, 4>(w, xq, xd, M, y, y_stride, ep, st);
        } else {
            if (q8) gemv_launch<T_Q8_0, 8>(w, xq, xd, M, y, y_stride, ep, st);
            else gemv_launch<T_Q4_0, 8>(w, xq, xd, M, y, y_stride, ep, st);
        }
        return;
    }
    dim3 grid((unsigned)((w.N + 63) / 64), (unsigned)((M + 63) / 64));
    if (w.type == T_Q8_0)
        k_gemm_block<T_Q8_0><<<grid, 128, 0, st>>>((const uint8_t*)w.qs, w.d, w.N, w.K, xq, xd,
                                                   M, y, y_stride, ep);
    else
        k_gemm_block<T_Q4_0><<<grid, 128, 0, st>>>((const uint8_t*)w.qs, w.d, w.N, w.K, xq, xd,
                                                   M, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

void launch_matmul_f(const QWeight& w, const float* x, int64_t x_stride, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    if (M == 0 || w.N == 0) return;
    dim3 grid((unsigned)((w.N + 3) / 4), (unsigned)M);
    k_matmul_f<<<grid, 128, 0, st>>>(w, x, x_stride, M, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
