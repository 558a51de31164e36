// Quantized MUL_MAT kernels over the split-row weight layout (kernels.h).
//
// M <= 8 (the decode path) goes to the GEMV in k_gemv.cu.
//
// gemm_block (M > 8, prefill): int8 tensor-core tiles (mma m16n8k32, one instruction per
// 32-K block) give the exact int32 block dot; the block scale product is applied in fp32 right
// after each block.  Integer block sums are exact; the fp32 summation order differs from the
// CPU's lane order (within 1e-5 relative in tests/test_ops_gpu.py).
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

// exact int -> float for |p| < 2^22 with one integer add and one fp32 add
__device__ __forceinline__ float i2f_exact(int p) {
    return __fsub_rn(__int_as_float(0x4B400000 + p), 12582912.0f);
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
                                                    int64_t N,
                                                    int64_t K, const int8_t* __restrict__ xq,
                                                    const float* __restrict__ xd, int64_t M,
                                                    float* __restrict__ y, int64_t y_stride,
                                                    MatmulEpilogue ep) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int64_t m0 = (int64_t)blockIdx.y * 64 + (warp >> 1) * 32;
    const int64_t n0 = (int64_t)blockIdx.x * 64 + (warp & 1) * 32;
    const int64_t nb = K / QK;
    const int64_t wrow_bytes = qrow_bytes(WT, K);
    float acc[2][4][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.0f;
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
                bf[nt][0] = __ldg((const int*)(wr + w_word_off(T_Q8_0, nb, kb, tg)));      // k = 4tg..
                bf[nt][1] = __ldg((const int*)(wr + w_word_off(T_Q8_0, nb, kb, tg + 4)));  // k = 16+4tg..
            } else {
                const unsigned w = (unsigned)__ldg((const int*)(wr + w_word_off(T_Q4_0, nb, kb, tg)));
                bf[nt][0] = (int)__vsub4(w & 0x0F0F0F0Fu, 0x08080808u);
                bf[nt][1] = (int)__vsub4((w >> 4) & 0x0F0F0F0Fu, 0x08080808u);
            }
            const int64_t c0 = min(n0 + nt * 8 + 2 * tg, N - 1);
            const int64_t c1 = min(n0 + nt * 8 + 2 * tg + 1, N - 1);
            dwv[nt][0] = __half2float(*(const __half*)(qs + c0 * wrow_bytes + w_scale_off(WT, nb, kb)));
            dwv[nt][1] = __half2float(*(const __half*)(qs + c1 * wrow_bytes + w_scale_off(WT, nb, kb)));
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
                acc[mt][nt][0] = __fmaf_rn(__fmul_rn(dwv[nt][0], dxv[mt][0]), i2f_exact(c[0]), acc[mt][nt][0]);
                acc[mt][nt][1] = __fmaf_rn(__fmul_rn(dwv[nt][1], dxv[mt][0]), i2f_exact(c[1]), acc[mt][nt][1]);
                acc[mt][nt][2] = __fmaf_rn(__fmul_rn(dwv[nt][0], dxv[mt][1]), i2f_exact(c[2]), acc[mt][nt][2]);
                acc[mt][nt][3] = __fmaf_rn(__fmul_rn(dwv[nt][1], dxv[mt][1]), i2f_exact(c[3]), acc[mt][nt][3]);
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

}  // namespace

void launch_matmul_q(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    GB_CHECK(w.K % QK == 0, "matmul: K must be a multiple of 32");
    if (M == 0 || w.N == 0) return;
    const bool q8 = w.type == T_Q8_0;
    if (M <= 8 && gemv_fused_fits(w.K, (int)M)) {
        GemvArgs a;
        a.w = w;
        a.M = (int)M;
        a.xq = xq;
        a.xd = xd;
        a.y = y;
        a.y_stride = y_stride;
        a.bias = ep.bias;
        a.residual = ep.residual;
        a.res_stride = ep.res_stride;
        launch_gemv_fused(a, st);
        return;
    }
    dim3 grid((unsigned)((w.N + 63) / 64), (unsigned)((M + 63) / 64));
    if (q8)
        k_gemm_block<T_Q8_0><<<grid, 128, 0, st>>>((const uint8_t*)w.qs, w.N, w.K, xq, xd,
                                                   M, y, y_stride, ep);
    else
        k_gemm_block<T_Q4_0><<<grid, 128, 0, st>>>((const uint8_t*)w.qs, w.N, w.K, xq, xd,
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
