// Quantized MUL_MAT kernels over the split-row weight layout (kernels.h).
//
// M <= 16 (decode and batched decode) goes to the GEMV (k_gemv.cu, M <= 2) or the tensor-core
// decode kernel (k_mmv.cu).
//
// M > 16 (prefill) runs the tcgen05 GEMM (k_gemm_tc.cu) when K % 128 == 0, else k_gemm_q:
// int8 tensor-core tiles (mma m16n8k32, one instruction per 32-K block) give the exact int32
// block dot; the block scale product is applied in fp32 right after each block.  Integer block
// sums are exact; the fp32 summation order differs from the CPU's lane order.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

// ---- block GEMM on int8 tensor cores (prefill, M > 16) -------------------------------------
// CTA tile 128 activation rows (m) x 128 weight rows (n), 8 warps as 2 (m) x 4 (n), warp tile
// 64 x 32.  K advances in stages of 4 blocks, streamed by cp.async through a 4-stage shared-memory
// ring; fragments come from swizzled shared memory with ldmatrix.  Each 32-element block is one
// mma.sync m16n8k32 (s8 x s8 -> exact s32 block dot) per 16x8 sub-tile, started from the
// 1.5*2^23 bias so the int -> float conversion is one add; the block term is then scaled by
// d_w * d_x and accumulated in fp32 registers.
//
// K order: a stage takes blocks {64g+2j, 64g+2j+1, 64g+32+2j, 64g+32+2j+1}, the order in which
// the weight scale region stores them, so one 8-byte copy brings a row's four scales.
constexpr int kBM = 128, kBN = 128, kGThreads = 256, kGStages = 4;

// BM: activation rows per tile (128, or 64 for launches of at most 64 rows)
template <int WT, int BM = kBM>
struct GStage {
    static constexpr int kRowB = WT == T_Q8_0 ? 128 : 64;  // weight bytes per row and stage
    static constexpr int kA = BM * 128;                     // activations: 4 blocks x 32 B per row
    static constexpr int kB = kBN * kRowB;
    static constexpr int kWs = kBN * 8;                     // 4 fp16 weight scales per row
    static constexpr int kXs = BM * 16;                     // 4 fp32 activation scales per row
    static constexpr int kBytes = kA + kB + kWs + kXs;
};

__device__ __forceinline__ unsigned s_addr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
// cp.async of `bytes` (4, 8 or 16) with zero fill when !valid
template <int BYTES>
__device__ __forceinline__ void cp_zfill(void* dst, const void* src, bool valid) {
    const int n = valid ? BYTES : 0;
    if (BYTES == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s_addr(dst)), "l"(src),
                     "r"(n)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(s_addr(dst)), "l"(src),
                     "n"(BYTES), "r"(n)
                     : "memory");
}
__device__ __forceinline__ void ldsm_x4(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s_addr(p)));
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const unsigned (&a)[4], unsigned b0,
                                       unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0x4B400000));
}

// SwiGLU epilogue: the tile's weight rows are gate rows p..p+63 and up rows F+p..F+p+63
// (p = 64 * blockIdx.x); the CTA writes silu(gate) * up of its 64 units as f32 (y) and/or Q8_0
// (yq, yd), the arithmetic of launch_swiglu on the plain GEMM's outputs.
struct SwiOut {
    int F = 0;
    float* y = nullptr;
    int64_t y_stride = 0;
    int8_t* yq = nullptr;
    float* yd = nullptr;
};

// OCC = CTAs per SM the kernel is built for: 2 keeps the block loop rolled (128 registers).
// BM = 64: the warps' tiles are 32 x 32 (two m16 rows of sub-tiles instead of four).
template <int WT, int SWI, int OCC, int BM = kBM>
__global__ void __launch_bounds__(kGThreads, OCC)
    k_gemm_q(const uint8_t* __restrict__ qs, int N, int K, const int8_t* __restrict__ xq,
             const float* __restrict__ xd, int M, float* __restrict__ y, int64_t y_stride,
             MatmulEpilogue ep, SwiOut so, float* __restrict__ part) {
    extern __shared__ __align__(128) uint8_t gsm[];
    using S = GStage<WT, BM>;
    constexpr int WR = BM / 2, MT = WR / 16;  // activation rows per warp, m16 sub-tiles
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int wm = warp >> 2, wn = warp & 3;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * kBN;
    const int p0 = blockIdx.x * (kBN / 2);
    // weight row of tile row r
    auto wrow = [&](int r) {
        if (SWI) return r < kBN / 2 ? p0 + r : so.F + p0 + r - kBN / 2;
        return min(n0 + r, N - 1);
    };
    const int nb = K / QK;
    const int ng = (nb + 63) / 64;
    const int ns = 16 * (ng - 1) + min(16, (nb - 64 * (ng - 1) + 1) / 2);  // stages with a valid block
    const int64_t rb = qrow_bytes(WT, K);
    const int64_t scale_base = (int64_t)nb * quant_bytes(WT);

    // stage t: g = t / 16, j = t % 16; local block lb -> global block gblk(lb)
    auto gblk = [&](int t, int lb) { return 64 * (t >> 4) + 2 * (t & 15) + (lb & 1) + 32 * (lb >> 1); };

    auto load = [&](int t, int buf) {
        uint8_t* st = gsm + buf * S::kBytes;
        uint8_t* sA = st;
        uint8_t* sB = sA + S::kA;
        uint8_t* sW = sB + S::kB;
        float* sX = (float*)(sW + S::kWs);
        // activations: 128 rows x 8 chunks of 16 B (chunk c: local block c/2, half c%2)
        for (int e = tid; e < BM * 8; e += kGThreads) {
            const int r = e >> 3, c = e & 7;
            const int gb = gblk(t, c >> 1);
            const int m = min(m0 + r, M - 1);
            cp_zfill<16>(sA + r * 128 + ((c ^ (r & 7)) << 4),
                         xq + (int64_t)m * K + (int64_t)gb * 32 + (c & 1) * 16, gb < nb);
        }
        for (int e = tid; e < BM * 4; e += kGThreads) {
            const int r = e >> 2, lb = e & 3;
            const int gb = gblk(t, lb);
            const int m = min(m0 + r, M - 1);
            cp_zfill<4>(sX + r * 4 + lb, xd + (int64_t)m * nb + gb, gb < nb);
        }
        // weights: Q4_0 rows of 4 chunks (one per local block), Q8_0 rows of 8 (4 low, 4 high)
        constexpr int CH = WT == T_Q8_0 ? 8 : 4;
        for (int e = tid; e < kBN * CH; e += kGThreads) {
            const int r = e / CH, c = e % CH;
            const int lb = c & 3;
            const int gb = gblk(t, lb);
            const int n = wrow(r);
            const uint8_t* src = qs + (int64_t)n * rb + (int64_t)((c >> 2) * nb + gb) * 16;
            const int phys = WT == T_Q8_0 ? (c ^ (r & 7)) : (c ^ ((r >> 1) & 3));
            cp_zfill<16>(sB + r * S::kRowB + phys * 16, src, gb < nb);
        }
        for (int r = tid; r < kBN; r += kGThreads) {
            const int n = wrow(r);
            cp_zfill<8>(sW + r * 8, qs + (int64_t)n * rb + scale_base + (t >> 4) * 128 + (t & 15) * 8,
                        true);
        }
    };

    float2 acc[MT][4][2];  // [m16][n8][row g / g+8] x (col 2tg, 2tg+1)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = make_float2(0.0f, 0.0f);

    // split K (gridDim.z > 1): this CTA's stages [tb, te), its partial sums to part
    const int tb = (int)((int64_t)ns * blockIdx.z / gridDim.z);
    const int te = (int)((int64_t)ns * (blockIdx.z + 1) / gridDim.z);
#pragma unroll
    for (int s = 0; s < kGStages - 1; ++s) {
        if (tb + s < te) load(tb + s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const float wsc = WT == T_Q4_0 ? 0.0625f : 1.0f;  // Q4_0 fragments hold 16 * (q - 8)
    for (int t = tb; t < te; ++t) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kGStages - 2) : "memory");
        __syncthreads();
        if (t + kGStages - 1 < te) load(t + kGStages - 1, (t - tb + kGStages - 1) % kGStages);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint8_t* st = gsm + ((t - tb) % kGStages) * S::kBytes;
        const uint8_t* sA = st;
        const uint8_t* sB = sA + S::kA;
        const __half* sW = (const __half*)(sB + S::kB);
        const float* sX = (const float*)((const uint8_t*)sW + S::kWs);
#pragma unroll(OCC == 2 ? 1 : 4)
        for (int lb = 0; lb < 4; ++lb) {
            unsigned af[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int q = lane >> 3;
                const int r = wm * WR + mt * 16 + (lane & 7) + ((q & 1) << 3);
                const int c = lb * 2 + (q >> 1);
                ldsm_x4(af[mt], sA + r * 128 + ((c ^ (r & 7)) << 4));
            }
            unsigned blo[4], bhi[4];
            {
                const int r = wn * 32 + lane;
                if (WT == T_Q8_0) {
                    unsigned t0[4], t1[4];
                    ldsm_x4(t0, sB + r * 128 + ((lb ^ (r & 7)) << 4));
                    ldsm_x4(t1, sB + r * 128 + (((4 + lb) ^ (r & 7)) << 4));
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) {
                        blo[nt] = t0[nt];
                        bhi[nt] = t1[nt];
                    }
                } else {
                    unsigned w4[4];
                    ldsm_x4(w4, sB + r * 64 + ((lb ^ ((r >> 1) & 3)) << 4));
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) {
                        blo[nt] = ((w4[nt] << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                        bhi[nt] = (w4[nt] & 0xF0F0F0F0u) ^ 0x80808080u;
                    }
                }
            }
            // scales of this block: sW/sX hold local blocks in the order [0, 2, 1, 3]
            const int si = ((lb & 1) << 1) | (lb >> 1);
            float2 dxv[MT][2], dwv[4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const float a0 = sX[(wm * WR + mt * 16 + g) * 4 + lb];
                const float a1 = sX[(wm * WR + mt * 16 + g + 8) * 4 + lb];
                dxv[mt][0] = make_float2(a0, a0);
                dxv[mt][1] = make_float2(a1, a1);
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int n = wn * 32 + nt * 8 + 2 * tg;
                dwv[nt] = make_float2(__fmul_rn(__half2float(sW[n * 4 + si]), wsc),
                                      __fmul_rn(__half2float(sW[(n + 1) * 4 + si]), wsc));
            }
            const float2 bias2 = make_float2(12582912.0f, 12582912.0f);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    int d[4];
                    mma_s8(d, af[mt], blo[nt], bhi[nt]);
                    // (dot * d_w) * d_x + acc, two outputs per packed instruction
                    const float2 v0 = sub2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), bias2);
                    const float2 v1 = sub2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), bias2);
                    acc[mt][nt][0] = fma2(mul2(v0, dwv[nt]), dxv[mt][0], acc[mt][nt][0]);
                    acc[mt][nt][1] = fma2(mul2(v1, dwv[nt]), dxv[mt][1], acc[mt][nt][1]);
                }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if constexpr (SWI != 0) {
        // the tile's results through shared memory (the stage ring is free now), then one warp
        // per (activation row, 32-unit block): ggml_vec_swiglu_f32 (vec.cpp:417-426) and
        // quantize_row_q8_0 of the block
        constexpr int kLd = kBN + 4;
        float* tile = (float*)gsm;
        __syncthreads();
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = wm * WR + mt * 16 + g + ((e >> 1) << 3);
                    const int n = wn * 32 + nt * 8 + 2 * tg + (e & 1);
                    const float2 pv = acc[mt][nt][e >> 1];
                    tile[m * kLd + n] = (e & 1) ? pv.y : pv.x;
                }
        __syncthreads();
        for (int task = warp; task < BM * 2; task += kGThreads / 32) {
            const int m = task >> 1, j = (task & 1) * 32 + lane;
            if (m0 + m >= M) continue;  // warp-uniform
            const float h = __fmul_rn(ref_v_silu(tile[m * kLd + j]), tile[m * kLd + kBN / 2 + j]);
            const int64_t gm = m0 + m, col = p0 + j;
            if (so.y) so.y[gm * so.y_stride + col] = h;
            if (so.yq) {
                float d16, q;
                q8_block(h, lane, d16, q);
                so.yq[gm * so.F + col] = (int8_t)__float2int_rn(q);
                if (lane == 0) so.yd[gm * (so.F / 32) + col / 32] = d16;
            }
        }
    } else if (gridDim.z > 1) {  // split K: the partial sums, finished by k_splitk_sum
        float* pz = part + (int64_t)blockIdx.z * M * N;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = m0 + wm * WR + mt * 16 + g + ((e >> 1) << 3);
                    const int n = n0 + wn * 32 + nt * 8 + 2 * tg + (e & 1);
                    if (m < M && n < N) {
                        const float2 p = acc[mt][nt][e >> 1];
                        pz[(int64_t)m * N + n] = (e & 1) ? p.y : p.x;
                    }
                }
    } else {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = m0 + wm * WR + mt * 16 + g + ((e >> 1) << 3);
                    const int n = n0 + wn * 32 + nt * 8 + 2 * tg + (e & 1);
                    if (m < M && n < N) {
                        const float2 p = acc[mt][nt][e >> 1];
                        float r = (e & 1) ? p.y : p.x;
                        if (ep.bias) r = __fadd_rn(r, ep.bias[n]);
                        if (ep.residual) r = __fadd_rn(ep.residual[(int64_t)m * ep.res_stride + n], r);
                        y[(int64_t)m * y_stride + n] = r;
                    }
                }
    }
}

// The split-K partial sums of a plain GEMM added in split order, then bias and residual as in
// k_gemm_q's own epilogue.  One thread per output element.
__global__ void k_splitk_sum(const float* __restrict__ part, int S, int M, int N, float* y,
                             int64_t y_stride, MatmulEpilogue ep) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)M * N) return;
    const int m = (int)(i / N), n = (int)(i % N);
    float r = part[i];
    for (int z = 1; z < S; ++z) r = __fadd_rn(r, part[(int64_t)z * M * N + i]);
    if (ep.bias) r = __fadd_rn(r, ep.bias[n]);
    if (ep.residual) r = __fadd_rn(ep.residual[(int64_t)m * ep.res_stride + n], r);
    y[(int64_t)m * y_stride + n] = r;
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

template <int WT, int SWI, int OCC, int BM = kBM>
void run_gemm(dim3 grid, const uint8_t* qs, int N, int K, const int8_t* xq, const float* xd,
              int M, float* y, int64_t y_stride, const MatmulEpilogue& ep, const SwiOut& so,
              cudaStream_t st, float* part = nullptr) {
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    {
        static std::mutex mu;
        static bool configured[64] = {};
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev & 63]) {
            GB_CUDA(cudaFuncSetAttribute(k_gemm_q<WT, SWI, OCC, BM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kGStages * GStage<WT, BM>::kBytes));
            configured[dev & 63] = true;
        }
    }
    k_gemm_q<WT, SWI, OCC, BM><<<grid, kGThreads, kGStages * GStage<WT, BM>::kBytes, st>>>(
        qs, N, K, xq, xd, M, y, y_stride, ep, so, part);
}

// 64-row tiles for launches of at most 64 rows (GGMLC_B200_GEMM64=0: off)
bool gemm64_enabled() {
    static const bool v = [] {
        const char* e = getenv("GGMLC_B200_GEMM64");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return v;
}

void launch_gemm_block(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                       int64_t y_stride, const MatmulEpilogue& ep, const SwiOut& so,
                       cudaStream_t st) {
    GB_CHECK(w.N < (1LL << 31) && w.K < (1LL << 31) && M < (1LL << 31), "matmul: shape too large");
    GB_CHECK(((uintptr_t)xq & 15) == 0, "matmul: xq must be 16-byte aligned");
    const bool swi = so.F > 0;
    const int64_t tiles = swi ? so.F / (kBN / 2) : (w.N + kBN - 1) / kBN;
    // launches of at most 64 activation rows take 64-row tiles (half of a 128-row tile would be
    // padding), two CTAs per SM
    const bool half = M <= 64 && gemm64_enabled();
    const int bm = half ? 64 : kBM;
    dim3 grid((unsigned)tiles, (unsigned)((M + bm - 1) / bm));
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    const uint8_t* qs = (const uint8_t*)w.qs;
    const int N = (int)w.N, K = (int)w.K, m = (int)M;
    const int sms = sm_count(dev);
    // A plain GEMM with tiles for at most half the SMs (few weight rows and few activation rows,
    // as in the operator sweep's M = 64 cells) splits K over gridDim.z: at most one wave (two
    // CTAs per SM for Q4_0, whose stages fit two, one for Q8_0) and at least 8 stages a split;
    // the partial sums are added in split order by k_splitk_sum.  Measured: Q4_0 4096 x 4096 at
    // 64 rows 76 -> 38 us, 4096 x 14336 246 -> 76 us; with 112-128 tiles (the 512-row prefill's
    // O and down projections) splitting measured slower, so those run whole.
    const int64_t ntile = tiles * grid.y;
    const int ns = (int)((K / QK + 3) / 4);
    const int64_t slots = (w.type == T_Q4_0 ? 2 : 1) * (int64_t)sms;
    int splits = 1;
    if (!swi && 2 * ntile <= sms && splitk_enabled())
        splits = (int)std::max<int64_t>(
            1, std::min<int64_t>(std::min<int64_t>(slots / ntile, ns / 8), 16));
    float* part = nullptr;
    if (splits > 1) {
        grid.z = (unsigned)splits;
        GB_CUDA(cudaMallocAsync((void**)&part, (size_t)splits * M * w.N * sizeof(float), st));
    }
    // Q4_0 stages fit two CTAs per SM: worth it once there are tiles for two per SM
    const bool two = w.type == T_Q4_0 && (splits > 1 || ntile >= 2 * (int64_t)sms);
    if (half && w.type == T_Q8_0) {
        if (swi) run_gemm<T_Q8_0, 1, 2, 64>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st);
        else run_gemm<T_Q8_0, 0, 2, 64>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st, part);
    } else if (half) {
        if (swi) run_gemm<T_Q4_0, 1, 2, 64>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st);
        else run_gemm<T_Q4_0, 0, 2, 64>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st, part);
    } else if (w.type == T_Q8_0) {
        if (swi) run_gemm<T_Q8_0, 1, 1>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st);
        else run_gemm<T_Q8_0, 0, 1>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st, part);
    } else if (two) {
        if (swi) run_gemm<T_Q4_0, 1, 2>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st);
        else run_gemm<T_Q4_0, 0, 2>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st, part);
    } else {
        if (swi) run_gemm<T_Q4_0, 1, 1>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st);
        else run_gemm<T_Q4_0, 0, 1>(grid, qs, N, K, xq, xd, m, y, y_stride, ep, so, st, part);
    }
    GB_CUDA(cudaGetLastError());
    if (splits > 1) {
        launch_splitk_sum(part, splits, m, N, y, y_stride, ep, st);
        GB_CUDA(cudaFreeAsync(part, st));
    }
}

}  // namespace

bool splitk_enabled() {
    static const bool v = [] {
        const char* e = getenv("GGMLC_B200_SPLITK");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return v;
}

void launch_splitk_sum(const float* part, int splits, int M, int N, float* y, int64_t y_stride,
                       const MatmulEpilogue& ep, cudaStream_t st) {
    const int64_t n = (int64_t)M * N;
    if (n == 0) return;
    k_splitk_sum<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, splits, M, N, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

// Prefill GEMM path (M > 16 rows), chosen by measurement on B200: Q8_0 weights go to the tcgen05
// kernel (k_gemm_tc.cu, 10-12% faster than the mma.sync kernel at every prefill shape measured),
// Q4_0 weights to the mma.sync block kernel (7-10% faster there: the tcgen05 path widens the
// nibbles to int8 in shared memory first).  The tcgen05 kernel needs K % 128 == 0.  The
// environment variable GGMLC_B200_GEMM = "mma" or "tc" forces one path; it is read at every
// launch, so one process can time both.
static bool use_gemm_tc(const QWeight& w) {
    if (!gemm_tc_fits(w.K)) return false;
    const char* e = std::getenv("GGMLC_B200_GEMM");
    if (e && std::strcmp(e, "mma") == 0) return false;
    if (e && std::strcmp(e, "tc") == 0) return true;
    return w.type == T_Q8_0;
}

void launch_gemm_swiglu(const GemvArgs& a, cudaStream_t st) {
    GB_CHECK(a.xq && a.xd && !a.xf, "gemm swiglu: Q8_0 input required");
    GB_CHECK(a.w.type == T_Q8_0 || a.w.type == T_Q4_0, "gemm swiglu: quantized weights required");
    GB_CHECK(a.w.N == 2 * a.F && a.F % (kBN / 2) == 0, "gemm swiglu: N == 2F with F % 64 == 0");
    GB_CHECK(!a.bias && !a.residual, "gemm swiglu: no bias / residual");
    GB_CHECK(a.y || a.yq, "gemm swiglu: no output");
    GB_CHECK(!a.yq == !a.yd, "gemm swiglu: Q8_0 output needs quants and scales");
    if (a.M == 0) return;
    if (use_gemm_tc(a.w)) {  // the tcgen05 GEMM with the same epilogue
        launch_gemm_tc_swiglu(a, st);
        return;
    }
    SwiOut so;
    so.F = (int)a.F;
    so.y = a.y;
    so.y_stride = a.y_stride;
    so.yq = a.yq;
    so.yd = a.yd;
    launch_gemm_block(a.w, a.xq, a.xd, a.M, nullptr, 0, MatmulEpilogue(), so, st);
}

void launch_matmul_q(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    GB_CHECK(w.K % QK == 0, "matmul: K must be a multiple of 32");
    if (M == 0 || w.N == 0) return;
    if (M <= kMmvMaxRows) {
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
    if (use_gemm_tc(w)) {  // prefill on tcgen05 (TMA stages of 4 blocks: K % 128 == 0)
        launch_gemm_tc(w, xq, xd, M, y, y_stride, ep, st);
        return;
    }
    launch_gemm_block(w, xq, xd, M, y, y_stride, ep, SwiOut(), st);
}

void launch_matmul_f(const QWeight& w, const float* x, int64_t x_stride, int64_t M, float* y,
                     int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    if (M == 0 || w.N == 0) return;
    dim3 grid((unsigned)((w.N + 3) / 4), (unsigned)M);
    k_matmul_f<<<grid, 128, 0, st>>>(w, x, x_stride, M, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
