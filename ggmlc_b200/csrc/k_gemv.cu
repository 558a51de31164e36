// Decode GEMV (M <= 8) over the super-group weight layout, bit-exact with the reference CPU
// kernels, with optional fused RMSNorm+quantize prologue and SwiGLU+quantize epilogue.
//
// Arithmetic order.  The reference's x86 kernels (ggml_vec_dot_q{8,4}_0_q8_0,
// arch/x86/quants.c:1308-1342 and :701; llamafile tinyBLAS_Q0_AVX, sgemm.cpp:1353) keep 8 fp32
// lanes per output: lane i accumulates, block after block, fma(d_w*d_x, float(int dot of
// elements 4i..4i+3), acc_i); the lanes are reduced ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)).  A
// quad of consumer threads owns an output row; thread t carries lanes t and t+4.
//
// Data movement.  A producer warp streams each tile of R weight rows through a 4-stage shared
// memory ring: one cp.async.bulk per row and stage (a contiguous run of C super-groups of that
// row), completion tracked by mbarrier transaction counts; consumers release a stage with an
// mbarrier arrive.  No TMA multicast is used.  Every wait is bounded: on timeout the kernel
// records an error code in *err and returns instead of hanging.
//
// Q4_0 nibbles become int8 with a shift and two bitwise ops: (q<<4) ^ 0x80 read as int8 is
// 16*(q-8), so dp4a yields 16x the lane dot; the activation scales are staged pre-divided by 16
// (exact: a power of two), which makes fma(d_w*(d_x/16), 16p, acc) the same rounding as the
// CPU's fma(d_w*d_x, p, acc).
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kStages = 4;
constexpr int kStageTarget = 18 * 1024;  // bytes of weights per stage
constexpr size_t kSmemMax = 220 * 1024;
constexpr long long kSpinLimit = 1LL << 26;  // bounded mbarrier waits (then error + exit)

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// returns false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
    const unsigned addr = smem_u32(bar);
    for (long long i = 0; i < kSpinLimit; ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void consumers_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ float h2f_lo(unsigned v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(unsigned v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// 4 blocks of one row (group) against the staged activations of blocks b0..b0+3
template <int WT, int MAXM>
__device__ __forceinline__ void consume_group(const uint8_t* grp, const float dw[4], int b0, int nb,
                                              int t, int M, const uint8_t* sx, const float* sxd,
                                              int nbx, float (&acc0)[MAXM], float (&acc1)[MAXM]) {
    int wl[4], wh[4];
    if (WT == T_Q8_0) {
        const uint4 a = *(const uint4*)(grp + t * 32);
        const uint4 b = *(const uint4*)(grp + t * 32 + 16);
        wl[0] = a.x; wh[0] = a.y; wl[1] = a.z; wh[1] = a.w;
        wl[2] = b.x; wh[2] = b.y; wl[3] = b.z; wh[3] = b.w;
    } else {
        const uint4 a = *(const uint4*)(grp + t * 16);
        const unsigned wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wl[j] = (int)(((wv[j] << 4) & 0xF0F0F0F0u) ^ 0x80808080u);  // 16*(q_lo - 8)
            wh[j] = (int)((wv[j] & 0xF0F0F0F0u) ^ 0x80808080u);         // 16*(q_hi - 8)
        }
    }
    const int jmax = min(4, nb - b0);
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
            const uint8_t* xs = sx + m * nbx * 32 + (b0 >> 2) * 128 + t * 32;
            const uint4 xa = *(const uint4*)xs, xb = *(const uint4*)(xs + 16);
            const float4 dx = *(const float4*)(sxd + m * nbx + b0);
            const int xl[4] = {(int)xa.x, (int)xa.z, (int)xb.x, (int)xb.z};
            const int xh[4] = {(int)xa.y, (int)xa.w, (int)xb.y, (int)xb.w};
            const float dxf[4] = {dx.x, dx.y, dx.z, dx.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < jmax) {
                    const float s = __fmul_rn(dw[j], dxf[j]);
                    acc0[m] = __fmaf_rn(s, __int2float_rn(__dp4a(wl[j], xl[j], 0)), acc0[m]);
                    acc1[m] = __fmaf_rn(s, __int2float_rn(__dp4a(wh[j], xh[j], 0)), acc1[m]);
                }
            }
        }
    }
}

__device__ double cons_sum_d(double v, double* sh, int nthreads) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    consumers_sync(nthreads);
    if (l == 0) sh[w] = v;
    consumers_sync(nthreads);
    double t = 0.0;
    for (int i = 0; i < nthreads / 32; ++i) t += sh[i];
    return t;
}

// Activation staging by the consumer threads: Q8_0 words at x_word_off, scales (divided by 16
// for Q4_0 weights) as fp32.
template <int WT, int IN>
__device__ void stage_inputs(const GemvArgs& a, int nb, int nbx, uint8_t* sx, float* sxd,
                             double* shd, int nthreads) {
    const int K = (int)a.w.K;
    const float dscale = WT == T_Q4_0 ? 0.0625f : 1.0f;
    if (IN == 0) {
        for (int idx = threadIdx.x; idx < a.M * nbx * 8; idx += nthreads) {
            const int m = idx / (nbx * 8), r = idx % (nbx * 8), b = r >> 3, w = r & 7;
            const int v = b < nb ? __ldg((const int*)(a.xq + (int64_t)m * K + b * 32) + w) : 0;
            *(int*)(sx + m * nbx * 32 + x_word_off(b, w)) = v;
        }
        for (int idx = threadIdx.x; idx < a.M * nbx; idx += nthreads) {
            const int m = idx / nbx, b = idx % nbx;
            sxd[idx] = b < nb ? __fmul_rn(a.xd[(int64_t)m * nb + b], dscale) : 0.0f;
        }
    } else {
        // RMSNorm (ggml-cpu/ops.cpp:3859-3920) then Q8_0 (arch/x86/quants.c:302-392)
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = nthreads >> 5;
        for (int m = 0; m < a.M; ++m) {
            const float* xr = a.xf + (int64_t)m * a.xf_stride;
            double s = 0.0;
            for (int k = threadIdx.x; k < K; k += nthreads) {
                const float v = xr[k];
                s += (double)__fmul_rn(v, v);
            }
            s = cons_sum_d(s, shd, nthreads);
            const float mean = (float)(s / (double)K);
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            for (int b = warp; b < nbx; b += nw) {
                float d16 = 0.0f, q = 0.0f;
                if (b < nb) {
                    float v = __fmul_rn(xr[b * 32 + lane], scale);
                    if (a.gamma) v = __fmul_rn(v, a.gamma[b * 32 + lane]);
                    q8_block(v, lane, d16, q);
                }
                sx[m * nbx * 32 + x_word_off(b, lane >> 2) + (lane & 3)] =
                    (uint8_t)(int8_t)__float2int_rn(q);
                if (lane == 0) sxd[m * nbx + b] = __fmul_rn(d16, dscale);
            }
        }
    }
}

struct Geo {
    int R;           // rows per tile (32, or 64 for SwiGLU: 32 gate + 32 up)
    int C;           // super-groups per row and stage
    int nsg;         // super-groups per row
    int nchunk;      // stages per tile
    int ntiles;
    int row_chunk;   // bytes per row and stage (C * sg bytes)
};

template <int WT, int SWI>
__host__ __device__ inline Geo make_geo(int64_t N, int64_t K, int64_t F) {
    Geo g;
    g.R = SWI ? 64 : 32;
    const int sgb = (int)sg_bytes(WT);
    g.C = kStageTarget / (g.R * sgb);
    if (g.C < 1) g.C = 1;
    g.nsg = (int)n_sg(K);
    if (g.C > g.nsg) g.C = g.nsg;
    g.nchunk = (g.nsg + g.C - 1) / g.C;
    g.ntiles = SWI ? (int)(F / 32) : (int)((N + 31) / 32);
    g.row_chunk = g.C * sgb;
    return g;
}

template <int WT, int MAXM, int IN, int SWI>
__global__ void k_gemv_fused(GemvArgs a, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double shd[8];
    __shared__ float sres[SWI ? MAXM * 64 : 1];
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
    const int K = (int)a.w.K;
    const int N = (int)a.w.N;
    const int nb = K / QK;
    const int nbx = (nb + 3) & ~3;
    const Geo geo = make_geo<WT, SWI>(a.w.N, a.w.K, a.F);
    const int nthreads = geo.R * 4;  // consumer threads; the last warp is the producer
    const int sgb = (int)sg_bytes(WT);
    const int64_t rb = qrow_bytes(WT, K);
    uint8_t* sx = smem;
    float* sxd = (float*)(smem + (size_t)MAXM * nbx * 32);
    const size_t act_bytes = ((size_t)MAXM * nbx * 36 + 127) & ~(size_t)127;
    uint8_t* stages = smem + act_bytes;
    const int stage_bytes = geo.R * geo.row_chunk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], nthreads / 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint8_t* qs = (const uint8_t*)a.w.qs;
    if (threadIdx.x >= nthreads) {
        // ---------------- producer warp ----------------
        if (threadIdx.x != nthreads) return;
        int it = 0;
        for (int tile = blockIdx.x; tile < geo.ntiles; tile += gridDim.x) {
            for (int c = 0; c < geo.nchunk; ++c, ++it) {
                const int st = it % kStages;
                if (it >= kStages && !mbar_wait(&empty_bar[st], ((it / kStages) - 1) & 1)) {
                    atomicExch(err, 1);
                    return;
                }
                const int nsg_here = min(geo.C, geo.nsg - c * geo.C);
                const unsigned bytes = (unsigned)(nsg_here * sgb);
                mbar_expect_tx(&full_bar[st], bytes * geo.R);
                uint8_t* dst = stages + (size_t)st * stage_bytes;
                for (int r = 0; r < geo.R; ++r) {
                    int row;
                    if (SWI) row = r < 32 ? tile * 32 + r : (int)a.F + tile * 32 + (r - 32);
                    else row = tile * 32 + r;
                    if (row >= N) row = N - 1;
                    bulk_g2s(dst + r * geo.row_chunk, qs + (int64_t)row * rb + (int64_t)c * geo.C * sgb,
                             bytes, &full_bar[st]);
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    stage_inputs<WT, IN>(a, nb, nbx, sx, sxd, shd, nthreads);
    consumers_sync(nthreads);
    const int t = threadIdx.x & 3;
    const int quad = threadIdx.x >> 2;
    const int lane = threadIdx.x & 31;
    int it = 0;
    for (int tile = blockIdx.x; tile < geo.ntiles; tile += gridDim.x) {
        float acc0[MAXM], acc1[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc0[m] = acc1[m] = 0.0f;
        for (int c = 0; c < geo.nchunk; ++c, ++it) {
            const int st = it % kStages;
            if (!mbar_wait(&full_bar[st], (it / kStages) & 1)) {
                atomicExch(err, 2);
                return;
            }
            const uint8_t* rowbuf = stages + (size_t)st * stage_bytes + quad * geo.row_chunk;
            const int nsg_here = min(geo.C, geo.nsg - c * geo.C);
            for (int sg = 0; sg < nsg_here; ++sg) {
                const uint8_t* sgp = rowbuf + sg * sgb;
                const int b0 = (c * geo.C + sg) * 8;
                const uint4 sc = *(const uint4*)(sgp + (WT == T_Q8_0 ? 256 : 128));
                const float d0[4] = {h2f_lo(sc.x), h2f_hi(sc.x), h2f_lo(sc.y), h2f_hi(sc.y)};
                const float d1[4] = {h2f_lo(sc.z), h2f_hi(sc.z), h2f_lo(sc.w), h2f_hi(sc.w)};
                consume_group<WT, MAXM>(sgp, d0, b0, nb, t, a.M, sx, sxd, nbx, acc0, acc1);
                if (b0 + 4 < nb)
                    consume_group<WT, MAXM>(sgp + (WT == T_Q8_0 ? 128 : 64), d1, b0 + 4, nb, t, a.M,
                                            sx, sxd, nbx, acc0, acc1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[st]);
        }
        // reduce the quad: t_t = a_t + a_{t+4}, then (t0 + t2) + (t1 + t3)
        const int row = SWI ? 0 : tile * 32 + quad;
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < a.M) {
                const float tt = __fadd_rn(acc0[m], acc1[m]);
                const float u = __fadd_rn(tt, __shfl_down_sync(0xffffffffu, tt, 2, 4));
                float res = __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 1, 4));
                if (t == 0) {
                    if (SWI) {
                        sres[m * 64 + quad] = res;
                    } else if (row < N) {
                        if (a.bias) res = __fadd_rn(res, a.bias[row]);
                        if (a.residual) res = __fadd_rn(a.residual[(int64_t)m * a.res_stride + row], res);
                        a.y[(int64_t)m * a.y_stride + row] = res;
                    }
                }
            }
        }
        if (SWI) {
            consumers_sync(nthreads);
            const int warp = threadIdx.x >> 5;
            for (int m = warp; m < a.M; m += nthreads / 32) {
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
            consumers_sync(nthreads);
        }
    }
}

template <int WT, int SWI>
size_t smem_bytes(int maxm, int64_t N, int64_t K, int64_t F) {
    const Geo g = make_geo<WT, SWI>(N, K, F);
    const int64_t nbx = ((K / 32) + 3) & ~3;
    const size_t act = ((size_t)maxm * nbx * 36 + 127) & ~(size_t)127;
    return act + (size_t)kStages * g.R * g.row_chunk;
}

int* g_err_dev[32] = {nullptr};

int* err_slot(int dev) {
    if (!g_err_dev[dev & 31]) {
        GB_CUDA(cudaMalloc(&g_err_dev[dev & 31], sizeof(int)));
        GB_CUDA(cudaMemset(g_err_dev[dev & 31], 0, sizeof(int)));
    }
    return g_err_dev[dev & 31];
}

template <int WT, int MAXM, int IN, int SWI>
void launch_t(const GemvArgs& a, cudaStream_t st) {
    const size_t smem = smem_bytes<WT, SWI>(MAXM, a.w.N, a.w.K, a.F);
    GB_CHECK(smem <= kSmemMax, "gemv: shared-memory stage too large");
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static unsigned configured = 0;
    if (!(configured & (1u << (dev & 31)))) {
        GB_CUDA(cudaFuncSetAttribute(k_gemv_fused<WT, MAXM, IN, SWI>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax));
        configured |= 1u << (dev & 31);
    }
    const Geo g = make_geo<WT, SWI>(a.w.N, a.w.K, a.F);
    const int per_sm = smem <= 110 * 1024 ? 2 : 1;
    const int blocks = g.ntiles < 148 * per_sm ? g.ntiles : 148 * per_sm;
    k_gemv_fused<WT, MAXM, IN, SWI><<<blocks, g.R * 4 + 32, smem, st>>>(a, err_slot(dev));
    GB_CUDA(cudaGetLastError());
}

template <int WT, int IN, int SWI>
void launch_m(const GemvArgs& a, cudaStream_t st) {
    if (a.M == 1) launch_t<WT, 1, IN, SWI>(a, st);
    else if (a.M <= 4) launch_t<WT, 4, IN, SWI>(a, st);
    else launch_t<WT, 8, IN, SWI>(a, st);
}

}  // namespace

void gemv_prepare_device(int dev) { (void)err_slot(dev); }

int gemv_error_code(int dev) {
    if (!g_err_dev[dev & 31]) return 0;
    int v = 0;
    GB_CUDA(cudaMemcpy(&v, g_err_dev[dev & 31], sizeof(int), cudaMemcpyDeviceToHost));
    return v;
}

bool gemv_fused_fits(int64_t K, int M) {
    if (M < 1 || M > 8 || K % QK != 0) return false;
    const int maxm = M == 1 ? 1 : (M <= 4 ? 4 : 8);
    const size_t worst = std::max(smem_bytes<T_Q8_0, 1>(maxm, 64, K, 32),
                                  smem_bytes<T_Q4_0, 1>(maxm, 64, K, 32));
    return worst <= kSmemMax;
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
