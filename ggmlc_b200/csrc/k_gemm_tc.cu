// Prefill MUL_MAT (M > 16 activation rows) on the 5th-generation tensor cores: tcgen05.mma
// kind::i8 with accumulators in tensor memory, per-block fp16 scales applied by epilogue warps.
//
// Arithmetic.  One tcgen05.mma (M = 128 weight rows, N = 128 activation rows, K = 32) per
// 32-element block writes every exact int32 block dot of a 128 x 128 tile into a tensor-memory
// accumulator.  Epilogue warps load it, add the 1.5*2^23 bias as an integer (so the bits read as
// the float 12582912 + sumi) and subtract it in fp32, multiply by d_w * d_x and accumulate the
// block terms in fp32 registers — the block formula of the reference's vec_dot
// (ggml-cpu/quants.c:225-256, :451-477) with the integer part exact.  Q4_0 nibbles are widened
// in shared memory to 16 * (q - 8) (exact in int8); their weight scales are divided by 16 to
// compensate.
//
// Work split per CTA (128 weight rows x 128 activation rows, 12 warps):
//   warps 0-2   producers: cp.async of activations / weights / scales for a stage of 4 blocks
//               into the canonical no-swizzle K-major layout (8-row x 16-byte core matrices,
//               K-adjacent core matrices 2048 B apart, row groups 128 B apart), Q4_0 nibble
//               widening and scale conversion, then mbarrier "full";
//   warp 3      MMA issuer (one thread) and tensor-memory owner: 4 accumulators of 128 columns,
//               one tcgen05.mma + tcgen05.commit per block;
//   warps 4-11  epilogue: warp w reads tensor-memory lanes 32*(w%4).. (its weight rows) and
//               columns 64*((w-4)/4).. (activation rows) of each finished block with
//               tcgen05.ld, releases the accumulator as soon as the loads land, then scales.
// Every wait on an mbarrier is bounded: past the limit the kernel records an error in
// gemm_tc_error, stops issuing, waits (bounded) for its tensor-core work to drain, frees the
// tensor memory and returns.
//
// K order: a stage takes blocks {64g+2j, 64g+2j+1, 64g+32+2j, 64g+32+2j+1}, the order in which
// the weight scale region stores them, so one 8-byte copy brings a row's four scales.
#include <cuda_fp16.h>

#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kTM = 128;            // weight rows per tile (MMA M, tensor-memory lanes)
constexpr int kTN = 128;            // activation rows per tile (MMA N, tensor-memory columns)
constexpr int kTB = 4;              // blocks per stage
constexpr int kTS = 4;              // stages in the ring
constexpr int kTBufs = 4;           // tensor-memory accumulators (128 columns each)
constexpr int kProd = 96;           // producer threads (warps 0-2)
constexpr int kMmaWarp = 3;
constexpr int kEpiWarp0 = 4, kEpiWarps = 8;
constexpr int kTThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kTmemCols = 512;
constexpr uint32_t kBiasBits = 0x4B400000u;      // 1.5 * 2^23
constexpr long long kSpinCycles = 4000000000LL;  // about 2 s at 1.9 GHz

template <int WT>
struct TcStage {
    static constexpr int kA = kTB * 4096;                           // weights, widened to int8
    static constexpr int kB = kTB * 4096;                           // activations
    static constexpr int kRaw = WT == T_Q4_0 ? kTB * kTM * 16 : 0;  // packed Q4_0 nibbles
    static constexpr int kWsr = kTM * 8;                            // 4 fp16 weight scales per row
    static constexpr int kWs = kTB * kTM * 4;                       // fp32 weight scales [block][row]
    static constexpr int kXs = kTB * kTN * 4;                       // fp32 activation scales
    static constexpr int kBytes = kA + kB + kRaw + kWsr + kWs + kXs;
    static_assert(kBytes % 128 == 0, "stage alignment");
};

__device__ int gemm_tc_error_word;

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp16z(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp8z(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(su32(dst)), "l"(src),
                 "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp4z(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(su32(dst)), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return done != 0;
}
// bounded wait on phase parity; false (and the CTA abort flag set) when it runs out
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_test(b, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kSpinCycles) {
            *abort = 1;
            atomicExch(&gemm_tc_error_word, 1);
            return false;
        }
    }
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(b))
                 : "memory");
}
// K-major, no swizzle: core matrices of 8 rows x 16 B; K-adjacent ones 2048 B apart (leading
// byte offset), row groups 128 B apart (stride byte offset); descriptor version 1 (tcgen05)
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
    const uint32_t a = su32(p);
    return (uint64_t)((a & 0x3FFFF) >> 4) | ((uint64_t)(2048 >> 4) << 16) |
           ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}
// kind::i8, D s32, A / B signed 8-bit, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);

// D = A * B (enable-input-d false: each block's dots overwrite the accumulator)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(0)
        : "memory");
}

#define GB_TC_R32(v)                                                                          \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),      \
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),           \
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),        \
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),        \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])

// issue a load of 32 consecutive columns of this thread's tensor-memory lane (no wait)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : GB_TC_R32(v)
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 block terms of one accumulator slice: acc[j] += (v - bias) * (dw * dx)
__device__ __forceinline__ void scale_acc(const uint32_t (&v)[32], float dw, const float* dx,
                                          float2* acc) {
    const float2 bias2 = make_float2(12582912.0f, 12582912.0f);
    const float2 dw2 = make_float2(dw, dw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 x4 = *(const float4*)(dx + 4 * j);
        const float2 p0 = mul2(dw2, make_float2(x4.x, x4.y));
        const float2 p1 = mul2(dw2, make_float2(x4.z, x4.w));
        const float2 f0 = sub2(make_float2(__uint_as_float(v[4 * j] + kBiasBits),
                                           __uint_as_float(v[4 * j + 1] + kBiasBits)),
                               bias2);
        const float2 f1 = sub2(make_float2(__uint_as_float(v[4 * j + 2] + kBiasBits),
                                           __uint_as_float(v[4 * j + 3] + kBiasBits)),
                               bias2);
        acc[2 * j] = fma2(f0, p0, acc[2 * j]);
        acc[2 * j + 1] = fma2(f1, p1, acc[2 * j + 1]);
    }
}

template <int WT>
__global__ void __launch_bounds__(kTThreads, 1)
    k_gemm_tc(const uint8_t* __restrict__ qs, int N, int K, const int8_t* __restrict__ xq,
              const float* __restrict__ xd, int M, float* __restrict__ y, int64_t y_stride,
              MatmulEpilogue ep) {
    using S = TcStage<WT>;
    extern __shared__ __align__(128) uint8_t tsm[];
    __shared__ __align__(8) uint64_t bar_full[kTS], bar_empty[kTS], bar_tfull[kTBufs],
        bar_tempty[kTBufs], bar_done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    volatile int* abort = &s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTM, m0 = blockIdx.y * kTN;
    const int nb = K / QK;
    const int ng = (nb + 63) / 64;
    const int ns = 16 * (ng - 1) + min(16, (nb - 64 * (ng - 1) + 1) / 2);
    const int64_t rb = qrow_bytes(WT, K);
    const int64_t scale_base = (int64_t)nb * quant_bytes(WT);
    auto gblk = [](int t, int lb) { return 64 * (t >> 4) + 2 * (t & 15) + (lb & 1) + 32 * (lb >> 1); };
    auto stage = [&](int s) { return tsm + s * S::kBytes; };

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kTS; ++s) {
            mbar_init(&bar_full[s], kProd);
            mbar_init(&bar_empty[s], 1 + kEpiWarps);
        }
        for (int b = 0; b < kTBufs; ++b) {
            mbar_init(&bar_tfull[b], 1);
            mbar_init(&bar_tempty[b], kEpiWarps);
        }
        mbar_init(&bar_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(&s_tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp < kMmaWarp) {
        // ---------------------------------------------------------------- producers
        // Copies run rows-fastest (consecutive threads fill consecutive 16-byte slots of a core
        // matrix column); a thread widens and converts only what it copied itself, so its own
        // cp.async.wait_group is all the ordering a hand-off needs.
        const int p = tid;
        constexpr int L = 2;  // stages between issue and hand-off
        for (int t = 0; t < ns + L && !*abort; ++t) {
            if (t < ns) {
                const int s = t % kTS;
                if (t >= kTS && !mbar_wait(&bar_empty[s], ((t / kTS) - 1) & 1, abort)) break;
                uint8_t* st = stage(s);
                uint8_t* sA = st;
                uint8_t* sB = st + S::kA;
                uint8_t* sRaw = sB + S::kB;
                uint8_t* sWsr = sRaw + S::kRaw;
                float* sXs = (float*)(sWsr + S::kWsr + S::kWs);
                // activations: [block][half][row]
                for (int c = p; c < kTB * 2 * kTN; c += kProd) {
                    const int r = c & (kTN - 1), lh = c >> 7, lb = lh >> 1, half = lh & 1;
                    const int gb = gblk(t, lb);
                    const int m = min(m0 + r, M - 1);
                    cp16z(sB + lb * 4096 + half * 2048 + r * 16,
                          xq + (int64_t)m * K + (int64_t)min(gb, nb - 1) * 32 + half * 16,
                          gb < nb && m0 + r < M);
                }
                if (WT == T_Q8_0) {
                    for (int c = p; c < kTB * 2 * kTM; c += kProd) {
                        const int r = c & (kTM - 1), lh = c >> 7, lb = lh >> 1, half = lh & 1;
                        const int gb = gblk(t, lb);
                        const int n = min(n0 + r, N - 1);
                        cp16z(sA + lb * 4096 + half * 2048 + r * 16,
                              qs + (int64_t)n * rb + ((int64_t)half * nb + min(gb, nb - 1)) * 16,
                              gb < nb);
                    }
                } else {
                    for (int c = p; c < kTB * kTM; c += kProd) {
                        const int r = c & (kTM - 1), lb = c >> 7;
                        const int gb = gblk(t, lb);
                        const int n = min(n0 + r, N - 1);
                        cp16z(sRaw + (lb * kTM + r) * 16,
                              qs + (int64_t)n * rb + (int64_t)min(gb, nb - 1) * 16, gb < nb);
                    }
                }
                for (int r = p; r < kTM; r += kProd) {  // weight scales: one 8-byte run per row
                    const int n = min(n0 + r, N - 1);
                    cp8z(sWsr + r * 8,
                         qs + (int64_t)n * rb + scale_base + (t >> 4) * 128 + (t & 15) * 8, true);
                }
                for (int c = p; c < kTB * kTN; c += kProd) {  // activation scales [block][row]
                    const int r = c & (kTN - 1), lb = c >> 7;
                    const int gb = gblk(t, lb);
                    const int m = min(m0 + r, M - 1);
                    cp4z(sXs + lb * kTN + r, xd + (int64_t)m * nb + min(gb, nb - 1),
                         gb < nb && m0 + r < M);
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            if (t >= L) {
                const int tl = t - L, s = tl % kTS;
                asm volatile("cp.async.wait_group %0;" ::"n"(L) : "memory");
                uint8_t* st = stage(s);
                uint8_t* sA = st;
                uint8_t* sRaw = st + S::kA + S::kB;
                uint8_t* sWsr = sRaw + S::kRaw;
                float* sWs = (float*)(sWsr + S::kWsr);
                if (WT == T_Q4_0) {  // widen nibbles to int8 16*(q-8): low -> k 0..15, high -> 16..31
                    for (int c = p; c < kTB * kTM; c += kProd) {
                        const int r = c & (kTM - 1), lb = c >> 7;
                        const uint4 w = *(const uint4*)(sRaw + (lb * kTM + r) * 16);
                        uint4 lo, hi;
                        lo.x = ((w.x << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                        lo.y = ((w.y << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                        lo.z = ((w.z << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                        lo.w = ((w.w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                        hi.x = (w.x & 0xF0F0F0F0u) ^ 0x80808080u;
                        hi.y = (w.y & 0xF0F0F0F0u) ^ 0x80808080u;
                        hi.z = (w.z & 0xF0F0F0F0u) ^ 0x80808080u;
                        hi.w = (w.w & 0xF0F0F0F0u) ^ 0x80808080u;
                        uint8_t* d = sA + lb * 4096 + r * 16;
                        *(uint4*)d = lo;
                        *(uint4*)(d + 2048) = hi;
                    }
                }
                const float wsc = WT == T_Q4_0 ? 0.0625f : 1.0f;
                for (int r = p; r < kTM; r += kProd) {  // a row's scales to fp32, local block order
                    const __half* hs = (const __half*)(sWsr + r * 8);
#pragma unroll
                    for (int lb = 0; lb < kTB; ++lb) {
                        const int si = ((lb & 1) << 1) | (lb >> 1);
                        sWs[lb * kTM + r] = __fmul_rn(__half2float(hs[si]), wsc);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&bar_full[s]);
            }
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = true;
            for (int t = 0; t < ns && ok; ++t) {
                const int s = t % kTS;
                if (!mbar_wait(&bar_full[s], (t / kTS) & 1, abort)) break;
                tc_fence_after();
                const uint8_t* st = stage(s);
                for (int lb = 0; lb < kTB; ++lb) {
                    const int b = t * kTB + lb, buf = b & (kTBufs - 1);
                    if (!mbar_wait(&bar_tempty[buf], (b >> 2) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tc_mma(tmem + buf * kTN, smem_desc(st + lb * 4096),
                           smem_desc(st + S::kA + lb * 4096));
                    tc_commit(&bar_tfull[buf]);
                }
                if (ok) tc_commit(&bar_empty[s]);
            }
            // every issued MMA has completed once this commit arrives
            tc_commit(&bar_done);
            const long long t0 = clock64();
            bool done = false;
            while (!done && clock64() - t0 < kSpinCycles) done = mbar_test(&bar_done, 0);
            if (!done) {
                *abort = 1;
                atomicExch(&gemm_tc_error_word, 2);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
        const int r = q * 32 + lane;  // weight row of the tile (tensor-memory lane)
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + h * 64;
        // every accumulator starts free
        if (lane == 0)
            for (int buf = 0; buf < kTBufs; ++buf) mbar_arrive(&bar_tempty[buf]);
        float2 acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.0f, 0.0f);
        // waits are made warp-uniform by a vote: tensor-memory loads and stores need the whole
        // warp converged
        for (int t = 0; t < ns && !*abort; ++t) {
            const int s = t % kTS;
            if (!__all_sync(0xffffffffu, mbar_wait(&bar_full[s], (t / kTS) & 1, abort))) break;
            const uint8_t* st = stage(s);
            const float* sWs = (const float*)(st + S::kA + S::kB + S::kRaw + S::kWsr);
            const float* sXs = sWs + kTB * kTM;
            bool ok = true;
#pragma unroll 1
            for (int lb = 0; lb < kTB; ++lb) {
                const int b = t * kTB + lb, buf = b & (kTBufs - 1);
                if (!__all_sync(0xffffffffu, mbar_wait(&bar_tfull[buf], (b >> 2) & 1, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float dw = sWs[lb * kTM + r];
                const float* dx = sXs + lb * kTN + h * 64;
                const uint32_t ta = lane_base + buf * kTN;
                uint32_t v0[32], v1[32];
                tmem_ld32(ta, v0);
                tmem_ld32(ta + 32, v1);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_tempty[buf]);  // the MMA may refill it now
                scale_acc(v0, dw, dx, acc);
                scale_acc(v1, dw, dx + 32, acc + 16);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[s]);
        }
        if (!*abort) {
            const int n = n0 + r;
            if (n < N) {
                const float bn = ep.bias ? ep.bias[n] : 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int m = m0 + h * 64 + 2 * j + e;
                        if (m < M) {
                            float o = e ? acc[j].y : acc[j].x;
                            if (ep.bias) o = __fadd_rn(o, bn);
                            if (ep.residual)
                                o = __fadd_rn(ep.residual[(int64_t)m * ep.res_stride + n], o);
                            y[(int64_t)m * y_stride + n] = o;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

void launch_gemm_tc(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                    int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    GB_CHECK(w.type == T_Q8_0 || w.type == T_Q4_0, "gemm_tc: quantized weights required");
    GB_CHECK(w.K % QK == 0 && w.K > 0, "gemm_tc: K must be a positive multiple of 32");
    GB_CHECK(w.N < (1LL << 31) && w.K < (1LL << 31) && M < (1LL << 31), "gemm_tc: shape too large");
    GB_CHECK(((uintptr_t)xq & 15) == 0 && ((uintptr_t)w.qs & 15) == 0,
             "gemm_tc: xq and weights must be 16-byte aligned");
    if (M == 0 || w.N == 0) return;
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lock(mu);
        GB_CHECK(dev >= 0 && dev < 64, "gemm_tc: device ordinal out of range");
        if (!configured[dev]) {
            GB_CUDA(cudaFuncSetAttribute(k_gemm_tc<T_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kTS * TcStage<T_Q8_0>::kBytes));
            GB_CUDA(cudaFuncSetAttribute(k_gemm_tc<T_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kTS * TcStage<T_Q4_0>::kBytes));
            configured[dev] = true;
        }
    }
    dim3 grid((unsigned)((w.N + kTM - 1) / kTM), (unsigned)((M + kTN - 1) / kTN));
    if (w.type == T_Q8_0)
        k_gemm_tc<T_Q8_0><<<grid, kTThreads, kTS * TcStage<T_Q8_0>::kBytes, st>>>(
            (const uint8_t*)w.qs, (int)w.N, (int)w.K, xq, xd, (int)M, y, y_stride, ep);
    else
        k_gemm_tc<T_Q4_0><<<grid, kTThreads, kTS * TcStage<T_Q4_0>::kBytes, st>>>(
            (const uint8_t*)w.qs, (int)w.N, (int)w.K, xq, xd, (int)M, y, y_stride, ep);
    GB_CUDA(cudaGetLastError());
}

int gemm_tc_error() {
    int v = 0;
    GB_CUDA(cudaMemcpyFromSymbol(&v, gemm_tc_error_word, sizeof(int)));
    return v;
}

}  // namespace gb
