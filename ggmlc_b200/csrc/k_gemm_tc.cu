// Prefill MUL_MAT (M > 16 activation rows) on the 5th-generation tensor cores: tcgen05.mma
// kind::i8 with accumulators in tensor memory, operands brought in by the TMA engine, per-block
// fp16 scales applied by epilogue warps.
//
// Arithmetic.  One tcgen05.mma (M = 128 weight rows, N = 128 activation rows, K = 32) per
// 32-element block writes every exact int32 block dot of a 128 x 128 tile into a tensor-memory
// accumulator; the epilogue adds 0x4B400000 (1.5 * 2^23) to the bits, which makes them the
// float 12582912 + sumi, forms sumi * d_x with one fma against the exact constant
// -12582912 * d_x, multiplies by d_w and accumulates the block terms in fp32 registers — the
// block formula of the reference's vec_dot (ggml-cpu/quants.c:225-256, :451-477) with the
// integer part exact.
// Q4_0 nibbles are widened in shared memory to 16 * (q - 8) (exact in int8); their weight scales
// are divided by 16 to compensate.
//
// A K stage is 4 consecutive blocks.  Per stage the TMA engine loads (tile mode, no multicast)
// the activation quants, 128 contiguous bytes per row, with the 128-byte swizzle the MMA reads
// directly (a block's 32 bytes selected by the descriptor's start address); the weight quants,
// 64 contiguous bytes per row (Q4_0 nibbles; Q8_0 first and second halves in two boxes), which
// helper warps widen (Q4_0) or copy (Q8_0) into the canonical no-swizzle K-major layout
// (8-row x 16-byte core matrices, the two 16-byte halves of a block 2048 B apart); the 16-byte
// scale word of every weight row (4 fp16 scales of the stage) and the 4 fp32 activation scales
// of every activation row.
//
// Warps (12, one CTA per SM):
//   warp 0      TMA producer (one thread), stage ring of 3-4 stages;
//   warp 1      MMA issuer (one thread) and tensor-memory owner: 4 accumulators of 128 columns,
//               one per block of a stage, one tcgen05.mma + tcgen05.commit per block;
//   warps 2-3   weight quants into the MMA layout (Q4_0 widened), weight scales to fp32 pairs
//               [block][row], activation scales transposed to [block][row pair], then mbarrier
//               "ready" (the MMA and the epilogue wait on it);
//   warps 4-11  epilogue: warp w reads tensor-memory lanes 32*(w%4).. (its weight rows) and 64
//               columns (activation rows) 64*((w-4)/4).. of each finished block with the
//               16x256b tcgen05.ld shape (a thread holds 4 weight rows x 16 columns, so one
//               shared-memory read of activation scales serves 4 rows), releases the
//               accumulator as soon as the values are in registers, scales.
// Every wait on an mbarrier is bounded: past the limit the kernel records an error in
// gemm_tc_error, stops issuing, waits (bounded) for its tensor-core work to drain, frees the
// tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kTM = 128;            // weight rows per tile (MMA M, tensor-memory lanes)
constexpr int kTN = 128;            // activation rows per tile (MMA N, tensor-memory columns)
constexpr int kTB = 4;              // blocks per stage = tensor-memory accumulators
// stages in the ring: 4 (Q4_0) or 3 (Q8_0, whose raw halves take more room)
template <int WT>
constexpr int stages() { return WT == T_Q8_0 ? 3 : 4; }
constexpr int kMmaWarp = 1;
constexpr int kHelpWarp0 = 2, kHelpWarps = 2;
#ifndef GB_TC_COLS
#define GB_TC_COLS 32
#endif
constexpr int kCols = GB_TC_COLS;              // accumulator columns per epilogue warp
static_assert(kCols == 32 || kCols == 64, "epilogue width");
constexpr int kJ = kCols / 8;                  // 8-column groups per epilogue thread
constexpr int kEpiWarp0 = 4, kEpiWarps = 4 * (128 / kCols);
constexpr int kTThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kTmemCols = kTB * kTN;
constexpr uint32_t kBiasBits = 0x4B400000u;      // 1.5 * 2^23
constexpr long long kSpinCycles = 4000000000LL;  // about 2 s at 1.9 GHz

// one stage in shared memory (1024-byte aligned: the activation tile is 128-byte swizzled)
template <int WT>
struct TcStage {
    static constexpr int kA = kTB * 4096;   // weights as int8, canonical no-swizzle MMA layout
    static constexpr int kB = kTN * 128;    // activations [row][4 blocks x 32 B], 128 B swizzle
    static constexpr int kRaw = kTM * 64 * (WT == T_Q8_0 ? 2 : 1);  // TMA rows: [row][4 x 16 B]
    static constexpr int kWs = kTM * 16;    // a row's scale word
    static constexpr int kXr = kTN * 16;    // 4 fp32 scales per activation row
    static constexpr int kXt = kTB * kTN * 8;  // (d_x, -1.5*2^23*d_x) pairs [block][row]
    static constexpr int kWf = kTB * kTM * 8;  // (d_w, d_w) fp32 pairs [block][row]
    static constexpr int kBytes = kA + kB + kRaw + kWs + kXr + kXt + kWf;
    static constexpr uint32_t kTx = kRaw + kB + kWs + kXr;  // TMA bytes
    static_assert(kBytes % 1024 == 0, "stage alignment");
};
template <int WT>
constexpr int tc_smem() { return stages<WT>() * TcStage<WT>::kBytes + 1024; }

struct TcArgs {
    int N, K, M;        // weight rows (SwiGLU: 2F), K, activation rows
    int swi_F;          // > 0: SwiGLU tiles of 64 pairs (gate p, up F + p)
    float* y;           // plain output [M][y_stride], or SwiGLU f32 output [M][F]
    int64_t y_stride;
    const float* bias;
    const float* residual;
    int64_t res_stride;
    int8_t* yq;         // SwiGLU Q8_0 output [M][F], yd [M][F / 32]
    float* yd;
    float* part;        // split K (gridDim.z > 1): partial sums [z][M][N], finished by
                        // launch_splitk_sum
};

__device__ int gemm_tc_error_word;

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)),
                 "r"(bytes)
                 : "memory");
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
// TMA tile load of box (x, y) of a 2-D tensor map into shared memory, completion on bar
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, int x, int y,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
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
// K-major, 128-byte swizzle (the TMA's CU_TENSOR_MAP_SWIZZLE_128B pattern): rows of 128 B, 8-row
// groups 1024 B apart; a block's 32 bytes are selected by advancing the start address by 32 B
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
    const uint32_t a = su32(p);
    return (uint64_t)((a & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::i8, D s32, A / B signed 8-bit, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);

// D = A * B (the accumulator is overwritten: one block per accumulator)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(0)
        : "memory");
}

// 16 lanes x 32 columns from lane `taddr.lane` (16x256b shape, 4 repeats): thread t gets, for
// each 8-column group j, rows t/4 and t/4 + 8 at columns 8j + 2(t%4) + {0, 1}:
// v[4j + 0..1] = row t/4, v[4j + 2..3] = row t/4 + 8
__device__ __forceinline__ void tmem_ld_16x256(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
// wait for this thread's tensor-memory loads; the registers the loads fill are operands, so no
// use of them is scheduled before the wait
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]),
          "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]),
          "+r"(a[14]), "+r"(a[15]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]),
          "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]),
          "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])
        :
        : "memory");
}
// the epilogue warps only (named barrier 1)
__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

// SPLIT: the CTA takes stages [tb, te) of K and writes partial sums (gridDim.z splits); the
// whole-K build is compiled separately so its code is the same as without split K.
template <int WT, bool SPLIT>
__global__ void __launch_bounds__(kTThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmws,
              const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tms,
              TcArgs a) {
    using S = TcStage<WT>;
    constexpr int kTS = stages<WT>();
    extern __shared__ __align__(1024) uint8_t tsm_raw[];
    // the stages start on a 1024-byte boundary (the launch adds 1024 bytes of room)
    uint8_t* tsm = tsm_raw + ((1024 - (su32(tsm_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t bar_full[4], bar_ready[4], bar_empty[4], bar_tfull[kTB],
        bar_tempty[kTB], bar_done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    volatile int* abort = &s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool swi = a.swi_F > 0;
    const int n0 = blockIdx.x * (swi ? kTM / 2 : kTM), m0 = blockIdx.y * kTN;
    const int nb = a.K / QK;
    const int ns = nb / kTB;  // stages (K % 128 == 0)
    // split K: this CTA's stages [tb, te); stage slots and barrier phases count from tb
    const int tb = SPLIT ? (int)((int64_t)ns * blockIdx.z / gridDim.z) : 0;
    const int te = SPLIT ? (int)((int64_t)ns * (blockIdx.z + 1) / gridDim.z) : ns;
    const int qsz = WT == T_Q8_0 ? 32 : 16;
    auto stage = [&](int s) { return tsm + s * S::kBytes; };

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kTS; ++s) {
            mbar_init(&bar_full[s], 1);
            mbar_init(&bar_ready[s], kHelpWarps);
            mbar_init(&bar_empty[s], 1 + kEpiWarps);
        }
        for (int b = 0; b < kTB; ++b) {
            mbar_init(&bar_tfull[b], 1);
            mbar_init(&bar_tempty[b], kEpiWarps);
        }
        mbar_init(&bar_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            for (int t = tb; t < te && !*abort; ++t) {
                const int i = t - tb, s = i % kTS;
                if (i >= kTS && !mbar_wait(&bar_empty[s], ((i / kTS) - 1) & 1, abort)) break;
                uint8_t* st = stage(s);
                uint8_t* sB = st + S::kA;
                uint8_t* sRaw = sB + S::kB;
                uint8_t* sWs = sRaw + S::kRaw;
                uint8_t* sXr = sWs + S::kWs;
                const int b0 = t * kTB;
                mbar_expect_tx(&bar_full[s], S::kTx);
                // weight rows of the tile: 128 rows, or gate rows then up rows (64 each)
                // weight rows of the tile: 128 rows, or gate rows then up rows (64 each); per row
                // the stage's 4 blocks of quants are 64 contiguous bytes (Q8_0: first halves,
                // then second halves in a second box)
                for (int part = 0; part < (swi ? 2 : 1); ++part) {
                    const int wy = swi ? n0 + part * a.swi_F : n0;
                    tma_load(sRaw + part * 64 * 64, &tmw, b0 * 16, wy, &bar_full[s]);
                    if (WT == T_Q8_0)
                        tma_load(sRaw + kTM * 64 + part * 64 * 64, &tmw, (nb + b0) * 16, wy,
                                 &bar_full[s]);
                    tma_load(sWs + part * 64 * 16, &tmws, nb * qsz + (b0 >> 6) * 128 + (b0 & 31) * 4,
                             wy, &bar_full[s]);
                }
                tma_load(sB, &tmx, b0 * 32, m0, &bar_full[s]);  // 128 B per row, swizzled
                tma_load(sXr, &tms, b0, m0, &bar_full[s]);
            }
        }
        __syncwarp();
    } else if (warp >= kHelpWarp0 && warp < kHelpWarp0 + kHelpWarps) {
        // ---------------------------------------------------------------- helpers
        const int p = tid - kHelpWarp0 * 32;  // 0..63
        for (int t = tb; t < te && !*abort; ++t) {
            const int i = t - tb, s = i % kTS;
            if (!__all_sync(0xffffffffu, mbar_wait(&bar_full[s], (i / kTS) & 1, abort))) break;
            uint8_t* st = stage(s);
            uint8_t* sA = st;
            uint8_t* sRaw = st + S::kA + S::kB;
            const float* sXr = (const float*)(sRaw + S::kRaw + S::kWs);
            float* sXt = (float*)(sRaw + S::kRaw + S::kWs + S::kXr);
            if (WT == T_Q8_0) {  // both halves into the MMA layout
                for (int c = p; c < kTB * kTM; c += 32 * kHelpWarps) {
                    const int r = c & (kTM - 1), lb = c >> 7;
                    uint8_t* d = sA + lb * 4096 + r * 16;
                    *(uint4*)d = *(const uint4*)(sRaw + r * 64 + lb * 16);
                    *(uint4*)(d + 2048) = *(const uint4*)(sRaw + kTM * 64 + r * 64 + lb * 16);
                }
            }
            if (WT == T_Q4_0) {  // nibbles to int8 16*(q-8): low -> k 0..15, high -> 16..31
                for (int c = p; c < kTB * kTM; c += 32 * kHelpWarps) {
                    const int r = c & (kTM - 1), lb = c >> 7;
                    const uint4 w = *(const uint4*)(sRaw + r * 64 + lb * 16);
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
            // activation scales [row][block] -> [block][row pair]: (d_x, d_x', c, c') for rows
            // 2k, 2k+1 with c = -1.5*2^23 * d_x (exact: d_x carries the 11 significant bits of an
            // fp16 scale), so the epilogue's packed pairs load as they are
            for (int k = p; k < kTN / 2; k += 32 * kHelpWarps) {
                const float4 v0 = *(const float4*)(sXr + (2 * k) * 4);
                const float4 v1 = *(const float4*)(sXr + (2 * k + 1) * 4);
                const float e0[4] = {v0.x, v0.y, v0.z, v0.w}, e1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int lb = 0; lb < kTB; ++lb)
                    *(float4*)(sXt + 4 * (lb * (kTN / 2) + k)) =
                        make_float4(e0[lb], e1[lb], __fmul_rn(e0[lb], -12582912.0f),
                                    __fmul_rn(e1[lb], -12582912.0f));
            }
            // weight scales to (d_w, d_w) fp32 pairs [block][row] (Q4_0: d_w / 16, the widened
            // quants being 16 * (q - 8)); a row's 16-byte scale word holds the stage's 4 fp16
            // scales in its low halves for the first 32 blocks of a 64-block group, else the high
            {
                const int sh = (((t * kTB) >> 5) & 1) * 16;
                const float wsc = WT == T_Q4_0 ? 0.0625f : 1.0f;
                const uint32_t* sWs = (const uint32_t*)(sRaw + S::kRaw);
                float2* sWf = (float2*)(sRaw + S::kRaw + S::kWs + S::kXr + S::kXt);
                for (int c = p; c < kTB * kTM; c += 32 * kHelpWarps) {
                    const int r = c & (kTM - 1), lb = c >> 7;
                    const float d = __fmul_rn(
                        __half2float(__ushort_as_half((unsigned short)(sWs[r * 4 + lb] >> sh))), wsc);
                    sWf[lb * kTM + r] = make_float2(d, d);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // A -> MMA
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_ready[s]);
        }
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = true;
            for (int t = tb; t < te && ok; ++t) {
                const int i = t - tb, s = i % kTS;
                if (!mbar_wait(&bar_ready[s], (i / kTS) & 1, abort)) break;
                tc_fence_after();
                const uint8_t* st = stage(s);
                for (int lb = 0; lb < kTB; ++lb) {
                    if (!mbar_wait(&bar_tempty[lb], i & 1, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tc_mma(tmem + lb * kTN, smem_desc(st + lb * 4096),
                           smem_desc_sw128(st + S::kA + lb * 32));
                    tc_commit(&bar_tfull[lb]);
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
        // warp (q, ch): tensor-memory lanes 32q.. and columns kCols*ch.. of every accumulator;
        // thread (g, cp) = (lane / 4, lane % 4) holds weight rows 32q + 8k + g (k = 0..3) at
        // columns kCols*ch + 8j + 2cp + {0, 1} (j < kCols / 8) in acc[k][j]
        const int q = warp & 3, ch = (warp - kEpiWarp0) >> 2;
        const int g = lane >> 2, cp = lane & 3;
        const uint32_t wbase = tmem + ((uint32_t)(q * 32) << 16) + ch * kCols;
        constexpr uint32_t kHalfLanes = 16u << 16;
        // every accumulator starts free
        if (lane == 0)
            for (int b = 0; b < kTB; ++b) mbar_arrive(&bar_tempty[b]);
        float2 acc[4][kJ];
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int j = 0; j < kJ; ++j) acc[k][j] = make_float2(0.0f, 0.0f);
        // 32 columns (j0.. j0 + 3) of the thread's 4 rows: per column the bits sumi + 0x4B400000
        // are the float 12582912 + sumi (|sumi| < 2^22), t = fma(that, d_x, c) = sumi * d_x (one
        // rounding: c = -12582912 * d_x exactly), then acc = fma(t, d_w, acc); one
        // (d_x, d_x', c, c') read serves 4 rows
        auto scale = [&](const uint32_t(&va)[16], const uint32_t(&vb)[16], const float* dx,
                         const float2(&dw)[4], int j0) {
            auto u = [](uint32_t bits) { return __uint_as_float(bits + kBiasBits); };
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float4 a4 = *(const float4*)(dx + 4 * (4 * jj + cp));
                const float2 x2 = make_float2(a4.x, a4.y), c2 = make_float2(a4.z, a4.w);
                float2& a0 = acc[0][j0 + jj];
                float2& a1 = acc[1][j0 + jj];
                float2& a2 = acc[2][j0 + jj];
                float2& a3 = acc[3][j0 + jj];
                a0 = fma2(fma2(make_float2(u(va[4 * jj]), u(va[4 * jj + 1])),
                               x2, c2), dw[0], a0);
                a1 = fma2(fma2(make_float2(u(va[4 * jj + 2]), u(va[4 * jj + 3])),
                               x2, c2), dw[1], a1);
                a2 = fma2(fma2(make_float2(u(vb[4 * jj]), u(vb[4 * jj + 1])),
                               x2, c2), dw[2], a2);
                a3 = fma2(fma2(make_float2(u(vb[4 * jj + 2]), u(vb[4 * jj + 3])),
                               x2, c2), dw[3], a3);
            }
        };
        // waits are made warp-uniform by a vote: tensor-memory loads and stores need the whole
        // warp converged
        for (int t = tb; t < te && !*abort; ++t) {
            const int i = t - tb, s = i % kTS;
            if (!__all_sync(0xffffffffu, mbar_wait(&bar_ready[s], (i / kTS) & 1, abort))) break;
            const uint8_t* st = stage(s);
            const float* sXt = (const float*)(st + S::kA + S::kB + S::kRaw + S::kWs + S::kXr);
            const float2* sWf = (const float2*)(sXt + S::kXt / 4);
            bool ok = true;
#pragma unroll 1
            for (int lb = 0; lb < kTB; ++lb) {
                float2 dw[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) dw[k] = sWf[lb * kTM + q * 32 + 8 * k + g];
                if (!__all_sync(0xffffffffu, mbar_wait(&bar_tfull[lb], i & 1, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ta = wbase + lb * kTN;
                const float* dx = sXt + 4 * (lb * (kTN / 2) + ch * (kCols / 2));
                uint32_t va[16], vb[16];
                tmem_ld_16x256(ta, va);
                tmem_ld_16x256(ta + kHalfLanes, vb);
                tmem_wait_ld(va, vb);
                if constexpr (kCols == 32) {
                    // the accumulator is released as soon as its values are in registers
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_tempty[lb]);  // the MMA may use it again
                    scale(va, vb, dx, dw, 0);
                } else {
                    // columns 32..63 load while 0..31 are scaled; the accumulator is released
                    // once both reads are done, before the last scaling
                    uint32_t wa[16], wb[16];
                    tmem_ld_16x256(ta + 32, wa);
                    tmem_ld_16x256(ta + kHalfLanes + 32, wb);
                    scale(va, vb, dx, dw, 0);
                    tmem_wait_ld(wa, wb);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_tempty[lb]);
                    scale(wa, wb, dx + 4 * 16, dw, 4);
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty[s]);  // this stage's scales are read
        }
        if (!*abort && !swi) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int n = n0 + q * 32 + 8 * k + g;
                if (n < a.N) {
                    const float bn = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
                    for (int j = 0; j < kJ; ++j) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int m = m0 + ch * kCols + 8 * j + 2 * cp + e;
                            if (SPLIT && m < a.M) {  // split K: the partial sum
                                a.part[((int64_t)blockIdx.z * a.M + m) * a.N + n] =
                                    e ? acc[k][j].y : acc[k][j].x;
                            } else if (m < a.M) {
                                float o = e ? acc[k][j].y : acc[k][j].x;
                                if (a.bias) o = __fadd_rn(o, bn);
                                if (a.residual)
                                    o = __fadd_rn(a.residual[(int64_t)m * a.res_stride + n], o);
                                a.y[(int64_t)m * a.y_stride + n] = o;
                            }
                        }
                    }
                }
            }
        }
        if (swi) {
            // SwiGLU: lanes 0-63 hold gate rows n0.., lanes 64-127 the up rows of the same pairs.
            // The up warps hand their sums over in shared memory (the stage ring is free now:
            // every MMA and every TMA load has completed before the last stage's "ready").
            constexpr int kXs = kTN + 8;  // padded row stride in floats
            float* xch = (float*)tsm;     // [64 pairs][kXs]
            epi_sync();
            if (q >= 2 && !*abort) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
#pragma unroll
                    for (int j = 0; j < kJ; ++j)
                        *(float2*)(xch + ((q - 2) * 32 + 8 * k + g) * kXs + ch * kCols + 8 * j + 2 * cp) =
                            acc[k][j];
            }
            epi_sync();
            if (q < 2 && !*abort) {
                // pairs n0 + 32q + 8k + g: for each activation row m the warp's lanes with one cp
                // hold the 32 pairs of one Q8_0 block (8 row groups g x 4 rows k)
#pragma unroll
                for (int j = 0; j < kJ; ++j) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int col = ch * kCols + 8 * j + 2 * cp + e, m = m0 + col;
                        float h[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float up = xch[(q * 32 + 8 * k + g) * kXs + col];
                            h[k] = __fmul_rn(ref_v_silu(e ? acc[k][j].y : acc[k][j].x), up);
                        }
                        float amax = fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3])));
                        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
                        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 16));
                        if (m < a.M) {
                            const int pr0 = n0 + q * 32 + g;
                            if (a.y) {
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    a.y[(int64_t)m * a.y_stride + pr0 + 8 * k] = h[k];
                            }
                            if (a.yq) {  // Q8_0 quantization of the block (q8_block's formula)
                                const float d = __fdiv_rn(amax, 127.0f);
                                const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    a.yq[(int64_t)m * a.swi_F + pr0 + 8 * k] =
                                        (int8_t)__float2int_rn(rintf(__fmul_rn(h[k], id)));
                                if (g == 0)
                                    a.yd[(int64_t)m * (a.swi_F / 32) + (n0 + q * 32) / 32] =
                                        __half2float(__float2half_rn(d));
                            }
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

// ---- tensor maps (host) -------------------------------------------------------------------------

// 2-D tiled tensor map of `dtype` elements: dims {d0, d1}, row pitch `pitch` bytes, box {b0, b1};
// no swizzle or the 128-byte swizzle, out-of-range elements read as zero.  Cached per argument
// set.
CUtensorMap tensor_map(const void* base, CUtensorMapDataType dtype, uint64_t d0, uint64_t d1,
                       uint64_t pitch, uint32_t b0, uint32_t b1, bool sw128) {
    using Key = std::tuple<const void*, int, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, (int)dtype, d0, d1, pitch, b0, b1, sw128};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    if (cache.size() > 4096) cache.clear();
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t es[2] = {1, 1};
    // the driver entry point, looked up through the runtime: the library does not link libcuda
    using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static Encode encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        GB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        GB_CHECK(fn != nullptr && q == cudaDriverEntryPointSuccess,
                 "gemm_tc: cuTensorMapEncodeTiled is not available from the driver");
        encode = (Encode)fn;
    }
    const CUresult rc = encode(
        &m, dtype, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
        sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    GB_CHECK(rc == CUDA_SUCCESS, "gemm_tc: cuTensorMapEncodeTiled failed (" + std::to_string((int)rc) + ")");
    cache.emplace(key, m);
    return m;
}

template <int WT>
void run_tc(const QWeight& w, const int8_t* xq, const float* xd, const TcArgs& a, cudaStream_t st) {
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lock(mu);
        GB_CHECK(dev >= 0 && dev < 64, "gemm_tc: device ordinal out of range");
        if (!configured[dev]) {
            GB_CUDA(cudaFuncSetAttribute(k_gemm_tc<WT, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem<WT>()));
            GB_CUDA(cudaFuncSetAttribute(k_gemm_tc<WT, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem<WT>()));
            configured[dev] = true;
        }
    }
    const int64_t rb = qrow_bytes(WT, w.K);
    const bool swi = a.swi_F > 0;
    const uint32_t rows = swi ? kTM / 2 : kTM;
    const CUtensorMap mw = tensor_map(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)rb,
                                      (uint64_t)w.N, (uint64_t)rb, 64, rows, false);
    const CUtensorMap mws = tensor_map(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)rb,
                                       (uint64_t)w.N, (uint64_t)rb, 16, rows, false);
    const CUtensorMap mx = tensor_map(xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w.K,
                                      (uint64_t)a.M, (uint64_t)w.K, 128, kTN, true);
    const CUtensorMap ms = tensor_map(xd, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)(w.K / QK),
                                      (uint64_t)a.M, (uint64_t)(w.K / QK) * 4, kTB, kTN, false);
    const int64_t ntiles = swi ? a.swi_F / (kTM / 2) : (w.N + kTM - 1) / kTM;
    dim3 grid((unsigned)ntiles, (unsigned)((a.M + kTN - 1) / kTN));
    // a plain GEMM with tiles for at most half the SMs splits K (one CTA per SM, at least 8
    // stages a split); the partial sums are added in split order by launch_splitk_sum
    const int sms = sm_count(dev), ns = (int)(w.K / QK / kTB);
    const int64_t ntile = (int64_t)grid.x * grid.y;
    int splits = 1;
    if (!swi && 2 * ntile <= sms && splitk_enabled())
        splits = (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(sms / ntile, ns / 8), 16));
    TcArgs b = a;
    if (splits > 1) {
        grid.z = (unsigned)splits;
        GB_CUDA(cudaMallocAsync((void**)&b.part, (size_t)splits * a.M * a.N * sizeof(float), st));
    }
    if (splits > 1) k_gemm_tc<WT, true><<<grid, kTThreads, tc_smem<WT>(), st>>>(mw, mws, mx, ms, b);
    else k_gemm_tc<WT, false><<<grid, kTThreads, tc_smem<WT>(), st>>>(mw, mws, mx, ms, b);
    GB_CUDA(cudaGetLastError());
    if (splits > 1) {
        MatmulEpilogue ep;
        ep.bias = a.bias;
        ep.residual = a.residual;
        ep.res_stride = a.res_stride;
        launch_splitk_sum(b.part, splits, a.M, a.N, a.y, a.y_stride, ep, st);
        GB_CUDA(cudaFreeAsync(b.part, st));
    }
}

void check_tc(const QWeight& w, const int8_t* xq, const float* xd) {
    GB_CHECK(w.type == T_Q8_0 || w.type == T_Q4_0, "gemm_tc: quantized weights required");
    GB_CHECK(gemm_tc_fits(w.K), "gemm_tc: K must be a positive multiple of 128");
    GB_CHECK(w.N < (1LL << 31) && w.K < (1LL << 31), "gemm_tc: shape too large");
    GB_CHECK(((uintptr_t)xq & 15) == 0 && ((uintptr_t)w.qs & 15) == 0 && ((uintptr_t)xd & 15) == 0,
             "gemm_tc: xq, xd and weights must be 16-byte aligned");
}

}  // namespace

bool gemm_tc_fits(int64_t K) { return K > 0 && K % (QK * kTB) == 0; }

void launch_gemm_tc(const QWeight& w, const int8_t* xq, const float* xd, int64_t M, float* y,
                    int64_t y_stride, const MatmulEpilogue& ep, cudaStream_t st) {
    check_tc(w, xq, xd);
    GB_CHECK(M < (1LL << 31), "gemm_tc: shape too large");
    if (M == 0 || w.N == 0) return;
    TcArgs a{};
    a.N = (int)w.N;
    a.K = (int)w.K;
    a.M = (int)M;
    a.swi_F = 0;
    a.y = y;
    a.y_stride = y_stride;
    a.bias = ep.bias;
    a.residual = ep.residual;
    a.res_stride = ep.res_stride;
    if (w.type == T_Q8_0) run_tc<T_Q8_0>(w, xq, xd, a, st);
    else run_tc<T_Q4_0>(w, xq, xd, a, st);
}

void launch_gemm_tc_swiglu(const GemvArgs& g, cudaStream_t st) {
    check_tc(g.w, g.xq, g.xd);
    GB_CHECK(g.w.N == 2 * g.F && g.F % (kTM / 2) == 0, "gemm_tc swiglu: N == 2F with F % 64 == 0");
    GB_CHECK(!g.bias && !g.residual, "gemm_tc swiglu: no bias / residual");
    GB_CHECK(g.y || g.yq, "gemm_tc swiglu: no output");
    GB_CHECK(!g.yq == !g.yd, "gemm_tc swiglu: Q8_0 output needs quants and scales");
    if (g.M == 0) return;
    TcArgs a{};
    a.N = (int)g.w.N;
    a.K = (int)g.w.K;
    a.M = g.M;
    a.swi_F = (int)g.F;
    a.y = g.y;
    a.y_stride = g.y_stride;
    a.yq = g.yq;
    a.yd = g.yd;
    if (g.w.type == T_Q8_0) run_tc<T_Q8_0>(g.w, g.xq, g.xd, a, st);
    else run_tc<T_Q4_0>(g.w, g.xq, g.xd, a, st);
}

int gemm_tc_error() {
    int v = 0;
    GB_CUDA(cudaMemcpyFromSymbol(&v, gemm_tc_error_word, sizeof(int)));
    return v;
}

}  // namespace gb
