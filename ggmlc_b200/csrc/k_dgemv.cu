// Decode GEMV for one or two activation rows (batch-1/2 decode): y = W x over the split-row
// layout, the weights streamed from HBM by bulk copies (cp.async.bulk, the TMA engine's linear
// mode).
//
// Work mapping.  Each CTA owns a contiguous range of output units (rows, or SwiGLU row pairs
// gate n / up n+F).  A row is cut into chunks of up to 128 blocks (K = 4096); a chunk is a few
// contiguous byte ranges of the split-row layout (quants, Q8_0 second halves, scales), fetched
// by one bulk copy each into a slot of a per-warp ring with its own mbarrier.  Every warp works
// on one fixed chunk index of the rows (rows of up to 128 blocks: every warp takes whole rows;
// longer rows: the warps split into one group per chunk), so its activation blocks stay in
// registers; lane 0 refills a slot as soon as the warp has consumed it.  Lanes run along K: lane l
// takes blocks l, l+32, l+64, l+96 of the chunk, whose quants are 16 consecutive bytes (Q4_0;
// Q8_0 two 16-byte halves), so the lanes' shared-memory reads are conflict-free, and whose fp16
// scales come two to a 32-bit word.  A chunk's lane sums are combined by a fixed xor-butterfly;
// the chunks of a row are added in chunk order at the end of the CTA.
//
// Activations come quantized (xq, xd) or as f32 (xf), quantized by every CTA in its prologue
// after an optional RMSNorm (+gamma): the same arithmetic as launch_rms_norm and the x86
// activation quantizer (ggml-cpu/arch/x86/quants.c:302-392).
//
// Arithmetic per 32-element block: the integer dot is exact.  Q4_0: the low nibbles (elements
// 0-15) and the high nibbles (16-31) are masked out of each 32-bit word as unsigned bytes and
// dotted with the signed activation bytes (dp4a.u32.s32); the high-nibble chain sees 16 * q, so
// its sum is shifted right by 4 (exact), and the -8 offset of every weight is folded into the
// chain's start value, -8 * sum(x) of the block.  The chain starts at 1.5 * 2^23, so the int sum
// becomes a float by one subtraction (exact for |sum| < 2^22).  The block term sumi * (d_w * d_x)
// accumulates in fp32 per lane.  This is the reference's block formula (ggml-cpu/quants.c:225-256
// Q4_0, :451-477 Q8_0); the x86 build adds the same terms in another order, so fp32 results agree
// to rounding.
//
// Epilogues: f32 rows (+bias, +residual), or SwiGLU of each pair, silu(gate) * up (the vector
// silu of the CPU build, ggml-cpu/vec.h:1255-1262), written as f32 rows of length F.
//
// Launch: one CTA of 8 warps per SM, programmatic dependent launch.  The rings stay under half of
// the shared memory, so the next kernel's CTAs start on an SM while this one finishes; every
// warp requests its first ring of chunks before griddepcontrol.wait, so the weight stream
// overlaps the previous kernel; activations are read and outputs written after the wait.  Every
// mbarrier wait is bounded (about 2 s): past the limit the kernel records an error in
// dgemv_error (gb_gemv_error), waits (bounded) for the copies it issued and returns.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kdot.cuh"
#include "kutil.cuh"

namespace gb {

__device__ int dgemv_error_word;

// Optional per-CTA timeline (built with -DGB_DGEMV_TRACE only; not part of the shipped library):
// for the n-th launch CTA b reaches, %globaltimer at entry (0), after the wait for the previous
// launch (1), after its prologue (2), when warp 0 has consumed its items (3) and at exit (4).
#ifdef GB_DGEMV_TRACE
constexpr int kTrLaunches = 1024, kTrCtas = 160;
__device__ unsigned g_dgemv_tr_n[kTrCtas];
__device__ unsigned long long g_dgemv_tr[kTrLaunches][kTrCtas][5];
#define DGEMV_TRACE(slot)                                                                   \
    do {                                                                                    \
        if (threadIdx.x == 0 && blockIdx.x < kTrCtas && tr_n < kTrLaunches) {              \
            unsigned long long t_;                                                          \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                          \
            g_dgemv_tr[tr_n][blockIdx.x][(slot)] = t_;                                      \
        }                                                                                   \
    } while (0)
#define DGEMV_TRACE_BEGIN                                                                   \
    unsigned tr_n = kTrLaunches;                                                            \
    if (threadIdx.x == 0 && blockIdx.x < kTrCtas) tr_n = atomicAdd(&g_dgemv_tr_n[blockIdx.x], 1u); \
    DGEMV_TRACE(0)
#else
#define DGEMV_TRACE(slot) ((void)0)
#define DGEMV_TRACE_BEGIN ((void)0)
#endif

namespace {

constexpr int kW = 16;           // warps per CTA
constexpr int kT = kW * 32;
constexpr int kMaxSlots = 8;     // ring slots per warp
// blocks per chunk: 128 for Q4_0 (2304-byte slots), 64 for Q8_0 (2176-byte slots)
template <int WT>
constexpr int chunk_blocks() { return WT == T_Q8_0 ? 64 : 128; }
constexpr int kMaxChunks = 16;   // chunks per row at most (a warp group per chunk)
constexpr size_t kRingBudget = 112 * 1024;

struct DArgs {
    GemvAllReduce ar;  // T > 0: y summed over the tensor-parallel ranks in the epilogue
    // L2 prefetch of the next GEMV's weights: rows pf_rb bytes apart, split over pf_grid CTAs
    // like this kernel splits its own (SwiGLU: a second range pf_F rows on); at most pf_cap bytes
    // per next-launch CTA; pf null: none
    const uint8_t* pf;
    int64_t pf_rb, pf_units, pf_F, pf_cap;
    int pf_grid;
    const uint8_t* w;
    int64_t rb;        // bytes per weight row
    int nb;            // blocks per row
    int nc;            // chunks per row (chunk_blocks each, the last one shorter)
    int rows_cta;      // most rows one CTA owns (sizes the chunk partials)
    int units;         // rows, or SwiGLU pairs
    int F;             // SwiGLU: up row of pair n is n + F
    int slots;         // ring slots per warp
    int M;             // activation rows (1 or 2)
    const int8_t* xq;  // Q8_0 input [M][K], or
    const float* xd;
    const float* xf;   // f32 input [M][xf_stride], quantized in the prologue
    int64_t xf_stride;
    int rms;
    float eps;
    const float* gamma;
    int swiglu;
    float* y;          // [M][y_stride]
    int64_t y_stride;
    const float* bias;
    const float* residual;  // [M][res_stride]
    int64_t res_stride;
};

__device__ double cta_sum_d(double v, double* sh) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < kW; ++i) t += sh[i];
    return t;
}

// Quantize f32 input row m (after RMSNorm / gamma) into the shared-memory activation stage:
// two threads per block, elements 0-15 and 16-31 (quantize_row_q8_0, x86 AVX2 build).
template <int WT>
__device__ void stage_f32(const DArgs& a, int m, int4* sxa, int4* sxb, float* sxd, int* sxi,
                          double* shd) {
    const int nb = a.nb, K = nb * 32;
    const float* xr = a.xf + (size_t)m * a.xf_stride;
    float scale = 1.0f;
    if (a.rms) {
        // RMSNorm (ggml-cpu/ops.cpp:3859-3920): fp32 squares summed in double
        double s = 0.0;
        const float4* x4 = (const float4*)xr;
        for (int k4 = threadIdx.x; k4 < K / 4; k4 += kT) {
            const float4 t = x4[k4];
            s += (double)__fmul_rn(t.x, t.x) + (double)__fmul_rn(t.y, t.y);
            s += (double)__fmul_rn(t.z, t.z) + (double)__fmul_rn(t.w, t.w);
        }
        const double tot = cta_sum_d(s, shd);
        const float mean = (float)(tot / (double)K);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    }
    // two threads per block; whole warps take part (the pair shares its amax by a shuffle)
    const int items = (2 * nb + 31) / 32 * 32;
    for (int it = threadIdx.x; it < items; it += kT) {
        const int b = it >> 1, hh = it & 1;
        float v[16];
        float amax = 0.0f;
        if (b < nb) {
            const float4* src = (const float4*)(xr + (size_t)b * 32 + hh * 16);
            const float4* gsrc = a.gamma ? (const float4*)(a.gamma + (size_t)b * 32 + hh * 16) : nullptr;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 t = src[i];
                const float e[4] = {t.x, t.y, t.z, t.w};
                float g[4] = {1.0f, 1.0f, 1.0f, 1.0f};
                if (gsrc) {
                    const float4 gg = __ldg(gsrc + i);
                    g[0] = gg.x; g[1] = gg.y; g[2] = gg.z; g[3] = gg.w;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float u = e[j];
                    if (a.rms) u = __fmul_rn(u, scale);
                    if (gsrc) u = __fmul_rn(u, g[j]);
                    v[4 * i + j] = u;
                    amax = fmaxf(amax, fabsf(u));
                }
            }
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        int4 qw = make_int4(0, 0, 0, 0);
        float d16 = 0.0f;
        if (b < nb) {
            d16 = __half2float(__float2half_rn(__fdiv_rn(amax, 127.0f)));
            const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            unsigned w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w[j] = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    w[j] |= ((unsigned)__float2int_rn(__fmul_rn(v[4 * j + e], id)) & 0xFF) << (8 * e);
            }
            qw = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
        }
        const int one = 0x01010101;
        int part = __dp4a(qw.x, one, __dp4a(qw.y, one, __dp4a(qw.z, one, __dp4a(qw.w, one, 0))));
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        if (b < nb) {
            if (hh == 0) {
                sxa[b] = qw;
                sxd[b] = d16;
                sxi[b] = WT == T_Q4_0 ? kMagic - 8 * part : kMagic;
            } else {
                sxb[b] = qw;
            }
        }
    }
}

// bytes of one chunk slot: quants (Q8_0: first halves, then second halves), then scales
template <int WT>
constexpr int slot_bytes() {
    return chunk_blocks<WT>() * (WT == T_Q8_0 ? 32 : 16) + (chunk_blocks<WT>() / 64) * 128;
}

// The bulk copies of one item (chunk ch of a weight row), worked out once per warp: byte offsets
// in the row and sizes of the quants (Q8_0: two halves) and of the scale group(s).
struct ChunkCopy {
    uint32_t qoff, qoff2, soff, qb, sb, tx;
};
template <int WT>
__device__ __forceinline__ ChunkCopy chunk_copy(const DArgs& a, int c) {
    constexpr int kCB = chunk_blocks<WT>();
    constexpr int qsz = WT == T_Q8_0 ? 32 : 16;
    const int c0 = c * kCB, cb = min(kCB, a.nb - c0);
    ChunkCopy cc;
    cc.qoff = (uint32_t)c0 * 16;
    cc.qoff2 = (uint32_t)(a.nb + c0) * 16;
    cc.soff = (uint32_t)(a.nb * qsz + (c0 / 64) * 128);
    cc.qb = (uint32_t)cb * 16;
    cc.sb = (uint32_t)((cb + 63) / 64) * 128;
    cc.tx = cc.qb * (WT == T_Q8_0 ? 2u : 1u) + cc.sb;
    return cc;
}

// bulk copies of one item (weight row `row`, the warp's chunk) into a slot
template <int WT>
__device__ __forceinline__ void fetch_chunk(uint8_t* slot, const DArgs& a, int64_t row,
                                            const ChunkCopy& cc, uint64_t* bar) {
    constexpr int kCB = chunk_blocks<WT>();
    constexpr int qsz = WT == T_Q8_0 ? 32 : 16;
    const uint8_t* src = a.w + row * a.rb;
    mbar_expect_tx(bar, cc.tx);
    auto copy = [&](void* dst, const void* from, uint32_t bytes) {
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
            "[%3];" ::"r"(su32(dst)),
            "l"(from), "r"(bytes), "r"(su32(bar))
            : "memory");
    };
    copy(slot, src + cc.qoff, cc.qb);
    if (WT == T_Q8_0) copy(slot + kCB * 16, src + cc.qoff2, cc.qb);
    copy(slot + kCB * qsz, src + cc.soff, cc.sb);
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The all-reduce of the epilogue (GemvAllReduce, kernels.h) over this CTA's rows [u0, u1) of y
// (one activation row): slot [parity][rank] of every rank, flags, bounded wait, rank-order sum.
__device__ void gemv_allreduce(const GemvAllReduce& ar, float* y, int u0, int u1) {
    __shared__ uint32_t s_e;
    __syncthreads();  // this CTA's rows of y are written
    if (threadIdx.x == 0) s_e = ar.epochs[blockIdx.x] + 1;
    __syncthreads();
    const uint32_t e = s_e;
    const int par = (int)(e & 1u), T = ar.T, me = ar.rank;
    for (int p = 0; p < T; ++p) {
        float* dst = ar.peers.grecv[p] + ((int64_t)par * T + me) * ar.cap;
        for (int i = u0 + threadIdx.x; i < u1; i += kT) dst[i] = y[i];
    }
    __syncthreads();
    if (threadIdx.x < T) {  // thread p tells rank p that this CTA's rows of slot [par][me] are in
        __threadfence_system();
        st_release_sys_u32(ar.peers.gflags[threadIdx.x] + ((int64_t)par * T + me) * kGemvArCtas + blockIdx.x, e);
    }
    if (threadIdx.x < T) {  // thread r waits for rank r's rows in this rank's memory
        const uint32_t* f = ar.peers.gflags[me] + ((int64_t)par * T + threadIdx.x) * kGemvArCtas + blockIdx.x;
        const long long t0 = clock64();
        while (ld_acquire_sys_u32(f) != e) {
            if (clock64() - t0 > kSpinCycles / 2) {  // about 1 s
                *(volatile int*)ar.err = 1;     // host-mapped word
                __threadfence_system();
                break;
            }
        }
    }
    __syncthreads();
    const float* src = ar.peers.grecv[me] + (int64_t)par * T * ar.cap;
    for (int i = u0 + threadIdx.x; i < u1; i += kT) {
        float v = __ldcg(src + i);
        for (int r = 1; r < T; ++r) v = __fadd_rn(v, __ldcg(src + (int64_t)r * ar.cap + i));
        y[i] = v;
    }
    if (threadIdx.x == 0) ar.epochs[blockIdx.x] = e;
}

// MAXM: activation rows (1 or 2; M <= MAXM at run time).
template <int WT, int MAXM>
__global__ void __launch_bounds__(kT, 1) k_dgemv(DArgs a) {
    DGEMV_TRACE_BEGIN;
    constexpr int kCB = chunk_blocks<WT>();
    constexpr int BPL = kCB / 32;  // activation blocks per lane
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[kW][kMaxSlots];
    __shared__ double shd[kW];
    constexpr int SB = slot_bytes<WT>();
    constexpr int QS = WT == T_Q8_0 ? 32 : 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb, M = a.M, nc = a.nc, D = a.slots;
    uint8_t* ring = smem + (size_t)warp * D * SB;
    // activation stage of row m: [sxa nb][sxb nb][sxd nb][sxi nb]; then the chunk partials
    uint8_t* stage = smem + (size_t)kW * D * SB;
    auto sxa = [&](int m) { return (int4*)(stage + (size_t)m * nb * 40); };
    auto sxb = [&](int m) { return sxa(m) + nb; };
    auto sxd = [&](int m) { return (float*)(sxb(m) + nb); };
    auto sxi = [&](int m) { return (int*)(sxd(m) + nb); };
    float* part = (float*)(stage + (size_t)(a.xf ? M : 0) * nb * 40);  // [row][chunk][m]

    // this CTA's units and rows (SwiGLU: local row 2k is gate k, 2k+1 is up k)
    const int u0 = (int)((int64_t)a.units * blockIdx.x / gridDim.x);
    const int u1 = (int)((int64_t)a.units * (blockIdx.x + 1) / gridDim.x);
    const int per = a.swiglu ? 2 : 1;
    const int sh = a.swiglu ? 1 : 0;  // log2(per)
    // this warp: chunk `ch` of units g, g + G, g + 2G, ... (nc <= kW: every warp has a chunk);
    // item k is row `per * unit + k % per` of unit g + (k / per) * G, so a SwiGLU pair's gate
    // and up rows go through the same warp, one after the other
    const int ch = warp % nc, g = warp / nc, G = (kW - ch + nc - 1) / nc;
    const int nu = u1 - u0;
    const int nmine = (nu > g ? (nu - g + G - 1) / G : 0) * per;
    // item q: local unit g + (q >> sh) * G; its local row (unit << sh) + (q & sh); its weight row
    // u0 + unit, or F rows on for the up row of a SwiGLU pair (no division in the item loop)
    auto item_row = [&](int q) { return ((g + (q >> sh) * G) << sh) + (q & sh); };
    auto item_wrow = [&](int q) -> int64_t {
        const int64_t r = (int64_t)u0 + g + (q >> sh) * G;
        return (q & sh) ? r + a.F : r;
    };
    const ChunkCopy cc = chunk_copy<WT>(a, ch);
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    uint64_t* bar = bars[warp];
    if (lane == 0) {
        for (int s = 0; s < D; ++s) mbar_init(&bar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int k = 0; k < D && k < nmine; ++k)
            fetch_chunk<WT>(ring + (size_t)k * SB, a, item_wrow(k), cc, &bar[k]);
    }
    __syncwarp();
    // this CTA's share of the next weights into L2, requested before the wait for the previous
    // launch: those bytes stream while this launch's prologue and rows run
    if (a.pf && threadIdx.x == kT - 32) {
        for (int nb = blockIdx.x; nb < a.pf_grid; nb += gridDim.x) {
            const int64_t v0 = a.pf_units * nb / a.pf_grid, v1 = a.pf_units * (nb + 1) / a.pf_grid;
            const int nr = a.pf_F ? 2 : 1;
            const int64_t len = min((v1 - v0) * a.pf_rb, a.pf_cap / nr) & ~(int64_t)15;
            for (int r = 0; r < nr; ++r) {
                const uint8_t* src = a.pf + (v0 + r * a.pf_F) * a.pf_rb;
                for (int64_t o = 0; o < len; o += 32768) {
                    const uint32_t n = (uint32_t)min((int64_t)32768, len - o);
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src + o), "r"(n)
                                 : "memory");
                }
            }
        }
    }

    pdl_wait();
    DGEMV_TRACE(1);
    for (int m = 0; m < M && a.xf; ++m) {
        stage_f32<WT>(a, m, sxa(m), sxb(m), sxd(m), sxi(m), shd);
        if (a.rms) __syncthreads();  // shd is reused by the next row's reduction
    }
    if (a.xf) __syncthreads();
    pdl_launch();
    DGEMV_TRACE(2);

    // the activation blocks of this warp's chunk: b = 128 ch + lane + 32 j
    XBlk x[MAXM][BPL];
    const int c0 = ch * kCB, cb = min(kCB, nb - c0);
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
#pragma unroll
        for (int j = 0; j < BPL; ++j) {
            const int bl = lane + 32 * j, b = c0 + bl;
            XBlk& xb = x[m][j];
            xb.lo = xb.hi = make_int4(0, 0, 0, 0);
            xb.d = 0.0f;
            xb.init = kMagic;
            if (m < M && bl < cb) {
                if (a.xf) {
                    xb.lo = sxa(m)[b];
                    xb.hi = sxb(m)[b];
                    xb.d = sxd(m)[b];
                    xb.init = sxi(m)[b];
                } else {
                    const int4* src = (const int4*)(a.xq + (size_t)m * nb * 32 + (size_t)b * 32);
                    xb.lo = src[0];
                    xb.hi = src[1];
                    xb.d = a.xd[(size_t)m * nb + b];
                    xb.init = chain_init<WT>(xb.lo, xb.hi);
                }
            }
        }
    }

    float gate[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) gate[m] = 0.0f;
    bool ok = true;
    int k = 0;
    int rs = 0;        // ring slot of item k
    uint32_t rph = 0;  // its mbarrier phase
    for (; k < nmine; ++k) {
        const int s = rs;
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], rph))) {
            ok = false;
            break;
        }
        if (++rs == D) {
            rs = 0;
            rph ^= 1u;
        }
        const uint8_t* slot = ring + (size_t)s * SB;
        const uint8_t* sc = slot + kCB * QS;
        float acc[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
#pragma unroll
        for (int jp = 0; jp < BPL / 2; ++jp) {
            const unsigned sw = 64 * jp + lane < cb ? *(const unsigned*)(sc + jp * 128 + lane * 4) : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * jp + h, bl = lane + 32 * j;
                if (bl < cb) {
                    WBlk wb;
                    if (WT == T_Q4_0) {
                        const uint4 q = *(const uint4*)(slot + (size_t)bl * 16);
                        wb.a = make_uint4(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu);
                        wb.b = make_uint4(q.x & 0xF0F0F0F0u, q.y & 0xF0F0F0F0u, q.z & 0xF0F0F0F0u, q.w & 0xF0F0F0F0u);
                    } else {
                        wb.a = *(const uint4*)(slot + (size_t)bl * 16);
                        wb.b = *(const uint4*)(slot + (size_t)(kCB + bl) * 16);
                    }
                    const float dw = h ? half_hi(sw) : half_lo(sw);
#pragma unroll
                    for (int m = 0; m < MAXM; ++m)
                        if (m < M) block_term<WT>(wb, dw, x[m][j], acc[m]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && k + D < nmine) {  // the slot is consumed: refill it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fetch_chunk<WT>(ring + (size_t)s * SB, a, item_wrow(k + D), cc, &bar[s]);
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                acc[m] = __fadd_rn(acc[m], __shfl_xor_sync(0xffffffffu, acc[m], off));
        }
        const int i = item_row(k);  // local row
        if (nc > 1) {             // chunk partial: rows are finished below
            if (lane < M) part[((size_t)i * nc + ch) * MAXM + lane] = lane == 0 ? acc[0] : acc[MAXM - 1];
            continue;
        }
        if (a.swiglu) {
            if (i & 1) {
#pragma unroll
                for (int m = 0; m < MAXM; ++m)
                    if (m < M && lane == m)
                        a.y[(size_t)m * a.y_stride + u0 + (i >> 1)] = __fmul_rn(ref_v_silu(gate[m]), acc[m]);
            } else {
#pragma unroll
                for (int m = 0; m < MAXM; ++m) gate[m] = acc[m];
            }
        } else {
            const int64_t row = u0 + i;
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M && lane == m) {
                    float r = acc[m];
                    if (a.bias) r = __fadd_rn(r, a.bias[row]);
                    if (a.residual) r = __fadd_rn(a.residual[(size_t)m * a.res_stride + row], r);
                    a.y[(size_t)m * a.y_stride + row] = r;
                }
            }
        }
    }
    DGEMV_TRACE(3);
    if (!ok) {
        if (lane == 0) {
            atomicExch(&dgemv_error_word, 1);
            s_fail = 1;
            // the copies this warp issued and did not consume: wait for them (bounded)
            for (int q = k; q < nmine && q < k + D; ++q) mbar_wait(&bar[q % D], (uint32_t)(q / D) & 1u);
        }
        __syncwarp();
    }
    if (nc > 1) {
        // rows cut into chunks: every row's chunk sums in chunk order, then the epilogue
        __syncthreads();
        if (s_fail) return;  // a wait ran out in this CTA: its partials are incomplete
        for (int t = threadIdx.x; t < (u1 - u0) * M; t += kT) {
            const int uu = t / M, m = t % M;
            float r[2];
            for (int hh = 0; hh < per; ++hh) {
                const int i = uu * per + hh;
                float v = part[((size_t)i * nc) * MAXM + m];
                for (int c = 1; c < nc; ++c) v = __fadd_rn(v, part[((size_t)i * nc + c) * MAXM + m]);
                r[hh] = v;
            }
            if (a.swiglu) {
                a.y[(size_t)m * a.y_stride + u0 + uu] = __fmul_rn(ref_v_silu(r[0]), r[1]);
            } else {
                const int64_t row = u0 + uu;
                float v = r[0];
                if (a.bias) v = __fadd_rn(v, a.bias[row]);
                if (a.residual) v = __fadd_rn(a.residual[(size_t)m * a.res_stride + row], v);
                a.y[(size_t)m * a.y_stride + row] = v;
            }
        }
    }
    if (a.ar.T > 0) gemv_allreduce(a.ar, a.y, u0, u1);
    DGEMV_TRACE(4);
}

template <int WT, int MAXM>
void launch_t(const DArgs& a, size_t smem, int grid, cudaStream_t st) {
    auto kern = k_dgemv<WT, MAXM>;
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "dgemv: device ordinal out of range");
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024));
            configured[dev] = true;
        }
    }
    launch_pdl(kern, (unsigned)grid, kT, smem, st, a);
}

template <int WT>
void launch_w(const DArgs& a, size_t smem, int grid, cudaStream_t st) {
    if (a.M == 1) launch_t<WT, 1>(a, smem, grid, st);
    else launch_t<WT, 2>(a, smem, grid, st);
}


// bytes of the next GEMV's weights requested into L2 ahead of it (GGMLC_B200_L2PF, MiB; default
// 0, off: 24-96 MiB measured no faster at the Llama-3-8B decode shape)
size_t l2_prefetch_budget() {
    static const size_t v = [] {
        const char* e = getenv("GGMLC_B200_L2PF");
        return (size_t)(e ? std::max(0LL, atoll(e)) : 0LL) << 20;
    }();
    return v;
}

// activation stage: per row and block 16 + 16 quant bytes, the scale and the chain start
size_t stage_bytes(int nb, int M) { return (size_t)M * nb * (16 + 16 + 4 + 4); }

size_t ring_budget() {
    static const size_t v = [] {
        const char* e = getenv("GGMLC_B200_DGEMV_RING");  // tuning: ring bytes per CTA
        const long long b = e ? atoll(e) : 0;
        return b > 0 ? (size_t)b : kRingBudget;
    }();
    return v;
}

}  // namespace

bool dgemv_eligible(const GemvArgs& a) {
    if (a.M < 1 || a.M > 2 || (a.w.type != T_Q4_0 && a.w.type != T_Q8_0) || a.w.K % QK != 0)
        return false;
    const int64_t cbk = a.w.type == T_Q8_0 ? chunk_blocks<T_Q8_0>() : chunk_blocks<T_Q4_0>();
    if (a.w.N <= 0 || a.w.N >= (1LL << 30) || a.w.K > cbk * QK * kMaxChunks) return false;
    if (((uintptr_t)a.w.qs & 15) != 0) return false;
    if (a.yq || a.yd) return false;  // Q8_0 output of the SwiGLU: the tiled GEMV
    if (a.swiglu && (a.w.N != 2 * a.F || !a.y || a.y_stride != a.F)) return false;
    if (!a.swiglu && !a.y) return false;
    if (a.xf) {
        if (((uintptr_t)a.xf & 15) != 0 || (a.gamma && ((uintptr_t)a.gamma & 15) != 0)) return false;
        if (a.M > 1 && (a.xf_stride % 4) != 0) return false;
    } else if (!a.xq || !a.xd || ((uintptr_t)a.xq & 15) != 0) {
        return false;
    }
    return true;
}

void launch_dgemv(const GemvArgs& a, cudaStream_t st) {
    GB_CHECK(dgemv_eligible(a), "dgemv: arguments outside the single-row bulk-copy GEMV");
    DArgs d;
    d.pf = nullptr;
    d.pf_rb = d.pf_units = d.pf_F = d.pf_cap = 0;
    d.pf_grid = 0;
    const PfNext& nx = a.pf;
    if (nx.qs && l2_prefetch_budget() > 0 && (nx.type == T_Q4_0 || nx.type == T_Q8_0) &&
        ((uintptr_t)nx.qs & 15) == 0 && nx.N > 0 && nx.K % QK == 0) {
        int dv = 0;
        GB_CUDA(cudaGetDevice(&dv));
        const int64_t units = nx.F ? nx.F : nx.N;
        d.pf = (const uint8_t*)nx.qs;
        d.pf_rb = qrow_bytes(nx.type, nx.K);
        d.pf_units = units;
        d.pf_F = nx.F;
        d.pf_grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(dv), (units + kW - 1) / kW));
        d.pf_cap = (int64_t)l2_prefetch_budget() / d.pf_grid;
    }
    d.w = (const uint8_t*)a.w.qs;
    d.rb = qrow_bytes(a.w.type, a.w.K);
    d.nb = (int)(a.w.K / QK);
    const int64_t cbk = a.w.type == T_Q8_0 ? chunk_blocks<T_Q8_0>() : chunk_blocks<T_Q4_0>();
    d.nc = (d.nb + (int)cbk - 1) / (int)cbk;
    d.M = a.M;
    d.xf_stride = a.xf_stride;
    d.y_stride = a.y_stride;
    d.res_stride = a.res_stride;
    d.ar = a.ar;
    if (a.ar.T > 0) {
        GB_CHECK(a.M == 1 && !a.swiglu && a.y_stride == a.w.N,
                 "dgemv all-reduce: one activation row, plain output");
        GB_CHECK(a.ar.T <= kMaxTp && a.ar.rank >= 0 && a.ar.rank < a.ar.T && a.w.N <= a.ar.cap,
                 "dgemv all-reduce: bad rank / size or vector larger than the peer slots");
    }
    d.swiglu = a.swiglu ? 1 : 0;
    d.F = (int)a.F;
    d.units = (int)(a.swiglu ? a.F : a.w.N);
    d.xq = a.xq;
    d.xd = a.xd;
    d.xf = a.xf;
    d.rms = a.xf && a.xf_rms ? 1 : 0;
    d.eps = a.eps;
    d.gamma = a.xf ? a.gamma : nullptr;
    d.y = a.y;
    d.bias = a.swiglu ? nullptr : a.bias;
    d.residual = a.swiglu ? nullptr : a.residual;
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    // one CTA per SM, fewer when there are not 8 units per CTA
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(dev), (d.units + kW - 1) / kW));
    GB_CHECK(a.ar.T == 0 || grid <= kGemvArCtas, "dgemv all-reduce: more CTAs than flag slots");
    d.rows_cta = (int)((d.units + grid - 1) / grid + 1) * (d.swiglu ? 2 : 1);
    const size_t sb = a.w.type == T_Q8_0 ? slot_bytes<T_Q8_0>() : slot_bytes<T_Q4_0>();
    d.slots = (int)std::max<int64_t>(1, std::min<int64_t>(kMaxSlots, (int64_t)(ring_budget() / (kW * sb))));
    const size_t smem = (size_t)kW * d.slots * sb + (a.xf ? stage_bytes(d.nb, d.M) : 0) +
                        (d.nc > 1 ? (size_t)d.rows_cta * d.nc * 2 * sizeof(float) : 0);
    GB_CHECK(smem <= 200 * 1024, "dgemv: shared memory plan too large");
    if (a.w.type == T_Q4_0) launch_w<T_Q4_0>(d, smem, grid, st);
    else launch_w<T_Q8_0>(d, smem, grid, st);
}

#ifdef GB_DGEMV_TRACE
extern "C" int gb_dgemv_trace_read(unsigned long long* out, size_t bytes) {
    if (bytes < sizeof(g_dgemv_tr)) return -1;
    return cudaMemcpyFromSymbol(out, g_dgemv_tr, sizeof(g_dgemv_tr)) == cudaSuccess ? 0 : -1;
}
extern "C" int gb_dgemv_trace_reset() {
    static const unsigned zero[kTrCtas] = {};
    return cudaMemcpyToSymbol(g_dgemv_tr_n, zero, sizeof(zero)) == cudaSuccess ? 0 : -1;
}
#endif

int dgemv_error() {
    int v = 0;
    GB_CUDA(cudaMemcpyFromSymbol(&v, dgemv_error_word, sizeof(int)));
    return v;
}

}  // namespace gb
