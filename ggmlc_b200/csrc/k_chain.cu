// Decode chain: the launches of one single-sequence decode step as ONE persistent launch.
//
// Why.  A batch-1 decode step of a Llama-3-8B-shaped model is ~160 small launches (5 per layer).
// Each one ramps its weight stream up from nothing, pays a prologue (RMSNorm + Q8_0 of the
// activation row) before its first dot product and drains at its tail, so HBM idles between
// launches even with programmatic dependent launch.  Here one CTA per SM runs every op of the
// step in order, separated by grid-wide barriers; the weight stream never stops, because the
// weights do not depend on activations: every warp keeps a ring of bulk copies (cp.async.bulk,
// the TMA engine's linear mode) filled with the chunks it will consume next, across op
// boundaries — while its CTA waits at a barrier, quantizes the next activation row or works on
// attention, the copies of the following GEMVs are already in flight.
//
// Ops (ChainOp, kernels.h):
//   CH_GEMV  one-row matmul over the split-row Q4_0 / Q8_0 layout, exactly k_dgemv's work split
//            per CTA (contiguous units), per warp (chunk index fixed per warp, rows dealt in turn)
//            and arithmetic (kdot.cuh block terms, lane butterfly, chunks added in chunk order),
//            so its outputs are bit-identical to launch_dgemv's.  Prologue: f32 row quantized
//            to Q8_0 in shared memory, after RMSNorm (+gamma) when asked; or a Q8_0 row.
//            Epilogue: f32 (+bias, +residual) or SwiGLU.
//   CH_ATTN  decode attention of one row over the F16 KV cache: every (KV head, split) unit
//            rotates the q heads of its GQA group (RoPE from the host table, q rounded to fp16
//            as the CPU kernel does), the unit holding the new position also rotates k and
//            writes k, v into the cache; positions are staged 32 at a time (cp.async) with an
//            fp32 online softmax; the last unit of a KV head to finish (an atomic counter,
//            threadfence-reduction pattern) merges the splits and writes f32 and/or Q8_0.
//   CH_ROW   one row, RMSNorm (+gamma) or plain, to f32 and/or Q8_0 (the output norm and the
//            quantization in front of the output projection); CTA 0 only.
//
// Memory model.  Activations written by other CTAs during the launch are read with ld.global.cg
// (L2), never through L1.  The grid barrier is a counter plus a generation word: each CTA's
// thread 0 adds one with acquire-release semantics after a fence; the last to arrive resets the
// counter and releases the next generation, the others spin (acquire loads) until it changes.
//
// Bounded waits.  Every mbarrier wait and every spin is bounded (about 2 s).  On expiry the CTA
// records chain_error_word (chain_error()), its peers see the word in their barrier spin and
// stop, every warp waits (bounded) for the copies it still has in flight, and the launch ends;
// later launches see the word and return at once (the counters are not trusted after an error).
//
// Launch: cooperative (all CTAs co-resident), grid = SM count, 16 warps, 1 CTA per SM.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kdot.cuh"
#include "krope.cuh"
#include "kutil.cuh"

namespace gb {

__device__ int chain_error_word;

// Optional per-CTA timeline (built with -DGB_CHAIN_TRACE only; not part of the shipped library):
// %globaltimer of CTA b when it reaches op j's barrier (slot 0) and when it leaves it (slot 1);
// inside a GEMV op: prologue done (2), warp 0's items done (3), every warp's items done (4).
#ifdef GB_CHAIN_TRACE
constexpr int kTraceOps = 256, kTraceCtas = 160;
__device__ unsigned long long g_chain_trace[kTraceOps][kTraceCtas][6];
#define CHAIN_TRACE(j, k)                                                                   \
    do {                                                                                    \
        if (threadIdx.x == 0 && (j) < kTraceOps && blockIdx.x < kTraceCtas) {               \
            unsigned long long t_;                                                          \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                          \
            g_chain_trace[(j)][blockIdx.x][(k)] = t_;                                       \
        }                                                                                   \
    } while (0)
#else
#define CHAIN_TRACE(j, k) ((void)0)
#endif

namespace {

constexpr int kW = 16;            // warps per CTA
constexpr int kT = kW * 32;
constexpr int kMaxSlots = 8;      // ring slots per warp
constexpr int kSlotBytes = 2304;  // one chunk: Q4_0 128 blocks (2048 + 256), Q8_0 64 (2048 + 128)
constexpr int kAC = 32;           // attention: positions staged per step
constexpr int kMaxRk = 8;         // q heads per KV head
constexpr int kMaxSplits = 64;    // attention splits per KV head

__host__ __device__ constexpr int cblocks(int wt) { return wt == T_Q8_0 ? 64 : 128; }

struct ChainArgs {
    const ChainOp* __restrict__ ops;
    int nops;
    int slots;  // ring slots per warp
    ChainSync* sync;
    float* part;  // attention partials
    int* err;     // set to 1 (besides chain_error_word) when the launch fails; may be null
};

// ------------------------------------------------------------------ GEMV work split per warp
struct Plan {
    int nb, nc, per, u0, nu, ch, g, gw, nmine;
};
__device__ __forceinline__ Plan plan_of(const ChainOp& op, int warp) {
    Plan p;
    p.nb = (int)(op.K / QK);
    const int cb = cblocks(op.wtype);
    p.nc = (p.nb + cb - 1) / cb;
    const int units = (int)(op.swiglu ? op.F : op.N);
    p.per = op.swiglu ? 2 : 1;
    p.u0 = (int)((int64_t)units * blockIdx.x / gridDim.x);
    p.nu = (int)((int64_t)units * (blockIdx.x + 1) / gridDim.x) - p.u0;
    p.ch = warp % p.nc;  // this warp's chunk index (nc <= kW)
    p.g = warp / p.nc;   // its place among the warps of that chunk index
    p.gw = (kW - p.ch + p.nc - 1) / p.nc;
    p.nmine = (p.nu > p.g ? (p.nu - p.g + p.gw - 1) / p.gw : 0) * p.per;
    return p;
}
// local row of a warp's item k: units g, g + gw, ...; a SwiGLU pair's gate and up rows in turn
__device__ __forceinline__ int item_row(const Plan& p, int k) {
    const int sh = p.per - 1;  // per is 1 or 2: shifts and masks, no division in the item loop
    return ((p.g + (k >> sh) * p.gw) << sh) + (k & sh);
}

// A warp's producer cursor (lane 0 only; kept in shared memory, off the register budget): the
// GEMV op whose items it requests next, with that op's plan for this warp reduced to the
// offsets one request needs, so a request is a few integer operations and the bulk copies.
struct Cursor {
    const uint8_t* w;   // weight rows
    int64_t rb, F;      // row bytes; SwiGLU: rows of the up half start F rows after the gate's
    int ug, gw, shift;  // first unit of this warp (u0 + g), unit step, log2(rows per unit)
    int swiglu, q8;
    int nmine, fk, fop; // items of this warp in op fop, next item to request
    uint32_t qoff, qoff2, soff, qb, sb;  // byte offsets / sizes of the chunk's copies in a row
    uint32_t tx;        // bytes one item brings
};

// point the cursor at the next GEMV op after c.fop (nmine = 0 past the last one)
__device__ void cursor_next(Cursor& c, const ChainArgs& A, int warp) {
    int j = c.fop + 1;
    while (j < A.nops && A.ops[j].kind != CH_GEMV) ++j;
    c.fop = j;
    c.fk = 0;
    c.nmine = 0;
    if (j >= A.nops) return;
    const ChainOp& op = A.ops[j];
    const Plan p = plan_of(op, warp);
    const bool q8 = op.wtype == T_Q8_0;
    const int cbf = cblocks(op.wtype);
    const int c0 = p.ch * cbf, cb = min(cbf, p.nb - c0);
    const int qs = q8 ? 32 : 16;
    c.w = op.w;
    c.rb = op.rb;
    c.F = op.F;
    c.ug = p.u0 + p.g;
    c.gw = p.gw;
    c.shift = p.per == 2 ? 1 : 0;
    c.swiglu = op.swiglu;
    c.q8 = q8 ? 1 : 0;
    c.nmine = p.nmine;
    c.qoff = (uint32_t)c0 * 16;
    c.qoff2 = (uint32_t)(p.nb + c0) * 16;
    c.soff = (uint32_t)(p.nb * qs + (c0 / 64) * 128);
    c.qb = (uint32_t)cb * 16;
    c.sb = (uint32_t)((cb + 63) / 64) * 128;
    c.tx = c.qb * (q8 ? 2u : 1u) + c.sb;
}

// A warp's ring: consumer position (slot, phase; the same in every lane) and, in lane 0, the
// producer's slot and the copies in flight.
struct Ring {
    uint8_t* base;
    uint64_t* bar;
    Cursor* cur;
    int cs, cph;   // consumer slot and phase
    int fs;        // producer slot
    int inflight;  // requested, not yet consumed
};

// lane 0: request items (in op order, GEMV ops only) until every slot is taken.  Item k of the
// cursor's op is chunk ch of unit ug + (k >> shift) * gw (the gate row, then the up row, of a
// SwiGLU unit).
__device__ void top_up(Ring& r, const ChainArgs& A, int warp) {
    Cursor& c = *r.cur;
    while (r.inflight < A.slots) {
        if (c.fk >= c.nmine) {
            if (c.fop >= A.nops) return;
            cursor_next(c, A, warp);
            continue;
        }
        const int k = c.fk;
        int64_t row = c.ug + (int64_t)(k >> c.shift) * c.gw;
        if (c.swiglu && (k & 1)) row += c.F;
        const uint8_t* src = c.w + row * c.rb;
        uint8_t* slot = r.base + (size_t)r.fs * kSlotBytes;
        uint64_t* bar = &r.bar[r.fs];
        const int cbf = c.q8 ? 64 : 128;
        mbar_expect_tx(bar, c.tx);
        bulk_g2s(slot, src + c.qoff, c.qb, bar);
        if (c.q8) bulk_g2s(slot + cbf * 16, src + c.qoff2, c.qb, bar);
        bulk_g2s(slot + cbf * (c.q8 ? 32 : 16), src + c.soff, c.sb, bar);
        ++c.fk;
        ++r.inflight;
        if (++r.fs == A.slots) r.fs = 0;
    }
}

// lane 0: wait (bounded) for every copy still in flight, so none lands after the CTA exits
__device__ void drain(Ring& r, int slots) {
    int s = r.cs, ph = r.cph;
    for (int q = 0; q < r.inflight; ++q) {
        mbar_wait(&r.bar[s], (uint32_t)ph);
        if (++s == slots) {
            s = 0;
            ph ^= 1;
        }
    }
    r.inflight = 0;
}

// ------------------------------------------------------------------ grid barrier
__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_rel(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_ar(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ bool chain_failed() {
    return ld_acq((const unsigned*)&chain_error_word) != 0;
}

// All CTAs reach this point before any leaves it; the writes before it are visible after it.
// False when the wait ran out or another CTA recorded an error.
__device__ bool grid_sync(ChainSync* sy, int* s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned gen = ld_acq(&sy->gen);  // cannot advance before this CTA arrives
        __threadfence();
        const unsigned a = atom_add_ar(&sy->count, 1u);
        if (a == gridDim.x - 1) {
            sy->count = 0u;
            st_rel(&sy->gen, gen + 1u);
        } else {
            const long long t0 = clock64();
            while (ld_acq(&sy->gen) == gen) {
                if (clock64() - t0 > kSpinCycles || chain_failed()) {
                    ok = 0;
                    break;
                }
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

__device__ double cta_sum_d(double v, double* sh) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < kW; ++i) t += sh[i];
    return t;
}

// ------------------------------------------------------------------ CH_GEMV
// Quantize the f32 input row (after RMSNorm / gamma) into the activation stage, two threads per
// block — k_dgemv's prologue with the same thread count, so the same sums and the same bits.
template <int WT>
__device__ void stage_f32(const ChainOp& op, int nb, int4* sxa, int4* sxb, float* sxd, int* sxi,
                          double* shd) {
    const int K = nb * 32;
    const float* xr = op.xf;
    float scale = 1.0f;
    if (op.rms) {
        // RMSNorm (ggml-cpu/ops.cpp:3859-3920): fp32 squares summed in double
        double s = 0.0;
        const float4* x4 = (const float4*)xr;
        for (int k4 = threadIdx.x; k4 < K / 4; k4 += kT) {
            const float4 t = __ldcg(x4 + k4);
            s += (double)__fmul_rn(t.x, t.x) + (double)__fmul_rn(t.y, t.y);
            s += (double)__fmul_rn(t.z, t.z) + (double)__fmul_rn(t.w, t.w);
        }
        const double tot = cta_sum_d(s, shd);
        const float mean = (float)(tot / (double)K);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, op.eps)));
    }
    const int items = (2 * nb + 31) / 32 * 32;
    for (int it = threadIdx.x; it < items; it += kT) {
        const int b = it >> 1, hh = it & 1;
        float v[16];
        float amax = 0.0f;
        if (b < nb) {
            const float4* src = (const float4*)(xr + (size_t)b * 32 + hh * 16);
            const float4* gsrc = op.gamma ? (const float4*)(op.gamma + (size_t)b * 32 + hh * 16) : nullptr;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 t = __ldcg(src + i);
                const float e[4] = {t.x, t.y, t.z, t.w};
                float g[4] = {1.0f, 1.0f, 1.0f, 1.0f};
                if (gsrc) {
                    const float4 gg = __ldg(gsrc + i);
                    g[0] = gg.x; g[1] = gg.y; g[2] = gg.z; g[3] = gg.w;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float u = e[j];
                    if (op.rms) u = __fmul_rn(u, scale);
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

// the epilogue of a GEMV op, read from the op table once per op
struct Epi {
    float* y;
    const float* bias;
    const float* residual;
    bool swiglu;
};
__device__ __forceinline__ float gemv_out(const Epi& e, int64_t row, float acc) {
    float r = acc;
    if (e.bias) r = __fadd_rn(r, __ldg(e.bias + row));
    if (e.residual) r = __fadd_rn(__ldcg(e.residual + row), r);
    return r;
}

// One GEMV op.  Returns false (in every thread of the CTA) when a wait ran out in any warp.
template <int WT>
__device__ bool gemv_op(const ChainArgs& A, const ChainOp& op, Ring& r, uint8_t* work,
                        double* shd, int* s_fail, int warp, int lane, int jop) {
    constexpr int kCB = cblocks(WT);
    constexpr int BPL = kCB / 32;  // activation blocks per lane
    constexpr int QS = WT == T_Q8_0 ? 32 : 16;
    const Plan p = plan_of(op, warp);
    const int nb = p.nb, nc = p.nc;
    Epi ep;
    ep.y = op.y;
    ep.bias = op.bias;
    ep.residual = op.residual;
    ep.swiglu = op.swiglu != 0;
    // activation stage [sxa nb][sxb nb][sxd nb][sxi nb], then the chunk partials [rows][nc]
    int4* sxa = (int4*)work;
    int4* sxb = sxa + nb;
    float* sxd = (float*)(sxb + nb);
    int* sxi = (int*)(sxd + nb);
    float* part = (float*)(work + (op.xf ? (size_t)nb * 40 : 0));
    if (op.xf) {
        stage_f32<WT>(op, nb, sxa, sxb, sxd, sxi, shd);
        __syncthreads();
    }
    // the activation blocks of this warp's chunk: b = kCB * ch + lane + 32 j
    XBlk x[BPL];
    const int c0 = p.ch * kCB, cb = min(kCB, nb - c0);
#pragma unroll
    for (int j = 0; j < BPL; ++j) {
        const int bl = lane + 32 * j, b = c0 + bl;
        XBlk& xb = x[j];
        xb.lo = xb.hi = make_int4(0, 0, 0, 0);
        xb.d = 0.0f;
        xb.init = kMagic;
        if (bl < cb) {
            if (op.xf) {
                xb.lo = sxa[b];
                xb.hi = sxb[b];
                xb.d = sxd[b];
                xb.init = sxi[b];
            } else {
                const int4* src = (const int4*)(op.xq + (size_t)b * 32);
                xb.lo = __ldcg(src);
                xb.hi = __ldcg(src + 1);
                xb.d = __ldcg(op.xd + b);
                xb.init = chain_init<WT>(xb.lo, xb.hi);
            }
        }
    }
    float gate = 0.0f;
    bool ok = true;
    CHAIN_TRACE(jop, 2);
    for (int k = 0; k < p.nmine; ++k) {
        if (!__all_sync(0xffffffffu, mbar_wait(&r.bar[r.cs], (uint32_t)r.cph))) {
            ok = false;
            break;
        }
        const uint8_t* slot = r.base + (size_t)r.cs * kSlotBytes;
        const uint8_t* sc = slot + kCB * QS;
        float acc = 0.0f;
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
                    block_term<WT>(wb, dw, x[j], acc);
                }
            }
        }
        __syncwarp();
        // the slot is consumed: advance, and lane 0 refills the ring (possibly from later ops)
        if (++r.cs == A.slots) {
            r.cs = 0;
            r.cph ^= 1;
        }
        --r.inflight;
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            top_up(r, A, warp);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        const int i = item_row(p, k);  // local row
        if (nc > 1) {                  // chunk partial: rows are finished below
            if (lane == 0) part[i * nc + p.ch] = acc;
            continue;
        }
        if (ep.swiglu) {
            if (i & 1) {
                if (lane == 0) ep.y[p.u0 + i / 2] = __fmul_rn(ref_v_silu(gate), acc);
            } else {
                gate = acc;
            }
        } else if (lane == 0) {
            const int64_t row = p.u0 + i;
            ep.y[row] = gemv_out(ep, row, acc);
        }
    }
    if (!ok && lane == 0) *s_fail = 1;
    CHAIN_TRACE(jop, 3);
    __syncthreads();
    CHAIN_TRACE(jop, 4);
    if (*s_fail) return false;
    if (nc > 1) {
        // rows cut into chunks: every row's chunk sums in chunk order, then the epilogue
        for (int t = threadIdx.x; t < p.nu; t += kT) {
            float rr[2] = {0.0f, 0.0f};
            for (int hh = 0; hh < p.per; ++hh) {
                const int i = t * p.per + hh;
                float v = part[i * nc];
                for (int c = 1; c < nc; ++c) v = __fadd_rn(v, part[i * nc + c]);
                rr[hh] = v;
            }
            if (ep.swiglu) ep.y[p.u0 + t] = __fmul_rn(ref_v_silu(rr[0]), rr[1]);
            else ep.y[p.u0 + t] = gemv_out(ep, p.u0 + t, rr[0]);
        }
    }
    return true;
}

// ------------------------------------------------------------------ CH_ATTN
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}

// shared-memory plan of the attention op for head_dim HD
template <int HD>
struct AttnSmem {
    static constexpr size_t k_off = 0;                                  // [kAC][HD] half
    static constexpr size_t v_off = k_off + (size_t)kAC * HD * 2;       // [kAC][HD] half
    static constexpr size_t new_off = v_off + (size_t)kAC * HD * 2;     // [2][HD] half: new k, v
    static constexpr size_t raw_off = new_off + (size_t)2 * HD * 2;     // [kMaxRk + 2][HD] f32
    static constexpr size_t q_off = raw_off + (size_t)(kMaxRk + 2) * HD * 4;  // [kMaxRk][HD] f32
    static constexpr size_t s_off = q_off + (size_t)kMaxRk * HD * 4;    // [kMaxRk][kAC] f32
    static constexpr size_t st_off = s_off + (size_t)kMaxRk * kAC * 4;  // [kMaxRk][4] f32
    static constexpr size_t bytes = st_off + (size_t)kMaxRk * 4 * 4;
};

// Decode attention of one row, all (KV head, split) units of the launch dealt to CTAs in turn.
// Partials of q head qh, split sp: part[(qh * S + sp) * (HD + 2)] = running max, sum, then HD
// accumulators.
template <int HD>
__device__ void attn_op(const ChainArgs& A, const ChainOp& op, uint8_t* work, int* s_flag,
                        int warp, int lane) {
    using SM = AttnSmem<HD>;
    const AttnDecArgs& a = op.at;
    __half* sk = (__half*)(work + SM::k_off);
    __half* sv = (__half*)(work + SM::v_off);
    __half* snew = (__half*)(work + SM::new_off);
    float* sraw = (float*)(work + SM::raw_off);
    float* sq = (float*)(work + SM::q_off);
    float* ss = (float*)(work + SM::s_off);
    float* sst = (float*)(work + SM::st_off);  // per head: max, sum, correction
    const int rk = a.Hq / a.Hkv;
    const int S = op.splits;
    const int64_t pos = a.step->pos + a.pos_off;
    const int64_t nkv = pos + 1;
    const int64_t per = (nkv + S - 1) / S;
    const int nout = rk * HD;  // outputs of a unit: at most 2 per thread
    for (int u = blockIdx.x; u < a.Hkv * S; u += gridDim.x) {
        const int h = u / S, sp = u % S;
        const int64_t c0 = min((int64_t)sp * per, nkv), c1 = min(c0 + per, nkv);
        __half* kb = a.kc + (int64_t)h * a.ctx * HD;
        __half* vb = a.vc + (int64_t)h * a.ctx * HD;
        const bool has_new = c0 <= pos && pos < c1;
        __syncthreads();  // the previous unit is done with the shared memory
        // the group's q heads (and k, v of the new position) from the projection row
        for (int e = threadIdx.x; e < (rk + 2) * HD; e += kT) {
            const int i = e / HD, d = e % HD;
            int64_t off;
            if (i < rk) off = a.q_off + (int64_t)(h * rk + i) * HD;
            else if (i == rk) off = a.k_off + (int64_t)h * HD;
            else off = a.v_off + (int64_t)h * HD;
            if (i < rk || has_new) sraw[e] = __ldcg(a.qkv + off + d);
        }
        if (threadIdx.x < rk) {
            sst[threadIdx.x * 4 + 0] = -INFINITY;
            sst[threadIdx.x * 4 + 1] = 0.0f;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nout; e += kT) {
            const int i = e / HD, d = e % HD;
            const float v = rope_elem(sraw + i * HD, d, HD, a.tab, pos);
            sq[e] = __half2float(__float2half_rn(v));  // Q in fp16, as the CPU kernel
        }
        if (has_new) {
            for (int d = threadIdx.x; d < HD; d += kT) {
                const __half kn = __float2half_rn(rope_elem(sraw + rk * HD, d, HD, a.tab, pos));
                const __half vn = __float2half_rn(sraw[(rk + 1) * HD + d]);
                snew[d] = kn;
                snew[HD + d] = vn;
                kb[pos * HD + d] = kn;
                vb[pos * HD + d] = vn;
            }
        }
        float acc[2] = {0.0f, 0.0f};
        for (int64_t cs = c0; cs < c1; cs += kAC) {
            const int rows = (int)min((int64_t)kAC, c1 - cs);
            __syncthreads();  // the previous step's K, V and probabilities are consumed
            for (int e = threadIdx.x; e < rows * (HD / 8); e += kT) {
                const int rr = e / (HD / 8), pc = e % (HD / 8);
                if (cs + rr == pos) continue;  // the new row comes from snew
                cp_async16(sk + rr * HD + pc * 8, kb + (cs + rr) * HD + pc * 8);
                cp_async16(sv + rr * HD + pc * 8, vb + (cs + rr) * HD + pc * 8);
            }
            asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
            __syncthreads();
            // scores: a warp per position, lanes across head_dim
            for (int rr = warp; rr < rows; rr += kW) {
                const __half* kr = cs + rr == pos ? snew : sk + rr * HD;
                float kv[HD / 32];
#pragma unroll
                for (int j = 0; j < HD / 32; ++j) kv[j] = __half2float(kr[lane + 32 * j]);
                for (int i = 0; i < rk; ++i) {
                    float t = 0.0f;
#pragma unroll
                    for (int j = 0; j < HD / 32; ++j) t = __fmaf_rn(sq[i * HD + lane + 32 * j], kv[j], t);
                    t = warp_sum(t);
                    if (lane == 0) ss[i * kAC + rr] = __fmul_rn(t, a.scale);
                }
            }
            __syncthreads();
            // online softmax: warp i updates head i
            if (warp < rk) {
                const float sc = lane < rows ? ss[warp * kAC + lane] : -INFINITY;
                const float m_old = sst[warp * 4 + 0];
                const float m_new = fmaxf(m_old, warp_max(sc));
                const float corr = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
                const float pr = lane < rows ? expf(sc - m_new) : 0.0f;
                ss[warp * kAC + lane] = pr;
                const float l = warp_sum(pr);
                if (lane == 0) {
                    sst[warp * 4 + 0] = m_new;
                    sst[warp * 4 + 1] = sst[warp * 4 + 1] * corr + l;
                    sst[warp * 4 + 2] = corr;
                }
            }
            __syncthreads();
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                const int e = threadIdx.x + o * kT;
                if (e < nout) {
                    const int i = e / HD, d = e % HD;
                    float t = __fmul_rn(acc[o], sst[i * 4 + 2]);
                    for (int rr = 0; rr < rows; ++rr) {
                        const __half* vr = cs + rr == pos ? snew + HD : sv + rr * HD;
                        t = __fmaf_rn(ss[i * kAC + rr], __half2float(vr[d]), t);
                    }
                    acc[o] = t;
                }
            }
        }
        // this unit's partials
        float* pu = A.part + ((int64_t)(h * rk) * S + sp) * (HD + 2);
        const int64_t hstride = (int64_t)S * (HD + 2);  // next q head of the group
#pragma unroll
        for (int o = 0; o < 2; ++o) {
            const int e = threadIdx.x + o * kT;
            if (e < nout) pu[(e / HD) * hstride + 2 + e % HD] = acc[o];
        }
        if (threadIdx.x < rk) {
            pu[threadIdx.x * hstride + 0] = sst[threadIdx.x * 4 + 0];
            pu[threadIdx.x * hstride + 1] = sst[threadIdx.x * 4 + 1];
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned old = atomicAdd(&A.sync->attn_cnt[h], 1u);
            *s_flag = old == (unsigned)S - 1;
            if (*s_flag) atomicExch(&A.sync->attn_cnt[h], 0u);
        }
        __syncthreads();
        if (!*s_flag) continue;
        // the last unit of KV head h merges the splits of its q heads
        __threadfence();
#pragma unroll
        for (int o = 0; o < 2; ++o) {
            const int e = threadIdx.x + o * kT;
            if (e < nout) {  // warp-uniform: nout is a multiple of 32
                const int i = e / HD, d = e % HD;
                const int qh = h * rk + i;
                const float* base = A.part + (int64_t)qh * hstride;
                float M = -INFINITY;
                for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, __ldcg(base + s2 * (HD + 2)));
                float L = 0.0f, v = 0.0f;
                for (int s2 = 0; s2 < S; ++s2) {
                    const float m = __ldcg(base + s2 * (HD + 2));
                    const float w = m == -INFINITY ? 0.0f : expf(m - M);
                    L = __fmaf_rn(__ldcg(base + s2 * (HD + 2) + 1), w, L);
                    v = __fmaf_rn(__ldcg(base + s2 * (HD + 2) + 2 + d), w, v);
                }
                v = v * (L == 0.0f ? 0.0f : 1.0f / L);
                const int64_t oi = (int64_t)qh * HD + d;
                if (a.o) a.o[oi] = v;
                if (a.oq) {  // the warp holds one 32-element block of one head
                    float d16, q;
                    q8_block(v, lane, d16, q);
                    a.oq[oi] = (int8_t)__float2int_rn(q);
                    if (lane == 0) a.od[oi / 32] = d16;
                }
            }
        }
    }
}

// ------------------------------------------------------------------ CH_ROW (CTA 0)
__device__ void row_op(const ChainOp& op, uint8_t* work, double* shd) {
    if (blockIdx.x != 0) return;
    float* srow = (float*)work;
    const int64_t D = op.D;
    double s = 0.0;
    for (int64_t k = threadIdx.x; k < D; k += kT) {
        const float v = __ldcg(op.xf + k);
        srow[k] = v;
        s += (double)__fmul_rn(v, v);
    }
    float scale = 1.0f;
    if (op.rms) {
        const double tot = cta_sum_d(s, shd);
        const float mean = (float)(tot / (double)D);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, op.eps)));
    }
    __syncthreads();
    for (int64_t k = threadIdx.x; k < D; k += kT) {
        float t = srow[k];
        if (op.rms) t = __fmul_rn(t, scale);
        if (op.gamma) t = __fmul_rn(t, __ldg(op.gamma + k));
        srow[k] = t;
        if (op.y) op.y[k] = t;
    }
    __syncthreads();
    if (op.yq) {
        const int lane = threadIdx.x & 31;
        for (int64_t b = threadIdx.x >> 5; b < D / QK; b += kW) {
            float d16, q;
            q8_block(srow[b * QK + lane], lane, d16, q);
            op.yq[b * QK + lane] = (int8_t)__float2int_rn(q);
            if (lane == 0) op.yd[b] = d16;
        }
    }
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kT, 1) k_chain(ChainArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[kW][kMaxSlots];
    __shared__ Cursor curs[kW];
    __shared__ double shd[kW];
    __shared__ int s_flag, s_fail, s_dead;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        s_fail = 0;
        s_dead = chain_failed() ? 1 : 0;
    }
    __syncthreads();
    // a launch after a failed one does nothing: its barrier counters are not trusted
    if (s_dead) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && A.err) *(volatile int*)A.err = 1;
        return;
    }
    Ring r;
    r.base = smem + (size_t)warp * A.slots * kSlotBytes;
    r.bar = bars[warp];
    r.cur = &curs[warp];
    r.cs = r.cph = r.fs = r.inflight = 0;
    uint8_t* work = smem + (size_t)kW * A.slots * kSlotBytes;
    if (lane == 0) {
        r.cur->fop = -1;
        r.cur->fk = r.cur->nmine = 0;
        for (int s = 0; s < A.slots; ++s) mbar_init(&r.bar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        top_up(r, A, warp);
    }
    __syncwarp();
    bool ok = true;
    for (int j = 0; j < A.nops; ++j) {
        const ChainOp& op = A.ops[j];
        CHAIN_TRACE(j, 0);
        if (j > 0 && !grid_sync(A.sync, &s_flag)) {
            ok = false;
            break;
        }
        CHAIN_TRACE(j, 1);
        if (op.kind == CH_GEMV) {
            ok = op.wtype == T_Q4_0 ? gemv_op<T_Q4_0>(A, op, r, work, shd, &s_fail, warp, lane, j)
                                    : gemv_op<T_Q8_0>(A, op, r, work, shd, &s_fail, warp, lane, j);
            if (!ok) break;
        } else if (op.kind == CH_ATTN) {
            if (op.at.hd == 128) attn_op<128>(A, op, work, &s_flag, warp, lane);
            else attn_op<64>(A, op, work, &s_flag, warp, lane);
        } else {
            row_op(op, work, shd);
        }
    }
    CHAIN_TRACE(A.nops, 0);
    if (!ok) {
        if (threadIdx.x == 0) {
            atomicExch(&chain_error_word, 1);
            if (A.err) *(volatile int*)A.err = 1;
        }
        if (lane == 0) drain(r, A.slots);
        __syncwarp();
    }
}

size_t attn_smem(int hd) { return hd == 128 ? AttnSmem<128>::bytes : AttnSmem<64>::bytes; }

// shared memory one op needs beside the rings
size_t work_bytes(const ChainOp& op, int grid) {
    if (op.kind == CH_GEMV) {
        const int64_t nb = op.K / QK, cb = cblocks(op.wtype), nc = (nb + cb - 1) / cb;
        const int64_t units = op.swiglu ? op.F : op.N;
        const int64_t rows = ((units + grid - 1) / grid) * (op.swiglu ? 2 : 1);
        return (op.xf ? (size_t)nb * 40 : 0) + (nc > 1 ? (size_t)rows * nc * 4 : 0);
    }
    if (op.kind == CH_ATTN) return attn_smem(op.at.hd);
    return (size_t)op.D * 4;
}

}  // namespace

bool chain_gemv_ok(const GemvArgs& a) {
    if (a.M != 1 || (a.w.type != T_Q4_0 && a.w.type != T_Q8_0) || a.w.K % QK != 0) return false;
    const int64_t nb = a.w.K / QK, cb = cblocks(a.w.type);
    if ((nb + cb - 1) / cb > kW || a.w.N <= 0 || a.w.N >= (1LL << 30)) return false;
    if (((uintptr_t)a.w.qs & 15) != 0 || a.yq || a.yd) return false;
    if (a.swiglu ? (a.w.N != 2 * a.F || !a.y) : !a.y) return false;
    if (a.xf) {
        if (((uintptr_t)a.xf & 15) != 0 || (a.gamma && ((uintptr_t)a.gamma & 15) != 0)) return false;
    } else if (!a.xq || !a.xd || ((uintptr_t)a.xq & 15) != 0) {
        return false;
    }
    return true;
}

bool chain_attn_ok(const AttnDecArgs& a) {
    return a.rows == 1 && !a.batched && !a.pg.pages && a.step && (a.hd == 64 || a.hd == 128) &&
           a.Hkv > 0 &&
           a.Hkv <= kChainMaxKvHeads && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRk &&
           a.tab.n_dims <= a.hd && a.tab.n_dims % 2 == 0 && (a.o || (a.oq && a.od));
}

bool chain_gemv_op(const GemvArgs& a, ChainOp& c) {
    if (!chain_gemv_ok(a)) return false;
    c.kind = CH_GEMV;
    c.w = (const uint8_t*)a.w.qs;
    c.wtype = a.w.type;
    c.N = a.w.N;
    c.K = a.w.K;
    c.swiglu = a.swiglu ? 1 : 0;
    c.F = a.F;
    c.xq = a.xf ? nullptr : a.xq;
    c.xd = a.xf ? nullptr : a.xd;
    c.xf = a.xf;
    c.rms = a.xf && a.xf_rms ? 1 : 0;
    c.eps = a.eps;
    c.gamma = a.xf ? a.gamma : nullptr;
    c.y = a.y;
    c.bias = a.swiglu ? nullptr : a.bias;
    c.residual = a.swiglu ? nullptr : a.residual;
    return true;
}

bool chain_row_ok(int64_t M, int64_t D) { return M == 1 && D > 0 && D % QK == 0 && D <= 16384; }

int64_t chain_prepare(ChainOp* ops, int n, int dev) {
    const int grid = sm_count(dev);
    int64_t part = 0;
    for (int i = 0; i < n; ++i) {
        ChainOp& op = ops[i];
        if (op.kind == CH_GEMV) {
            op.rb = qrow_bytes(op.wtype, op.K);
        } else if (op.kind == CH_ATTN) {
            GB_CHECK(chain_attn_ok(op.at), "chain: attention op outside the chain's shapes");
            op.splits = std::max(1, std::min(kMaxSplits, grid / op.at.Hkv));
            part = std::max<int64_t>(part, (int64_t)op.at.Hq * op.splits * (op.at.hd + 2));
        }
    }
    return part;
}

void launch_chain(const ChainOp* ops, const ChainOp* host_ops, int n, ChainSync* sync, float* part,
                  int* err, cudaStream_t st) {
    if (n <= 0) return;
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "chain: device ordinal out of range");
    // dynamic shared memory the kernel may take on this device: the opt-in limit per block minus
    // the kernel's static shared memory (set once per device)
    static std::mutex mu;
    static size_t dyn_cap[64] = {};
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!dyn_cap[dev]) {
            int optin = 0;
            GB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
            cudaFuncAttributes fa;
            GB_CUDA(cudaFuncGetAttributes(&fa, k_chain));
            const size_t cap = (size_t)optin - fa.sharedSizeBytes;
            GB_CUDA(cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap));
            dyn_cap[dev] = cap;
        }
    }
    const int grid = sm_count(dev);
    size_t work = 0;
    for (int i = 0; i < n; ++i) work = std::max(work, work_bytes(host_ops[i], grid));
    work = (work + 127) / 128 * 128;
    GB_CHECK(work + 2 * (size_t)kW * kSlotBytes <= dyn_cap[dev], "chain: shared memory plan too large");
    const int slots = (int)std::min<size_t>(kMaxSlots, (dyn_cap[dev] - work) / ((size_t)kW * kSlotBytes));
    const size_t smem = (size_t)kW * slots * kSlotBytes + work;
    ChainArgs A;
    A.ops = ops;
    A.nops = n;
    A.slots = slots;
    A.sync = sync;
    A.part = part;
    A.err = err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GB_CUDA(cudaLaunchKernelEx(&cfg, k_chain, A));
}

#ifdef GB_CHAIN_TRACE
extern "C" int gb_chain_trace_read(unsigned long long* out, size_t bytes) {
    if (bytes < sizeof(g_chain_trace)) return -1;
    return cudaMemcpyFromSymbol(out, g_chain_trace, sizeof(g_chain_trace)) == cudaSuccess ? 0 : -1;
}
#endif

int chain_error() {
    int v = 0;
    GB_CUDA(cudaMemcpyFromSymbol(&v, chain_error_word, sizeof(int)));
    return v;
}

}  // namespace gb
