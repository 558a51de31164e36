// Decode and small-batch matmul (M <= 16 activation rows) on int8 tensor cores, over the
// split-row weight layout (kernels.h), with a bias / residual or SwiGLU (f32 and/or Q8_0 output)
// epilogue.
//
// Arithmetic.  Each 32-element block is one mma.sync m16n8k32 (16 weight rows x 8 activation rows,
// s8 x s8 -> exact s32), started from the 1.5*2^23 bias so the int -> float conversion is one
// subtraction.  Every output then accumulates fp32 block terms sumi * (d_w * d_x), the block
// formula of ggml_vec_dot_q4_0_q8_0 / ggml_vec_dot_q8_0_q8_0 (ggml-cpu/quants.c:225-256,
// :451-477).  Per output the terms are summed block by block within a warp's K range, then the
// K ranges in a fixed order, so a row's result does not depend on how many rows run with it (a
// sequence decodes to the same logits alone or inside a batch) nor on the grid size.
//
// Work mapping.  A CTA tile is 16 weight rows (plain) or 32 SwiGLU output pairs (gate rows
// p..p+31 and up rows F+p..F+p+31, four 16-row tiles).  Its K range is cut into steps of 8
// blocks {j0..j0+3, j0+32..j0+35} of one 64-block group, the blocks whose weight scales share one
// 16-byte word run of the scale region.  Plain tiles deal the steps to all 8 warps; SwiGLU tiles
// give each warp one 16-row tile and half of the steps.  The Q8_0 activations and their scales
// are staged once per CTA in shared memory, a phase of whole 64-block groups at a time (one
// phase covers K unless K is long and M large; then every tile restages its phases).  A warp
// streams only the weights and weight scales of its steps through its own cp.async ring (6 slots
// for Q4_0, 4 for Q8_0) and reads them back with ldmatrix / 32-bit shared loads; warps meet at
// phase boundaries and at the end of a tile, to add their partial sums in shared memory.  CTAs
// are persistent over tiles, so a warp's ring runs on into its next tile.
//
// Q4_0 nibbles become int8 with a shift and two bitwise ops: (q<<4) ^ 0x80 read as int8 is
// 16*(q-8); activation scales are divided by 16 (exact) to compensate.
//
// Launch: programmatic dependent launch.  The weights of the first ring slots are requested
// before griddepcontrol.wait; activations are read and outputs written after it.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kVW = 16;           // warps per CTA: two teams of kTW
constexpr int kTW = 8;            // warps per team (one tile at a time)
constexpr int kVT = kVW * 32;     // threads per CTA
constexpr int kTT = kTW * 32;     // threads per team
constexpr int kVSB = 8;           // blocks per step
constexpr size_t kVSmemMax = 227 * 1024;
constexpr int kActBytes = 72 * 1024;  // shared-memory budget of one activation phase

template <int WT>
struct WSlot {  // one ring slot: the weights of one step of one 16-row tile
    static constexpr int kQ = WT == T_Q8_0 ? 2 : 1;   // 16-byte chunks per block and weight row
    static constexpr int kW = kVSB * kQ * 16 * 16;     // [block][chunk][row 16][16 B]
    static constexpr int kWs = 16 * 16;                // [row 16][4 words of 2 fp16 scales]
    static constexpr int kBytes = kW + kWs;
    static constexpr int kDepth = WT == T_Q8_0 ? 2 : 3;  // ring slots per warp
};
__device__ __forceinline__ unsigned v_saddr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
// cp.async of 16 (or 4) bytes; zero fill when !valid (the source address stays in bounds)
__device__ __forceinline__ void v_cp16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(v_saddr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void v_cp4(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(v_saddr(dst)), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void v_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void v_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void v_ldsm4(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(v_saddr(p)));
}
__device__ __forceinline__ void v_mma(int (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0x4B400000));
}

// global block of local block lb (0..7) of step s
__device__ __forceinline__ int step_block(int s, int lb) {
    return 64 * (s >> 3) + 32 * (lb >> 2) + (s & 7) * 4 + (lb & 3);
}

// weights and weight scales of step s for the 16 rows starting at row0
template <int WT>
__device__ __forceinline__ void issue_w(uint8_t* slot, const uint8_t* qs, int64_t rb, int row0,
                                        int N, int nb, int s, int lane) {
    using S = WSlot<WT>;
    constexpr int Q = S::kQ;
#pragma unroll
    for (int it = 0; it < Q * 4; ++it) {
        const int c = it * 32 + lane;  // [row][chunk][half][block of 4]
        const int b4 = c & 3, h = (c >> 2) & 1, q = Q == 2 ? (c >> 3) & 1 : 0;
        const int r = Q == 2 ? c >> 4 : c >> 3;
        const int lb = h * 4 + b4;
        const int blk = step_block(s, lb);
        const int n = min(row0 + r, N - 1);
        const uint8_t* src = qs + (int64_t)n * rb + ((int64_t)q * nb + min(blk, nb - 1)) * 16;
        v_cp16(slot + ((lb * Q + q) * 16 + r) * 16, src, blk < nb);
    }
    if (lane < 16) {
        const int n = min(row0 + lane, N - 1);
        v_cp16(slot + S::kW + lane * 16,
               qs + (int64_t)n * rb + (int64_t)nb * quant_bytes(WT) + (s >> 3) * 128 + (s & 7) * 16,
               true);
    }
}

// staged activation rows: ldmatrix reads B fragments as 8-row matrices
template <int MAXM>
constexpr int stage_rows() { return MAXM < 8 ? 8 : MAXM; }

// Stage the Q8_0 activations of blocks [pbase, pbase + KC), rows 0..M-1, by the whole CTA, all by
// cp.async in one commit group per thread: sx [block][half][row SR][16 B] and sxs [block][row SR]
// fp32 scales.  Blocks past nb and scale rows M..SR-1 are zero filled; quant rows M..SR-1 are
// left as they are (their scales are zero, so they contribute exact zeros).
template <int MAXM>
__device__ __forceinline__ void stage_act(uint8_t* sx, float* sxs, const int8_t* xq,
                                          const float* xd, int M, int K, int nb, int pbase, int KC) {
    constexpr int SR = stage_rows<MAXM>();
    for (int e = threadIdx.x; e < KC * 2 * SR; e += kVT) {
        const int m = e % SR, hb = e / SR, half = hb & 1, pb = hb >> 1;
        if (m < M) {
            const int blk = pbase + pb;
            v_cp16(sx + (size_t)e * 16,
                   xq + (int64_t)m * K + (int64_t)min(blk, nb - 1) * 32 + half * 16, blk < nb);
        }
    }
    for (int e = threadIdx.x; e < KC * SR; e += kVT) {
        const int m = e % SR, blk = pbase + e / SR;
        const bool ok = m < M && blk < nb;
        v_cp4(sxs + e, xd + (ok ? (int64_t)m * nb + blk : 0), ok);
    }
    v_commit();
}

// wait until at most n of this thread's newest commit groups are pending (0 <= n <= 5)
__device__ __forceinline__ void v_wait_dyn(int n) {
    switch (n) {
        case 0: v_wait<0>(); break;
        case 1: v_wait<1>(); break;
        case 2: v_wait<2>(); break;
        case 3: v_wait<3>(); break;
        case 4: v_wait<4>(); break;
        default: v_wait<5>(); break;
    }
}

__device__ __forceinline__ void v_ldsm2(unsigned (&r)[2], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(v_saddr(p)));
}

// accumulate the 8 blocks of a landed step; pb0 = stage-local index of the step's first block
template <int WT, int MAXM>
__device__ __forceinline__ void consume(const uint8_t* slot, const uint8_t* sX, const float* sXs,
                                        int pb0, int lane, float2 (&acc)[(MAXM + 7) / 8][2]) {
    using S = WSlot<WT>;
    constexpr int NT = (MAXM + 7) / 8;
    constexpr int SR = stage_rows<MAXM>();
    const int g = lane >> 2, tg = lane & 3;
    const uint8_t* sW = slot;
    const float2 bias2 = make_float2(12582912.0f, 12582912.0f);
    // the 8 weight scales of rows g and g + 8 (fp16, block lb at half (lb & 3) * 2 + (lb >> 2))
    const uint4 ws0 = *(const uint4*)(slot + S::kW + g * 16);
    const uint4 ws1 = *(const uint4*)(slot + S::kW + (g + 8) * 16);
    const unsigned wa[4] = {ws0.x, ws0.y, ws0.z, ws0.w}, wb[4] = {ws1.x, ws1.y, ws1.z, ws1.w};
    // ldmatrix row address of this lane: matrix lane>>3, row lane&7
    const int lm = lane >> 3, lr = lane & 7;
    unsigned t[4] = {0, 0, 0, 0};
#pragma unroll
    for (int lb = 0; lb < kVSB; ++lb) {
        unsigned af[4];
        if (WT == T_Q8_0) {
            // matrices: (lo, rows 0-7), (lo, rows 8-15), (hi, rows 0-7), (hi, rows 8-15)
            v_ldsm4(af, sW + ((lb * 2 + (lm >> 1)) * 16 + (lm & 1) * 8 + lr) * 16);
        } else {
            // one ldmatrix brings blocks lb, lb+1: (lb, 0-7), (lb, 8-15), (lb+1, 0-7), (lb+1, 8-15)
            if ((lb & 1) == 0) v_ldsm4(t, sW + ((lb + (lm >> 1)) * 16 + (lm & 1) * 8 + lr) * 16);
            const unsigned w0 = t[(lb & 1) * 2], w1 = t[(lb & 1) * 2 + 1];
            af[0] = ((w0 << 4) & 0xF0F0F0F0u) ^ 0x80808080u;  // row g, k 4tg..: low nibbles
            af[1] = ((w1 << 4) & 0xF0F0F0F0u) ^ 0x80808080u;  // row g+8
            af[2] = (w0 & 0xF0F0F0F0u) ^ 0x80808080u;         // row g, k 16+4tg..: high nibbles
            af[3] = (w1 & 0xF0F0F0F0u) ^ 0x80808080u;
        }
        const int hw = (lb & 3) * 2 + (lb >> 2);
        const unsigned sh = (hw & 1) * 16;
        const float dw0 = __half2float(__ushort_as_half((unsigned short)(wa[hw >> 1] >> sh)));
        const float dw1 = __half2float(__ushort_as_half((unsigned short)(wb[hw >> 1] >> sh)));
        const int pb = pb0 + 32 * (lb >> 2) + (lb & 3);
        // B fragments: matrices (half 0, rows 0-7), (half 1, rows 0-7), (half 0, rows 8-15), ...
        unsigned bq[2 * NT];
        const uint8_t* brow = sX + ((pb * 2 + (lm & 1)) * SR + (lm >> 1) * 8 + lr) * 16;
        if (NT == 2) {
            unsigned r4[4];
            v_ldsm4(r4, brow);
#pragma unroll
            for (int i = 0; i < 2 * NT; ++i) bq[i] = r4[i];
        } else {
            unsigned r2[2];
            v_ldsm2(r2, sX + ((pb * 2 + (lm & 1)) * SR + lr) * 16);
            bq[0] = r2[0];
            bq[1] = r2[1];
        }
        (void)brow;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            int d[4];
            v_mma(d, af, bq[2 * nt], bq[2 * nt + 1]);
            float2 dx = *(const float2*)(sXs + pb * SR + nt * 8 + 2 * tg);
            if (WT == T_Q4_0) dx = mul2(dx, make_float2(0.0625f, 0.0625f));  // 16 * (q - 8)
            const float2 p0 = mul2(make_float2(dw0, dw0), dx);
            const float2 p1 = mul2(make_float2(dw1, dw1), dx);
            const float2 v0 = sub2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), bias2);
            const float2 v1 = sub2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), bias2);
            acc[nt][0] = fma2(v0, p0, acc[nt][0]);
            acc[nt][1] = fma2(v1, p1, acc[nt][1]);
        }
    }
}

// Work order.  A CTA's tiles are blockIdx.x + i * gridDim.x; its two teams of 8 warps take the
// even and the odd i, so two tiles run at once over one activation stage.  Per team: its tiles in
// chunks of TM; per chunk, the activation phases (shared by the CTA); per phase, each tile of the
// chunk; per tile, this warp's steps of the phase (s = ph * sp + kw + KW * j).  Accumulators of
// the whole chunk stay in registers across phases, so each tile still sums its steps in
// ascending order.  The weight issue cursor walks the same order D - 1 steps ahead.
struct VCursor {
    int c, ph, tt, s;  // chunk (first team-local tile index), phase, tile in chunk, step
};

template <int WT, int MAXM, int SWI>
__global__ void __launch_bounds__(kVT, 1) k_mmv(GemvArgs a, int ns, int ntiles, int KC, int nphase) {
    using S = WSlot<WT>;
    constexpr int D = S::kDepth;
    constexpr int NT = (MAXM + 7) / 8;
    constexpr int SR = stage_rows<MAXM>();
    constexpr int KW = SWI ? 2 : 8;   // K ranges per tile
    constexpr int MT = SWI ? 4 : 1;   // 16-row tiles per CTA tile
    constexpr int RC = 8 * NT;        // partial-sum columns
    constexpr int KS = 8 / KW;        // partial sums held per warp
    constexpr int TM = SWI ? 1 : 4;   // tiles per chunk
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int team = warp / kTW, wt = warp % kTW, ttid = tid % kTT;
    const int g = lane >> 2, tg = lane & 3;
    const int kw = SWI ? wt >> 2 : wt;
    const int mt = SWI ? wt & 3 : 0;
    const int nbuf = nphase > 1 ? 2 : 1;
    const size_t stage_bytes = (size_t)KC * SR * 36;
    uint8_t* ring = smem + nbuf * stage_bytes + warp * D * S::kBytes;
    float* red = (float*)(smem + nbuf * stage_bytes + kVW * D * S::kBytes) + team * 1024 * NT;
    auto sx_of = [&](int b) { return smem + b * stage_bytes; };
    auto sxs_of = [&](int b) { return (float*)(smem + b * stage_bytes + (size_t)KC * 2 * SR * 16); };
    const int N = (int)a.w.N, K = (int)a.w.K, nb = K / QK, M = a.M;
    const int F = (int)a.F;
    const int64_t rb = qrow_bytes(WT, K);
    const uint8_t* qs = (const uint8_t*)a.w.qs;
    const int sp = KC / 8;                             // steps per phase
    const int ntc = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int ntt0 = (ntc + 1) / 2;                    // tiles of team 0 (team 1 has ntc / 2)
    const int ntt = team == 0 ? ntt0 : ntc / 2;
    const int tmc = nphase > 1 ? TM : 1;               // tiles per chunk at run time
    auto tile_of = [&](int j) { return (int)blockIdx.x + (2 * j + team) * (int)gridDim.x; };
    auto row0 = [&](int tile) {
        return SWI ? (mt < 2 ? 0 : F) + tile * 32 + (mt & 1) * 16 : tile * 16;
    };
    auto s_end = [&](int ph) { return min(ns, (ph + 1) * sp); };
    // move a cursor to the next (tile, step) of this warp; c >= ntt once the work is done
    auto advance = [&](VCursor& u) {
        u.s += KW;
        while (u.c < ntt && u.s >= s_end(u.ph)) {
            if (++u.tt >= min(tmc, ntt - u.c)) {
                u.tt = 0;
                if (++u.ph >= nphase) {
                    u.ph = 0;
                    u.c += tmc;
                }
            }
            u.s = u.ph * sp + kw;
        }
    };
    VCursor iu{0, 0, 0, kw - KW};
    advance(iu);  // first step of this warp (none if kw >= ns or the team has no tile)
    int islot = 0;
#pragma unroll
    for (int d = 0; d < D - 1; ++d) {
        if (iu.c < ntt)
            issue_w<WT>(ring + d * S::kBytes, qs, rb, row0(tile_of(iu.c + iu.tt)), N, nb, iu.s, lane);
        v_commit();
        if (iu.c < ntt) advance(iu);
    }
    islot = D - 1;
    int cslot = 0;
    pdl_wait();
    pdl_launch();
    // the first phase, then (several phases) the next one ahead of use
    stage_act<MAXM>(sx_of(0), sxs_of(0), a.xq, a.xd, M, K, nb, 0, KC);
    v_wait<0>();
    __syncthreads();
    int q = 0;  // phases started so far (over all chunks); phase q uses buffer q & 1
    const int nq = nphase > 1 ? ((ntt0 + tmc - 1) / tmc) * nphase : 1;

    // chunks follow team 0 (it has at least as many tiles as team 1); both teams meet at every
    // phase boundary and tile epilogue
    for (int c = 0; c < ntt0; c += tmc) {
        const int nt_c = max(0, min(tmc, ntt - c));    // this team's tiles in the chunk
        const int nt_max = min(tmc, ntt0 - c);
        float2 acc[TM][KS][NT][2];
#pragma unroll
        for (int u = 0; u < TM; ++u)
#pragma unroll
            for (int i = 0; i < KS; ++i)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    acc[u][i][nt][0] = acc[u][i][nt][1] = make_float2(0.0f, 0.0f);
        for (int ph = 0; ph < nphase; ++ph, ++q) {
            const int buf = nphase > 1 ? (q & 1) : 0;
            int after = 0;  // commit groups of this thread since the next phase's stage
            if (nphase > 1) {
                if (q > 0) __syncthreads();  // phase q - 1 done: its buffer takes phase q + 1
                if (q + 1 < nq) {
                    const int nph = (ph + 1) % nphase;
                    stage_act<MAXM>(sx_of(buf ^ 1), sxs_of(buf ^ 1), a.xq, a.xd, M, K, nb,
                                    nph * KC, KC);
                }
            }
            const uint8_t* sX = sx_of(buf);
            const float* sXs = sxs_of(buf);
            for (int u = 0; u < nt_c; ++u) {
                for (int s = ph * sp + kw; s < s_end(ph); s += KW) {
                    v_wait<D - 2>();
                    __syncwarp();
                    // refill the slot the previous step consumed
                    if (iu.c < ntt) {
                        issue_w<WT>(ring + islot * S::kBytes, qs, rb, row0(tile_of(iu.c + iu.tt)),
                                    N, nb, iu.s, lane);
                        advance(iu);
                    }
                    v_commit();
                    ++after;
                    islot = islot + 1 == D ? 0 : islot + 1;
                    const int i = ((s - kw) / KW) % KS;
                    const int pb0 = 64 * (s >> 3) + (s & 7) * 4 - ph * KC;
#pragma unroll
                    for (int uu = 0; uu < TM; ++uu)
#pragma unroll
                        for (int j = 0; j < KS; ++j)
                            if (uu == u && j == i)
                                consume<WT, MAXM>(ring + cslot * S::kBytes, sX, sXs, pb0, lane,
                                                  acc[uu][j]);
                    cslot = cslot + 1 == D ? 0 : cslot + 1;
                }
            }
            // the next phase's stage has landed once D - 1 groups followed it; else wait for it
            if (nphase > 1 && after < D - 1) v_wait_dyn(after);
        }
#pragma unroll
        for (int u = 0; u < TM; ++u) {
            if (u >= nt_max) break;
            const bool mine = u < nt_c;  // this team has a tile at this position
            const int tile = mine ? tile_of(c + u) : 0;
            // SwiGLU warps fold their four partials: ((P_kw + P_kw+2) + P_kw+4) + P_kw+6
#pragma unroll
            for (int i = 1; i < KS; ++i)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[u][0][nt][0] = add2(acc[u][0][nt][0], acc[u][i][nt][0]);
                    acc[u][0][nt][1] = add2(acc[u][0][nt][1], acc[u][i][nt][1]);
                }
            if (mine) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float* r0 = red + (kw * MT * 16 + mt * 16 + g) * RC + nt * 8 + 2 * tg;
                    *(float2*)r0 = acc[u][0][nt][0];
                    *(float2*)(r0 + 8 * RC) = acc[u][0][nt][1];
                }
            }
            __syncthreads();
            if (mine && !SWI) {
                for (int t = ttid; t < 16 * M; t += kTT) {
                    const int r = t & 15, cc = t >> 4;
                    auto P = [&](int w) { return red[(w * 16 + r) * RC + cc]; };
                    // (((P0 + P2) + P4) + P6) + (((P1 + P3) + P5) + P7)
                    const float ev = __fadd_rn(__fadd_rn(__fadd_rn(P(0), P(2)), P(4)), P(6));
                    const float od = __fadd_rn(__fadd_rn(__fadd_rn(P(1), P(3)), P(5)), P(7));
                    float v = __fadd_rn(ev, od);
                    const int n = tile * 16 + r;
                    if (n < N) {
                        if (a.bias) v = __fadd_rn(v, a.bias[n]);
                        if (a.residual) v = __fadd_rn(a.residual[(int64_t)cc * a.res_stride + n], v);
                        a.y[(int64_t)cc * a.y_stride + n] = v;
                    }
                }
            } else if (mine) {
                // ggml_vec_swiglu_f32 (vec.cpp:417-426) on the tile's 32 pairs, f32 and/or Q8_0
                for (int t = ttid; t < 32 * M; t += kTT) {  // one warp per activation row
                    const int p = t & 31, cc = t >> 5;
                    const float gs = __fadd_rn(red[p * RC + cc], red[(64 + p) * RC + cc]);
                    const float us = __fadd_rn(red[(32 + p) * RC + cc], red[(96 + p) * RC + cc]);
                    const float h = __fmul_rn(ref_v_silu(gs), us);
                    const int64_t col = (int64_t)tile * 32 + p;
                    if (a.y) a.y[(int64_t)cc * a.y_stride + col] = h;
                    if (a.yq) {
                        float d16, qv;
                        q8_block(h, p, d16, qv);
                        a.yq[(int64_t)cc * a.F + col] = (int8_t)__float2int_rn(qv);
                        if (p == 0) a.yd[(int64_t)cc * (a.F / 32) + tile] = d16;
                    }
                }
            }
            __syncthreads();
        }
    }
    v_wait<0>();
}

template <int WT, int MAXM>
constexpr size_t v_fixed_smem() {  // rings and the two teams' partial sums
    return (size_t)kVW * WSlot<WT>::kDepth * WSlot<WT>::kBytes +
           (size_t)2 * 1024 * ((MAXM + 7) / 8) * 4;
}

template <int WT, int MAXM, int SWI>
void launch_v(const GemvArgs& a, cudaStream_t st) {
    auto kern = k_mmv<WT, MAXM, SWI>;
    constexpr int SR = stage_rows<MAXM>();
    // one phase when K fits the activation budget; else two buffers of whole 64-block groups
    constexpr int kOne = 64 * (kActBytes / (SR * 64 * 36));
    constexpr int kTwo = 64 * std::max(kActBytes / 2 / (SR * 64 * 36), 1);
    static_assert(kOne >= 64, "mmv: one 64-block group must fit the activation budget");
    constexpr size_t smem_max = (size_t)std::max(kOne, 2 * kTwo) * SR * 36 + v_fixed_smem<WT, MAXM>();
    static_assert(smem_max <= kVSmemMax, "mmv: stage and rings do not fit in shared memory");
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "mmv: device ordinal out of range");
    const int nb = (int)(a.w.K / QK);
    const int ng = (nb + 63) / 64;
    const int rem = nb - 64 * (ng - 1);
    const int ns = 8 * (ng - 1) + (std::min(rem, 32) + 3) / 4;
    const bool one = 64 * ng <= kOne;
    const int KC = one ? 64 * ng : kTwo;
    const int nphase = one ? 1 : (64 * ng + KC - 1) / KC;
    const size_t smem = (size_t)(one ? 1 : 2) * KC * SR * 36 + v_fixed_smem<WT, MAXM>();
    static std::mutex mu;
    static bool configured[64] = {};
    static int per_sm[64][kOne / 64 + 2] = {};  // [device][stage size]: resident CTAs per SM
    const int key = one ? KC / 64 : kOne / 64 + 1;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_max));
            configured[dev] = true;
        }
        if (!per_sm[dev][key]) {
            int n = 0;
            GB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kVT, smem));
            per_sm[dev][key] = std::max(n, 1);
        }
    }
    const int ntiles = SWI ? (int)(a.F / 32) : (int)((a.w.N + 15) / 16);
    if (ntiles == 0) return;
    const int grid = (int)std::min<int64_t>(ntiles, (int64_t)sm_count(dev) * per_sm[dev][key]);
    launch_pdl(kern, (unsigned)grid, kVT, smem, st, a, ns, ntiles, KC, nphase);
}

template <int WT, int SWI>
void launch_vm(const GemvArgs& a, cudaStream_t st) {
    if (a.M == 1) launch_v<WT, 1, SWI>(a, st);
    else if (a.M == 2) launch_v<WT, 2, SWI>(a, st);
    else if (a.M <= 4) launch_v<WT, 4, SWI>(a, st);
    else if (a.M <= 8) launch_v<WT, 8, SWI>(a, st);
    else launch_v<WT, 16, SWI>(a, st);
}

}  // namespace

void launch_mmv(const GemvArgs& a, cudaStream_t st) {
    GB_CHECK(a.w.type == T_Q8_0 || a.w.type == T_Q4_0, "mmv: quantized weights required");
    GB_CHECK(a.w.K % QK == 0 && a.w.K < (1LL << 30) && a.w.N < (1LL << 30), "mmv: bad shape");
    GB_CHECK(a.M >= 1 && a.M <= kMmvMaxRows, "mmv: 1..16 activation rows");
    GB_CHECK(a.xq && a.xd && !a.xf, "mmv: Q8_0 input required");
    GB_CHECK(((uintptr_t)a.xq & 15) == 0, "mmv: xq must be 16-byte aligned");
    GB_CHECK(!a.swiglu || (a.w.N == 2 * a.F && a.F % 32 == 0),
             "mmv: SwiGLU needs N == 2F, F % 32 == 0");
    GB_CHECK(a.swiglu || (!a.yq && !a.yd), "mmv: Q8_0 output only with SwiGLU");
    GB_CHECK(a.swiglu ? (a.y || a.yq) : a.y != nullptr, "mmv: no output");
    GB_CHECK(!a.yq == !a.yd, "mmv: Q8_0 output needs quants and scales");
    if (a.w.N == 0) return;
    if (a.w.type == T_Q8_0) {
        if (a.swiglu) launch_vm<T_Q8_0, 1>(a, st);
        else launch_vm<T_Q8_0, 0>(a, st);
    } else {
        if (a.swiglu) launch_vm<T_Q4_0, 1>(a, st);
        else launch_vm<T_Q4_0, 0>(a, st);
    }
}

}  // namespace gb
