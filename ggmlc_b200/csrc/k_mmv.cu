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

constexpr int kVW = 8;            // warps per CTA
constexpr int kVT = kVW * 32;     // threads per CTA
constexpr int kVSB = 8;           // blocks per step
constexpr size_t kVSmemMax = 227 * 1024;
constexpr int kActBytes = 72 * 1024;  // shared-memory budget of one activation phase

template <int WT>
struct WSlot {  // one ring slot: the weights of one step of one 16-row tile
    static constexpr int kQ = WT == T_Q8_0 ? 2 : 1;   // 16-byte chunks per block and weight row
    static constexpr int kW = kVSB * kQ * 16 * 16;     // [block][chunk][row 16][16 B]
    static constexpr int kWs = 16 * 16;                // [row 16][4 words of 2 fp16 scales]
    static constexpr int kBytes = kW + kWs;
    static constexpr int kDepth = WT == T_Q8_0 ? 4 : 6;  // ring slots per warp
};
// blocks of one activation phase: whole 64-block groups within the budget
template <int MAXM>
constexpr int phase_blocks_max() {
    return 64 * ((kActBytes / (MAXM * 64 * 36)) > 0 ? (kActBytes / (MAXM * 64 * 36)) : 1);
}

__device__ __forceinline__ unsigned v_saddr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
// cp.async of 16 bytes; zero fill when !valid (the source address stays in bounds)
__device__ __forceinline__ void v_cp16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(v_saddr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
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

// Q8_0 activations and scales of blocks [pbase, pbase + KC) of rows 0..M-1, by the whole CTA:
// sx [block][half][m][16 B], sxs [m][block]; blocks past nb are zero.  Rows run fastest so the
// 16-byte shared stores of a warp are contiguous.
template <int MAXM>
__device__ __forceinline__ void stage_act(uint8_t* sx, float* sxs, const int8_t* xq,
                                          const float* xd, int M, int K, int nb, int pbase, int KC) {
    for (int e = threadIdx.x; e < M * KC * 2; e += kVT) {
        const int m = e % M, rest = e / M, half = rest & 1, pb = rest >> 1;
        const int blk = pbase + pb;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (blk < nb) v = __ldcg((const uint4*)(xq + (int64_t)m * K + (int64_t)blk * 32 + half * 16));
        *(uint4*)(sx + ((pb * 2 + half) * MAXM + m) * 16) = v;
    }
    for (int e = threadIdx.x; e < M * KC; e += kVT) {
        const int m = e / KC, pb = e % KC;
        const int blk = pbase + pb;
        sxs[m * KC + pb] = blk < nb ? __ldcg(xd + (int64_t)m * nb + blk) : 0.0f;
    }
}

// accumulate the 8 blocks of a landed step; pb0 = phase-local index of the step's first block
template <int WT, int MAXM>
__device__ __forceinline__ void consume(const uint8_t* slot, const uint8_t* sX, const float* sXs,
                                        int KC, int pb0, int M, int lane,
                                        float2 (&acc)[(MAXM + 7) / 8][2]) {
    using S = WSlot<WT>;
    constexpr int NT = (MAXM + 7) / 8;
    const int g = lane >> 2, tg = lane & 3;
    const uint8_t* sW = slot;
    const uint8_t* sWs = slot + S::kW;
    const float xsc = WT == T_Q4_0 ? 0.0625f : 1.0f;  // Q4_0 fragments hold 16 * (q - 8)
    const float2 bias2 = make_float2(12582912.0f, 12582912.0f);
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
        const int so = (lb & 3) * 4 + (lb >> 2) * 2;
        const float dw0 = __half2float(*(const __half*)(sWs + g * 16 + so));
        const float dw1 = __half2float(*(const __half*)(sWs + (g + 8) * 16 + so));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int pb = pb0 + 32 * (lb >> 2) + (lb & 3);
            const int cb = nt * 8 + g;  // activation row feeding this lane's B fragment
            unsigned b0 = 0, b1 = 0;
            if (MAXM == 1 ? g == 0 : cb < M) {
                b0 = *(const unsigned*)(sX + ((pb * 2) * MAXM + cb) * 16 + tg * 4);
                b1 = *(const unsigned*)(sX + ((pb * 2 + 1) * MAXM + cb) * 16 + tg * 4);
            }
            int d[4];
            v_mma(d, af, b0, b1);
            const int c0 = nt * 8 + 2 * tg;
            const float dx0 = c0 < M ? __fmul_rn(sXs[c0 * KC + pb], xsc) : 0.0f;
            const float dx1 = c0 + 1 < M ? __fmul_rn(sXs[(c0 + 1) * KC + pb], xsc) : 0.0f;
            const float2 p0 = make_float2(__fmul_rn(dw0, dx0), __fmul_rn(dw0, dx1));
            const float2 p1 = make_float2(__fmul_rn(dw1, dx0), __fmul_rn(dw1, dx1));
            const float2 v0 = sub2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), bias2);
            const float2 v1 = sub2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), bias2);
            acc[nt][0] = fma2(v0, p0, acc[nt][0]);
            acc[nt][1] = fma2(v1, p1, acc[nt][1]);
        }
    }
}

template <int WT, int MAXM, int SWI>
__global__ void __launch_bounds__(kVT, 1) k_mmv(GemvArgs a, int ns, int ntiles, int KC) {
    using S = WSlot<WT>;
    constexpr int D = S::kDepth;
    constexpr int NT = (MAXM + 7) / 8;
    constexpr int KW = SWI ? 2 : 8;   // K ranges per tile
    constexpr int MT = SWI ? 4 : 1;   // 16-row tiles per CTA tile
    constexpr int RC = 8 * NT;        // partial-sum columns
    constexpr int KS = 8 / KW;        // partial sums held per warp
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int kw = SWI ? warp >> 2 : warp;
    const int mt = SWI ? warp & 3 : 0;
    uint8_t* sx = smem;                                             // activation phase
    float* sxs = (float*)(sx + (size_t)KC * 2 * MAXM * 16);
    uint8_t* ring = (uint8_t*)(sxs + (size_t)MAXM * KC) + warp * D * S::kBytes;
    float* red = (float*)((uint8_t*)(sxs + (size_t)MAXM * KC) + kVW * D * S::kBytes);
    const int N = (int)a.w.N, K = (int)a.w.K, nb = K / QK, M = a.M;
    const int F = (int)a.F;
    const int64_t rb = qrow_bytes(WT, K);
    const uint8_t* qs = (const uint8_t*)a.w.qs;
    const int sp = KC / 8;                     // steps per phase
    const int nphase = (ns + sp - 1) / sp;
    auto row0 = [&](int tile) {
        return SWI ? (mt < 2 ? 0 : F) + tile * 32 + (mt & 1) * 16 : tile * 16;
    };
    const bool active = kw < ns;  // a warp with no step in a tile only adds zeros
    // issue cursor over this warp's (tile, step) sequence: weights only
    int it = blockIdx.x, is = kw, islot = 0;
    auto advance = [&](int& t, int& s) {
        s += KW;
        if (s >= ns) {
            s = kw;
            t += gridDim.x;
        }
    };
#pragma unroll
    for (int d = 0; d < D - 1; ++d) {
        if (active && it < ntiles) issue_w<WT>(ring + d * S::kBytes, qs, rb, row0(it), N, nb, is, lane);
        v_commit();
        advance(it, is);
    }
    islot = D - 1;
    int cslot = 0;
    pdl_wait();
    pdl_launch();
    if (nphase == 1) {  // one phase: staged once for every tile
        stage_act<MAXM>(sx, sxs, a.xq, a.xd, M, K, nb, 0, KC);
        __syncthreads();
    }

    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        // acc[i] sums the steps s == kw + KW*i (mod 8): every output is built from the same eight
        // partial sums P_r (steps s == r mod 8) in plain and SwiGLU mode
        float2 acc[KS][NT][2];
#pragma unroll
        for (int i = 0; i < KS; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[i][nt][0] = acc[i][nt][1] = make_float2(0.0f, 0.0f);
        for (int ph = 0; ph < nphase; ++ph) {
            if (nphase > 1) {  // every warp is done with the previous phase's activations
                __syncthreads();
                stage_act<MAXM>(sx, sxs, a.xq, a.xd, M, K, nb, ph * KC, KC);
                __syncthreads();
            }
            const int s_end = min(ns, (ph + 1) * sp);
            int s = ph * sp + ((kw - ph * sp) % KW + KW) % KW;  // this warp's first step here
            for (; active && s < s_end; s += KW) {
                v_wait<D - 2>();
                __syncwarp();
                // refill the slot the previous step consumed
                if (it < ntiles) {
                    issue_w<WT>(ring + islot * S::kBytes, qs, rb, row0(it), N, nb, is, lane);
                    advance(it, is);
                }
                v_commit();
                islot = islot + 1 == D ? 0 : islot + 1;
                const int i = ((s - kw) / KW) % KS;
                const int pb0 = 64 * (s >> 3) + (s & 7) * 4 - ph * KC;
#pragma unroll
                for (int j = 0; j < KS; ++j)
                    if (j == i)
                        consume<WT, MAXM>(ring + cslot * S::kBytes, sx, sxs, KC, pb0, M, lane, acc[j]);
                cslot = cslot + 1 == D ? 0 : cslot + 1;
            }
        }
        // SwiGLU warps fold their four partials: ((P_kw + P_kw+2) + P_kw+4) + P_kw+6
#pragma unroll
        for (int i = 1; i < KS; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[0][nt][0] = add2(acc[0][nt][0], acc[i][nt][0]);
                acc[0][nt][1] = add2(acc[0][nt][1], acc[i][nt][1]);
            }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float* r0 = red + (kw * MT * 16 + mt * 16 + g) * RC + nt * 8 + 2 * tg;
            *(float2*)r0 = acc[0][nt][0];
            *(float2*)(r0 + 8 * RC) = acc[0][nt][1];
        }
        __syncthreads();
        if (!SWI) {
            for (int t = tid; t < 16 * M; t += kVT) {
                const int r = t & 15, c = t >> 4;
                auto P = [&](int w) { return red[(w * 16 + r) * RC + c]; };
                // (((P0 + P2) + P4) + P6) + (((P1 + P3) + P5) + P7)
                const float ev = __fadd_rn(__fadd_rn(__fadd_rn(P(0), P(2)), P(4)), P(6));
                const float od = __fadd_rn(__fadd_rn(__fadd_rn(P(1), P(3)), P(5)), P(7));
                float v = __fadd_rn(ev, od);
                const int n = tile * 16 + r;
                if (n < N) {
                    if (a.bias) v = __fadd_rn(v, a.bias[n]);
                    if (a.residual) v = __fadd_rn(a.residual[(int64_t)c * a.res_stride + n], v);
                    a.y[(int64_t)c * a.y_stride + n] = v;
                }
            }
        } else {
            // ggml_vec_swiglu_f32 (vec.cpp:417-426) on the tile's 32 pairs, f32 and/or Q8_0
            for (int t = tid; t < 32 * M; t += kVT) {  // one warp per activation row
                const int p = t & 31, c = t >> 5;
                const float gs = __fadd_rn(red[p * RC + c], red[(64 + p) * RC + c]);
                const float us = __fadd_rn(red[(32 + p) * RC + c], red[(96 + p) * RC + c]);
                const float h = __fmul_rn(ref_v_silu(gs), us);
                const int64_t col = (int64_t)tile * 32 + p;
                if (a.y) a.y[(int64_t)c * a.y_stride + col] = h;
                if (a.yq) {
                    float d16, q;
                    q8_block(h, p, d16, q);
                    a.yq[(int64_t)c * a.F + col] = (int8_t)__float2int_rn(q);
                    if (p == 0) a.yd[(int64_t)c * (a.F / 32) + tile] = d16;
                }
            }
        }
        __syncthreads();
    }
    v_wait<0>();
}

template <int WT, int MAXM>
constexpr size_t v_fixed_smem() {  // rings and partial sums
    return (size_t)kVW * WSlot<WT>::kDepth * WSlot<WT>::kBytes + (size_t)1024 * ((MAXM + 7) / 8) * 4;
}

template <int WT, int MAXM, int SWI>
void launch_v(const GemvArgs& a, cudaStream_t st) {
    auto kern = k_mmv<WT, MAXM, SWI>;
    constexpr int kPhaseMax = phase_blocks_max<MAXM>();
    constexpr size_t smem_max = (size_t)kPhaseMax * MAXM * 36 + v_fixed_smem<WT, MAXM>();
    static_assert(smem_max <= kVSmemMax, "mmv: stage and rings do not fit in shared memory");
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "mmv: device ordinal out of range");
    const int nb = (int)(a.w.K / QK);
    const int ng = (nb + 63) / 64;
    const int rem = nb - 64 * (ng - 1);
    const int ns = 8 * (ng - 1) + (std::min(rem, 32) + 3) / 4;
    const int KC = std::min(64 * ng, kPhaseMax);
    const size_t smem = (size_t)KC * MAXM * 36 + v_fixed_smem<WT, MAXM>();
    static std::mutex mu;
    static bool configured[64] = {};
    static int per_sm[64][kPhaseMax / 64 + 1] = {};  // [device][KC / 64]: resident CTAs per SM
    const int key = KC / 64;
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
    launch_pdl(kern, (unsigned)grid, kVT, smem, st, a, ns, ntiles, KC);
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
