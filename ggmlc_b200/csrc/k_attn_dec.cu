// Fused attention-side kernels over the F16 KV cache.
//
// k_rope_qkv (any s): RoPE of q and k read straight from the QKV projection output, rotated q to
//   an f32 buffer, rotated k and v rows to the F16 cache at rows pos..pos+s-1 (the reference's
//   ROPE x2 + SET_ROWS x2, executor.cpp:2132-2184, in one launch).
// k_attn_decode (s == 1): split-KV flash decoding.  grid = (splits, Hkv); each CTA rotates the q
//   heads of its GQA group itself, the CTA whose range holds the new position also rotates the
//   new k and writes k, v into the cache, then the CTA walks its positions in chunks of 64: the
//   chunk's K and V rows are staged in shared memory with cp.async (one memory round trip per
//   chunk), scores come from one warp per position (lanes across head_dim), and an online
//   softmax rescales the per-thread V accumulators.  Partials (m, l, acc) go to a workspace.
// k_attn_combine: merges the splits of each head (all splits read in parallel) and writes the
//   head's output as f32 and/or as Q8_0 blocks for the output projection (head_dim % 32 == 0,
//   so blocks never straddle heads).
//
// RoPE arithmetic is the reference's (ops.cpp:5910-5923, 5998-6015) with the host cos/sin table;
// attention accumulates in fp32 (the CPU rounds its V accumulator to fp16 per position).
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.h"
#include "kernels.h"
#include "krope.cuh"
#include "kutil.cuh"

namespace gb {

namespace {

__global__ void k_rope_qkv(QkvRopeArgs a) {
    const int hd = a.hd;
    const int64_t base = (a.step ? a.step->pos : 0) + a.pos_off;
    const int64_t heads = (int64_t)a.Hq + 2 * a.Hkv;
    const int64_t total = (int64_t)a.s * heads * hd;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(idx % hd);
        const int64_t hh = (idx / hd) % heads;
        const int64_t t = idx / (hd * heads);
        const float* row = a.qkv + t * a.qkv_stride;
        const int64_t p = base + t;
        if (hh < a.Hq) {
            const float* src = row + a.q_off + hh * hd;
            a.q_out[(t * a.Hq + hh) * hd + d] = rope_elem(src, d, hd, a.tab, p);
        } else if (hh < a.Hq + a.Hkv) {
            const int64_t h = hh - a.Hq;
            const float* src = row + a.k_off + h * hd;
            a.kc[kv_row_off(a.pages, a.page_shift, a.Hkv, a.ctx, h, p, hd) + d] =
                __float2half_rn(rope_elem(src, d, hd, a.tab, p));
        } else {
            const int64_t h = hh - a.Hq - a.Hkv;
            a.vc[kv_row_off(a.pages, a.page_shift, a.Hkv, a.ctx, h, p, hd) + d] =
                __float2half_rn(row[a.v_off + h * hd + d]);
        }
    }
}

constexpr int kDecThreads = 128;
constexpr int kMaxRk = 8;     // q heads per KV head handled by one CTA
constexpr int kChunk = 32;    // positions per staged chunk (two chunk buffers)
constexpr int kMaxSplits = 64;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

// Split-KV decode attention for head_dim HD, one CTA per (split, KV head), 4 warps.
// Launched as a programmatic dependent launch: the first chunk of cached K/V rows (written by
// earlier steps) is requested before griddepcontrol.wait; the q/k/v projection row after it.
// Scores: a warp per position, lane l holding dims [l*PL, l*PL+PL) of q (registers) and K.
// Values: thread t owns 4 consecutive dims of one q head (HD/4 threads per head).
template <int HD>
__global__ void __launch_bounds__(kDecThreads) k_attn_decode(AttnDecArgs a) {
    constexpr int PL = HD / 32;             // dims per lane in the score dot
    constexpr int VEC = HD / 8;             // 16-byte pieces per K or V row
    constexpr int TPH = HD / 4;             // value threads per q head
    constexpr int HPP = kDecThreads / TPH;  // q heads per value pass
    constexpr int NPASS = (kMaxRk + HPP - 1) / HPP;
    extern __shared__ __align__(16) uint8_t smem[];
    __half* sk = (__half*)smem;              // [2][kChunk][HD]
    __half* sv = sk + 2 * kChunk * HD;       // [2][kChunk][HD]
    __half* snew = sv + 2 * kChunk * HD;     // [2][HD] new k (rotated), new v
    float* ss = (float*)(snew + 2 * HD);     // [kMaxRk][kChunk] scores / probabilities
    float* sstat = ss + kMaxRk * kChunk;     // [kMaxRk][3] running max, sum, correction
    float* sq = sstat + kMaxRk * 3;          // [kMaxRk][HD] rotated q (fp16-rounded)
    const int rk = a.Hq / a.Hkv;
    const int hk = blockIdx.y;
    const int row = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // position of the new token and the KV window of its sequence
    const int64_t pos = a.batched ? (int64_t)a.step->row_pos[row]
                                  : (a.step ? a.step->pos : 0) + a.pos_off;
    // the sequence's rows: its page list in a paged cache, else its contiguous window
    const int32_t* plist =
        a.pg.pages ? a.pg.pages + (a.batched ? (int64_t)a.step->row_slot[row] * a.pg.stride : 0)
                   : nullptr;
    const int64_t slot_off =
        !plist && a.batched ? (int64_t)a.step->row_slot[row] * a.slot_elems : 0;
    __half* kslot = a.kc + slot_off;
    __half* vslot = a.vc + slot_off;
    auto krow = [&](int64_t t) { return kv_row_off(plist, a.pg.shift, a.Hkv, a.ctx, hk, t, HD); };
    const int64_t nkv = pos + 1;
    const int64_t per = (nkv + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = min((int64_t)blockIdx.x * per, nkv);
    const int64_t c1 = min(c0 + per, nkv);
    auto stage = [&](int buf, int64_t cs, int rows) {
        __half* dk = sk + buf * kChunk * HD;
        __half* dv = sv + buf * kChunk * HD;
        for (int e = threadIdx.x; e < rows * VEC; e += kDecThreads) {
            const int r = e / VEC, pc = e % VEC;
            if (cs + r == pos) continue;  // the new row is taken from snew
            const int64_t off = krow(cs + r) + pc * 8;
            cp_async16(dk + r * HD + pc * 8, kslot + off);
            cp_async16(dv + r * HD + pc * 8, vslot + off);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int nch = (int)((c1 - c0 + kChunk - 1) / kChunk);
    if (nch > 0) stage(0, c0, (int)min((int64_t)kChunk, c1 - c0));
    pdl_wait();
    pdl_launch();

    const float* qrow = a.qkv + (int64_t)row * a.qkv_stride;
    for (int e = threadIdx.x; e < rk * HD; e += kDecThreads) {
        const int h = e / HD, d = e % HD;
        const float* src = qrow + a.q_off + (int64_t)(hk * rk + h) * HD;
        sq[e] = __half2float(__float2half_rn(rope_elem(src, d, HD, a.tab, pos)));
    }
    if (c0 <= pos && pos < c1) {
        // this split holds the new position: rotate its k, write k and v to the cache
        const float* ks = qrow + a.k_off + (int64_t)hk * HD;
        for (int d = threadIdx.x; d < HD; d += kDecThreads) {
            const __half kh = __float2half_rn(rope_elem(ks, d, HD, a.tab, pos));
            const __half vh = __float2half_rn(qrow[a.v_off + (int64_t)hk * HD + d]);
            kslot[krow(pos) + d] = kh;
            vslot[krow(pos) + d] = vh;
            snew[d] = kh;
            snew[HD + d] = vh;
        }
    }
    if (threadIdx.x < kMaxRk) {
        sstat[threadIdx.x * 3 + 0] = -INFINITY;
        sstat[threadIdx.x * 3 + 1] = 0.0f;
        sstat[threadIdx.x * 3 + 2] = 1.0f;
    }
    __syncthreads();  // sq ready
    float qr[kMaxRk][PL];
#pragma unroll
    for (int h = 0; h < kMaxRk; ++h)
#pragma unroll
        for (int j = 0; j < PL; ++j) qr[h][j] = h < rk ? sq[h * HD + lane * PL + j] : 0.0f;
    float4 acc[NPASS];
#pragma unroll
    for (int p = 0; p < NPASS; ++p) acc[p] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int vh0 = threadIdx.x / TPH, vd = (threadIdx.x % TPH) * 4;

    for (int c = 0; c < nch; ++c) {
        const int buf = c & 1;
        const int64_t cs = c0 + (int64_t)c * kChunk;
        const int rows = (int)min((int64_t)kChunk, c1 - cs);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();  // chunk c landed; the previous chunk's reads are finished
        if (c + 1 < nch) stage(buf ^ 1, cs + kChunk, (int)min((int64_t)kChunk, c1 - cs - kChunk));
        const __half* ck = sk + buf * kChunk * HD;
        const __half* cv = sv + buf * kChunk * HD;
        for (int r = warp; r < rows; r += kDecThreads / 32) {
            const __half* kr = (cs + r == pos ? snew : ck + r * HD) + lane * PL;
            float kv[PL];
#pragma unroll
            for (int j = 0; j < PL; j += 2) {
                const float2 f = __half22float2(*(const __half2*)(kr + j));
                kv[j] = f.x;
                kv[j + 1] = f.y;
            }
#pragma unroll
            for (int h = 0; h < kMaxRk; ++h) {
                if (h < rk) {
                    float dot = 0.0f;
#pragma unroll
                    for (int j = 0; j < PL; ++j) dot = __fmaf_rn(kv[j], qr[h][j], dot);
                    dot = warp_sum(dot);
                    if (lane == 0) ss[h * kChunk + r] = __fmul_rn(dot, a.scale);
                }
            }
        }
        __syncthreads();
        // online softmax statistics per head (one warp per head)
        for (int h = warp; h < rk; h += kDecThreads / 32) {
            const float sc = lane < rows ? ss[h * kChunk + lane] : -INFINITY;
            const float mx = warp_max(sc);
            const float mold = sstat[h * 3 + 0];
            const float mnew = fmaxf(mold, mx);
            const float p = lane < rows ? expf(sc - mnew) : 0.0f;
            ss[h * kChunk + lane] = p;
            const float l = warp_sum(p);
            if (lane == 0) {
                const float corr = expf(mold - mnew);
                sstat[h * 3 + 0] = mnew;
                sstat[h * 3 + 1] = sstat[h * 3 + 1] * corr + l;
                sstat[h * 3 + 2] = corr;
            }
        }
        __syncthreads();
#pragma unroll
        for (int p = 0; p < NPASS; ++p) {
            const int h = vh0 + p * HPP;
            if (h < rk) {
                const float corr = sstat[h * 3 + 2];
                float4 v = make_float4(acc[p].x * corr, acc[p].y * corr, acc[p].z * corr,
                                       acc[p].w * corr);
                const float* ph = ss + h * kChunk;
                for (int r = 0; r < rows; ++r) {
                    const __half* vr = (cs + r == pos ? snew + HD : cv + r * HD) + vd;
                    const uint2 raw = *(const uint2*)vr;
                    const float2 f0 = __half22float2(*(const __half2*)&raw.x);
                    const float2 f1 = __half22float2(*(const __half2*)&raw.y);
                    const float pr = ph[r];
                    v.x = __fmaf_rn(pr, f0.x, v.x);
                    v.y = __fmaf_rn(pr, f0.y, v.y);
                    v.z = __fmaf_rn(pr, f1.x, v.z);
                    v.w = __fmaf_rn(pr, f1.y, v.w);
                }
                acc[p] = v;
            }
        }
    }
    __syncthreads();
    float* part = a.part + (int64_t)row * gridDim.x * a.Hq * (HD + 4) +
                  ((int64_t)blockIdx.x * a.Hq + (int64_t)hk * rk) * (HD + 4);
    if (threadIdx.x < rk) {
        part[threadIdx.x * (HD + 4) + 0] = c0 < c1 ? sstat[threadIdx.x * 3 + 0] : -INFINITY;
        part[threadIdx.x * (HD + 4) + 1] = c0 < c1 ? sstat[threadIdx.x * 3 + 1] : 0.0f;
    }
#pragma unroll
    for (int p = 0; p < NPASS; ++p) {
        const int h = vh0 + p * HPP;
        if (h < rk) *(float4*)(part + h * (HD + 4) + 4 + vd) = acc[p];
    }
}

// Split-KV decode attention on tensor cores (mma.sync m16n8k16, f16 inputs, f32 accumulation),
// head_dim 64 or 128; one CTA per (split, KV head, row), 4 warps.  The q heads of the GQA group
// are the rows of a 16-row A tile (rows >= the group size are zero).  Each warp walks its own
// 16-position blocks of the split (blocks warp, warp + 4, ...) through a two-slot cp.async ring
// and keeps its own online-softmax state, so warps never wait on one another inside the loop:
//   scores  S[16 x 16] = Q[16 x HD] K^T   (K rows by ldmatrix, scaled, masked past the split)
//   P = expf(S - m), the running max m and sum l per head, O rescaled by expf(m_old - m_new)
//   O[16 x HD] += P V, with P entered as hi + lo fp16 halves (two products), so the f32 result
//   keeps the probabilities' fp32 precision (V by ldmatrix.trans).
// At the end the four warps' (m, l, O) are merged in shared memory in warp order and written as
// the split's partial, in the layout k_attn_combine reads.  The new position's k and v rows are
// written to the cache by the CTA that holds it and taken from shared memory, never re-read.
constexpr int kTcPos = 16;    // positions per block
constexpr int kTcDepth = 2;   // ring slots per warp
constexpr int kMaxCluster = 16;  // 8 portable; 16 with the non-portable cluster attribute

template <int HD, int NW>
struct TcAttnSmem {
    static constexpr int kRow = HD * 2 + 16;              // bytes per staged K / V / q row
    static constexpr int kSlot = 2 * kTcPos * kRow;       // K block, then V block
    static constexpr int kQ = 16 * kRow;
    static constexpr int kNew = 2 * HD * 2;               // new k, new v (fp16)
    static constexpr int kRing = NW * kTcDepth * kSlot;
    static constexpr int kMerge = NW * kMaxRk * (HD + 2) * 4;
    static constexpr int kCm = kMaxRk * (HD + 2) * 4;     // the CTA's merged (acc, M, L)
    static constexpr int kBytes = kQ + kNew + (kRing > kMerge ? kRing : kMerge) + kCm;
};

__device__ __forceinline__ void cp_async16z(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void tc_ldsm4(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((unsigned)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void tc_ldsm4t(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((unsigned)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void tc_mma(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned pack_h2(__half2 h) { return *(unsigned*)&h; }
// all threads of all CTAs of the cluster; release / acquire orders the shared-memory partials
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// float at the same shared-memory offset as p in the CTA of cluster rank `rank`
__device__ __forceinline__ float ld_peer(const float* p, int rank) {
    unsigned addr;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(addr)
                 : "r"((unsigned)__cvta_generic_to_shared(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// CL: the CTAs of one (KV head, row) form a thread-block cluster (gridDim.x of them) and merge
// their partials through distributed shared memory at the end (no workspace, no merge launch);
// otherwise each CTA writes its partial for k_attn_combine.
template <int HD, int NW, bool CL>
__global__ void __launch_bounds__(NW * 32) k_attn_decode_tc(AttnDecArgs a) {
    static_assert(NW * 32 >= HD, "one thread per element of the new k / v row");
    constexpr int kTcWarps = NW;
    using SM = TcAttnSmem<HD, NW>;
    constexpr int KS = HD / 16;   // k-steps of the score product = 16-dim groups of the output
    constexpr int NTO = HD / 8;   // output n-tiles
    constexpr int R = SM::kRow;
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* sq = smem;                                  // [16][R] rotated q, fp16
    __half* snew = (__half*)(smem + SM::kQ);             // [2][HD]
    uint8_t* ring_all = smem + SM::kQ + SM::kNew;
    const int rk = a.Hq / a.Hkv;
    const int hk = blockIdx.y;
    const int row = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tg = lane & 3;
    uint8_t* ring = ring_all + warp * kTcDepth * SM::kSlot;
    const int64_t pos = a.batched ? (int64_t)a.step->row_pos[row]
                                  : (a.step ? a.step->pos : 0) + a.pos_off;
    // the sequence's rows: its page list in a paged cache, else its contiguous window
    const int32_t* plist =
        a.pg.pages ? a.pg.pages + (a.batched ? (int64_t)a.step->row_slot[row] * a.pg.stride : 0)
                   : nullptr;
    const int64_t slot_off =
        !plist && a.batched ? (int64_t)a.step->row_slot[row] * a.slot_elems : 0;
    __half* kslot = a.kc + slot_off;
    __half* vslot = a.vc + slot_off;
    auto krow = [&](int64_t t) { return kv_row_off(plist, a.pg.shift, a.Hkv, a.ctx, hk, t, HD); };
    const int64_t nkv = pos + 1;
    const int64_t per = (nkv + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = min((int64_t)blockIdx.x * per, nkv);
    const int64_t c1 = min(c0 + per, nkv);
    const int nblk = (int)((c1 - c0 + kTcPos - 1) / kTcPos);
    // block b of the split into a ring slot: rows past the split and the new position read as 0
    auto stage = [&](int slot, int b) {
        uint8_t* dk = ring + slot * SM::kSlot;
        uint8_t* dv = dk + kTcPos * R;
        const int64_t ps = c0 + (int64_t)b * kTcPos;
        // paged: lane j < kTcPos finds row j's offset (one page-table read a row, not one a
        // chunk); contiguous: rows are HD apart from the head's first row
        const int64_t mine = plist && lane < kTcPos && ps + lane < c1 ? krow(ps + lane) : 0;
        const int64_t head0 = (int64_t)hk * a.ctx * HD;
        for (int e = lane; e < kTcPos * (HD / 8); e += 32) {  // the same trip count on every lane
            const int r = e / (HD / 8), pc = e % (HD / 8);
            const int64_t roff = plist ? __shfl_sync(0xffffffffu, mine, r)  // warp-uniform branch
                                       : head0 + (ps + r) * HD;
            const bool ok = ps + r < c1 && ps + r != pos;
            const int64_t off = ok ? roff + pc * 8 : 0;
            cp_async16z(dk + r * R + pc * 16, kslot + off, ok);
            cp_async16z(dv + r * R + pc * 16, vslot + off, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // cached rows were written by earlier steps: both ring slots (the warp's first two blocks) are
    // requested before the wait, so at batch 1 (at most two blocks a warp) every K / V byte of
    // the CTA is in flight while the previous launch finishes
    if (warp < nblk) stage(0, warp);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    if (warp + kTcWarps < nblk) stage(1, warp + kTcWarps);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_wait();
    pdl_launch();

    const float* qrow = a.qkv + (int64_t)row * a.qkv_stride;
    // the new position's k and v (the CTA whose range holds it): this thread's element, loaded
    // with the q heads below, so the CTA pays one round trip for both
    const bool has_new = c0 <= pos && pos < c1;
    const int nd = threadIdx.x;  // its element (head_dim <= the CTA's threads)
    float nk0 = 0.0f, nk1 = 0.0f, nv = 0.0f;
    if (has_new && nd < HD) {
        const float* ks = qrow + a.k_off + (int64_t)hk * HD;
        const int half = a.tab.n_dims / 2;
        if (nd >= a.tab.n_dims) {
            nk0 = ks[nd];
        } else {
            const int i = nd < half ? nd : nd - half;
            nk0 = ks[i];
            nk1 = ks[i + half];
        }
        nv = qrow[a.v_off + (int64_t)hk * HD + nd];
    }
    {
        // rotated q heads (rope_elem's arithmetic): every load of this thread's elements is
        // issued before the first is used, so the rotation costs one round trip; rows >= rk zero
        constexpr int NT = kTcWarps * 32;
        constexpr int NE = kMaxRk * HD / NT;
        const int half = a.tab.n_dims / 2;
        const bool tab = a.tab.cs && pos >= 0 && pos < a.tab.n_pos;
        float x0[NE], x1[NE];
        float2 cs[NE];
#pragma unroll
        for (int k = 0; k < NE; ++k) {
            const int e = threadIdx.x + k * NT, h = e / HD, d = e % HD;
            x0[k] = x1[k] = 0.0f;
            cs[k] = make_float2(1.0f, 0.0f);
            if (h < rk) {
                const float* src = qrow + a.q_off + (int64_t)(hk * rk + h) * HD;
                if (d >= a.tab.n_dims) {
                    x0[k] = src[d];
                } else {
                    const int i = d < half ? d : d - half;
                    x0[k] = src[i];
                    x1[k] = src[i + half];
                    if (tab) cs[k] = a.tab.cs[pos * half + i];
                }
            }
        }
#pragma unroll
        for (int k = 0; k < NE; ++k) {
            const int e = threadIdx.x + k * NT, h = e / HD, d = e % HD;
            float v = 0.0f;
            if (h < rk) {
                if (d >= a.tab.n_dims) {
                    v = x0[k];
                } else {
                    const int i = d < half ? d : d - half;
                    float c = cs[k].x, sn = cs[k].y;
                    if (!tab) rope_cs(a.tab, pos, i, c, sn);
                    v = d < half ? __fmaf_rn(x0[k], c, -__fmul_rn(x1[k], sn))
                                 : __fmaf_rn(x0[k], sn, __fmul_rn(x1[k], c));
                }
            }
            *(__half*)(sq + h * R + d * 2) = __float2half_rn(v);
        }
        for (int e = kMaxRk * HD + threadIdx.x; e < 16 * HD; e += NT)
            *(__half*)(sq + (e / HD) * R + (e % HD) * 2) = __float2half_rn(0.0f);
    }
    if (has_new && nd < HD) {
        // rope_elem's arithmetic on the values loaded above
        float kr = nk0;
        if (nd < a.tab.n_dims) {
            const int half = a.tab.n_dims / 2;
            const int i = nd < half ? nd : nd - half;
            float c, sn;
            rope_cs(a.tab, pos, i, c, sn);
            kr = nd < half ? __fmaf_rn(nk0, c, -__fmul_rn(nk1, sn)) : __fmaf_rn(nk0, sn, __fmul_rn(nk1, c));
        }
        const __half kh = __float2half_rn(kr);
        const __half vh = __float2half_rn(nv);
        kslot[krow(pos) + nd] = kh;
        vslot[krow(pos) + nd] = vh;
        snew[nd] = kh;
        snew[HD + nd] = vh;
    }
    __syncthreads();  // sq and snew ready
    unsigned qf[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
        tc_ldsm4(qf[ks], sq + ((lane & 7) + ((lane >> 3) & 1) * 8) * R + (ks * 16 + (lane >> 4) * 8) * 2);
    float o[NTO][4];
#pragma unroll
    for (int n = 0; n < NTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_r = -INFINITY, l_r = 0.0f;  // row g: running max, this thread's share of the sum
    int j = 0;                           // blocks of this warp done
    for (int b = warp; b < nblk; b += kTcWarps, ++j) {
        // blocks j and j + 1 of this warp are requested (groups in order): block j has landed
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncwarp();
        uint8_t* ck = ring + (j & 1) * SM::kSlot;
        uint8_t* cv = ck + kTcPos * R;
        const int64_t ps = c0 + (int64_t)b * kTcPos;
        if (has_new && ps <= pos && pos < ps + kTcPos) {
            const int r = (int)(pos - ps);
            for (int d = lane; d < HD; d += 32) {
                *(__half*)(ck + r * R + d * 2) = snew[d];
                *(__half*)(cv + r * R + d * 2) = snew[HD + d];
            }
            __syncwarp();
        }
        float s[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            unsigned kb[4];  // (pos 0-7, dims lo), (pos 0-7, dims hi), (pos 8-15, lo), (8-15, hi)
            tc_ldsm4(kb, ck + ((lane & 7) + (lane >> 4) * 8) * R + (ks * 16 + ((lane >> 3) & 1) * 8) * 2);
            tc_mma(s[0], qf[ks], kb[0], kb[1]);
            tc_mma(s[1], qf[ks], kb[2], kb[3]);
        }
        float v[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int64_t p = ps + nt * 8 + 2 * tg + e;
                v[nt * 2 + e] = p < c1 ? __fmul_rn(s[nt][e], a.scale) : -INFINITY;
            }
        float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_r, mx);  // finite: every block holds a position of the split
        const float corr = expf(m_r - m_new);
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = expf(v[e] - m_new);
        l_r = __fadd_rn(__fmul_rn(l_r, corr), __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])));
        m_r = m_new;
#pragma unroll
        for (int n = 0; n < NTO; ++n) {
            o[n][0] = __fmul_rn(o[n][0], corr);
            o[n][1] = __fmul_rn(o[n][1], corr);
        }
        const __half2 h0 = __floats2half2_rn(p[0], p[1]), h1 = __floats2half2_rn(p[2], p[3]);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        const __half2 r0 = __floats2half2_rn(p[0] - f0.x, p[1] - f0.y);
        const __half2 r1 = __floats2half2_rn(p[2] - f1.x, p[3] - f1.y);
        const unsigned ahi[4] = {pack_h2(h0), 0u, pack_h2(h1), 0u};
        const unsigned alo[4] = {pack_h2(r0), 0u, pack_h2(r1), 0u};
#pragma unroll
        for (int dg = 0; dg < KS; ++dg) {
            unsigned vb[4];  // (pos 0-7, dims 16dg..), (pos 8-15, same), (0-7, +8..), (8-15, +8..)
            tc_ldsm4t(vb, cv + ((lane & 7) + ((lane >> 3) & 1) * 8) * R + (dg * 16 + (lane >> 4) * 8) * 2);
            tc_mma(o[2 * dg], ahi, vb[0], vb[1]);
            tc_mma(o[2 * dg], alo, vb[0], vb[1]);
            tc_mma(o[2 * dg + 1], ahi, vb[2], vb[3]);
            tc_mma(o[2 * dg + 1], alo, vb[2], vb[3]);
        }
        __syncwarp();  // every lane is done with slot j & 1: block j + 2 goes there
        const int bn = b + 2 * kTcWarps;
        if (bn < nblk) stage(j & 1, bn);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    l_r = __fadd_rn(l_r, __shfl_xor_sync(0xffffffffu, l_r, 1));
    l_r = __fadd_rn(l_r, __shfl_xor_sync(0xffffffffu, l_r, 2));
    __syncthreads();  // every warp is done with its ring: the area holds the merge
    float* mo = (float*)ring_all;                        // [warp][kMaxRk][HD]
    float* mm = mo + kTcWarps * kMaxRk * HD;              // [warp][kMaxRk] max
    float* ml = mm + kTcWarps * kMaxRk;                   // [warp][kMaxRk] sum
    if (g < rk) {
#pragma unroll
        for (int n = 0; n < NTO; ++n)
            *(float2*)(mo + (warp * kMaxRk + g) * HD + n * 8 + 2 * tg) = make_float2(o[n][0], o[n][1]);
        if (tg == 0) {
            mm[warp * kMaxRk + g] = m_r;
            ml[warp * kMaxRk + g] = l_r;
        }
    }
    __syncthreads();
    // this CTA's merged partial: to the workspace (split path) or to its own shared memory
    // (cluster path: [kMaxRk][HD] acc, then [kMaxRk] M, [kMaxRk] L)
    float* cm = (float*)(ring_all + (SM::kRing > SM::kMerge ? SM::kRing : SM::kMerge));
    float* part = CL ? nullptr
                     : a.part + (int64_t)row * gridDim.x * a.Hq * (HD + 4) +
                           ((int64_t)blockIdx.x * a.Hq + (int64_t)hk * rk) * (HD + 4);
    for (int e = threadIdx.x; e < rk * HD; e += kTcWarps * 32) {
        const int h = e / HD, d = e % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, mm[w * kMaxRk + h]);
        float acc = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kTcWarps; ++w) {
                const float mw = mm[w * kMaxRk + h];
                if (mw != -INFINITY)
                    acc = __fmaf_rn(mo[(w * kMaxRk + h) * HD + d], expf(mw - M), acc);
            }
        }
        if (CL) cm[h * HD + d] = acc;
        else part[h * (HD + 4) + 4 + d] = acc;
        if (d == 0) {
            float L = 0.0f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < kTcWarps; ++w) {
                    const float mw = mm[w * kMaxRk + h];
                    if (mw != -INFINITY) L = __fmaf_rn(ml[w * kMaxRk + h], expf(mw - M), L);
                }
            }
            if (CL) {
                cm[kMaxRk * HD + h] = M;
                cm[kMaxRk * HD + kMaxRk + h] = L;
            } else {
                part[h * (HD + 4) + 0] = M;
                part[h * (HD + 4) + 1] = L;
            }
        }
    }
    if (CL) {
        // every CTA of the cluster has its partial in shared memory; the rk * HD outputs, in
        // 32-element blocks (one Q8_0 block each), are dealt to the warps of the cluster, and
        // each lane merges one element over the cluster's CTAs in rank order (the weights and
        // the order of k_attn_combine)
        cluster_sync_all();
        const int C = (int)gridDim.x, me = (int)blockIdx.x;
        const int nob = rk * HD / 32;
        for (int ob = me + C * warp; ob < nob; ob += C * kTcWarps) {
            const int e = ob * 32 + lane, h = e / HD, d = e % HD;
            float Mc[kMaxCluster], Lc[kMaxCluster], Ac[kMaxCluster];
#pragma unroll
            for (int c = 0; c < kMaxCluster; ++c) {
                Mc[c] = -INFINITY;
                Lc[c] = Ac[c] = 0.0f;
                if (c < C) {
                    Ac[c] = ld_peer(cm + h * HD + d, c);
                    Mc[c] = ld_peer(cm + kMaxRk * HD + h, c);
                    Lc[c] = ld_peer(cm + kMaxRk * HD + kMaxRk + h, c);
                }
            }
            float M = -INFINITY;
#pragma unroll
            for (int c = 0; c < kMaxCluster; ++c) M = fmaxf(M, Mc[c]);
            float L = 0.0f, v = 0.0f;
#pragma unroll
            for (int c = 0; c < kMaxCluster; ++c) {
                const float w = Mc[c] == -INFINITY ? 0.0f : expf(Mc[c] - M);
                L += Lc[c] * w;
                v += Ac[c] * w;
            }
            v = v * (L == 0.0f ? 0.0f : 1.0f / L);
            const int64_t oi = ((int64_t)row * a.Hq + (int64_t)hk * rk + h) * HD + d;
            if (a.o) a.o[oi] = v;
            if (a.oq) {  // the warp holds one 32-element block of one head
                float d16, q;
                q8_block(v, lane, d16, q);
                a.oq[oi] = (int8_t)__float2int_rn(q);
                if (lane == 0) a.od[oi / 32] = d16;
            }
        }
        cluster_sync_all();  // no CTA leaves while a peer may still read its shared memory
    }
}

// Merge the splits of each q head; one CTA per q head, one thread per dim.  Every load is issued
// before the first dependent step: thread d reads its value of each split, warp 0 the (m, l)
// pairs.
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_combine(AttnDecArgs a) {
    __shared__ float sw[kMaxSplits];
    __shared__ float sL;
    pdl_wait();
    pdl_launch();
    const int h = blockIdx.x;  // q head
    const int row = blockIdx.y;
    const int S = a.splits;
    const int d = threadIdx.x;
    const float* base = a.part + (int64_t)row * S * a.Hq * (HD + 4) + (int64_t)h * (HD + 4);
    const int64_t sstride = (int64_t)a.Hq * (HD + 4);
    float pv[kMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp) pv[sp] = sp < S ? __ldcg(base + sp * sstride + 4 + d) : 0.0f;
    if (threadIdx.x < 32) {
        const int l = threadIdx.x;
        const float2 ml0 = l < S ? __ldcg((const float2*)(base + l * sstride)) : make_float2(-INFINITY, 0.0f);
        const float2 ml1 = l + 32 < S ? __ldcg((const float2*)(base + (l + 32) * sstride))
                                      : make_float2(-INFINITY, 0.0f);
        const float M = warp_max(fmaxf(ml0.x, ml1.x));
        const float w0 = ml0.x == -INFINITY ? 0.0f : expf(ml0.x - M);
        const float w1 = ml1.x == -INFINITY ? 0.0f : expf(ml1.x - M);
        sw[l] = w0;
        sw[l + 32] = w1;
        const float L = warp_sum(ml0.y * w0 + ml1.y * w1);
        if (l == 0) sL = L;
    }
    __syncthreads();
    const float inv = sL == 0.0f ? 0.0f : 1.0f / sL;
    float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f, v3 = 0.0f;
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; sp += 4) {
        v0 += pv[sp] * sw[sp];
        v1 += pv[sp + 1] * sw[sp + 1];
        v2 += pv[sp + 2] * sw[sp + 2];
        v3 += pv[sp + 3] * sw[sp + 3];
    }
    const float v = ((v0 + v1) + (v2 + v3)) * inv;
    const int64_t oi = ((int64_t)row * a.Hq + h) * HD + d;
    if (a.o) a.o[oi] = v;
    if (a.oq) {  // warp w owns elements 32w..32w+31 of the head: one Q8_0 block
        const int lane = threadIdx.x & 31;
        float d16, q;
        q8_block(v, lane, d16, q);
        a.oq[oi] = (int8_t)__float2int_rn(q);
        if (lane == 0) a.od[oi / 32] = d16;
    }
}

template <int HD>
size_t dec_smem() {
    return (size_t)4 * kChunk * HD * 2 + (size_t)2 * HD * 2 + (size_t)kMaxRk * kChunk * 4 +
           kMaxRk * 12 + (size_t)kMaxRk * HD * 4;
}

// cudaFuncAttributeMaxDynamicSharedMemorySize of one kernel, set once per device
template <auto KERN>
void set_max_smem(size_t bytes) {
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static bool done[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev & 63]) {
        GB_CUDA(cudaFuncSetAttribute(KERN, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
        done[dev & 63] = true;
    }
}

// programmatic dependent launch of a cluster kernel: clusters of cx CTAs along x
template <typename... P>
void launch_cluster_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, unsigned cx,
                        cudaStream_t st, const AttnDecArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cx;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cx > 8)
        GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    GB_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
}

template <int HD, int NW>
void launch_cluster(const AttnDecArgs& a, int C, cudaStream_t st) {
    constexpr size_t tsm = TcAttnSmem<HD, NW>::kBytes;
    auto kern = k_attn_decode_tc<HD, NW, true>;
    set_max_smem<k_attn_decode_tc<HD, NW, true>>(tsm);
    if (C > 8) {
        // clusters beyond the portable 8 CTAs: only where this device can hold one (asked once
        // per device), else 8
        static int fits[64] = {};  // 0 unknown, 1 yes, -1 no
        int dev = 0;
        GB_CUDA(cudaGetDevice(&dev));
        if (dev >= 0 && dev < 64 && fits[dev] == 0) {
            GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)C, (unsigned)a.Hkv, 1);
            cfg.blockDim = dim3(NW * 32);
            cfg.dynamicSmemBytes = tsm;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)C;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
            if (e != cudaSuccess) cudaGetLastError();
            fits[dev] = e == cudaSuccess && n >= 1 ? 1 : -1;
        }
        if (dev < 0 || dev >= 64 || fits[dev] < 0) C = 8;
    }
    launch_cluster_pdl(k_attn_decode_tc<HD, NW, true>,
                       dim3((unsigned)C, (unsigned)a.Hkv, (unsigned)a.rows), NW * 32, tsm,
                       (unsigned)C, st, a);
}

template <int HD>
void launch_dec(const AttnDecArgs& a, cudaStream_t st) {
    if (HD <= 128) {
        constexpr int H = HD <= 128 ? HD : 128;
        const int C = attn_decode_cluster(a.Hkv, HD, a.ctx, a.rows);
        if (C > 0) {  // one launch: the cluster merges its CTAs' partials
            launch_cluster<H, 4>(a, C, st);
            return;
        }
        constexpr size_t tsm = TcAttnSmem<H, 4>::kBytes;
        set_max_smem<k_attn_decode_tc<H, 4, false>>(tsm);
        launch_pdl(k_attn_decode_tc<H, 4, false>,
                   dim3((unsigned)a.splits, (unsigned)a.Hkv, (unsigned)a.rows), 4 * 32, tsm, st, a);
    } else {
        const size_t smem = dec_smem<HD>();
        set_max_smem<k_attn_decode<HD>>(smem);
        launch_pdl(k_attn_decode<HD>, dim3((unsigned)a.splits, (unsigned)a.Hkv, (unsigned)a.rows),
                   kDecThreads, smem, st, a);
    }
    GB_CHECK(a.part != nullptr, "attn_decode: this shape needs the split workspace");
    launch_pdl(k_attn_combine<HD>, dim3((unsigned)a.Hq, (unsigned)a.rows), HD, 0, st, a);
}

}  // namespace

void launch_rope_qkv(const QkvRopeArgs& a, cudaStream_t st) {
    const int64_t total = (int64_t)a.s * (a.Hq + 2 * a.Hkv) * a.hd;
    if (!total) return;
    GB_CHECK(a.tab.n_dims <= a.hd && a.tab.n_dims % 2 == 0, "rope_qkv: bad n_dims");
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_rope_qkv<<<(unsigned)blocks, 256, 0, st>>>(a);
    GB_CUDA(cudaGetLastError());
}

int attn_decode_splits(int64_t Hkv, int64_t max_kv, int rows) {
    // about two CTAs per SM over the launch; each split then walks max_kv / splits positions
    const int64_t units = Hkv * std::max(rows, 1);
    if (units <= 0 || max_kv <= 0) return 1;  // invalid shapes are rejected by the launch checks
    int64_t s = (296 + units - 1) / units;
    if (s > max_kv) s = max_kv;
    if (s > kMaxSplits) s = kMaxSplits;
    return (int)(s < 1 ? 1 : s);
}

int attn_decode_cluster(int64_t Hkv, int64_t hd, int64_t ctx, int rows) {
    if ((hd != 64 && hd != 128) || Hkv <= 0 || ctx <= 0) return 0;
    // about one CTA per SM over the launch, at most kMaxCluster per (row, KV head)
    const int64_t units = Hkv * std::max(rows, 1);
    int64_t C = (148 + units - 1) / units;
    // CTAs per cluster at most: 16 (GGMLC_B200_ATTN_CLUSTER; 16 measured 1 % faster than the
    // portable 8 at batch 1 on the 8B shape; launch_cluster falls back to 8 where the device
    // cannot hold a 16-CTA cluster)
    static const int64_t cmax = [] {
        const char* e = getenv("GGMLC_B200_ATTN_CLUSTER");
        const int64_t v = e ? atoll(e) : 16;
        return std::max<int64_t>(1, std::min<int64_t>(v, kMaxCluster));
    }();
    C = std::max<int64_t>(1, std::min<int64_t>(C, cmax));
    // each of a CTA's 4 warps walks at most 4 blocks of 16 positions (a CTA stays under 80 KB of
    // shared memory, so the GEMVs before and after it share the SM); longer caches take the
    // wider split with the merge launch
    if ((ctx + C * kTcPos - 1) / (C * kTcPos) > 16) return 0;
    return (int)C;
}

size_t attn_decode_workspace(int64_t Hq, int64_t hd, int splits) {
    return (size_t)splits * Hq * (hd + 4) * sizeof(float);
}

void launch_attn_decode(const AttnDecArgs& a, cudaStream_t st) {
    GB_CHECK(a.hd == 64 || a.hd == 128 || a.hd == 256, "attn_decode: head_dim must be 64, 128 or 256");
    GB_CHECK(a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRk,
             "attn_decode: GQA group too large");
    GB_CHECK(a.splits >= 1 && a.splits <= kMaxSplits, "attn_decode: bad split count");
    GB_CHECK(a.rows >= 1 && a.rows <= kMaxRows && (a.rows == 1 || a.batched),
             "attn_decode: 1..16 rows, several only in batched mode");
    GB_CHECK(!a.batched || a.step, "attn_decode: batched mode reads positions from step params");
    switch (a.hd) {
        case 64: launch_dec<64>(a, st); break;
        case 128: launch_dec<128>(a, st); break;
        default: launch_dec<256>(a, st); break;
    }
}

}  // namespace gb

// Fixed scratch for gb_attn_decode_noalloc: the split partials of one decode-attention call.
// Every partial the combine reads is written by k_attn_decode earlier on the same stream, so the
// array needs no initial contents.  One array per device, shared by every call on that device.
namespace gb {
namespace {
__device__ __align__(256) float g_dec_static_work[kAttnDecStaticWorkBytes / sizeof(float)];
}  // namespace

float* attn_decode_static_work(size_t need) {
    GB_CHECK(need <= kAttnDecStaticWorkBytes,
             "attn_decode: needs " + std::to_string(need) + " bytes of split scratch, more than the " +
                 std::to_string(kAttnDecStaticWorkBytes) + "-byte static array");
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "attn_decode: device ordinal out of range");
    static std::mutex mu;
    static void* addr[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        GB_CUDA(cudaGetSymbolAddress(&p, g_dec_static_work));
        GB_CHECK(p != nullptr, "attn_decode: static scratch has no device address");
        addr[dev] = p;
    }
    return (float*)addr[dev];
}

}  // namespace gb
