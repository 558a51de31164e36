// RoPE, KV-cache writes and attention over the F16 KV cache.
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

__device__ __forceinline__ float load_f(const TView& v, int64_t i0, int64_t i1, int64_t i2) {
    const char* p = v.data + i0 * v.nb[0] + i1 * v.nb[1] + i2 * v.nb[2];
    if (v.type == T_F16) return __half2float(*(const __half*)p);
    return *(const float*)p;
}

// NEOX RoPE (ggml-cpu/ops.cpp:5910-5923 cache init, :5998-6015 rotate_pairs): pair (i, i+nd/2),
// out0 = fma(x0, cos, -(x1*sin)), out1 = fma(x0, sin, x1*cos) — the contracted form the
// reference's GNU build computes.  cos/sin come from the host table built with the CPU's own
// fp32 theta recurrence and libm; positions outside it fall back to an on-device recurrence.
__global__ void k_rope_neox(TView x, const int32_t* __restrict__ pos_src, int use_step,
                            const StepParams* __restrict__ step, RopeTable tab, TView y,
                            int to_kv, KVDst kv) {
    const int64_t hd = x.ne[0], H = x.ne[1], s = x.ne[2];
    const int half = tab.n_dims / 2;
    const int64_t total = (hd / 2) * H * s;
    const int64_t base = use_step ? step->pos : 0;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = idx % (hd / 2);
        const int64_t h = (idx / (hd / 2)) % H;
        const int64_t t = idx / ((hd / 2) * H);
        float o0, o1;
        int64_t d0, d1;
        if (i < half) {
            d0 = i;
            d1 = i + half;
            const int32_t p = pos_src ? pos_src[base + t] : (int32_t)(base + t);
            float c, sn;
            if (tab.cs && p >= 0 && p < tab.n_pos) {
                const float2 cs = tab.cs[(int64_t)p * half + i];
                c = cs.x;
                sn = cs.y;
            } else {
                float theta = (float)p;
                for (int64_t k = 0; k < i; ++k) theta = __fmul_rn(theta, tab.theta_scale);
                c = (float)cos((double)theta);
                sn = (float)sin((double)theta);
            }
            const float x0 = load_f(x, d0, h, t), x1 = load_f(x, d1, h, t);
            o0 = __fmaf_rn(x0, c, -__fmul_rn(x1, sn));
            o1 = __fmaf_rn(x0, sn, __fmul_rn(x1, c));
        } else {
            // dims past n_dims are copied through (rope_f32 tail)
            d0 = 2 * half + 2 * (i - half);
            d1 = d0 + 1;
            o0 = load_f(x, d0, h, t);
            o1 = load_f(x, d1, h, t);
        }
        if (to_kv) {
            __half* row = kv.base + kv_row_off(kv.pages, kv.shift, H, kv.ctx, h, base + t, hd);
            row[d0] = __float2half_rn(o0);
            row[d1] = __float2half_rn(o1);
        } else {
            *(float*)(y.data + d0 * y.nb[0] + h * y.nb[1] + t * y.nb[2]) = o0;
            *(float*)(y.data + d1 * y.nb[0] + h * y.nb[1] + t * y.nb[2]) = o1;
        }
    }
}

// SET_ROWS of K or V into the F16 cache (ggml-cpu/ops.cpp:5156-5224; fp32 -> fp16 RNE).
__global__ void k_kv_write(TView src, const StepParams* __restrict__ step, int use_step,
                           KVDst kv) {
    const int64_t hd = src.ne[0], H = src.ne[1], s = src.ne[2];
    const int64_t total = hd * H * s;
    const int64_t base = use_step ? step->pos : 0;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = idx % hd, h = (idx / hd) % H, t = idx / (hd * H);
        kv.base[kv_row_off(kv.pages, kv.shift, H, kv.ctx, h, base + t, hd) + d] =
            __float2half_rn(load_f(src, d, h, t));
    }
}

// ---- attention -----------------------------------------------------------------------------
// Flash-decoding over the F16 cache.  grid = (splits, query-vector tiles, Hkv); a CTA holds
// `nq` query vectors (rows x heads of one GQA group), one warp each, and walks its split of
// the KV positions in 32-row tiles staged in shared memory: lane j scores position tile+j,
// the warp keeps an online softmax and lanes accumulate V for dims lane, lane+32, ...
// Split results (m, l, acc) are merged by k_attn_combine.
constexpr int kTile = 32;
constexpr int kMaxHd = 256;
constexpr int kSplitLen = 128;

struct AttnArgs {
    TView q;              // f32 [hd, s, Hq]
    const __half* kc;     // [Hkv][ctx][hd], or page pools (pages != nullptr, KvPages)
    const __half* vc;
    const int32_t* pages;
    int shift;
    int64_t ctx, Hkv, Hq, hd, s;
    const StepParams* step;
    int use_step;
    int64_t kv_off;
    float scale;
    int64_t splits;       // number of KV splits (gridDim.x)
    float* o;             // [s][Hq][hd]
    float* part;          // [splits][s*Hq][hd+2] partials (m, l, acc) when splits > 1
};

__global__ void k_attn(AttnArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t hd = a.hd;
    const int64_t rk = a.Hq / a.Hkv;
    const int nq = blockDim.x / 32;
    const int64_t hk = blockIdx.z;
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int64_t kstride = hd + 2;  // halves per staged K row (odd word count: no conflicts)
    __half* sk = (__half*)smem;
    __half* sv = sk + kTile * kstride;
    float* sq = (float*)(sv + kTile * hd);

    // query vector owned by this warp: qv = tile*nq + warp -> (row t, head h)
    const int64_t qv = (int64_t)blockIdx.y * nq + warp;
    const bool qvalid = qv < a.s * rk;
    const int64_t t = qvalid ? qv / rk : 0;
    const int64_t h = hk * rk + (qvalid ? qv % rk : 0);
    const int64_t kv_base = (a.use_step ? a.step->pos : 0) + a.kv_off;
    const int64_t limit = kv_base + t;  // last visible cache row for this query

    // stage q rounded to fp16 (q_to_vec_dot of the CPU kernel)
    for (int64_t d = lane; d < hd; d += 32)
        sq[warp * hd + d] = qvalid ? __half2float(__float2half_rn(load_f(a.q, d, t, h))) : 0.0f;

    // KV range of this split, clipped to what any query of the CTA can see
    const int64_t t_last = min((int64_t)(blockIdx.y + 1) * nq - 1, a.s * rk - 1) / rk;
    const int64_t cta_limit = kv_base + t_last;
    const int64_t per_split = ((cta_limit + 1) + a.splits - 1) / a.splits;
    const int64_t c0 = (int64_t)blockIdx.x * per_split;
    const int64_t c1 = min(c0 + per_split, cta_limit + 1);

    float m = -INFINITY, l = 0.0f;
    float acc[kMaxHd / 32];
#pragma unroll
    for (int k = 0; k < kMaxHd / 32; ++k) acc[k] = 0.0f;
    const int nd = (int)((hd + 31) / 32);

    for (int64_t tile = c0; tile < c1; tile += kTile) {
        __syncthreads();
        const int64_t rows = min((int64_t)kTile, c1 - tile);
        for (int64_t e = threadIdx.x; e < rows * hd; e += blockDim.x) {
            const int64_t r = e / hd, d = e % hd;
            const int64_t off = kv_row_off(a.pages, a.shift, a.Hkv, a.ctx, hk, tile + r, hd) + d;
            sk[r * kstride + d] = a.kc[off];
            sv[r * hd + d] = a.vc[off];
        }
        __syncthreads();
        if (!qvalid) continue;
        const int64_t c = tile + lane;
        float sc = -INFINITY;
        if (lane < rows && c <= limit) {
            float dot = 0.0f;
            const __half* kr = sk + lane * kstride;
            const float* qr = sq + warp * hd;
            for (int64_t d = 0; d < hd; d += 2) {
                const float2 kf = __half22float2(*(const __half2*)(kr + d));
                dot = __fmaf_rn(kf.x, qr[d], dot);
                dot = __fmaf_rn(kf.y, qr[d + 1], dot);
            }
            sc = __fmul_rn(dot, a.scale);
        }
        const float tmax = warp_max(sc);
        if (tmax == -INFINITY) continue;
        const float mnew = fmaxf(m, tmax);
        const float corr = expf(m - mnew);
        const float p = sc == -INFINITY ? 0.0f : expf(sc - mnew);
        l = l * corr + warp_sum(p);
#pragma unroll
        for (int k = 0; k < kMaxHd / 32; ++k) acc[k] *= corr;
        for (int j = 0; j < rows; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            if (pj == 0.0f) continue;
            const __half* vr = sv + j * hd;
#pragma unroll
            for (int k = 0; k < kMaxHd / 32; ++k)
                if (k < nd && lane + 32 * k < hd)
                    acc[k] = __fmaf_rn(pj, __half2float(vr[lane + 32 * k]), acc[k]);
        }
        m = mnew;
    }
    if (!qvalid) return;
    if (a.splits == 1) {
        const float inv = l == 0.0f ? 0.0f : 1.0f / l;
        float* orow = a.o + (t * a.Hq + h) * hd;
#pragma unroll
        for (int k = 0; k < kMaxHd / 32; ++k)
            if (k < nd && lane + 32 * k < hd) orow[lane + 32 * k] = acc[k] * inv;
    } else {
        float* pr = a.part + ((int64_t)blockIdx.x * a.s * a.Hq + t * a.Hq + h) * (hd + 2);
        if (lane == 0) {
            pr[0] = m;
            pr[1] = l;
        }
#pragma unroll
        for (int k = 0; k < kMaxHd / 32; ++k)
            if (k < nd && lane + 32 * k < hd) pr[2 + lane + 32 * k] = acc[k];
    }
}

__global__ void k_attn_combine(AttnArgs a) {
    const int64_t vec = blockIdx.x;  // t*Hq + h
    const int64_t hd = a.hd;
    const int64_t n = a.s * a.Hq;
    float M = -INFINITY;
    for (int64_t sp = 0; sp < a.splits; ++sp) M = fmaxf(M, a.part[(sp * n + vec) * (hd + 2)]);
    float L = 0.0f;
    for (int64_t sp = 0; sp < a.splits; ++sp) {
        const float* pr = a.part + (sp * n + vec) * (hd + 2);
        if (pr[0] != -INFINITY) L += pr[1] * expf(pr[0] - M);
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    for (int64_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float v = 0.0f;
        for (int64_t sp = 0; sp < a.splits; ++sp) {
            const float* pr = a.part + (sp * n + vec) * (hd + 2);
            if (pr[0] != -INFINITY) v += pr[2 + d] * expf(pr[0] - M);
        }
        a.o[vec * hd + d] = v * inv;
    }
}

// ---- tensor-core flash attention for prefill (s >= 16, head_dim 64 or 128) ------------------
// One warp owns 16 query rows of one q head; a CTA's 4 warps share one KV head (GQA), so each
// K/V tile of 64 cache rows is staged once (cp.async, double-buffered, XOR-swizzled rows) for all
// of them.  S = Q K^T and O += P V run on mma.sync m16n8k16 with fp16 inputs and fp32
// accumulators: Q is rounded to fp16 as the CPU kernel does (q_to_vec_dot), the probabilities P
// are rounded to fp16 for the second product (the CPU rounds its whole V accumulator to fp16
// after every position, a larger error).  Online softmax in fp32 per row; causal limit per
// query at absolute positions (query t sees cache rows 0 .. kv_base + t).
constexpr int kFaKeys = 64;
constexpr int kFaWarps = 4;

__device__ __forceinline__ unsigned fa_saddr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void fa_cp16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(fa_saddr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void fa_ldsm4(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(fa_saddr(p)));
}
__device__ __forceinline__ void fa_ldsm4t(unsigned (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(fa_saddr(p)));
}
__device__ __forceinline__ void fa_mma(float (&d)[4], const unsigned (&a)[4], unsigned b0,
                                       unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *(const unsigned*)&h;
}

template <int HD>
__global__ void __launch_bounds__(kFaWarps * 32) k_fa(AttnArgs a) {
    constexpr int CH = HD / 8;  // 16-byte chunks per K/V row
    extern __shared__ __align__(16) uint8_t smem[];
    __half* sK = (__half*)smem;                      // [2][kFaKeys][HD]
    __half* sV = sK + 2 * kFaKeys * HD;              // [2][kFaKeys][HD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int rk = (int)(a.Hq / a.Hkv);
    const int hk = blockIdx.y;
    const int nqb = (int)((a.s + 15) / 16);
    // work items of this KV head: (query block, head in group); 4 per CTA
    const int item = blockIdx.x * kFaWarps + warp;
    const bool active = item < nqb * rk;
    const int qb = active ? item / rk : 0;
    const int h = hk * rk + (active ? item % rk : 0);
    const int64_t kv_base = (a.use_step ? a.step->pos : 0) + a.kv_off;
    // rows this CTA must see: up to the last query of its last item
    const int last_item = min((int)(blockIdx.x + 1) * kFaWarps, nqb * rk) - 1;
    const int64_t last_q = min((int64_t)(last_item / rk) * 16 + 15, a.s - 1);
    const int64_t nkv = kv_base + last_q + 1;
    const int ntile = (int)((nkv + kFaKeys - 1) / kFaKeys);
    auto stage = [&](int tile, int buf) {
        __half* dk = sK + buf * kFaKeys * HD;
        __half* dv = sV + buf * kFaKeys * HD;
        for (int e = threadIdx.x; e < kFaKeys * CH; e += kFaWarps * 32) {
            const int r = e / CH, c = e % CH;
            const int64_t key = (int64_t)tile * kFaKeys + r;
            const bool ok = key < nkv;
            const int64_t off = kv_row_off(a.pages, a.shift, a.Hkv, a.ctx, hk, ok ? key : 0, HD);
            const int sw = (c ^ (r & 7)) * 8;
            fa_cp16(dk + r * HD + sw, a.kc + off + c * 8, ok);
            fa_cp16(dv + r * HD + sw, a.vc + off + c * 8, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0, 0);

    // Q fragments (fp16) of this warp's 16 rows: [k16 step][a0..a3]
    unsigned qf[HD / 16][4];
    const int64_t t0 = (int64_t)qb * 16;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t t = t0 + g + ((r & 1) << 3);
            const int d = ks * 16 + 2 * tg + ((r >> 1) << 3);
            float2 v = make_float2(0.0f, 0.0f);
            if (active && t < a.s) {
                const char* p = a.q.data + d * a.q.nb[0] + t * a.q.nb[1] + h * a.q.nb[2];
                v = *(const float2*)p;
            }
            qf[ks][r] = pack_h2(v.x, v.y);
        }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
    const int64_t lim0 = kv_base + t0 + g, lim1 = lim0 + 8;  // last visible row per owned row

    for (int tile = 0; tile < ntile; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < ntile) {
            stage(tile + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const __half* cK = sK + buf * kFaKeys * HD;
        const __half* cV = sV + buf * kFaKeys * HD;
        const int64_t key0 = (int64_t)tile * kFaKeys;
        if (active && key0 <= kv_base + t0 + 15) {
            // S = Q K^T: 8 key tiles of 8
            float sc[kFaKeys / 8][4];
#pragma unroll
            for (int nt = 0; nt < kFaKeys / 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
                for (int np = 0; np < kFaKeys / 16; ++np) {
                    // keys np*16 .. +15, dims ks*16 .. +15: matrices (k0-7,d0-7) (k0-7,d8-15)
                    // (k8-15,d0-7) (k8-15,d8-15)
                    const int q4 = lane >> 3;
                    const int r = np * 16 + (lane & 7) + ((q4 >> 1) << 3);
                    const int c = ks * 2 + (q4 & 1);
                    unsigned bk[4];
                    fa_ldsm4(bk, cK + r * HD + ((c ^ (r & 7)) << 3));
                    fa_mma(sc[2 * np], qf[ks], bk[0], bk[1]);
                    fa_mma(sc[2 * np + 1], qf[ks], bk[2], bk[3]);
                }
            }
            // scale, causal mask, online softmax (rows g and g+8 of the warp's block)
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int nt = 0; nt < kFaKeys / 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int64_t key = key0 + nt * 8 + 2 * tg + (e & 1);
                    const int64_t lim = (e >> 1) ? lim1 : lim0;
                    const float v = key <= lim ? __fmul_rn(sc[nt][e], a.scale) : -INFINITY;
                    sc[nt][e] = v;
                    mx[e >> 1] = fmaxf(mx[e >> 1], v);
                }
            float corr[2], mnew[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                mnew[r] = fmaxf(mrow[r], mx[r]);
                corr[r] = mnew[r] == -INFINITY ? 1.0f : expf(mrow[r] - mnew[r]);
                mrow[r] = mnew[r];
            }
            float ls[2] = {0.0f, 0.0f};
            unsigned pf[kFaKeys / 16][4];
#pragma unroll
            for (int nt = 0; nt < kFaKeys / 8; ++nt) {
                float p[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float mr = mnew[e >> 1];
                    p[e] = sc[nt][e] == -INFINITY ? 0.0f : expf(sc[nt][e] - mr);
                    ls[e >> 1] += p[e];
                }
                // C layout of key tile nt -> A layout of the PV product (k16 step nt/2)
                pf[nt >> 1][(nt & 1) * 2 + 0] = pack_h2(p[0], p[1]);
                pf[nt >> 1][(nt & 1) * 2 + 1] = pack_h2(p[2], p[3]);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
                lrow[r] = lrow[r] * corr[r] + ls[r];
            }
#pragma unroll
            for (int i = 0; i < HD / 8; ++i) {
                o[i][0] *= corr[0];
                o[i][1] *= corr[0];
                o[i][2] *= corr[1];
                o[i][3] *= corr[1];
            }
            // O += P V: for each 16-key step, V^T fragments with ldmatrix.trans
#pragma unroll
            for (int ks = 0; ks < kFaKeys / 16; ++ks) {
#pragma unroll
                for (int dp = 0; dp < HD / 16; ++dp) {
                    const int q4 = lane >> 3;
                    const int r = ks * 16 + (lane & 7) + ((q4 & 1) << 3);
                    const int c = dp * 2 + (q4 >> 1);
                    unsigned bv[4];
                    fa_ldsm4t(bv, cV + r * HD + ((c ^ (r & 7)) << 3));
                    fa_mma(o[2 * dp], pf[ks], bv[0], bv[1]);
                    fa_mma(o[2 * dp + 1], pf[ks], bv[2], bv[3]);
                }
            }
        }
        __syncthreads();  // the buffer is restaged next
    }
    if (!active) return;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int64_t t = t0 + g + r * 8;
        if (t >= a.s) continue;
        const float inv = lrow[r] == 0.0f ? 0.0f : 1.0f / lrow[r];
        float* orow = a.o + (t * a.Hq + h) * HD;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            const int d = i * 8 + 2 * tg;
            *(float2*)(orow + d) = make_float2(o[i][r * 2] * inv, o[i][r * 2 + 1] * inv);
        }
    }
}

int64_t attn_splits(int64_t s, int64_t max_kv) {
    if (s > 4) return 1;
    int64_t sp = (max_kv + kSplitLen - 1) / kSplitLen;
    return sp < 1 ? 1 : (sp > 64 ? 64 : sp);
}

}  // namespace

void launch_rope_neox(const TView& x, const int32_t* pos_src, bool use_step_pos,
                      const StepParams* step, const RopeTable& tab, const TView* y,
                      const KVDst* kv, cudaStream_t st) {
    const int64_t total = (x.ne[0] / 2) * x.ne[1] * x.ne[2];
    if (!total) return;
    GB_CHECK(x.ne[0] % 2 == 0 && tab.n_dims <= x.ne[0], "rope: bad n_dims");
    TView yy = y ? *y : TView{};
    KVDst kk = kv ? *kv : KVDst{};
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_rope_neox<<<(unsigned)blocks, threads, 0, st>>>(x, pos_src, use_step_pos ? 1 : 0, step, tab,
                                                      yy, kv ? 1 : 0, kk);
    GB_CUDA(cudaGetLastError());
}

void launch_kv_write(const TView& src, const StepParams* step, const KVDst& kv, cudaStream_t st) {
    const int64_t total = src.ne[0] * src.ne[1] * src.ne[2];
    if (!total) return;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_kv_write<<<(unsigned)blocks, threads, 0, st>>>(src, step, step ? 1 : 0, kv);
    GB_CUDA(cudaGetLastError());
}

size_t attn_workspace_bytes(int64_t s, int64_t Hq, int64_t hd, int64_t max_kv) {
    const int64_t sp = attn_splits(s, max_kv);
    return sp > 1 ? (size_t)sp * s * Hq * (hd + 2) * sizeof(float) : 0;
}

void launch_attention(const TView& q, const __half* kc, const __half* vc, int64_t ctx,
                      int64_t Hkv, const StepParams* step, bool use_step, int64_t kv_off,
                      float scale, float* o, void* work, int64_t max_kv, cudaStream_t st,
                      const int32_t* pages, int page_shift) {
    AttnArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.pages = pages;
    a.shift = page_shift;
    a.ctx = ctx;
    a.Hkv = Hkv;
    a.hd = q.ne[0];
    a.s = q.ne[1];
    a.Hq = q.ne[2];
    a.step = step;
    a.use_step = use_step ? 1 : 0;
    a.kv_off = kv_off;
    a.scale = scale;
    a.o = o;
    a.part = (float*)work;
    GB_CHECK(a.hd <= kMaxHd && a.hd % 2 == 0, "attention: head_dim must be even and <= 256");
    GB_CHECK(a.Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
    if (!a.s) return;
    if (a.s >= 16 && (a.hd == 64 || a.hd == 128) && q.nb[0] == 4 &&
        ((uintptr_t)kc & 15) == 0 && ((uintptr_t)vc & 15) == 0) {
        // tensor-core flash attention; one KV split (every query block walks its own rows)
        a.splits = 1;
        const int64_t rk = a.Hq / Hkv;
        const int64_t items = ((a.s + 15) / 16) * rk;
        dim3 grid((unsigned)((items + kFaWarps - 1) / kFaWarps), (unsigned)Hkv);
        const size_t smem = (size_t)4 * kFaKeys * a.hd * 2;
        if (a.hd == 64) {
            k_fa<64><<<grid, kFaWarps * 32, smem, st>>>(a);
        } else {
            static bool configured[64] = {};
            int dev = 0;
            GB_CUDA(cudaGetDevice(&dev));
            if (!configured[dev & 63]) {
                GB_CUDA(cudaFuncSetAttribute(k_fa<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem));
                configured[dev & 63] = true;
            }
            k_fa<128><<<grid, kFaWarps * 32, smem, st>>>(a);
        }
        GB_CUDA(cudaGetLastError());
        return;
    }
    a.splits = attn_splits(a.s, max_kv);
    const int64_t rk = a.Hq / Hkv;
    const int nq = (int)(rk * a.s < 8 ? rk * a.s : 8);
    const int64_t qtiles = (a.s * rk + nq - 1) / nq;
    const size_t smem = (size_t)kTile * (a.hd + 2) * 2 + (size_t)kTile * a.hd * 2 +
                        (size_t)nq * a.hd * 4;
    dim3 grid((unsigned)a.splits, (unsigned)qtiles, (unsigned)Hkv);
    k_attn<<<grid, nq * 32, smem, st>>>(a);
    GB_CUDA(cudaGetLastError());
    if (a.splits > 1) {
        k_attn_combine<<<(unsigned)(a.s * a.Hq), 128, 0, st>>>(a);
        GB_CUDA(cudaGetLastError());
    }
}

}  // namespace gb
