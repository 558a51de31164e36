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
            __half* row = kv.base + (h * kv.ctx + base + t) * hd;
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
        kv.base[(h * kv.ctx + base + t) * hd + d] = __float2half_rn(load_f(src, d, h, t));
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
    const __half* kc;     // [Hkv][ctx][hd]
    const __half* vc;
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
        const __half* kb = a.kc + (hk * a.ctx + tile) * hd;
        const __half* vb = a.vc + (hk * a.ctx + tile) * hd;
        for (int64_t e = threadIdx.x; e < rows * hd; e += blockDim.x) {
            const int64_t r = e / hd, d = e % hd;
            sk[r * kstride + d] = kb[e];
            sv[r * hd + d] = vb[e];
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
                      float scale, float* o, void* work, int64_t max_kv, cudaStream_t st) {
    AttnArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
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
