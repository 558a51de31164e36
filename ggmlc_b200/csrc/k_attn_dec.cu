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

#include <mutex>
#include <string>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

__device__ __forceinline__ void rope_cs(const RopeTable& tab, int64_t p, int i, float& c, float& s) {
    if (tab.cs && p >= 0 && p < tab.n_pos) {
        const float2 v = tab.cs[p * (tab.n_dims / 2) + i];
        c = v.x;
        s = v.y;
    } else {
        float theta = (float)p;
        for (int k = 0; k < i; ++k) theta = __fmul_rn(theta, tab.theta_scale);
        c = (float)cos((double)theta);
        s = (float)sin((double)theta);
    }
}

// rotated value of element d (< hd) of a head vector src (f32, contiguous) at position p
__device__ __forceinline__ float rope_elem(const float* src, int d, int hd, const RopeTable& tab,
                                           int64_t p) {
    const int half = tab.n_dims / 2;
    if (d >= tab.n_dims) return src[d];
    const int i = d < half ? d : d - half;
    float c, s;
    rope_cs(tab, p, i, c, s);
    const float x0 = src[i], x1 = src[i + half];
    return d < half ? __fmaf_rn(x0, c, -__fmul_rn(x1, s)) : __fmaf_rn(x0, s, __fmul_rn(x1, c));
}

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
            a.kc[(h * a.ctx + p) * hd + d] = __float2half_rn(rope_elem(src, d, hd, a.tab, p));
        } else {
            const int64_t h = hh - a.Hq - a.Hkv;
            a.vc[(h * a.ctx + p) * hd + d] = __float2half_rn(row[a.v_off + h * hd + d]);
        }
    }
}

constexpr int kDecThreads = 128;
constexpr int kMaxRk = 8;     // q heads per KV head handled by one CTA
constexpr int kChunk = 64;    // positions staged per round trip
constexpr int kMaxOut = kMaxRk * 256 / kDecThreads;  // V outputs per thread

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

__global__ void __launch_bounds__(kDecThreads) k_attn_decode(AttnDecArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int hd = a.hd;
    const int rk = a.Hq / a.Hkv;
    __half* sk = (__half*)smem;                      // [kChunk][hd]
    __half* sv = sk + kChunk * hd;                   // [kChunk][hd]
    float* sq = (float*)(sv + kChunk * hd);          // [rk][hd] rotated q (fp16-rounded)
    float* ss = sq + rk * hd;                        // [rk][kChunk] scores / probabilities
    float* sstat = ss + rk * kChunk;                 // [rk][3] running max, sum, correction
    const int hk = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pos = (a.step ? a.step->pos : 0) + a.pos_off;  // position of the new token
    const int64_t nkv = pos + 1;
    const int64_t per = (nkv + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = (int64_t)blockIdx.x * per;
    const int64_t c1 = min(c0 + per, nkv);
    const float* row = a.qkv;
    const __half* kbase = a.kc + ((int64_t)hk * a.ctx) * hd;
    const __half* vbase = a.vc + ((int64_t)hk * a.ctx) * hd;
    const int vec = hd / 8;  // 16-byte pieces per row
    // the split holding the new position writes its k, v rows into the cache first
    const bool owns_new = c0 <= pos && pos < c1;
    if (owns_new) {
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            const float* ks = row + a.k_off + (int64_t)hk * hd;
            a.kc[((int64_t)hk * a.ctx + pos) * hd + d] = __float2half_rn(rope_elem(ks, d, hd, a.tab, pos));
            a.vc[((int64_t)hk * a.ctx + pos) * hd + d] = __float2half_rn(row[a.v_off + (int64_t)hk * hd + d]);
        }
        __syncthreads();  // the new row is read back below
    }
    // first chunk in flight while q is rotated
    auto stage = [&](int64_t cs, int rows) {
        for (int e = threadIdx.x; e < rows * vec * 2; e += blockDim.x) {
            const int r = e / (vec * 2), piece = e % (vec * 2);
            const int kv = piece >= vec;
            const int pc = piece - kv * vec;
            const __half* src = (kv ? vbase : kbase) + (cs + r) * hd + pc * 8;
            __half* dst = (kv ? sv : sk) + r * hd + pc * 8;
            cp_async16(dst, src);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (c0 < c1) stage(c0, (int)min((int64_t)kChunk, c1 - c0));
    for (int e = threadIdx.x; e < rk * hd; e += blockDim.x) {
        const int h = e / hd, d = e % hd;
        const float* src = row + a.q_off + (int64_t)(hk * rk + h) * hd;
        sq[h * hd + d] = __half2float(__float2half_rn(rope_elem(src, d, hd, a.tab, pos)));
    }
    for (int h = threadIdx.x; h < rk; h += blockDim.x) {
        sstat[h * 3 + 0] = -INFINITY;
        sstat[h * 3 + 1] = 0.0f;
        sstat[h * 3 + 2] = 1.0f;
    }
    float acc[kMaxOut];
#pragma unroll
    for (int k = 0; k < kMaxOut; ++k) acc[k] = 0.0f;
    const int per_lane = hd / 32;
    for (int64_t cs = c0; cs < c1; cs += kChunk) {
        const int rows = (int)min((int64_t)kChunk, c1 - cs);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // scores: one warp per position, lanes across head_dim
        for (int r = warp; r < rows; r += kDecThreads / 32) {
            float kv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < per_lane) kv[j] = __half2float(sk[r * hd + lane * per_lane + j]);
            for (int h = 0; h < rk; ++h) {
                float dot = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (j < per_lane) dot = __fmaf_rn(kv[j], sq[h * hd + lane * per_lane + j], dot);
                dot = warp_sum(dot);
                if (lane == 0) ss[h * kChunk + r] = __fmul_rn(dot, a.scale);
            }
        }
        __syncthreads();
        // online softmax statistics per head (one warp per head)
        for (int h = warp; h < rk; h += kDecThreads / 32) {
            float mx = -INFINITY;
            for (int r = lane; r < rows; r += 32) mx = fmaxf(mx, ss[h * kChunk + r]);
            mx = warp_max(mx);
            const float mold = sstat[h * 3 + 0];
            const float mnew = fmaxf(mold, mx);
            float l = 0.0f;
            for (int r = lane; r < rows; r += 32) {
                const float p = expf(ss[h * kChunk + r] - mnew);
                ss[h * kChunk + r] = p;
                l += p;
            }
            l = warp_sum(l);
            if (lane == 0) {
                const float corr = expf(mold - mnew);
                sstat[h * 3 + 0] = mnew;
                sstat[h * 3 + 1] = sstat[h * 3 + 1] * corr + l;
                sstat[h * 3 + 2] = corr;
            }
        }
        __syncthreads();
        // V accumulation: thread owns outputs e = tid + k*128 of the group's [rk][hd]
#pragma unroll
        for (int k = 0; k < kMaxOut; ++k) {
            const int e = threadIdx.x + k * kDecThreads;
            if (e < rk * hd) {
                const int h = e / hd, d = e % hd;
                float v = acc[k] * sstat[h * 3 + 2];
                for (int r = 0; r < rows; ++r)
                    v = __fmaf_rn(ss[h * kChunk + r], __half2float(sv[r * hd + d]), v);
                acc[k] = v;
            }
        }
        __syncthreads();  // chunk buffers are free again
        if (cs + kChunk < c1) stage(cs + kChunk, (int)min((int64_t)kChunk, c1 - cs - kChunk));
    }
    __syncthreads();
    float* part = a.part + ((int64_t)blockIdx.x * a.Hq + (int64_t)hk * rk) * (hd + 2);
    for (int h = threadIdx.x; h < rk; h += blockDim.x) {
        part[h * (hd + 2) + 0] = c0 < c1 ? sstat[h * 3 + 0] : -INFINITY;
        part[h * (hd + 2) + 1] = c0 < c1 ? sstat[h * 3 + 1] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kMaxOut; ++k) {
        const int e = threadIdx.x + k * kDecThreads;
        if (e < rk * hd) part[(e / hd) * (hd + 2) + 2 + e % hd] = acc[k];
    }
}

__global__ void k_attn_combine(AttnDecArgs a) {
    __shared__ float sw[256];
    __shared__ float sL;
    const int h = blockIdx.x;  // q head
    const int hd = a.hd;
    const int S = a.splits;
    const float* base = a.part + (int64_t)h * (hd + 2);
    const int64_t sstride = (int64_t)a.Hq * (hd + 2);
    if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (int sp = threadIdx.x; sp < S; sp += 32) M = fmaxf(M, base[sp * sstride]);
        M = warp_max(M);
        float L = 0.0f;
        for (int sp = threadIdx.x; sp < S; sp += 32) {
            const float m = base[sp * sstride];
            const float w = m == -INFINITY ? 0.0f : expf(m - M);
            sw[sp] = w;
            L += base[sp * sstride + 1] * w;
        }
        L = warp_sum(L);
        if (threadIdx.x == 0) sL = L;
    }
    __syncthreads();
    const float inv = sL == 0.0f ? 0.0f : 1.0f / sL;
    const int lane = threadIdx.x & 31;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f, v3 = 0.0f;
        int sp = 0;
        for (; sp + 4 <= S; sp += 4) {
            v0 += base[(sp + 0) * sstride + 2 + d] * sw[sp + 0];
            v1 += base[(sp + 1) * sstride + 2 + d] * sw[sp + 1];
            v2 += base[(sp + 2) * sstride + 2 + d] * sw[sp + 2];
            v3 += base[(sp + 3) * sstride + 2 + d] * sw[sp + 3];
        }
        for (; sp < S; ++sp) v0 += base[sp * sstride + 2 + d] * sw[sp];
        const float v = ((v0 + v1) + (v2 + v3)) * inv;
        if (a.o) a.o[(int64_t)h * hd + d] = v;
        if (a.oq) {  // blockDim.x == hd: warp w owns elements 32w..32w+31 of the head
            float d16, q;
            q8_block(v, lane, d16, q);
            a.oq[(int64_t)h * hd + d] = (int8_t)__float2int_rn(q);
            if (lane == 0) a.od[((int64_t)h * hd + d) / 32] = d16;
        }
    }
}

size_t dec_smem(int hd, int rk) {
    return (size_t)kChunk * hd * 2 * 2 + (size_t)rk * hd * 4 + (size_t)rk * kChunk * 4 + rk * 12;
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

int attn_decode_splits(int64_t Hkv, int64_t max_kv) {
    // about two CTAs per SM; each split then walks max_kv / splits positions
    int64_t s = (296 + Hkv - 1) / Hkv;
    if (s > max_kv) s = max_kv;
    if (s > 256) s = 256;
    return (int)(s < 1 ? 1 : s);
}

size_t attn_decode_workspace(int64_t Hq, int64_t hd, int splits) {
    return (size_t)splits * Hq * (hd + 2) * sizeof(float);
}

void launch_attn_decode(const AttnDecArgs& a, cudaStream_t st) {
    GB_CHECK(a.hd % 32 == 0 && a.hd <= 256, "attn_decode: head_dim must be a multiple of 32, <= 256");
    GB_CHECK(a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRk, "attn_decode: GQA group too large");
    GB_CHECK(a.splits >= 1 && a.splits <= 256, "attn_decode: bad split count");
    const size_t smem = dec_smem(a.hd, a.Hq / a.Hkv);
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    static unsigned configured = 0;
    if (!(configured & (1u << (dev & 31)))) {
        GB_CUDA(cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     100 * 1024));
        configured |= 1u << (dev & 31);
    }
    dim3 grid((unsigned)a.splits, (unsigned)a.Hkv);
    k_attn_decode<<<grid, kDecThreads, smem, st>>>(a);
    GB_CUDA(cudaGetLastError());
    k_attn_combine<<<(unsigned)a.Hq, (unsigned)a.hd, 0, st>>>(a);
    GB_CUDA(cudaGetLastError());
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
