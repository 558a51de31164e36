// Decode GEMV (M <= 4 activation rows; the engine sends it 1-2) over the split-row weight layout, with an optional fused
// RMSNorm + Q8_0 prologue and a bias / residual / SwiGLU epilogue.
//
// Arithmetic.  Per 32-element block the integer dot sumi = sum q_w * q_x is exact (dp4a chain),
// and the output accumulates fp32 block terms sumi * (d_w * d_x), the block formula of the
// reference's generic kernels (ggml-cpu/quants.c:225-256 Q4_0, :451-477 Q8_0).  The x86 build
// splits each block over 8 SIMD lanes instead; the fp32 results agree to rounding (the integer
// parts are identical).  Activations are quantized exactly like the x86 build
// (arch/x86/quants.c:302-392).
//
// Work mapping.  Lanes run along K: lane l of a warp takes blocks l, l+32, l+64, ... of a row, so
// each 16-byte load of a warp reads 512 contiguous bytes.  A lane holds G blocks of one row in
// registers ("group"); the next group (possibly of the warp's next row) is loaded before the
// current one is consumed, so every warp keeps one group of loads in flight.  The Q8_0
// activations live in shared memory, split into words 0-3 and 4-7 of each block so the lanes'
// 16-byte reads are conflict-free.  A row's lane sums are combined by a fixed xor-butterfly.
// Plain outputs: rows are dealt to all warps of the grid.  SwiGLU: a CTA owns 32 consecutive
// outputs (row pairs n, F+n) so it can emit each Q8_0 block of the result itself.
//
// Q4_0 nibbles become int8 with a shift and two bitwise ops: (q<<4) ^ 0x80 read as int8 is
// 16*(q-8); the activation scales are staged divided by 16 (exact), so the products are
// unchanged.  int -> float of the block sum uses the 1.5*2^23 bias trick (exact for |v| < 2^22).
//
// Launch: programmatic dependent launch.  The first group of weights is requested before
// griddepcontrol.wait, so the weight stream of this launch overlaps the tail of the previous one;
// all reads of activations and all writes happen after the wait.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr size_t kSmemMax = 224 * 1024;  // dynamic; static shared memory needs the rest of 227 KB


__device__ __forceinline__ float block_sum_f(int s) {
    return __fsub_rn(__int_as_float(s), 12582912.0f);
}

// A step covers 64 blocks of one row: lane l takes blocks 64g + l and 64g + 32 + l and their two
// scales (one 4-byte word of the scale region).  Each warp streams its steps through a ring of
// kDepth shared-memory slots with cp.async; a lane only ever reads what it copied itself, so no
// synchronization beyond cp.async.wait_group is needed.
constexpr int kDepth = 3;

template <int WT>
struct Slot {  // bytes of one ring slot (one step of one warp)
    static constexpr int kQuant = (WT == T_Q8_0 ? 4 : 2) * 32 * 16;  // [piece][lane][16 B]
    static constexpr int kBytes = kQuant + 32 * 4;                    // + [lane][2 scales]
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// copy step g of a row into a ring slot (blocks >= nb are skipped: their scales are zero)
template <int WT>
__device__ __forceinline__ void issue_step(uint8_t* slot, const uint8_t* row, int nb, int g,
                                           int lane) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int b = g * 64 + i * 32 + lane;
        if (b < nb) {
            if (WT == T_Q8_0) {
                cp_async16(slot + ((2 * i) * 32 + lane) * 16, row + (int64_t)b * 16);
                cp_async16(slot + ((2 * i + 1) * 32 + lane) * 16, row + (int64_t)(nb + b) * 16);
            } else {
                cp_async16(slot + (i * 32 + lane) * 16, row + (int64_t)b * 16);
            }
        }
    }
    cp_async4(slot + Slot<WT>::kQuant + lane * 4,
              row + (int64_t)nb * quant_bytes(WT) + (int64_t)g * 128 + lane * 4);
}

// accumulate the two blocks of a landed step against the staged activations
template <int WT, int MAXM>
__device__ __forceinline__ void consume(const uint8_t* slot, int g, int lane, int M,
                                        const uint4* sxa, const uint4* sxb, const float* sxd,
                                        int nbp, float (&acc)[MAXM]) {
    const unsigned sc = *(const unsigned*)(slot + Slot<WT>::kQuant + lane * 4);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int b = g * 64 + i * 32 + lane;
        int lo[4], hi[4];
        if (WT == T_Q4_0) {
            const uint4 q = *(const uint4*)(slot + (i * 32 + lane) * 16);
            const unsigned w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                lo[j] = (int)(((w[j] << 4) & 0xF0F0F0F0u) ^ 0x80808080u);  // 16*(q_lo - 8)
                hi[j] = (int)((w[j] & 0xF0F0F0F0u) ^ 0x80808080u);         // 16*(q_hi - 8)
            }
        } else {
            const uint4 qa = *(const uint4*)(slot + ((2 * i) * 32 + lane) * 16);
            const uint4 qb = *(const uint4*)(slot + ((2 * i + 1) * 32 + lane) * 16);
            lo[0] = (int)qa.x; lo[1] = (int)qa.y; lo[2] = (int)qa.z; lo[3] = (int)qa.w;
            hi[0] = (int)qb.x; hi[1] = (int)qb.y; hi[2] = (int)qb.z; hi[3] = (int)qb.w;
        }
        const float dw = __half2float(__ushort_as_half((unsigned short)(i ? sc >> 16 : sc & 0xFFFF)));
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                const uint4 xa = sxa[m * nbp + b];
                const uint4 xb = sxb[m * nbp + b];
                const float dx = sxd[m * nbp + b];
                int s = 0x4B400000;
                s = __dp4a(lo[0], (int)xa.x, s);
                s = __dp4a(lo[1], (int)xa.y, s);
                s = __dp4a(lo[2], (int)xa.z, s);
                s = __dp4a(lo[3], (int)xa.w, s);
                s = __dp4a(hi[0], (int)xb.x, s);
                s = __dp4a(hi[1], (int)xb.y, s);
                s = __dp4a(hi[2], (int)xb.z, s);
                s = __dp4a(hi[3], (int)xb.w, s);
                acc[m] = __fmaf_rn(block_sum_f(s), __fmul_rn(dw, dx), acc[m]);
            }
        }
    }
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ double block_sum_d(double v, double* sh) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < kWarps; ++i) t += sh[i];
    return t;
}

// Stage the M activation rows as Q8_0 in shared memory: sxa/sxb = words 0-3 / 4-7 of each block,
// sxd = fp32 scales (divided by 16 for Q4_0 weights); blocks nb..nbp-1 are zero.
struct StageIn {  // the GemvArgs fields the prologue reads, passed by value
    const int8_t* xq;
    const float* xd;
    const float* xf;
    int64_t xf_stride;
    const float* gamma;
    float eps;
    int M, K;
    bool xf_rms;
};

template <int WT>
__device__ __noinline__ void stage_x(const StageIn a, int nb, int nbp, uint4* sxa, uint4* sxb,
                                     float* sxd, float* sxf, const float* sgm, double* shd) {
    const int K = a.K;
    const float dscale = WT == T_Q4_0 ? 0.0625f : 1.0f;
    if (!a.xf) {
        for (int idx = threadIdx.x; idx < a.M * nbp; idx += kThreads) {
            const int m = idx / nbp, b = idx % nbp;
            uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
            float d = 0.0f;
            if (b < nb) {
                const int4* src = (const int4*)(a.xq + (int64_t)m * K + (int64_t)b * 32);
                const int4 p = src[0], q = src[1];
                va = make_uint4(p.x, p.y, p.z, p.w);
                vb = make_uint4(q.x, q.y, q.z, q.w);
                d = __fmul_rn(a.xd[(int64_t)m * nb + b], dscale);
            }
            sxa[idx] = va;
            sxb[idx] = vb;
            sxd[idx] = d;
        }
        return;
    }
    // f32 rows: the row is copied to shared memory with coalesced 16-byte loads (sxf: 33 floats
    // per block, so lanes walking their own half-blocks hit distinct banks), the sum of squares
    // taken on the way; then two lanes per block apply the scale and gamma (staged in sgm the same
    // way) and quantize — quantize_row_q8_0's per-block steps, each element's arithmetic
    // unchanged.
    const bool vec4 = ((uintptr_t)a.xf & 15) == 0 && (a.xf_stride & 3) == 0;
    for (int m = 0; m < a.M; ++m) {
        const float* xr = a.xf + (int64_t)m * a.xf_stride;
        double s0 = 0.0, s1 = 0.0;
        if (vec4) {
#pragma unroll 4
            for (int k4 = threadIdx.x; k4 < K / 4; k4 += kThreads) {
                const float4 t = __ldg((const float4*)xr + k4);
                float* d = sxf + (k4 >> 3) * 33 + (k4 & 7) * 4;
                d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
                s0 += (double)__fmul_rn(t.x, t.x) + (double)__fmul_rn(t.y, t.y);
                s1 += (double)__fmul_rn(t.z, t.z) + (double)__fmul_rn(t.w, t.w);
            }
        } else {
#pragma unroll 4
            for (int k = threadIdx.x; k < K; k += kThreads) {
                const float t = __ldg(xr + k);
                sxf[(k >> 5) * 33 + (k & 31)] = t;
                s0 += (double)__fmul_rn(t, t);
            }
        }
        float scale = 1.0f;
        if (a.xf_rms) {
            // RMSNorm (ggml-cpu/ops.cpp:3859-3920): fp32 squares summed in double
            const double s = block_sum_d(s0 + s1, shd);
            const float mean = (float)(s / (double)K);
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        } else {
            __syncthreads();
        }
        // two lanes per block (elements 0-15 and 16-31 = words 0-3 and 4-7); the block's amax
        // is combined with one shuffle.  2 * nbp is a multiple of 128, so whole warps take part.
        for (int it = threadIdx.x; it < 2 * nbp; it += kThreads) {
            const int b = it >> 1, hh = it & 1;
            float v[16];
            float amax = 0.0f;
            if (b < nb) {
                const float* xb = sxf + b * 33 + hh * 16;
                const float* gb_ = sgm + b * 33 + hh * 16;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float t = xb[i];
                    if (a.xf_rms) t = __fmul_rn(t, scale);
                    if (a.gamma) t = __fmul_rn(t, gb_[i]);
                    v[i] = t;
                    amax = fmaxf(amax, fabsf(t));
                }
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            uint4 qw = make_uint4(0, 0, 0, 0);
            float d16 = 0.0f;
            if (b < nb) {
                // quantize_row_q8_0, x86 AVX2 build (arch/x86/quants.c:302-392)
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
                qw = make_uint4(w[0], w[1], w[2], w[3]);
            }
            if (hh == 0) {
                sxa[m * nbp + b] = qw;
                sxd[m * nbp + b] = __fmul_rn(d16, dscale);
            } else {
                sxb[m * nbp + b] = qw;
            }
        }
        __syncthreads();  // sxf is reused by the next row
    }
}

// gamma staged like sxf (33 floats per block); it is a weight, so this runs before the
// dependency wait
__device__ __forceinline__ void stage_gamma(const float* gamma, int K, float* sgm) {
    for (int k = threadIdx.x; k < K; k += kThreads) sgm[(k >> 5) * 33 + (k & 31)] = __ldg(gamma + k);
}

struct Geo {
    int nb, nbp, ng;  // blocks per row, padded to whole steps (64 blocks), steps per row
};

__host__ __device__ inline Geo make_geo(int64_t K) {
    Geo g;
    g.nb = (int)(K / 32);
    g.ng = (g.nb + 63) / 64;
    g.nbp = g.ng * 64;
    return g;
}

// SWI = 0: rows dealt to the warps of the grid.  SWI = 1: CTA tiles of 32 SwiGLU outputs.
template <int WT, int MAXM, int SWI>
__global__ void __launch_bounds__(kThreads, MAXM <= 2 ? 4 : 2) k_gemv(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double shd[kWarps];
    __shared__ float sres[SWI ? MAXM * 32 : 1];
    const Geo geo = make_geo(a.w.K);
    const int nb = geo.nb, nbp = geo.nbp, ng = geo.ng;
    const int N = (int)a.w.N;
    const int64_t rb = qrow_bytes(WT, a.w.K);
    const uint8_t* qs = (const uint8_t*)a.w.qs;
    uint4* sxa = (uint4*)smem;
    uint4* sxb = sxa + MAXM * nbp;
    float* sxd = (float*)(sxb + MAXM * nbp);
    float* sxf = sxd + MAXM * nbp;                        // f32 input row, 33 floats per block
    float* sgm = sxf + (a.xf ? nbp * 33 : 0);             // gamma, same layout
    uint8_t* ring = (uint8_t*)(sgm + (a.xf && a.gamma ? nbp * 33 : 0));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* wring = ring + warp * kDepth * Slot<WT>::kBytes;

    const int F = (int)a.F;
    const int gw = blockIdx.x * kWarps + warp;
    const int tw = gridDim.x * kWarps;
    // row k of this warp's sequence in a tile
    auto row_of = [&](int tile, int k) -> int {
        if (SWI) {  // pair tile*32 + warp*4 + k/2: gate row, then up row
            const int p = tile * 32 + warp * 4 + (k >> 1);
            return (k & 1) ? F + p : p;
        }
        return gw + k * tw;
    };
    const int rpt = SWI ? 8 : (gw < N ? (N - gw + tw - 1) / tw : 0);  // rows per tile
    const int ntiles = SWI ? F / 32 : 1;
    const int tstep = SWI ? (int)gridDim.x : 1;
    const int tile0 = SWI ? (int)blockIdx.x : 0;
    // step cursors (tile, row, step of the row): issue runs kDepth - 1 steps ahead of consume
    int it = tile0, ik = 0, ig = 0, islot = 0;
    auto issue = [&]() {
        if (it < ntiles && ik < rpt) {
            issue_step<WT>(wring + islot * Slot<WT>::kBytes, qs + (int64_t)row_of(it, ik) * rb, nb,
                           ig, lane);
            if (++ig == ng) {
                ig = 0;
                if (++ik == rpt) {
                    ik = 0;
                    it += tstep;
                }
            }
        }
        cp_commit();
        islot = islot + 1 == kDepth ? 0 : islot + 1;
    };
#pragma unroll
    for (int d = 0; d < kDepth - 1; ++d) issue();
    if (a.xf && a.gamma) stage_gamma(a.gamma, (int)a.w.K, sgm);
    pdl_wait();
    pdl_launch();
    stage_x<WT>(StageIn{a.xq, a.xd, a.xf, a.xf_stride, a.gamma, a.eps, a.M, (int)a.w.K, a.xf_rms},
                nb, nbp, sxa, sxb, sxd, sxf, sgm, shd);
    __syncthreads();

    float acc[MAXM], gate[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) acc[m] = gate[m] = 0.0f;
    int ct = tile0, ck = 0, cg = 0, cslot = 0;
    while (ct < ntiles && ck < rpt) {
        issue();
        cp_wait<kDepth - 1>();
        consume<WT, MAXM>(wring + cslot * Slot<WT>::kBytes, cg, lane, a.M, sxa, sxb, sxd, nbp, acc);
        cslot = cslot + 1 == kDepth ? 0 : cslot + 1;
        if (cg == ng - 1) {  // row ck complete
            const int row = row_of(ct, ck);
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < a.M) {
                    float r = warp_allsum(acc[m]);
                    acc[m] = 0.0f;
                    if (SWI) {
                        if (ck & 1) {
                            if (lane == 0)
                                sres[m * 32 + warp * 4 + (ck >> 1)] = __fmul_rn(ref_v_silu(gate[m]), r);
                        } else {
                            gate[m] = r;
                        }
                    } else if (lane == m) {
                        if (a.bias) r = __fadd_rn(r, a.bias[row]);
                        if (a.residual) r = __fadd_rn(a.residual[(int64_t)m * a.res_stride + row], r);
                        a.y[(int64_t)m * a.y_stride + row] = r;
                    }
                }
            }
            if (SWI && ck == rpt - 1) {
                // ggml_vec_swiglu_f32 (vec.cpp:417-426) outputs of this tile, f32 and/or Q8_0
                __syncthreads();
                for (int m = warp; m < a.M; m += kWarps) {
                    const float h = sres[m * 32 + lane];
                    const int64_t col = (int64_t)ct * 32 + lane;
                    if (a.y) a.y[(int64_t)m * a.y_stride + col] = h;
                    if (a.yq) {
                        float d16, q;
                        q8_block(h, lane, d16, q);
                        a.yq[(int64_t)m * a.F + col] = (int8_t)__float2int_rn(q);
                        if (lane == 0) a.yd[(int64_t)m * (a.F / 32) + ct] = d16;
                    }
                }
                __syncthreads();
            }
        }
        if (++cg == ng) {
            cg = 0;
            if (++ck == rpt) {
                ck = 0;
                ct += tstep;
            }
        }
    }
}

template <int WT>
size_t smem_bytes(int maxm, int64_t K, bool xf, bool gamma) {
    const Geo g = make_geo(K);
    return (size_t)maxm * g.nbp * 36 + (xf ? (size_t)g.nbp * 33 * 4 * (gamma ? 2 : 1) : 0) +
           (size_t)kWarps * kDepth * Slot<WT>::kBytes;
}

template <int WT, int MAXM, int SWI>
void launch_t(const GemvArgs& a, cudaStream_t st) {
    auto kern = k_gemv<WT, MAXM, SWI>;
    const size_t smem = smem_bytes<WT>(MAXM, a.w.K, a.xf != nullptr, a.gamma != nullptr);
    GB_CHECK(smem <= kSmemMax, "gemv: activation stage too large for shared memory");
    int dev = 0;
    GB_CUDA(cudaGetDevice(&dev));
    GB_CHECK(dev >= 0 && dev < 64, "gemv: device ordinal out of range");
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemMax));
            configured[dev] = true;
        }
    }
    int per_sm = 0;
    GB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
    const int64_t want = SWI ? a.F / 32 : (a.w.N + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)sm_count(dev) * std::max(per_sm, 1);
    launch_pdl(kern, (unsigned)std::min(want, cap), kThreads, smem, st, a);
}

template <int WT, int SWI>
void launch_m(const GemvArgs& a, cudaStream_t st) {
    if (a.M == 1) launch_t<WT, 1, SWI>(a, st);
    else if (a.M == 2) launch_t<WT, 2, SWI>(a, st);
    else launch_t<WT, 4, SWI>(a, st);
}

}  // namespace

static int maxm_of(int M) { return M == 1 ? 1 : (M == 2 ? 2 : 4); }

bool gemv_fits(int type, int64_t K, int M, bool staged, bool gamma) {
    if (M < 1 || M > kGemvMaxRows || K % QK != 0) return false;
    const size_t b = type == T_Q8_0 ? smem_bytes<T_Q8_0>(maxm_of(M), K, staged, gamma)
                                    : smem_bytes<T_Q4_0>(maxm_of(M), K, staged, gamma);
    return b <= kSmemMax;
}

bool gemv_fused_fits(int64_t K, int M) {
    return gemv_fits(T_Q8_0, K, M, false, false) && gemv_fits(T_Q4_0, K, M, false, false);
}

void launch_gemv_fused(const GemvArgs& a, cudaStream_t st) {
    if (!a.xf && a.M > kMmvMaxRows) {  // prefill: the block GEMM
        if (a.swiglu) {
            launch_gemm_swiglu(a, st);
        } else {
            MatmulEpilogue ep;
            ep.bias = a.bias;
            ep.residual = a.residual;
            ep.res_stride = a.res_stride;
            launch_matmul_q(a.w, a.xq, a.xd, a.M, a.y, a.y_stride, ep, st);
        }
        return;
    }
    if (a.M <= kGemvRouteRows && dgemv_eligible(a)) {  // 1-2 rows: the bulk-copy GEMV
        launch_dgemv(a, st);
        return;
    }
    GB_CHECK(a.ar.T == 0, "gemv: the epilogue all-reduce needs the single-row decode GEMV");
    if (!a.xf && (a.M > kGemvRouteRows || !gemv_fits(a.w.type, a.w.K, a.M, false, false))) {
        launch_mmv(a, st);  // batched decode: the tensor-core kernel
        return;
    }
    GB_CHECK(a.w.type == T_Q8_0 || a.w.type == T_Q4_0, "gemv: quantized weights required");
    GB_CHECK(a.w.K % QK == 0 && a.w.K < (1LL << 30) && a.w.N < (1LL << 30), "gemv: bad shape");
    GB_CHECK(gemv_fits(a.w.type, a.w.K, a.M, a.xf != nullptr, a.gamma != nullptr),
             "gemv: M or K too large for the shared-memory stage");
    GB_CHECK(!a.swiglu || (a.w.N == 2 * a.F && a.F % 32 == 0),
             "gemv: SwiGLU needs N == 2F, F % 32 == 0");
    GB_CHECK(a.swiglu || (!a.yq && !a.yd), "gemv: Q8_0 output only with SwiGLU");
    GB_CHECK(a.swiglu ? (a.y || a.yq) : a.y != nullptr, "gemv: no output");
    GB_CHECK(!a.yq == !a.yd, "gemv: Q8_0 output needs quants and scales");
    GB_CHECK(a.xf || (a.xq && a.xd), "gemv: no input");
    if (a.w.N == 0 || a.M == 0) return;
    if (a.w.type == T_Q8_0) {
        if (a.swiglu) launch_m<T_Q8_0, 1>(a, st);
        else launch_m<T_Q8_0, 0>(a, st);
    } else {
        if (a.swiglu) launch_m<T_Q4_0, 1>(a, st);
        else launch_m<T_Q4_0, 0>(a, st);
    }
}

}  // namespace gb
