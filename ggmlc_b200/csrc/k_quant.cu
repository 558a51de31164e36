// Quantization-side kernels: Q8_0 activation quantization, GGUF block repack, GET_ROWS.
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

// One warp per 32-element block; lane j owns element j.  Reproduces quantize_row_q8_0 of the
// x86 AVX2 build (ggml-cpu/arch/x86/quants.c:302-392) bit for bit: amax = max|x|,
// d = fp16(amax / 127), id = amax ? 127 / amax : 0, q = round-half-even(x * id).
__global__ void k_quantize_q8_0(const float* __restrict__ x, int64_t x_stride, int64_t M,
                                int64_t K, int8_t* __restrict__ xq, float* __restrict__ xd) {
    const int64_t nb = K / QK;
    const int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (blk >= M * nb) return;
    const int lane = threadIdx.x & 31;
    const int64_t m = blk / nb, b = blk % nb;
    const float v = x[m * x_stride + b * QK + lane];
    float d16, q;
    q8_block(v, lane, d16, q);
    xq[m * K + b * QK + lane] = (int8_t)__float2int_rn(q);
    if (lane == 0) xd[m * nb + b] = d16;
}

void launch_quantize_q8_0(const float* x, int64_t x_stride, int64_t M, int64_t K, int8_t* xq,
                          float* xd, cudaStream_t st) {
    GB_CHECK(K % QK == 0, "quantize: K must be a multiple of 32");
    const int64_t blocks = M * (K / QK);
    if (blocks == 0) return;
    const int warps = 8;
    k_quantize_q8_0<<<(unsigned)((blocks + warps - 1) / warps), warps * 32, 0, st>>>(
        x, x_stride, M, K, xq, xd);
    GB_CUDA(cudaGetLastError());
}

// GGUF rows of 34-byte (Q8_0) / 18-byte (Q4_0) blocks -> split-row layout (kernels.h).  One
// thread per block; the source is 2-byte aligned, so it is read in 16-bit halves.
__global__ void k_repack(const uint8_t* __restrict__ src, int type, int64_t N, int64_t nb,
                         int64_t row_bytes, uint8_t* __restrict__ qs) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * nb) return;
    const int64_t row = i / nb, b = i % nb;
    const int bb = type == T_Q8_0 ? 34 : 18;
    const uint16_t* s = (const uint16_t*)(src + i * bb);
    uint8_t* rowp = qs + row * row_bytes;
    *(uint16_t*)(rowp + w_scale_off(type, nb, b)) = s[0];
    const int nwords = type == T_Q8_0 ? 8 : 4;
    for (int w = 0; w < nwords; ++w) {
        const uint32_t v = (uint32_t)s[1 + 2 * w] | ((uint32_t)s[2 + 2 * w] << 16);
        *(uint32_t*)(rowp + w_word_off(type, nb, b, w)) = v;
    }
}

void launch_repack_blocks(const uint8_t* gguf, int type, int64_t N, int64_t K, void* qs,
                          cudaStream_t st) {
    GB_CHECK(type == T_Q8_0 || type == T_Q4_0, "repack: not a block type");
    GB_CHECK(K % QK == 0, "repack: K must be a multiple of 32");
    const int64_t nb = K / QK;
    if (!N || !nb) return;
    const int64_t rb = qrow_bytes(type, K);
    GB_CUDA(cudaMemsetAsync(qs, 0, (size_t)(N * rb), st));
    const int64_t n = N * nb;
    k_repack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(gguf, type, N, nb, rb, (uint8_t*)qs);
    GB_CUDA(cudaGetLastError());
}

// GET_ROWS with dequantization: y = q * d (one rounded fp32 product, as dequantize_row_q8_0 /
// _q4_0 in ggml-quants.c:459-477, :553-567).
__global__ void k_get_rows(QWeight w, const int32_t* __restrict__ ids, int64_t n,
                           float* __restrict__ out, int64_t out_stride) {
    const int64_t r = blockIdx.y;
    if (r >= n) return;
    const int64_t K = w.K;
    int64_t row = ids[r];
    const bool ok = row >= 0 && row < w.N;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K;
         k += (int64_t)gridDim.x * blockDim.x) {
        float v = 0.0f;
        if (ok) {
            const int64_t b = k / QK, e = k % QK, nb = K / QK;
            const uint8_t* q = (const uint8_t*)w.qs + row * qrow_bytes(w.type, K);
            if (w.type == T_Q8_0 || w.type == T_Q4_0) {
                const float d = __half2float(*(const __half*)(q + w_scale_off(w.type, nb, b)));
                if (w.type == T_Q8_0) {
                    const int8_t qv = (int8_t)q[w_word_off(T_Q8_0, nb, b, (int)(e >> 2)) + (e & 3)];
                    v = __fmul_rn((float)qv, d);
                } else {
                    const int64_t j = e & 15;
                    const uint8_t byte = q[w_word_off(T_Q4_0, nb, b, (int)(j >> 2)) + (j & 3)];
                    const int nib = e < 16 ? (byte & 0x0F) : (byte >> 4);
                    v = __fmul_rn((float)(nib - 8), d);
                }
            } else if (w.type == T_F16) {
                v = __half2float(((const __half*)w.qs)[row * K + k]);
            } else {
                v = ((const float*)w.qs)[row * K + k];
            }
        }
        out[r * out_stride + k] = v;
    }
}

// Greedy token per row: the index of the first maximum (the reference's sample_next_token with
// temperature 0, batch_scheduler.cpp:94-106).  One CTA per row; ties keep the lowest index.
__global__ void k_argmax_rows(const float* __restrict__ x, int64_t n, int32_t* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int64_t si[32];
    const float* row = x + (int64_t)blockIdx.x * n;
    float best = -INFINITY;
    int64_t bi = n;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (v > best || (v == best && i < bi)) {
            best = v;
            bi = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, best, o);
        const int64_t j = __shfl_xor_sync(0xffffffffu, bi, o);
        if (v > best || (v == best && j < bi)) {
            best = v;
            bi = j;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
            if (sv[k] > best || (sv[k] == best && si[k] < bi)) {
                best = sv[k];
                bi = si[k];
            }
        out[blockIdx.x] = (int32_t)(bi < n ? bi : 0);
    }
}

void launch_argmax_rows(const float* x, int64_t rows, int64_t n, int32_t* out, cudaStream_t st) {
    if (!rows) return;
    k_argmax_rows<<<(unsigned)rows, 1024, 0, st>>>(x, n, out);
    GB_CUDA(cudaGetLastError());
}

void launch_get_rows(const QWeight& w, const int32_t* ids, int64_t n, float* out,
                     int64_t out_stride, cudaStream_t st) {
    if (!n) return;
    dim3 grid((unsigned)((w.K + 255) / 256), (unsigned)n);
    k_get_rows<<<grid, 256, 0, st>>>(w, ids, n, out, out_stride);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
