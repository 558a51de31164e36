// Elementwise kernels over strided 4-D views: ADD / MUL with ggml broadcasting (ggml_add /
// ggml_mul repeat src1 over src0) and CONT / CPY with type conversion.
#include <cuda_fp16.h>

#include <mutex>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

__device__ __forceinline__ float ld(const TView& v, const int64_t* i) {
    const char* p = v.data + i[0] * v.nb[0] + i[1] * v.nb[1] + i[2] * v.nb[2] + i[3] * v.nb[3];
    switch (v.type) {
        case T_F16: return __half2float(*(const __half*)p);
        case T_I32: return (float)*(const int32_t*)p;
        default: return *(const float*)p;
    }
}

__global__ void k_binary(TView a, TView b, TView d, int op) {
    const int64_t total = a.ne[0] * a.ne[1] * a.ne[2] * a.ne[3];
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i[4], j[4];
        int64_t r = idx;
        for (int k = 0; k < 4; ++k) {
            i[k] = r % a.ne[k];
            r /= a.ne[k];
            j[k] = i[k] % b.ne[k];
        }
        const float x = ld(a, i), y = ld(b, j);
        const float v = op == 0 ? __fadd_rn(x, y) : __fmul_rn(x, y);
        *(float*)(d.data + i[0] * d.nb[0] + i[1] * d.nb[1] + i[2] * d.nb[2] + i[3] * d.nb[3]) = v;
    }
}

__global__ void k_copy(TView s, TView d) {
    const int64_t total = s.ne[0] * s.ne[1] * s.ne[2] * s.ne[3];
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i[4], j[4];
        int64_t r = idx;
        for (int k = 0; k < 4; ++k) {
            i[k] = r % s.ne[k];
            r /= s.ne[k];
        }
        r = idx;  // destination walks its own shape in the same linear order
        for (int k = 0; k < 4; ++k) {
            j[k] = r % d.ne[k];
            r /= d.ne[k];
        }
        char* q = d.data + j[0] * d.nb[0] + j[1] * d.nb[1] + j[2] * d.nb[2] + j[3] * d.nb[3];
        if (s.type == T_I32 && d.type == T_I32) {
            const char* p = s.data + i[0] * s.nb[0] + i[1] * s.nb[1] + i[2] * s.nb[2] + i[3] * s.nb[3];
            *(int32_t*)q = *(const int32_t*)p;
            continue;
        }
        const float v = ld(s, i);
        if (d.type == T_F16) *(__half*)q = __float2half_rn(v);
        else if (d.type == T_I32) *(int32_t*)q = (int32_t)v;
        else *(float*)q = v;
    }
}

__global__ void k_gather_rows(const float* __restrict__ x, int64_t x_stride,
                              const StepParams* __restrict__ step, int64_t K, float* __restrict__ y) {
    const int r = blockIdx.x;
    const float* src = x + (int64_t)step->out_rows[r] * x_stride;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) y[(int64_t)r * K + k] = src[k];
}

unsigned grid_for(int64_t total) {
    int64_t b = (total + 255) / 256;
    if (b > 148 * 32) b = 148 * 32;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

void launch_binary(const TView& a, const TView& b, const TView& dst, int op, cudaStream_t st) {
    const int64_t total = a.ne[0] * a.ne[1] * a.ne[2] * a.ne[3];
    if (!total) return;
    for (int k = 0; k < 4; ++k)
        GB_CHECK(b.ne[k] > 0 && a.ne[k] % b.ne[k] == 0, "binary op: operand cannot be broadcast");
    k_binary<<<grid_for(total), 256, 0, st>>>(a, b, dst, op);
    GB_CUDA(cudaGetLastError());
}

void launch_gather_rows(const float* x, int64_t x_stride, const StepParams* step, int n, int64_t K,
                        float* y, cudaStream_t st) {
    GB_CHECK(n >= 1 && n <= kMaxOutRows, "gather rows: 1..64 rows");
    k_gather_rows<<<(unsigned)n, 256, 0, st>>>(x, x_stride, step, K, y);
    GB_CUDA(cudaGetLastError());
}

void launch_copy(const TView& src, const TView& dst, cudaStream_t st) {
    const int64_t total = src.ne[0] * src.ne[1] * src.ne[2] * src.ne[3];
    if (!total) return;
    k_copy<<<grid_for(total), 256, 0, st>>>(src, dst);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb

namespace gb {

int sm_count(int dev) {
    static std::mutex mu;
    static int cache[64] = {};
    GB_CHECK(dev >= 0 && dev < 64, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        GB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        cache[dev] = n > 0 ? n : 1;
    }
    return cache[dev];
}

}  // namespace gb
