// One-shot all-reduce (sum, fp32) of the tensor-parallel partial sums over peer memory.
//
// Every rank owns one device allocation, mapped into every other rank's process with CUDA IPC:
//   recv  [2][T][cap] floats   slot [parity][r] receives rank r's partial vector
//   flags [2][T][kArCtas]      epoch written by rank r once its part of slot [parity][r] is in
// A call with epoch e uses parity e & 1.  CTA c of every rank owns the same chunk of the vector:
// it stores its partial chunk into slot [parity][rank] of every rank (NVLink stores), raises its
// flag at every rank with a system-scope release, waits (bounded) until all T flags for its chunk
// in its own memory read e, and sums the T slots in rank order — so every rank ends with the
// same bits.  Epochs only grow (one counter per CTA, advanced by the CTA itself), so a flag
// left from an earlier call never matches; two parities suffice because a rank cannot start
// call k+1 before every peer has contributed to call k, which each does only after finishing
// call k-1 (the previous use of the same parity).
//
// A wait that runs past its limit (about 1 s) records 1 in the error word (mapped pinned host
// memory) and the call goes on, so the sum it writes is not valid; the executor raises on the
// next host synchronisation (every output read), and tp_allreduce_error reads the word.
#include <cuda_runtime.h>

#include "common.h"
#include "kernels.h"
#include "kutil.cuh"

namespace gb {

namespace {

constexpr int kArThreads = 512;
constexpr long long kArSpin = 2000000000LL;  // about 1 s at 1.9 GHz

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kArThreads)
    k_tp_allreduce(float* __restrict__ y, int64_t n, TpPeers peers, int rank, int T,
                   uint32_t* __restrict__ epochs, int64_t cap, int* __restrict__ err) {
    __shared__ uint32_t s_e;
    const int c = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) s_e = epochs[c] + 1;
    __syncthreads();
    const uint32_t e = s_e;
    const int par = (int)(e & 1u);
    // this CTA's chunk, in whole float4s
    const int64_t n4 = (n + 3) / 4;
    const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
    const int64_t a = (int64_t)c * per * 4, b = min(n, a + per * 4);
    const bool vec = (n % 4) == 0;
    for (int p = 0; p < T; ++p) {
        float* dst = peers.recv[p] + ((int64_t)par * T + rank) * cap;
        if (vec) {
            for (int64_t i = a + 4 * tid; i < b; i += 4 * kArThreads)
                *(float4*)(dst + i) = *(const float4*)(y + i);
        } else {
            for (int64_t i = a + tid; i < b; i += kArThreads) dst[i] = y[i];
        }
    }
    __syncthreads();
    if (tid < T) {  // thread p tells rank p that this chunk of slot [par][rank] is in
        __threadfence_system();
        st_release_sys(peers.flags[tid] + ((int64_t)par * T + rank) * kArCtas + c, e);
    }
    if (tid < T) {  // thread r waits for rank r's chunk in this rank's memory
        const uint32_t* f = peers.flags[rank] + ((int64_t)par * T + tid) * kArCtas + c;
        const long long t0 = clock64();
        while (ld_acquire_sys(f) != e) {
            if (clock64() - t0 > kArSpin) {
                *(volatile int*)err = 1;  // host-mapped word: a plain store, no atomic
                __threadfence_system();
                break;
            }
        }
    }
    __syncthreads();
    const float* src = peers.recv[rank] + (int64_t)par * T * cap;
    for (int64_t i = a + tid; i < b; i += kArThreads) {
        float s = __ldcg(src + i);
        for (int r = 1; r < T; ++r) s = __fadd_rn(s, __ldcg(src + (int64_t)r * cap + i));
        y[i] = s;
    }
    if (tid == 0) epochs[c] = e;
}

}  // namespace

void launch_tp_allreduce(float* y, int64_t n, const TpPeers& peers, int rank, int T,
                         uint32_t* epochs, int64_t cap, int* err, cudaStream_t st) {
    GB_CHECK(T >= 2 && T <= kMaxTp && rank >= 0 && rank < T, "tp all-reduce: bad rank / size");
    GB_CHECK(n >= 0 && n <= cap, "tp all-reduce: vector larger than the peer buffers");
    GB_CHECK(((uintptr_t)y & 15) == 0, "tp all-reduce: y must be 16-byte aligned");
    if (n == 0) return;
    k_tp_allreduce<<<kArCtas, kArThreads, 0, st>>>(y, n, peers, rank, T, epochs, cap, err);
    GB_CUDA(cudaGetLastError());
}

}  // namespace gb
