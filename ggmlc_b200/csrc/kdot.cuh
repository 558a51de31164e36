// Device helpers of the bulk-copy GEMVs (k_dgemv.cu, k_chain.cu): mbarrier waits with a bound,
// bulk copies of weight bytes into shared memory, and the exact Q4_0 / Q8_0 block dot against a
// Q8_0 activation block.
//
// Block dot.  The integer dot of a 32-element block is exact.  Q4_0: the low nibbles (elements
// 0-15) and the high nibbles (16-31) are masked out of each 32-bit word as unsigned bytes and
// dotted with the signed activation bytes (dp4a.u32.s32); the high-nibble chain sees 16 * q, so
// its sum is shifted right by 4 (exact), and the -8 offset of every weight is folded into the
// chain's start value, -8 * sum(x) of the block.  The chain starts at 1.5 * 2^23, so the int sum
// becomes a float by one subtraction (exact for |sum| < 2^22).  The block term
// sumi * (d_w * d_x) accumulates in fp32.  This is the reference's block formula
// (ggml-cpu/quants.c:225-256 Q4_0, :451-477 Q8_0).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "common.h"

namespace gb {
namespace {

constexpr long long kSpinCycles = 4000000000LL;  // bound of one wait: about 2 s at 1.9 GHz
constexpr int kMagic = 0x4B400000;               // 1.5 * 2^23

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// wait for phase `parity` of an mbarrier to complete; false when the bound ran out
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_test(b, parity))
        if (clock64() - t0 > kSpinCycles) return false;
    return true;
}
// bulk copy (the TMA engine's linear mode) of `bytes` global bytes into shared memory, completing
// on mbarrier `bar` (both addresses 16-byte aligned, bytes a multiple of 16)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One activation block as a lane holds it.
struct XBlk {
    int4 lo, hi;  // quants of elements 0-15, 16-31
    float d;      // scale
    int init;     // dot-chain start: 1.5 * 2^23 (Q8_0 weights), minus 8 * sum(q) for Q4_0
};

// sum(q) of a block's 32 quants
__device__ __forceinline__ int qsum(const int4& lo, const int4& hi) {
    const int one = 0x01010101;
    int s = __dp4a(lo.x, one, 0);
    s = __dp4a(lo.y, one, s);
    s = __dp4a(lo.z, one, s);
    s = __dp4a(lo.w, one, s);
    s = __dp4a(hi.x, one, s);
    s = __dp4a(hi.y, one, s);
    s = __dp4a(hi.z, one, s);
    return __dp4a(hi.w, one, s);
}

template <int WT>
__device__ __forceinline__ int chain_init(const int4& lo, const int4& hi) {
    return WT == T_Q4_0 ? kMagic - 8 * qsum(lo, hi) : kMagic;
}

// One weight block as the lanes consume it.  Q4_0: a = low nibbles (elements 0-15) and b = high
// nibbles times 16 (elements 16-31), both as unsigned bytes; Q8_0: a, b = quant bytes 0-15, 16-31.
struct WBlk {
    uint4 a, b;
};

// acc += sumi * (d_w * d_x) of a weight block against one activation block
template <int WT>
__device__ __forceinline__ void block_term(const WBlk& w, float dw, const XBlk& x, float& acc) {
    int s = x.init;
    if (WT == T_Q4_0) {
        int sh = 0;
        s = dp4a_us(w.a.x, x.lo.x, s);
        s = dp4a_us(w.a.y, x.lo.y, s);
        s = dp4a_us(w.a.z, x.lo.z, s);
        s = dp4a_us(w.a.w, x.lo.w, s);
        sh = dp4a_us(w.b.x, x.hi.x, sh);
        sh = dp4a_us(w.b.y, x.hi.y, sh);
        sh = dp4a_us(w.b.z, x.hi.z, sh);
        sh = dp4a_us(w.b.w, x.hi.w, sh);
        s += sh >> 4;
    } else {
        s = __dp4a((int)w.a.x, x.lo.x, s);
        s = __dp4a((int)w.a.y, x.lo.y, s);
        s = __dp4a((int)w.a.z, x.lo.z, s);
        s = __dp4a((int)w.a.w, x.lo.w, s);
        s = __dp4a((int)w.b.x, x.hi.x, s);
        s = __dp4a((int)w.b.y, x.hi.y, s);
        s = __dp4a((int)w.b.z, x.hi.z, s);
        s = __dp4a((int)w.b.w, x.hi.w, s);
    }
    acc = __fmaf_rn(__fsub_rn(__int_as_float(s), 12582912.0f), __fmul_rn(dw, x.d), acc);
}

__device__ __forceinline__ float half_lo(unsigned w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}
__device__ __forceinline__ float half_hi(unsigned w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

}  // namespace
}  // namespace gb
