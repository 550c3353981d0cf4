// Shared device pieces of the FP8 weight-streaming kernel (gemv_fp8.cu): the operand / shared-memory geometry, the
// tcgen05 wrappers (cta_group::1) and the e4m3 conversions.
#pragma once

#include <algorithm>

#include "qres_common.cuh"

namespace qres {

// PRO_RMSNORM_XACC / EPI_XACC: the counted fixed-point exchange between ranks (their own instantiations, so the
// one-rank kernels carry none of its code)
enum { PRO_RMSNORM = 0, PRO_BF16 = 1, PRO_RMSNORM_ADD = 2, PRO_SILU_ACC = 3, PRO_RMSNORM_XACC = 4 };
enum { EPI_BF16 = 0, EPI_SILU_MUL = 1, EPI_RESID = 2, EPI_F32 = 3, EPI_P2P = 4, EPI_ACC = 5, EPI_XACC = 6 };

constexpr int kMaxPeers = 8;

constexpr int kGemvThreads = 256;
constexpr int kTileRows = 128;
constexpr int kUnitBytes = 128 * 128;  // one 128-row x 128-K block of e4m3
constexpr int kDSlots = 4;             // TMEM accumulator slots, 16 fp32 columns each
constexpr int kTmemCols = 64;
constexpr int kMaxStages = 8;
constexpr int kSelBytes = 128;         // per tile: the selector of each row
constexpr int kHeadBytes = 1024;       // barriers and small shared state

// instruction descriptor of tcgen05.mma.kind::f8f6f4: D fp32 (bits 4-5 = 1), A and B e4m3 (bits 7-9, 10-12 =
// 0), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t kIdesc = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

// The activations' operand, per user group of 4 (columns 2b, 2b + 1 = user b's hi, lo) and 128-K block: 8
// K-chunks of 16 bytes, chunk j's 8 column rows at j * LBO. With B < 4 users only rows 0 .. 2B-1 are real and
// LBO = 32 B: rows 2B..7 of a chunk are the next chunks' real rows, read by the MMA into D columns nobody reads
// (a column of D depends only on its own operand column), which shrinks the operand 4x at one user.
__host__ __device__ constexpr int gemv_act_lbo(int B) { return B >= 4 ? 128 : 32 * B; }
__host__ __device__ inline size_t gemv_act_group(int B, int nkw) { return (size_t)nkw * 8 * gemv_act_lbo(B) + 128; }
__host__ __device__ inline size_t gemv_act_bytes(int B, int nkw) { return (size_t)(B > 4 ? 2 : 1) * gemv_act_group(B, nkw); }
__host__ __device__ inline size_t gemv_ainv_bytes(int nkw) { return ((size_t)nkw * 8 * 4 + 127) & ~size_t(127); }
__host__ __device__ inline size_t gemv_smem_bytes(int B, int nkw, int nstages) {
    const size_t pre = kHeadBytes + gemv_ainv_bytes(nkw) + gemv_act_bytes(B, nkw);
    return ((pre + 1023) & ~size_t(1023)) + (size_t)nstages * kUnitBytes;
}

// ---- tcgen05 wrappers (cta_group::1) ------------------------------------------------------------------------

// shared-memory matrix descriptor: start, leading (K) and stride (M/N) byte offsets, version 1, layout type
// (bits 61-63: 0 no swizzle, 2 = 128-byte swizzle; a swizzled operand's atoms are 1024-byte aligned)
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout = 0) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

__device__ __forceinline__ void tc_mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(kIdesc)
        : "memory");
}

// arrive on `bar` once every tcgen05 operation this thread issued so far has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// whole warp: allocate `cols` TMEM columns, base address written to *dst (shared memory)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// this warp's 32 TMEM lanes x NC consecutive fp32 columns (one lane per thread); the load and its wait are one
// statement, so no use of the values can be scheduled before the wait
template <int NC>
__device__ __forceinline__ void tmem_load(uint32_t taddr, float* v);

template <>
__device__ __forceinline__ void tmem_load<2>(uint32_t a, float* v) {
    uint32_t r0, r1;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];\n\ttcgen05.wait::ld.sync.aligned;"
                 : "=r"(r0), "=r"(r1)
                 : "r"(a)
                 : "memory");
    v[0] = __uint_as_float(r0);
    v[1] = __uint_as_float(r1);
}
template <>
__device__ __forceinline__ void tmem_load<4>(uint32_t a, float* v) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n\ttcgen05.wait::ld.sync.aligned;"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_load<8>(uint32_t a, float* v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(a)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_load<16>(uint32_t a, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n\ttcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(a)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// two floats -> two e4m3 bytes (round to nearest even, saturating), a in the low byte
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
    return r;
}
// two e4m3 bytes -> floats (exact)
__device__ __forceinline__ float2 e4m3x2_f32(uint32_t v) {
    uint32_t h2;
    asm("{\n\t.reg .b16 l;\n\tcvt.u16.u32 l, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\t}" : "=r"(h2) : "r"(v));
    return __half22float2(*reinterpret_cast<__half2*>(&h2));
}

// CTA owning unit u when U units are split over G CTAs (base = U / G, rem = U % G)
__device__ __forceinline__ int cta_of_unit(int u, int base, int rem) {
    const int big = rem * (base + 1);
    if (u < big) return u / (base + 1);
    return rem + (u - big) / base;
}

}  // namespace qres
