// Shared device helpers of libqres: sm_100a PTX wrappers (mbarrier, bulk async copies, programmatic
// dependent launch), bounded waits that report instead of hanging, and the numeric helpers every kernel of the
// resident decode step uses.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qres.h"

namespace qres {

constexpr int kHidden = 5120;
constexpr int kDK = 128, kDV = 128;
constexpr int kHD = 256, kRot = 64;
constexpr int kKvBlock = 64;
constexpr int kMaxRows = 8;  // users (or verify rows) per step
constexpr float kEps = 1e-6f;

// error bits written into the context's device error word (qres_dev_status)
enum : uint32_t {
    kErrTimeout = 1u << 0,   // a bounded wait ran out (mbarrier / peer flag)
    kErrBounds = 1u << 1,    // an index (position, page, token) outside its table
    kErrPeer = 1u << 2,      // a peer flag carried an unexpected epoch
};

// ---- numeric helpers -------------------------------------------------------------------------------------

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// IEEE-rounded helpers (no FMA contraction) where the reference's torch ops round each product / sum
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }
// torch.nn.functional.softplus (beta 1, threshold 20)
__device__ __forceinline__ float softplus_f(float v) { return v > 20.0f ? v : log1pf(expf(v)); }
__device__ __forceinline__ float rsqrt_ieee(float v) { return 1.0f / sqrtf(v); }

// 4 e4m3 bytes -> 4 floats (exact), through the packed e4m3x2 -> f16x2 conversion
__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float* f) {
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xffffu), __NV_E4M3);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3);
    float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
    float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Fixed-point accumulators (the GEMV's EPI_ACC): every CTA adds its fp32 partial of a row, rounded to a multiple of 2^-30,
// into a 64-bit integer with one atomic add. Integer addition is associative, so the sum does not depend on the
// order in which the CTAs' additions land (bit-reproducible without a ticket or a designated finisher); the
// consumer (the next launch) reads it back as one float rounding of the exact sum of the rounded partials.
// Range: |partial|, |sum| < 2^33.
constexpr float kAccScale = 1073741824.0f;    // 2^30
constexpr float kAccInv = 9.313225746154785e-10f;  // 2^-30
__device__ __forceinline__ unsigned long long acc_encode(float v) {
    return (unsigned long long)__float2ll_rn(v * kAccScale);
}
__device__ __forceinline__ float acc_decode(long long w) { return __ll2float_rn(w) * kAccInv; }
// Counted form (the row-parallel exchange): each contribution adds (value << 8) + 1, so the low byte counts the
// contributions that have landed and a consumer that knows how many to expect can read a word as soon as it is
// complete, whoever added it and in whatever order. Range: |sum| < 2^25.
__device__ __forceinline__ unsigned long long acc_encode_cnt(float v) {
    return ((unsigned long long)__float2ll_rn(v * kAccScale) << 8) + 1ull;
}
__device__ __forceinline__ float acc_decode_cnt(long long w) { return __ll2float_rn(w >> 8) * kAccInv; }

// the in-projection's output as the mixers read it: bf16 values, or (one rank) its fixed-point sums rounded to bf16
struct YIn {
    const uint16_t* y;
    const long long* acc;
    __device__ __forceinline__ uint16_t operator[](size_t i) const {
        return acc ? __bfloat16_as_ushort(__float2bfloat16_rn(acc_decode(acc[i]))) : y[i];
    }
    __device__ __forceinline__ YIn at(size_t off) const { return YIn{y ? y + off : nullptr, acc ? acc + off : nullptr}; }
};

// ---- programmatic dependent launch --------------------------------------------------------------------------
// wait: every prerequisite grid has completed and its memory is visible; launch_dependents: allow the next
// kernel in the stream to be scheduled (its pre-wait part -- weight prefetch -- overlaps this kernel's tail)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- mbarrier + bulk async copy (cp.async.bulk, no multicast) ----------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// spin budget of a bounded wait: ~2^22 try_wait rounds (each suspends for a while) -- far beyond any legitimate
// wait of this code, well short of a hang
constexpr uint32_t kSpinLimit = 1u << 22;

// wait for the phase with the given parity to complete; false (and the error bit set) when the budget runs out
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    if (err) atomicOr(err, kErrTimeout);
    return false;
}

// The tensor-parallel exchange of one GEMV launch over peer memory (gemv_launch's optional argument). The
// row-parallel projection's epilogue stores each partial as a tagged word -- {fp32 bits, tag} in one 8-byte store,
// so a word is either wholly old or wholly new -- into its region of every rank's window; the next projection's
// rmsnorm prologue re-reads the words until every one carries this exchange's tag and adds the ranks' partials
// in rank order. No fence, counter or barrier sits between the two GPUs' kernels.
struct GemvExchange {
    int nsrc = 1;                      // prologue: partial sources to add (red, red + src_stride, ...; fp32)
    size_t src_stride = 0;
    const uint2* tagged = nullptr;     // prologue: tagged sources [nsrc][users][K] in this rank's window, or null
    const uint32_t* epoch = nullptr;   // steps completed (device)
    uint32_t tag_mul = 0, tag_add = 0; // tag of this exchange: *epoch * tag_mul + tag_add (never 0)
    int p2p_n = 0;                     // epilogue: destinations (ranks)
    int peer_ld = 0;                   // words per user row in a destination region
    uint2* peer_data[8] = {};          // this rank's region in each rank's window
    // the rmsnorm prologue over two segments (the MTP fc, mtp.py:54-60 / streamer_common.hpp fc): K = 2 seg,
    // positions [0, seg) from the launch's input (fp32 [users][seg]), [seg, 2 seg) from seg2, each segment
    // normalised on its own; seg 0 = one segment
    const float* seg2 = nullptr;
    int seg = 0;
    // fixed-point accumulators (one rank): the prologue's partial source (PRO_RMSNORM_ADD, int64 [users][K])
    // instead of fp32 `red`; the SwiGLU prologue's gate|up sums (PRO_SILU_ACC, int64 [users][ld_gacc], rows in the
    // interleaved quads of the gate|up matrix); the epilogue's target (EPI_ACC, int64 [users][ld_out]); and a
    // buffer this launch zeroes after its dependency wait (the one a later launch accumulates into)
    const long long* racc = nullptr;
    const long long* gacc = nullptr;
    int ld_gacc = 0;
    long long* acc_out = nullptr;
    long long* zero = nullptr;
    size_t zero_words = 0;
    bool zero_sys = false;  // the zeroed buffer receives other GPUs' adds later: fence the zeroing at system scope
    // the counted row-parallel exchange (EPI_ACC with xn > 0): each partial goes, as a counted word, into every
    // rank's accumulator xdst[0..xn-1] (the peers' mapped over NVLink; xn = 1: this rank's alone), and the next
    // prologue reads its racc once every word holds rc_ranks x (the producing launch's CTAs over the row's tile)
    // contributions -- the producing launch split rc_units units of rc_nkb per tile over rc_grid CTAs
    long long* xdst[8] = {};
    int xn = 0;
    int rc_ranks = 0, rc_units = 0, rc_grid = 0, rc_nkb = 0;
};

// destinations of a small per-step peer exchange, double-buffered by step parity: this rank's region in each
// rank's window (slot 1 at + slot_words) and its counter there (slot 1 at + 8)
struct P2PDest {
    int n = 0;
    size_t slot_words = 0;
    uint32_t* data[8] = {};
    uint32_t* cnt[8] = {};
};

// ---- peer memory (another GPU's window mapped over NVLink) -------------------------------------------------

// acquire load at system scope: pairs with a peer GPU's release-add on this (local) memory
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// release add at system scope (the counter usually lives in a peer GPU's memory)
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 16 bytes (two tagged words) read past every cache level a peer's stores could be stale in
__device__ __forceinline__ uint4 ld_volatile128(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
                 : "memory");
    return v;
}

// spin budget on a peer counter: ~2^24 polls with a short sleep (about a second), far beyond a healthy step
constexpr uint32_t kPeerSpinLimit = 1u << 24;

// wait until the counter reaches `want` (wrap-safe compare); false (error bits set) when the budget of `limit`
// polls runs out
__device__ inline bool wait_count(const uint32_t* p, uint32_t want, uint32_t* err, uint32_t limit = kPeerSpinLimit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if ((int32_t)(ld_acquire_sys(p) - want) >= 0) return true;
        __nanosleep(64);
    }
    if (err) atomicOr(err, kErrPeer | kErrTimeout);
    return false;
}

// global -> shared bulk copy completing on an mbarrier (sizes and addresses multiples of 16 bytes)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// global -> shared bulk copy with an L2 cache policy (e.g. evict_first for data read exactly once)
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// L2 prefetch of [p, p + bytes) spread over `n` participants (participant i takes its share), 16-byte granules
__device__ __forceinline__ void l2_prefetch_share(const uint8_t* p, size_t bytes, int i, int n) {
    const size_t per = ((bytes + n - 1) / n + 15) & ~size_t(15);
    size_t a = (size_t)i * per;
    if (a >= bytes) return;
    size_t e = a + per < bytes ? a + per : bytes;
    for (; a < e; a += 65536) {
        const size_t len = (e - a) < 65536 ? (e - a) : 65536;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + a), "r"((uint32_t)((len + 15) & ~size_t(15))) : "memory");
    }
}

// L2 prefetch of a global range (no shared destination)
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// The heads of a weight-streaming projection's CTA runs: its `units` 16 KB units are split over `grid` CTAs in
// contiguous runs (the first units % grid runs one longer), and units k0 .. k0 + k - 1 of every run are pulled
// into L2, so that every CTA of that launch starts on L2 hits rather than only the first few.
struct L2Heads {
    const uint8_t* w;
    int units, grid, k0, k;
    int tiles, nkb, nq;  // the launch's unit order (see unit_offset)
};

// The order in which a weight-streaming launch walks its units (128-row x 128-K blocks of 16 KB; the weight is
// stored tile-major, K fastest): units are grouped by K block group (nq blocks each), then tile, then block in the
// group, and a launch splits that order over its CTAs in contiguous runs. nq = nkb is the plain storage order (a
// CTA's run covers about one tile's whole K); a smaller nq makes a run cover a few tiles of one K group, so the
// CTA needs the activations of nq K blocks only. Returns the unit's index in storage order.
__device__ __forceinline__ size_t unit_offset(int u, int tiles, int nkb, int nq) {
    const int per = tiles * nq, kq = u / per, r = u - kq * per, T = r / nq;
    return (size_t)T * nkb + kq * nq + (r - T * nq);
}

// prefetcher i of n takes the runs i, i + n, ...
__device__ __forceinline__ void l2_prefetch_heads(const L2Heads& h, int i, int n) {
    if (h.w == nullptr || h.k <= 0 || h.grid <= 0) return;
    const int base = h.units / h.grid, rem = h.units % h.grid;
    for (int c = i; c < h.grid; c += n) {
        const int u0 = c * base + min(c, rem), cnt = base + (c < rem ? 1 : 0);
        const int m = min(cnt, h.k0 + h.k);
        for (int u = h.k0; u < m; ++u)
            bulk_prefetch_l2(h.w + unit_offset(u0 + u, h.tiles, h.nkb, h.nq) * 16384, 16384u);
    }
}

// order this thread's generic-proxy shared-memory accesses before later async-proxy ones (tensor core, bulk copy)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// named barrier over a subset of warps (id 1.., count a multiple of 32)
__device__ __forceinline__ void bar_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_addr(p)));
    return v;
}

// streaming read-only global load (no L1 allocation)
__device__ __forceinline__ uint4 ldg_nc128(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace qres
