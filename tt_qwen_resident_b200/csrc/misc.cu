// Small kernels of the decode step and weight preparation for sm_100a:
//  - tile_weight: row-major e4m3 [rows][K] -> the GEMV tile/unit layout (gemv_fp8.cu);
//  - quantize_fp8: fp32 [N][K] -> e4m3 + one fp32 scale per 128 x 128 block (amax / 448);
//  - topk: per-row top-32 (key, index) list and argmax of bf16 logits, the order and tie rule of the
//    reference's sampling.hpp (:24-74): bf16 order keys descending, the smaller vocab index first on ties;
//  - embed_rows: the step's input rows, x0 or embed[token] (streamer_reader.cpp:117-128);
//  - feed: the device-fed next token state (mlp_hub.cpp:414-458): token = greedy pick, pos + 1.
#include <mutex>

#include "qres_common.cuh"

namespace qres {

// ------------------------------------------------------------------------------------------------ tiling
// 128-row tiles, 128-K units of 16 KB back to back per tile, inside a unit the tensor core's 128-byte-swizzled
// K-major rows: dst[(T * nkb + kb) * 16384 + r * 128 + ((c / 16) ^ (r % 8)) * 16 + c % 16] =
// src[(128 T + r) * K + 128 kb + c], zero past the last row. One thread per 16-byte granule.
__global__ void tile_weight_kernel(const uint8_t* __restrict__ src, int rows, int K, uint8_t* __restrict__ dst,
                                   size_t total16) {
    const int nkb = K / 128;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < total16; v += (size_t)gridDim.x * blockDim.x) {
        const size_t off = v * 16;
        const size_t unit = off / 16384;
        const int inner = (int)(off % 16384);
        const size_t T = unit / nkb;
        const int kb = (int)(unit % nkb);
        const int r = inner / 128, c = (((inner % 128) / 16) ^ (r % 8)) * 16;
        const size_t row = T * 128 + r;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (row < (size_t)rows) val = *reinterpret_cast<const uint4*>(src + row * K + (size_t)kb * 128 + c);
        *reinterpret_cast<uint4*>(dst + off) = val;
    }
}

// ------------------------------------------------------------------------------------------------ quantize
__global__ void quantize_fp8_kernel(const float* __restrict__ w, int N, int K, uint8_t* __restrict__ q,
                                    float* __restrict__ scales) {
    const int nb = blockIdx.y, kb = blockIdx.x;
    const int kbs = (K + 127) / 128;
    __shared__ float red[8];
    float amax = 0.f;
    for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
        const int r = nb * 128 + i / 128, c = kb * 128 + i % 128;
        if (r < N && c < K) amax = fmaxf(amax, fabsf(w[(size_t)r * K + c]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    const float scale = m > 0.f ? m / 448.0f : 1.0f;
    if (threadIdx.x == 0) scales[(size_t)nb * kbs + kb] = scale;
    for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
        const int r = nb * 128 + i / 128, c = kb * 128 + i % 128;
        if (r < N && c < K) {
            const float v = __fdiv_rn(w[(size_t)r * K + c], scale);
            q[(size_t)r * K + c] = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
        }
    }
}

// ------------------------------------------------------------------------------------------------ top-k
constexpr int kTopK = QRES_TOPK;
constexpr int kTopkThreads = 512;

__device__ __forceinline__ uint32_t key_of_bf16(uint32_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }

// Warp 0: scanning the 256 bins of hist from the top, the first bin b at which acc0 + (counts of bins above b) +
// hist[b] reaches kTopK; *bin = b (-1 if the total stays below kTopK) and *above = acc0 + the counts strictly
// above it (the total if none). Lane l holds bins 255 - 8 l .. 248 - 8 l: one scan over lanes, then the lane that
// crosses walks its 8 bins (a serial walk over 256 bins by one thread cost microseconds).
__device__ __forceinline__ void topk_bin(const int* hist, int acc0, int* bin, int* above) {
    const int lane = threadIdx.x & 31;
    int h[8], sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        h[q] = hist[255 - 8 * lane - q];
        sum += h[q];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, acc0 + incl >= kTopK);
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (hit == 0u) {
        if (lane == 0) {
            *bin = -1;
            *above = acc0 + total;
        }
        return;
    }
    if (lane == __ffs(hit) - 1) {
        int a = acc0 + incl - sum;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (a + h[q] >= kTopK) {
                *bin = 255 - 8 * lane - q;
                *above = a;
                return;
            }
            a += h[q];
        }
    }
}

// Select the top-32 of n candidates (key in [0, 65535], distinct indices) held in shared memory, in
// (key desc, index asc) order, into out_k / out_i. Radix select on the 16-bit key (high byte, then low byte),
// then the elements above the threshold plus the lowest-index ones equal to it, then a sort of those <= 32.
// All threads of the block call it.
__device__ void block_top32(const uint16_t* keys, const uint32_t* idx, int n, uint32_t* out_k, uint32_t* out_i,
                            int* hist, int* scratch) {
    const int tid = threadIdx.x, nt = blockDim.x;
    // pass 1: high byte
    for (int i = tid; i < 256; i += nt) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nt) atomicAdd(&hist[keys[i] >> 8], 1);
    __syncthreads();
    if (tid < 32) topk_bin(hist, 0, &scratch[0], &scratch[1]);  // bin (-1: fewer than 32, take all), count above
    __syncthreads();
    const int hb = scratch[0];
    int T = -1;  // threshold key: everything > T is in, == T partially
    if (hb >= 0) {
        for (int i = tid; i < 256; i += nt) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < n; i += nt)
            if ((keys[i] >> 8) == hb) atomicAdd(&hist[keys[i] & 0xff], 1);
        __syncthreads();
        // the low byte's bin (-1 never happens: the high byte's bin holds the crossing) and the count strictly
        // above T
        if (tid < 32) topk_bin(hist, scratch[1], &scratch[2], &scratch[3]);
        __syncthreads();
        T = (hb << 8) | max(scratch[2], 0);
    }
    // gather: key > T (any order), then key == T by ascending index (block prefix over index order)
    __shared__ uint64_t cand[kTopK];
    __shared__ int ncand;
    if (tid == 0) ncand = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nt) {
        if ((int)keys[i] > T) {
            const int s = atomicAdd(&ncand, 1);
            cand[s] = ((uint64_t)keys[i] << 32) | (0xffffffffu - idx[i]);
        }
    }
    __syncthreads();
    if (T >= 0) {
        const int above = ncand, need = kTopK - above;
        // equal keys: the `need` smallest indices (indices ascend with position in these arrays). Each thread
        // owns a contiguous segment; an exclusive scan of the per-segment counts gives every equal element its
        // rank in index order.
        const int seg = (n + nt - 1) / nt;
        const int a0 = min(tid * seg, n), a1 = min(a0 + seg, n);
        int cnt = 0;
        for (int i = a0; i < a1; ++i) cnt += (int)keys[i] == T;
        const int lane = tid & 31, warp = tid >> 5;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        __shared__ int wsum[32];
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        int wbase = 0;
        for (int w = 0; w < warp; ++w) wbase += wsum[w];
        int r = wbase + incl - cnt;
        for (int i = a0; i < a1 && r < need; ++i) {
            if ((int)keys[i] == T) {
                cand[above + r] = ((uint64_t)T << 32) | (0xffffffffu - idx[i]);
                ++r;
            }
        }
        __syncthreads();
        if (tid == 0) ncand = kTopK;
        __syncthreads();
    }
    // sort <= 32 candidates descending (one warp, bitonic over 32 lanes)
    if (tid < 32) {
        uint64_t v = tid < ncand ? cand[tid] : 0ull;  // empty: key 0, index 0xffffffff
        for (int k = 2; k <= 32; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
                const bool up = ((tid & k) == 0);  // descending overall
                const bool lower = (tid & j) == 0;
                const uint64_t mx = v > o ? v : o, mn = v > o ? o : v;
                v = (lower == up) ? mx : mn;
            }
        }
        out_k[tid] = (uint32_t)(v >> 32);
        out_i[tid] = 0xffffffffu - (uint32_t)(v & 0xffffffffu);
    }
    __syncthreads();
}

struct TopkParams {
    const uint16_t* logits;
    int n, ld, base, rows;
    uint32_t* cand;       // [rows][nblk][64]
    int* ticket;          // [rows]
    uint32_t* lists;      // [rows][64] keys then indices
    int32_t* argmax;      // [rows] or null
    int nblk;
};

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const TopkParams p) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int blk = blockIdx.x, row = blockIdx.y;
    const int per = (p.n + p.nblk - 1) / p.nblk;
    const int lo = blk * per, hi = min(lo + per, p.n);
    const int cnt = max(hi - lo, 0);
    uint16_t* keys = reinterpret_cast<uint16_t*>(sm);
    const int cap = max(per, p.nblk * kTopK);
    uint32_t* idx = reinterpret_cast<uint32_t*>(sm + ((cap * 2 + 15) & ~15));
    __shared__ int hist[256];
    __shared__ int scratch[4];
    __shared__ int last;
    pdl_launch();
    pdl_wait();
    const uint16_t* lg = p.logits + (size_t)row * p.ld;
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
        keys[i] = (uint16_t)key_of_bf16(lg[lo + i]);
        idx[i] = (uint32_t)(p.base + lo + i);
    }
    __syncthreads();
    uint32_t* mine = p.cand + ((size_t)row * p.nblk + blk) * 2 * kTopK;
    block_top32(keys, idx, cnt, mine, mine + kTopK, hist, scratch);
    // release / acquire through one thread (barrier, then thread 0's cumulative fence and atomic)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(p.ticket + row, 1) == p.nblk - 1;
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    // merge: the candidates of every block, in block order (indices ascend with block, then rank in list)
    const uint32_t* all = p.cand + (size_t)row * p.nblk * 2 * kTopK;
    int m = 0;
    // keep only real entries; lay them out in ascending index order per block (lists are key-sorted: re-sort
    // by index is unnecessary because equal keys inside one list are already in index order and blocks ascend)
    for (int i = threadIdx.x; i < p.nblk * kTopK; i += blockDim.x) {
        const int bb = i / kTopK, j = i % kTopK;
        keys[i] = (uint16_t)__ldcg(all + (size_t)bb * 2 * kTopK + j);
        idx[i] = __ldcg(all + (size_t)bb * 2 * kTopK + kTopK + j);
    }
    __syncthreads();
    m = p.nblk * kTopK;
    // entries with key 0 are empty fillers (index 0xffffffff): a real bf16 logit never has key 0 except -NaN
    __shared__ uint32_t ok_[kTopK], oi_[kTopK];
    block_top32(keys, idx, m, ok_, oi_, hist, scratch);
    if (threadIdx.x < kTopK) {
        p.lists[(size_t)row * 2 * kTopK + threadIdx.x] = ok_[threadIdx.x];
        p.lists[(size_t)row * 2 * kTopK + kTopK + threadIdx.x] = oi_[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        if (p.argmax) p.argmax[row] = (int32_t)oi_[0];
        p.ticket[row] = 0;
    }
}

// ------------------------------------------------------------------------------------------------ rows in / feed
__global__ void embed_rows_kernel(const qres_tok* tok, const float* x0, const uint16_t* embed, int vocab, float* x,
                                  int rows, uint32_t* err) {
    const int b = blockIdx.x;
    pdl_launch();
    pdl_wait();
    const int t = tok->token[b];
    if (t >= 0 && (embed == nullptr || t >= vocab)) {
        if (threadIdx.x == 0) atomicOr(err, kErrBounds);
        return;
    }
    for (int i = threadIdx.x; i < kHidden / 8; i += blockDim.x) {
        float4* dst = reinterpret_cast<float4*>(x + (size_t)b * kHidden) + 2 * i;
        if (t >= 0) {
            const uint4 e = reinterpret_cast<const uint4*>(embed + (size_t)t * kHidden)[i];
            dst[0] = make_float4(bf16lo(e.x), bf16hi(e.x), bf16lo(e.y), bf16hi(e.y));
            dst[1] = make_float4(bf16lo(e.z), bf16hi(e.z), bf16lo(e.w), bf16hi(e.w));
        } else {
            const float4* s = reinterpret_cast<const float4*>(x0 + (size_t)b * kHidden) + 2 * i;
            dst[0] = s[0];
            dst[1] = s[1];
        }
    }
}

// ------------------------------------------------------------------------------------------------ sampling draw
// The draw of the fed token from a row's final top-32 list (keys descending, then vocab indices; key 0 = empty),
// an integer contract with the reference's hub (sampling.hpp:77-143, bit-exact): temperature, then top-k, then
// top-p (vLLM's order) in Q16 fixed point. Parameter words: 1 / temperature in Q16 (0 = greedy), top-k (<= 1:
// greedy; at most 32), top-p in Q16 (65536 = off), seed. The random number hashes (seed, position), so a seeded
// request repeats and nothing carries over between steps. All arithmetic is 32 / 64-bit integer with the
// reference's wrap-around.

// bf16 bits -> Q16.16
__device__ __forceinline__ int32_t q16_of_bf16(uint32_t b) {
    const int32_t e = (b >> 7) & 0xff;
    if (e == 0) return 0;
    const int32_t m = (b & 0x7f) | 0x80;
    const int32_t sh = e - 118;  // value m * 2^(e - 134): m << (e - 118) in Q16
    const int32_t v = sh >= 0 ? (sh > 22 ? (m << 22) : (m << sh)) : (sh < -31 ? 0 : (m >> -sh));
    return (b & 0x8000) ? -v : v;
}

// exp(d) in Q16 for d <= 0 in Q16: 2^(d log2 e) with the fraction by the reference's degree-5 polynomial
__device__ __forceinline__ uint32_t exp_q16(int32_t d) {
    const int32_t t = (int32_t)(((int64_t)d * 94548) >> 16);
    const int32_t n = t >> 16;
    const uint32_t f = (uint32_t)t & 0xffffu;
    uint32_t p = 87u;
    p = 630u + ((p * f) >> 16);
    p = 3638u + ((p * f) >> 16);
    p = 15743u + ((p * f) >> 16);
    p = 45426u + ((p * f) >> 16);
    p = 65536u + ((p * f) >> 16);
    return n <= -31 ? 0u : p >> -n;
}

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ uint32_t bf16_of_key(uint32_t k) { return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu); }

// list: 32 keys then 32 indices; words: the 4 parameter words; pos: the position of the row being decoded
__device__ uint32_t draw_token(const uint32_t* list, const uint32_t* words, uint32_t pos) {
    const uint32_t inv_temp = words[0];
    const uint32_t k = words[1] < (uint32_t)kTopK ? words[1] : (uint32_t)kTopK;
    if (inv_temp == 0 || k <= 1) return list[kTopK];
    uint32_t w[kTopK];
    const int32_t l0 = q16_of_bf16(bf16_of_key(list[0]));
    uint32_t total = 0;
    for (uint32_t i = 0; i < k; ++i) {
        int64_t d = ((int64_t)(q16_of_bf16(bf16_of_key(list[i])) - l0) * (int64_t)inv_temp) >> 16;
        d = d < -(int64_t)(64 << 16) ? -(int64_t)(64 << 16) : d;
        w[i] = list[i] ? exp_q16((int32_t)d) : 0u;
        total += w[i];
    }
    const uint32_t limit = (uint32_t)(((uint64_t)total * words[2]) >> 16);
    uint32_t kept = 0, mass = 0;
    while (kept < k && (kept == 0 || mass < limit)) mass += w[kept++];
    uint32_t target = (uint32_t)(((uint64_t)mix32(words[3] ^ mix32(pos + 0x9e3779b9u)) * mass) >> 32);
    for (uint32_t i = 0; i < kept; ++i) {
        if (target < w[i]) return list[kTopK + i];
        target -= w[i];
    }
    return list[kTopK + kept - 1];
}

// standalone draws (qres_sample): one thread per row
__global__ void sample_kernel(int rows, const uint32_t* lists, const uint32_t* words, const int32_t* pos, int32_t* token) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < rows) token[b] = (int32_t)draw_token(lists + (size_t)b * 2 * kTopK, words + 4 * b, (uint32_t)pos[b]);
}

// out[b] = {next token, pos + 1, greedy argmax, 0}: the next token is the draw from the row's final list when
// sampling words are bound (words [rows][4]; a row with 1 / temperature 0 or top-k <= 1 draws its argmax), else
// the argmax. Feed mode writes it and pos + 1 into the token state (mlp_hub.cpp:414-458).
__global__ void feed_kernel(qres_tok* tok, const int32_t* argmax, int32_t* out, int rows, uint32_t* epoch,
                            const uint32_t* lists, const uint32_t* words) {
    pdl_launch();
    pdl_wait();
    const int b = threadIdx.x;
    if (b < rows) {
        const int a = argmax ? argmax[b] : -1;
        const int p = tok->pos[b], np = p + 1;
        const int t = (argmax && lists && words) ? (int)draw_token(lists + (size_t)b * 2 * kTopK, words + 4 * b, (uint32_t)p) : a;
        if (out) {
            out[b * 4 + 0] = t;
            out[b * 4 + 1] = np;
            out[b * 4 + 2] = a;
        }
        if (tok->feed && argmax) {
            tok->token[b] = t;
            tok->pos[b] = np;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        tok->step += 1;
        if (epoch) *epoch += 1;  // steps completed: the peer exchanges' expected counts derive from it
    }
}

// the peer exchange of the lm_head's top-32 lists (the hubs' list exchange, mlp_hub.cpp:366-411): this rank's
// [rows][64] list into its region of every rank's window, then one release-add per destination
__global__ void publish_lists_kernel(const uint32_t* __restrict__ list, int words, P2PDest dst, const uint32_t* epoch) {
    pdl_launch();
    pdl_wait();
    const uint32_t slot = *epoch & 1u;  // this step's half of the double buffer
    for (int d = 0; d < dst.n; ++d)
        for (int i = threadIdx.x; i < words; i += blockDim.x) dst.data[d][slot * dst.slot_words + i] = list[i];
    __syncthreads();
    if ((int)threadIdx.x < dst.n) {
        __threadfence_system();
        red_release_sys_add(dst.cnt[threadIdx.x] + slot * 8, 1u);
    }
}

// ------------------------------------------------------------------------------------------------ KV rows <-> pages
// One user's K / V rows of positions 0 .. npos-1 ([nkv][npos][256] bf16, contiguous) to or from the paged pool
// ([pages][nkv][64][256]): position p of head j is row p % 64 of page page_table[p / 64]. One CTA per (position,
// head, K or V), 32 threads x 16 bytes. to_pages: 1 = rows -> pool (load), 0 = pool -> rows (dump).
__global__ void kv_rows_kernel(uint16_t* kp, uint16_t* vp, uint16_t* k, uint16_t* v, const int32_t* page_table,
                               int npos, int nkv, int num_pages, int to_pages, uint32_t* err) {
    const int p = blockIdx.x, j = blockIdx.y;
    const int pg = page_table[p / kKvBlock];
    if (pg < 0 || pg >= num_pages) {
        if (threadIdx.x == 0) atomicOr(err, kErrBounds);
        return;
    }
    uint16_t* pool = blockIdx.z ? vp : kp;
    uint16_t* rows = blockIdx.z ? v : k;
    uint4* a = reinterpret_cast<uint4*>(pool + (((size_t)pg * nkv + j) * kKvBlock + p % kKvBlock) * kHD);
    uint4* b = reinterpret_cast<uint4*>(rows + ((size_t)j * npos + p) * kHD);
    if (to_pages) a[threadIdx.x] = b[threadIdx.x];
    else b[threadIdx.x] = a[threadIdx.x];
}

cudaError_t kv_rows_launch(uint16_t* kp, uint16_t* vp, uint16_t* k, uint16_t* v, const int32_t* page_table, int npos,
                           int nkv, int num_pages, bool to_pages, uint32_t* err, cudaStream_t st) {
    if (npos < 1 || nkv < 1) return cudaErrorInvalidValue;
    kv_rows_kernel<<<dim3(npos, nkv, 2), kHD * 2 / 16, 0, st>>>(kp, vp, k, v, page_table, npos, nkv, num_pages,
                                                                 to_pages ? 1 : 0, err);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ wait probe
// One bounded wait of the peer exchange's kind (wait_count on a counter word) with a caller-chosen budget: the
// failure path of a lost peer exercised on one GPU, with a word that nothing advances (qres_wait_probe).
__global__ void wait_probe_kernel(const uint32_t* flag, uint32_t want, uint32_t limit, uint32_t* err) {
    wait_count(flag, want, err, limit);
}

cudaError_t wait_probe_launch(const uint32_t* flag, uint32_t want, uint32_t limit, uint32_t* err, cudaStream_t st) {
    wait_probe_kernel<<<1, 1, 0, st>>>(flag, want, limit, err);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ launchers
static cudaLaunchConfig_t pdl_cfg(dim3 g, dim3 b, size_t smem, cudaStream_t st, cudaLaunchAttribute* at, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = b;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

cudaError_t tile_weight_launch(const uint8_t* src, int rows, int K, uint8_t* dst, cudaStream_t st) {
    const int rows_pad = (rows + 127) & ~127;
    const size_t total16 = (size_t)rows_pad * K / 16;
    tile_weight_kernel<<<1024, 256, 0, st>>>(src, rows, K, dst, total16);
    return cudaGetLastError();
}

cudaError_t quantize_fp8_launch(const float* w, int N, int K, uint8_t* q, float* scales, cudaStream_t st) {
    dim3 grid((K + 127) / 128, (N + 127) / 128);
    quantize_fp8_kernel<<<grid, 256, 0, st>>>(w, N, K, q, scales);
    return cudaGetLastError();
}

int topk_default_blocks(int n) {
    int nb = (n + 2047) / 2048;
    return nb < 1 ? 1 : (nb > 128 ? 128 : nb);
}

size_t topk_workspace_bytes(int rows, int nblk) {
    return (size_t)rows * nblk * 2 * kTopK * 4 + 256 + (size_t)rows * 4;
}

cudaError_t topk_launch(int rows, const uint16_t* logits, int n, int ld, int base, uint32_t* lists, int32_t* argmax,
                        void* work, int nblk, cudaStream_t st, bool pdl) {
    TopkParams p;
    p.logits = logits;
    p.n = n;
    p.ld = ld;
    p.base = base;
    p.rows = rows;
    p.nblk = nblk;
    p.cand = static_cast<uint32_t*>(work);
    p.ticket = reinterpret_cast<int*>(static_cast<uint8_t*>(work) + (size_t)rows * nblk * 2 * kTopK * 4 + 256);
    p.lists = lists;
    p.argmax = argmax;
    const int per = (n + nblk - 1) / nblk;
    const int cap = per > nblk * kTopK ? per : nblk * kTopK;
    const size_t smem = ((size_t)cap * 2 + 15) / 16 * 16 + (size_t)cap * 4;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(nblk, rows), dim3(kTopkThreads), smem, st, at, pdl);
    return cudaLaunchKernelEx(&cfg, topk_kernel, p);
}

cudaError_t embed_rows_launch(const qres_tok* tok, const float* x0, const uint16_t* embed, int vocab, float* x, int rows,
                              uint32_t* err, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(320), 0, st, at, pdl);
    return cudaLaunchKernelEx(&cfg, embed_rows_kernel, tok, x0, embed, vocab, x, rows, err);
}

cudaError_t feed_launch(qres_tok* tok, const int32_t* argmax, int32_t* out, int rows, cudaStream_t st, bool pdl,
                        uint32_t* epoch, const uint32_t* lists, const uint32_t* words) {
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(32), 0, st, at, pdl);
    return cudaLaunchKernelEx(&cfg, feed_kernel, tok, argmax, out, rows, epoch, lists, words);
}

cudaError_t sample_launch(int rows, const uint32_t* lists, const uint32_t* words, const int32_t* pos, int32_t* token,
                          cudaStream_t st) {
    if (rows < 1) return cudaErrorInvalidValue;
    sample_kernel<<<(rows + 127) / 128, 128, 0, st>>>(rows, lists, words, pos, token);
    return cudaGetLastError();
}

}  // namespace qres

namespace qres {

// merge nlists per-rank lists ([nlists][rows][64], keys then indices, ranks in vocab order) into one list per
// row and its argmax (the hubs' exchange + merge, mlp_hub.cpp:366-411 / sampling.hpp merge)
__global__ void __launch_bounds__(256) merge_lists_kernel(const uint32_t* lists, int nlists, int rows, uint32_t* out,
                                                          int32_t* argmax, const uint32_t* wait_cnt,
                                                          const uint32_t* epoch, uint32_t* err) {
    const int row = blockIdx.x;
    __shared__ uint16_t keys[8 * kTopK];
    __shared__ uint32_t idx[8 * kTopK];
    __shared__ int hist[256];
    __shared__ int scratch[4];
    __shared__ uint32_t ok_[kTopK], oi_[kTopK];
    pdl_launch();
    pdl_wait();
    if (wait_cnt != nullptr) {
        // the peer exchange: every rank's list of this step has arrived (one thread per rank, bounded); step s
        // uses half s % 2 of the double buffer for the (s / 2 + 1)-th time
        const uint32_t e = *epoch;
        lists += (size_t)(e & 1u) * 8 * rows * 2 * kTopK;
        if ((int)threadIdx.x < nlists) wait_count(wait_cnt + (e & 1u) * 8 + threadIdx.x, e / 2 + 1, err);
        __syncthreads();
    }
    const int n = nlists * kTopK;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int l = i / kTopK, j = i % kTopK;
        const uint32_t* src = lists + ((size_t)l * rows + row) * 2 * kTopK;
        keys[i] = (uint16_t)__ldcg(src + j);
        idx[i] = __ldcg(src + kTopK + j);
    }
    __syncthreads();
    block_top32(keys, idx, n, ok_, oi_, hist, scratch);
    if (threadIdx.x < kTopK) {
        out[(size_t)row * 2 * kTopK + threadIdx.x] = ok_[threadIdx.x];
        out[(size_t)row * 2 * kTopK + kTopK + threadIdx.x] = oi_[threadIdx.x];
    }
    if (threadIdx.x == 0 && argmax) argmax[row] = (int32_t)oi_[0];
}

cudaError_t merge_lists_launch(const uint32_t* lists, int nlists, int rows, uint32_t* out, int32_t* argmax,
                               cudaStream_t st, bool pdl, const uint32_t* wait_cnt, const uint32_t* epoch,
                               uint32_t* err) {
    if (nlists < 1 || nlists > 8 || (wait_cnt && !epoch)) return cudaErrorInvalidValue;
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(256), 0, st, at, pdl);
    return cudaLaunchKernelEx(&cfg, merge_lists_kernel, lists, nlists, rows, out, argmax, wait_cnt, epoch, err);
}

cudaError_t publish_lists_launch(const uint32_t* list, int words, const P2PDest& dst, const uint32_t* epoch,
                                 cudaStream_t st, bool pdl) {
    if (dst.n < 1 || dst.n > 8 || !epoch) return cudaErrorInvalidValue;
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(256), 0, st, at, pdl);
    return cudaLaunchKernelEx(&cfg, publish_lists_kernel, list, words, dst, epoch);
}

}  // namespace qres

namespace qres {

// ------------------------------------------------------------------------------------------------ top-k, no allocation
// The top-k of qres_topk_noalloc keeps its scratch (the per-block candidate lists and the per-row tickets) in this
// fixed device array instead of a caller-provided workspace. It is sized for 8 rows of the full 248,320-entry
// vocabulary (8 x 122 blocks of 256 bytes, plus the tickets): 256 KiB, held by every GPU that loads the library
// until the process exits. All calls share it and it keeps the last call's contents.
constexpr size_t kTopkStaticScratch = 256 * 1024;
static __device__ __align__(256) uint8_t g_topk_scratch[kTopkStaticScratch];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_topk_scratch_mu;
void* g_topk_scratch_ptr[kMaxDevices] = {};  // device address of g_topk_scratch, per device
}  // namespace

// the device address of the scratch array on the current device (looked up once per device; the host-side name
// g_topk_scratch is only a stand-in and must never be passed to a kernel)
cudaError_t topk_static_scratch(void** out, size_t* bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_topk_scratch_mu);
    if (g_topk_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_topk_scratch);
        if (e != cudaSuccess) return e;
        g_topk_scratch_ptr[dev] = p;
    }
    *out = g_topk_scratch_ptr[dev];
    *bytes = kTopkStaticScratch;
    return cudaSuccess;
}

// byte offset of the per-row tickets inside a top-k workspace (they must start every call at zero)
size_t topk_ticket_offset(int rows, int nblk) { return (size_t)rows * nblk * 2 * kTopK * 4 + 256; }

}  // namespace qres
