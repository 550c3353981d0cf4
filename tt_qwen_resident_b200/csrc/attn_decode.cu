// Gated GQA decode attention over a paged KV cache for sm_100a: split-K over pages (flash-decoding), the scores
// and the probability-weighted sum of V on the tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate), pages
// staged by TMA tensor copies.
//
// Replaces the reference's attention leader / tail / chunk workers (qwen36_resident/kernels/attn_leader_*.cpp,
// attn_worker_*.cpp, attn_compute_common.hpp:186-497), i.e. the math of model.py:233-247:
//   q  = rope(rmsnorm(q_h) * wq / 16)            (fp32; rope on dims 0..63 as pairs (i, i + 32), theta 1e7)
//   k  = bf16(rope(rmsnorm(k) * wk));  K[pos] = k, V[pos] = v
//   o  = bf16(softmax(q . K[0..pos]^T) @ V * sigmoid(gate))
// KV layout: per attention layer a pool [pages][kv_heads_local][64][256] bf16 per K and V; position p of user b
// lives in page page_table[b][p / 64], row p % 64 (pages of one head are 32 KB contiguous runs).
//
// Grid (chunks, kv heads, users). A CTA takes a contiguous run of the user's pages (the run length adapts to
// the current context). Warp 6 lane 0 streams each page's K and V into a ring of 3 stages with 8 TMA tensor
// copies (64 rows x 64 dims each, 128-byte swizzle, no multicast; an L2 evict-first hint: KV is read once per
// step). Warps 0..5 are three page groups of two warps; group j takes the pages that land in stage j and keeps
// its own online softmax (no barrier between groups until the end). For a page of 64 positions a group computes
//   S [16 x 64] = Q [16 x 256] . K^T          rows 0..7 = q_hi of the group's query heads, rows 8..15 = q_lo,
//                                              q = q_hi + q_lo two bf16 terms (exact to ~2^-16), heads >= G zero
//   s = S[h] + S[h + 8]                       the fp32 score of head h
//   P [16 x 64] = (p_hi ; p_lo),  p = exp(s - m)   the probabilities split the same way
//   O [16 x 256] += P . V                     each warp of the group half of the dims
// so the tensor cores take bf16 operands while scores and weights keep fp32 accuracy. K and V are read with
// ldmatrix (V transposed) from the swizzled stage, bank-conflict-free. At the end the three groups merge in
// group order through shared memory, the CTA writes its chunk's (max, sum, o[256]) per head, and the last CTA of
// a (user, kv head) -- an atomic ticket -- combines the chunks in order (deterministic) and applies the gate.
// The CTA whose pages hold `pos` appends k / v to the cache; a stage that holds positions this step writes gets
// those rows patched in shared memory from the step's own k / v before use.
//
// Verify step (R consecutive positions p .. p+R-1 of one user, attn_common.hpp:39-42 KV sharing; row r sees
// rows < r): all rows share user 0's page table; every CTA of row r computes k / v of rows 0..r itself and
// uses them for positions p .. p+r (the cache there may be mid-append by other rows' CTAs, so it is never read
// for those positions); each row still appends its own position.
#include <mutex>
#include <unordered_map>

#include "qres_common.cuh"

namespace qres {

constexpr int kAttnThreads = 256;  // warps 0..5 consumers (3 groups of 2), warp 6 the producer, warp 7 spare
constexpr int kAttnGroups = 3;
constexpr int kAttnStages = kAttnGroups;  // stage j is consumed by group j
constexpr int kMaxGroup = 6;  // query heads per KV head on a rank (24 / 4)
constexpr int kPageBytes = kKvBlock * kHD * 2;  // 32 KB per head page of K (or V)
constexpr int kStageBytes = 2 * kPageBytes;     // K page then V page, 4 swizzled boxes of 8 KB each
constexpr int kBoxBytes = kKvBlock * 128;       // one TMA box: 64 rows x 64 dims bf16
constexpr int kPartStride = 2 + kHD;  // a chunk's partial per head: max, sum, o[256]
// dynamic shared memory: the ring, q (16 rows x 256 bf16, swizzled), the new rows' k and v (bf16), barriers
constexpr int kOffQ = kAttnStages * kStageBytes;
constexpr int kOffKnew = kOffQ + 16 * kHD * 2;
constexpr int kOffVnew = kOffKnew + kMaxRows * kHD * 2;
constexpr int kOffBar = kOffVnew + kMaxRows * kHD * 2;
constexpr int kAttnSmem = kOffBar + 64 + 1024;  // + slack to align the base to 1024 bytes

struct AttnParams {
    int h, nkv, G;            // local query heads, local KV heads, heads per KV head
    int ld_y;
    const uint16_t* y;        // [B][ld_y]: q (h*256) | gate (h*256) | k (nkv*256) | v (nkv*256)
    const long long* yacc;    // or the in-projection's fixed-point sums, same layout (y null)
    const int32_t* pos;
    const int32_t* page_table;
    int max_pages, num_pages;
    const float* wq;          // [256] q-norm weight / 16
    const float* wk;          // [256]
    const float* cos_tab;     // [max_pos][32]
    const float* sin_tab;
    int max_pos;
    uint16_t* kp;             // K pool
    uint16_t* vp;             // V pool
    uint16_t* o;              // [B][h*256]
    uint16_t* mixer_copy;
    float* part;              // [B][nkv][nchunks][G][2 + 256]
    int* ticket;              // [B][nkv]
    int nchunks;
    int verify;               // 0, or R: rows are R consecutive positions of user 0
    const uint8_t* pf;        // the next projection's weights: prefetched into L2 while this kernel runs
    size_t pf_bytes;
    uint32_t* err;
};

// ---- tensor-core helpers (mma.sync / ldmatrix) ----------------------------------------------------------------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// c += a (16 x 16, row) * b (16 x 8, col), bf16 operands, fp32 accumulators
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}

// byte offset of (row, 16-byte chunk) in a stage page: 4 boxes of 64 dims, the TMA's 128-byte swizzle inside
__device__ __forceinline__ uint32_t page_off(int row, int chunk) {
    return (uint32_t)((chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}
// q rows: 512 bytes each, chunk c stored at c ^ (row % 8) (conflict-free ldmatrix)
__device__ __forceinline__ uint32_t q_off(int row, int chunk) { return (uint32_t)(row * 512 + ((chunk ^ (row & 7)) << 4)); }

// 2-D TMA tensor load (box 64 x 64 bf16) completing on an mbarrier, with an L2 cache policy
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void rms_rope_head(float v, float wd, float c, float s, float* dst, float* red, bool round_bf16) {
    // one head of 256 dims by 256 threads (v: this thread's dim d of the input, wd the weight there, c / s the
    // rope cos / sin of the dim for d < 32): dst = rope(rmsnorm(src) * w) (optionally rounded to bf16)
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
    float ss = warp_sum(v * v);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float r = rsqrt_ieee(t / (float)kHD + kEps);
    const float nv = mul_rn(mul_rn(v, r), wd);
    dst[d] = nv;
    __syncthreads();
    if (d < kRot / 2) {
        const float a = dst[d], b = dst[d + kRot / 2];
        const float ra = mul_rn(a, c) - mul_rn(b, s);
        const float rb = mul_rn(b, c) + mul_rn(a, s);
        dst[d] = round_bf16 ? bf16_round(ra) : ra;
        dst[d + kRot / 2] = round_bf16 ? bf16_round(rb) : rb;
    } else if (d >= kRot && round_bf16) {
        dst[d] = bf16_round(nv);
    }
    __syncthreads();
}

// the G query heads of a group at once (256 threads, one dim each): dst[j] = rope(rmsnorm(src_j) * w), fp32, one
// reduction round for every head; v[j] = this thread's dim of head j, wd the weight there, c / s the rope cos / sin
// of the dim (d < 32)
__device__ __forceinline__ void rms_rope_group(const float* v, int G, float wd, float c, float s, float (*dst)[kHD],
                                               float (*red)[kMaxGroup]) {
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        const float ss = warp_sum(v[j] * v[j]);
        if (lane == 0) red[warp][j] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        if (j >= G) break;
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) t += red[i][j];
        const float r = rsqrt_ieee(t / (float)kHD + kEps);
        dst[j][d] = mul_rn(mul_rn(v[j], r), wd);
    }
    __syncthreads();
    if (d < kRot / 2) {
#pragma unroll
        for (int j = 0; j < kMaxGroup; ++j) {
            if (j >= G) break;
            const float a = dst[j][d], b = dst[j][d + kRot / 2];
            dst[j][d] = mul_rn(a, c) - mul_rn(b, s);
            dst[j][d + kRot / 2] = mul_rn(b, c) + mul_rn(a, s);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_decode_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;  // [3 stages][K page | V page]
    uint16_t* q_s = reinterpret_cast<uint16_t*>(smem + kOffQ);
    uint16_t* knew_s = reinterpret_cast<uint16_t*>(smem + kOffKnew);  // [row j][256] bf16: k of position p0 + j
    uint16_t* vnew_s = reinterpret_cast<uint16_t*>(smem + kOffVnew);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* empty = full + kAttnStages;

    __shared__ float qf[kMaxGroup][kHD];
    __shared__ float kf[kHD];
    __shared__ float red[8];
    __shared__ float lrow[kMaxGroup];
    __shared__ int last_flag;

    const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.G;

    if (tid == 0) {
        for (int i = 0; i < kAttnStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 2);  // the group's two warps
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (p.pf && tid == 0) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        l2_prefetch_share(p.pf, p.pf_bytes, cta, gridDim.x * gridDim.y * gridDim.z);
    }
    const float wq_d = p.wq[tid], wk_d = p.wk[tid];  // immutable: read before the dependency wait
    pdl_wait();

    // Every input that does not depend on the position goes out with the position's load (one L2 round trip, not
    // a chain of them): the group's q rows, their gates, this row's new k and v. What depends on the position
    // (page table entries, rope cos / sin) is the second round.
    const YIn yall{p.y, p.yacc};
    const YIn y = yall.at((size_t)b * p.ld_y);
    const int kbase = 2 * p.h * kHD;
    float qin[kMaxGroup], gin[kMaxGroup];
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        const int hq = g * G + j;
        qin[j] = j < G ? __uint_as_float((uint32_t)y[(size_t)hq * kHD + tid] << 16) : 0.f;
        gin[j] = j < G ? __uint_as_float((uint32_t)y[(size_t)(p.h + hq) * kHD + tid] << 16) : 0.f;
    }
    const float kin = __uint_as_float((uint32_t)y[kbase + (size_t)g * kHD + tid] << 16);
    const uint16_t vin = y[kbase + (size_t)(p.nkv + g) * kHD + tid];
    const int pos = p.pos[b];
    const int p0 = p.verify ? p.pos[0] : pos;  // first position this step writes (new k / v from p0 on)
    if (pos < 0 || pos >= p.max_pos || pos / kKvBlock >= p.max_pages || (p.verify && pos != p0 + b)) {
        if (tid == 0) atomicOr(p.err, kErrBounds);
        return;
    }
    const int L = pos + 1;
    const int npg = (L + kKvBlock - 1) / kKvBlock;
    // at least one page per page group: the groups of a CTA take their pages in parallel, so a chunk of 3 pages
    // costs what a chunk of 1 does, and a short context leaves fewer chunks to combine
    const int ppc = max((npg + p.nchunks - 1) / p.nchunks, min(kAttnGroups, npg));
    const int pg0 = c * ppc, pg1 = min(pg0 + ppc, npg);
    // chunks that hold pages at this length: the others leave at once (no partial, no ticket), so a short
    // context costs what its pages do
    const int nce = (npg + ppc - 1) / ppc;
    if (c >= nce) return;
    const int* pt = p.page_table + (size_t)(p.verify ? 0 : b) * p.max_pages;
    const float* cs = p.cos_tab + (size_t)pos * (kRot / 2);
    const float* sn = p.sin_tab + (size_t)pos * (kRot / 2);
    const float cpos = tid < kRot / 2 ? cs[tid] : 0.f, spos = tid < kRot / 2 ? sn[tid] : 0.f;
    const size_t head_stride = (size_t)kKvBlock * kHD;  // elements per (page, head)

    const int npages = max(pg1 - pg0, 0);
    bool bad_page = false;
    for (int i = 0; i < npages; ++i) {
        const int pg = pt[pg0 + i];
        if (pg < 0 || pg >= p.num_pages) bad_page = true;
    }
    if (bad_page) {
        if (tid == 0) atomicOr(p.err, kErrBounds);
        return;
    }
    const uint64_t pol = policy_evict_first();
    // page i of the run into stage i % 3: 4 boxes of K, then 4 of V (rows of the (page, head) run of the pool)
    auto issue = [&](int i) {
        const int s = i % kAttnStages;
        const int row = (pt[pg0 + i] * p.nkv + g) * kKvBlock;
        uint8_t* dst = ring + (size_t)s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
#pragma unroll
        for (int bx = 0; bx < 4; ++bx) {
            tma_load_2d(dst + bx * kBoxBytes, &tm_k, 64 * bx, row, &full[s], pol);
            tma_load_2d(dst + kPageBytes + bx * kBoxBytes, &tm_v, 64 * bx, row, &full[s], pol);
        }
    };
    // the first pages' copies go out before the q / k math
    if (warp == 6 && lane == 0)
        for (int i = 0; i < min(npages, kAttnStages); ++i) issue(i);

    // q of the group's heads (fp32), then its bf16 hi / lo rows for the tensor cores
    {
        __shared__ float redg[8][kMaxGroup];
        rms_rope_group(qin, G, wq_d, cpos, spos, qf, redg);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float v = j < G ? qf[j < kMaxGroup ? j : 0][tid] : 0.f;
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        const int ch = tid >> 3, e = tid & 7;
        reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(q_s) + q_off(j, ch))[e] = hi;
        reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(q_s) + q_off(j + 8, ch))[e] = lo;
    }
    // k / v of the new positions p0 .. pos whose pages this CTA covers (row j's from its own y row; one step
    // writes the single row pos, whose inputs are loaded already)
    const int pg_lo = pg0 * kKvBlock, pg_hi = pg1 * kKvBlock;  // positions of this CTA's pages
    const int t_lo = max(p0, pg_lo), t_hi = min(pos, pg_hi - 1);
    for (int t = t_lo; t <= t_hi; ++t) {
        const int j = t - p0;
        const YIn yj = yall.at((size_t)(p.verify ? j : b) * p.ld_y);
        const float kv = p.verify ? __uint_as_float((uint32_t)yj[kbase + (size_t)g * kHD + tid] << 16) : kin;
        float ct = cpos, st = spos;  // one step: t = pos
        if (p.verify && tid < kRot / 2) {
            ct = p.cos_tab[(size_t)t * (kRot / 2) + tid];
            st = p.sin_tab[(size_t)t * (kRot / 2) + tid];
        }
        rms_rope_head(kv, wk_d, ct, st, kf, red, true);
        knew_s[j * kHD + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(kf[tid]));
        vnew_s[j * kHD + tid] = p.verify ? yj[kbase + (size_t)(p.nkv + g) * kHD + tid] : vin;
        __syncthreads();  // kf is reused by the next row
    }
    if (pg0 <= pos / kKvBlock && pos / kKvBlock < pg1) {
        // append this row to the cache
        const int pg = pt[pos / kKvBlock];
        const size_t off = ((size_t)pg * p.nkv + g) * head_stride + (size_t)(pos % kKvBlock) * kHD + tid;
        p.kp[off] = knew_s[(pos - p0) * kHD + tid];
        p.vp[off] = vnew_s[(pos - p0) * kHD + tid];
    }
    __syncthreads();

    // ---- the page loop: producer (warp 6) and the three page groups (warps 0..5)
    bool ok = true;
    const int grp = warp >> 1, half = warp & 1;
    const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates: row (head) g, column pair t
    float m_run = -INFINITY, l_run = 0.f;
    float O[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) O[n][0] = O[n][1] = O[n][2] = O[n][3] = 0.f;
    if (warp == 6) {
        if (lane == 0) {
            int issued = min(npages, kAttnStages);
            for (int i = kAttnStages; i < npages && ok; ++i) {
                const int s = i % kAttnStages;
                if (!mbar_wait(&empty[s], ((i / kAttnStages) - 1) & 1, p.err)) {
                    ok = false;
                    break;
                }
                issue(i);
                issued = i + 1;
            }
            // never reuse shared memory with a copy still landing in it (a consumer that timed out stops waiting)
            for (int i = max(0, issued - kAttnStages); i < issued; ++i)
                mbar_wait(&full[i % kAttnStages], (i / kAttnStages) & 1, nullptr);
        }
    } else if (warp < 6) {
        const uint32_t qa = smem_addr(q_s);
        for (int i = grp; i < npages; i += kAttnGroups) {
            const int s = grp;
            if (ok && !mbar_wait(&full[s], (i / kAttnStages) & 1, p.err)) ok = false;
            uint8_t* stage = ring + (size_t)s * kStageBytes;
            const int t0 = (pg0 + i) * kKvBlock;
            // rows this step writes: the step's own k / v (the cache there may be stale or mid-append)
            const int r_lo = max(p0, t0) - t0, r_hi = min(pos, t0 + kKvBlock - 1) - t0;
            if (r_lo <= r_hi) {
                for (int e = half * 32 + lane; e < (r_hi - r_lo + 1) * 32; e += 64) {
                    const int r = r_lo + e / 32, ch = e % 32;
                    const int j = t0 + r - p0;
                    *reinterpret_cast<uint4*>(stage + page_off(r, ch)) = reinterpret_cast<const uint4*>(knew_s + j * kHD)[ch];
                    *reinterpret_cast<uint4*>(stage + kPageBytes + page_off(r, ch)) =
                        reinterpret_cast<const uint4*>(vnew_s + j * kHD)[ch];
                }
                bar_sync(1 + grp, 64);
            }
            const uint32_t ka = smem_addr(stage), va = ka + kPageBytes;
            // S = Q K^T: 8 n-tiles of 8 positions, 16 k-steps of 16 dims
            float S[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n) S[n][0] = S[n][1] = S[n][2] = S[n][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 16; ++ks) {
                uint32_t a[4];
                ldsm_x4(qa + q_off((lane & 7) + 8 * ((lane >> 3) & 1), 2 * ks + (lane >> 4)), a);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t bk[4];
                    ldsm_x4(ka + page_off(16 * np + (lane & 7) + 8 * (lane >> 4), 2 * ks + ((lane >> 3) & 1)), bk);
                    mma_bf16(S[2 * np], a, bk[0], bk[1]);
                    mma_bf16(S[2 * np + 1], a, bk[2], bk[3]);
                }
            }
            // scores of head gq (hi + lo rows), masked past pos; the page's max over the quad
            float sc[8][2];
            float pm = -INFINITY;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = t0 + 8 * n + 2 * tq + e;
                    sc[n][e] = t <= pos ? S[n][e] + S[n][2 + e] : -INFINITY;
                    pm = fmaxf(pm, sc[n][e]);
                }
            }
            pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
            pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
            const float m_new = fmaxf(m_run, pm);
            const float corr = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
            m_run = m_new;
            // P = (p_hi ; p_lo) as the A operand of k-step j (positions 16 j .. 16 j + 15)
            uint32_t pa[4][4];
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int hsel = 0; hsel < 2; ++hsel) {
                    const int n = 2 * j + hsel;
                    const float e0 = sc[n][0] == -INFINITY ? 0.f : expf(sc[n][0] - m_new);
                    const float e1 = sc[n][1] == -INFINITY ? 0.f : expf(sc[n][1] - m_new);
                    ps += e0 + e1;
                    const float h0 = __bfloat162float(__float2bfloat16_rn(e0));
                    const float h1 = __bfloat162float(__float2bfloat16_rn(e1));
                    pa[j][2 * hsel] = pack_bf16(h0, h1);
                    pa[j][2 * hsel + 1] = pack_bf16(e0 - h0, e1 - h1);
                }
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l_run = l_run * corr + ps;
#pragma unroll
            for (int n = 0; n < 16; ++n) {
                O[n][0] *= corr;
                O[n][1] *= corr;
                O[n][2] *= corr;
                O[n][3] *= corr;
            }
            // O += P V over this warp's 128 dims (n-tiles 16 half .. 16 half + 15)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int np = 0; np < 8; ++np) {
                    uint32_t bv[4];
                    ldsm_x4_t(va + page_off(16 * j + (lane & 7) + 8 * ((lane >> 3) & 1), 16 * half + 2 * np + (lane >> 4)), bv);
                    mma_bf16(O[2 * np], pa[j], bv[0], bv[1]);
                    mma_bf16(O[2 * np + 1], pa[j], bv[2], bv[3]);
                }
            }
            // rows patched by generic stores: ordered before the next TMA write into the stage
            if (r_lo <= r_hi) fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    // the next launch (the out-projection, its weights pulled into L2 by this kernel) may start its CTAs from here
    // on: earlier, its CTAs' start-up work on the other SMs slowed this kernel's tail
    pdl_launch();
    // ---- merge the three groups in group order through shared memory (the ring is free: every copy landed)
    __syncthreads();
    float* mg = reinterpret_cast<float*>(ring);                 // [3][8]
    float* lg = mg + kAttnGroups * 8;                           // [3][8]
    float* Og = reinterpret_cast<float*>(ring + 1024);          // [3][8][256]
    if (warp < 6) {
        if (half == 0 && tq == 0) {
            mg[grp * 8 + gq] = m_run;
            lg[grp * 8 + gq] = l_run;
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            const int d = 8 * (16 * half + n) + 2 * tq;
            Og[(grp * 8 + gq) * kHD + d] = O[n][0] + O[n][2];
            Og[(grp * 8 + gq) * kHD + d + 1] = O[n][1] + O[n][3];
        }
    }
    __syncthreads();
    // partial of this chunk: per head (max, sum, o[256]); a single chunk is the result itself (the combine's
    // weights would be exp(0) = 1: the same arithmetic)
    float* part = p.part + ((((size_t)b * p.nkv + g) * p.nchunks + c) * G) * kPartStride;
    for (int j = 0; j < G; ++j) {
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < kAttnGroups; ++q) M = fmaxf(M, mg[q * 8 + j]);
        float Ls = 0.f, ov = 0.f;
#pragma unroll
        for (int q = 0; q < kAttnGroups; ++q) {
            const float mq = mg[q * 8 + j];
            const float wq_ = mq == -INFINITY ? 0.f : expf(mq - M);
            Ls = fmaf(wq_, lg[q * 8 + j], Ls);
            ov = fmaf(wq_, Og[(q * 8 + j) * kHD + tid], ov);
        }
        if (nce == 1) {
            const int hq = g * G + j;
            float gate = 0.f;
#pragma unroll
            for (int q = 0; q < kMaxGroup; ++q)
                if (q == j) gate = gin[q];
            const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(ov / Ls, sigmoid_f(gate)));
            const size_t idx = (size_t)b * p.h * kHD + hq * kHD + tid;
            reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
            if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
            continue;
        }
        if (tid == 0) {
            part[j * kPartStride] = M;
            part[j * kPartStride + 1] = Ls;
        }
        part[j * kPartStride + 2 + tid] = ov;
    }
    if (nce == 1) return;
    // release / acquire through one thread: the barrier orders every thread's stores before thread 0's fence
    // (cumulative) and atomic; the last CTA's fence before the barrier orders the other CTAs' parts before its
    // threads' reads (a fence in every thread costs microseconds)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const int t = atomicAdd(p.ticket + b * p.nkv + g, 1);
        last_flag = (t == nce - 1);
        if (last_flag) __threadfence();
    }
    __syncthreads();
    if (!last_flag) return;
    // combine the chunks in order: o = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, then the gate.
    const float* base = p.part + (((size_t)b * p.nkv + g) * p.nchunks) * G * kPartStride;
    // Every load of the combine is independent, so they go out in wide rounds (each an L2 round trip): the
    // chunks' (m, l) into shared memory in one, then each thread's dimension of every head over 8 chunks at a time.
    float* wch = reinterpret_cast<float*>(ring + kStageBytes);  // [nchunks][G] chunk maxima, then weights
    float* lch = wch + p.nchunks * G;                            // [nchunks][G] chunk sums
    for (int i = tid; i < nce * G; i += kAttnThreads) {
        wch[i] = __ldcg(base + (size_t)i * kPartStride);
        lch[i] = __ldcg(base + (size_t)i * kPartStride + 1);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int cc = 0; cc < nce; ++cc) M = fmaxf(M, wch[cc * G + tid]);
        float Lsum = 0.f;
        for (int cc = 0; cc < nce; ++cc) {
            const float mc = wch[cc * G + tid];
            const float w = mc == -INFINITY ? 0.f : expf(mc - M);
            wch[cc * G + tid] = w;
            Lsum = fmaf(w, lch[cc * G + tid], Lsum);
        }
        lrow[tid] = Lsum;
    }
    __syncthreads();
    constexpr int kCU = 8;  // chunks per round
    float Ov[kMaxGroup];
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) Ov[j] = 0.f;
    for (int cc = 0; cc < nce; cc += kCU) {
        float ov[kCU][kMaxGroup];
#pragma unroll
        for (int u = 0; u < kCU; ++u)
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j)
                ov[u][j] = (j < G && cc + u < nce) ? __ldcg(base + ((size_t)(cc + u) * G + j) * kPartStride + 2 + tid) : 0.f;
        // chunk weights applied in chunk order
#pragma unroll
        for (int u = 0; u < kCU; ++u)
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j) {
                const float w = (j < G && cc + u < nce) ? wch[(cc + u) * G + j] : 0.f;
                if (w != 0.f) Ov[j] = fmaf(w, ov[u][j], Ov[j]);
            }
    }
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        if (j >= G) break;
        const int hq = g * G + j;
        const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(Ov[j] / lrow[j], sigmoid_f(gin[j])));
        const size_t idx = (size_t)b * p.h * kHD + hq * kHD + tid;
        reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
        if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
    }
    if (tid == 0) p.ticket[b * p.nkv + g] = 0;
}

size_t attn_workspace_bytes(int nranks, int rows, int nchunks) {
    const int h = 24 / nranks, nkv = nranks <= 4 ? 4 / nranks : 1, G = h / nkv;
    size_t part = (size_t)rows * nkv * nchunks * G * kPartStride * 4;
    part = (part + 255) & ~size_t(255);
    return part + 256 + (size_t)rows * nkv * 4;
}

// CTAs per (user, kv head): one per SM over all of them (the kernel takes a whole SM's shared memory)
int attn_default_chunks(int nranks, int rows, int sm_count, int max_pages) {
    const int nkv = nranks <= 4 ? 4 / nranks : 1;
    int c = (sm_count + nkv * rows - 1) / (nkv * rows);
    if (c > max_pages) c = max_pages;
    return c < 1 ? 1 : c;
}

// ---- tensor maps of the KV pools (one per pool, made on first use and kept: a pool's pointer and page count
// identify it) -------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static cudaError_t kv_tensor_map(const uint16_t* pool, int num_pages, int nkv, CUtensorMap* out) {
    static std::mutex mu;
    static std::unordered_map<const void*, std::pair<uint64_t, CUtensorMap>> cache;
    static EncodeTiledFn encode = nullptr;
    const uint64_t rows = (uint64_t)num_pages * nkv * kKvBlock;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(pool);
    if (it != cache.end() && it->second.first == rows) {
        *out = it->second.second;
        return cudaSuccess;
    }
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    // the pool as a 2-D tensor [rows][256] bf16; boxes of 64 rows x 64 dims (128 bytes: the swizzle span)
    const cuuint64_t dims[2] = {(cuuint64_t)kHD, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kHD * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kKvBlock};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(pool), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    cache[pool] = {rows, m};
    *out = m;
    return cudaSuccess;
}

cudaError_t attn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const int32_t* page_table,
                        int max_pages, int num_pages, const float* wq, const float* wk, const float* cos_tab,
                        const float* sin_tab, int max_pos, uint16_t* kp, uint16_t* vp, uint16_t* o, uint16_t* mixer_copy,
                        void* work, size_t work_bytes, int nchunks, uint32_t* err, cudaStream_t st, bool pdl,
                        const void* pf, size_t pf_bytes, int verify, const long long* yacc) {
    if (nranks < 1 || 24 % nranks || rows < 1 || rows > kMaxRows || (verify && verify != rows)) return cudaErrorInvalidValue;
    if (work_bytes < attn_workspace_bytes(nranks, rows, nchunks)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) & 15) return cudaErrorInvalidValue;
    AttnParams p;
    p.h = 24 / nranks;
    p.nkv = nranks <= 4 ? 4 / nranks : 1;
    p.G = p.h / p.nkv;
    p.ld_y = ld_y;
    p.y = yacc ? nullptr : y;
    p.yacc = yacc;
    p.pos = pos;
    p.page_table = page_table;
    p.max_pages = max_pages;
    p.num_pages = num_pages;
    p.wq = wq;
    p.wk = wk;
    p.cos_tab = cos_tab;
    p.sin_tab = sin_tab;
    p.max_pos = max_pos;
    p.kp = kp;
    p.vp = vp;
    p.o = o;
    p.mixer_copy = mixer_copy;
    size_t part = (size_t)rows * p.nkv * nchunks * p.G * kPartStride * 4;
    part = (part + 255) & ~size_t(255);
    p.part = static_cast<float*>(work);
    p.ticket = reinterpret_cast<int*>(static_cast<uint8_t*>(work) + part + 256);
    p.nchunks = nchunks;
    p.verify = verify;
    p.pf = static_cast<const uint8_t*>(pf);
    p.pf_bytes = pf_bytes;
    p.err = err;
    CUtensorMap tk, tv;
    cudaError_t e = kv_tensor_map(kp, num_pages, p.nkv, &tk);
    if (e != cudaSuccess) return e;
    e = kv_tensor_map(vp, num_pages, p.nkv, &tv);
    if (e != cudaSuccess) return e;
    static bool smem_set = false;
    if (!smem_set) {
        e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
        if (e != cudaSuccess) return e;
        smem_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nchunks, p.nkv, rows);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kAttnSmem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel, p, tk, tv);
}

}  // namespace qres
