// Gated GQA decode attention over a paged KV cache for sm_100a (split-K over pages, flash-decoding).
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
// the current context, so every CTA works at any length), streams each page's K and V with one cp.async.bulk
// each into a double-buffered shared ring, scores it for the G query heads that share the KV head (K read once
// per group), and keeps an online softmax (m, l, o[256]) per head. Partials go to the workspace; the last CTA
// of a (user, kv head) -- an atomic ticket -- combines them in chunk order (deterministic) and applies the gate.
// The CTA whose pages hold `pos` appends k / v to the cache and uses them from shared memory for that row.
//
// Verify step (R consecutive positions p .. p+R-1 of one user, attn_common.hpp:39-42 KV sharing; row r sees
// rows < r): all rows share user 0's page table; every CTA of row r computes k / v of rows 0..r itself and
// uses them for positions p .. p+r (the cache there may be mid-append by other rows' CTAs, so it is never read
// for those positions); each row still appends its own position.
#include "qres_common.cuh"

namespace qres {

constexpr int kAttnThreads = 256;
constexpr int kMaxGroup = 6;  // query heads per KV head on a rank (24 / 4)
constexpr int kPageBytes = kKvBlock * kHD * 2;  // 32 KB per head page of K (or V)

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

__host__ __device__ inline size_t attn_smem_bytes() {
    return 2 * 2 * (size_t)kPageBytes /* K,V double buffer */ + 64 /* barriers */;
}

__device__ __forceinline__ void rms_rope_head(const YIn src, const float* w, const float* cs, const float* sn,
                                              float* dst, float* red, bool round_bf16) {
    // one head of 256 dims by 256 threads: dst = rope(rmsnorm(src) * w) (optionally rounded to bf16)
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
    const float v = __uint_as_float((uint32_t)src[d] << 16);
    float ss = warp_sum(v * v);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float r = rsqrt_ieee(t / (float)kHD + kEps);
    const float nv = mul_rn(mul_rn(v, r), w[d]);
    dst[d] = nv;
    __syncthreads();
    if (d < kRot / 2) {
        const float a = dst[d], b = dst[d + kRot / 2];
        const float c = cs[d], s = sn[d];
        const float ra = mul_rn(a, c) - mul_rn(b, s);
        const float rb = mul_rn(b, c) + mul_rn(a, s);
        dst[d] = round_bf16 ? bf16_round(ra) : ra;
        dst[d + kRot / 2] = round_bf16 ? bf16_round(rb) : rb;
    } else if (d >= kRot && round_bf16) {
        dst[d] = bf16_round(nv);
    }
    __syncthreads();
}

// the G query heads of a group at once (256 threads, one dim each): dst[j] = rope(rmsnorm(src_j) * w), fp32; all
// loads in flight together and one reduction round for every head
__device__ __forceinline__ void rms_rope_group(const YIn src, int G, const float* w, const float* cs,
                                               const float* sn, float (*dst)[kHD], float (*red)[kMaxGroup]) {
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
    float v[kMaxGroup];
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) v[j] = j < G ? __uint_as_float((uint32_t)src[(size_t)j * kHD + d] << 16) : 0.f;
    const float wd = w[d];
    float c = 0.f, s = 0.f;
    if (d < kRot / 2) {
        c = cs[d];
        s = sn[d];
    }
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

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;  // [2][K page | V page]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 4 * (size_t)kPageBytes);

    __shared__ float qf[kMaxGroup][kHD];
    __shared__ float knew[kMaxRows][kHD];  // k / v of the positions this step writes (row order)
    __shared__ float vnew[kMaxRows][kHD];
    __shared__ float sc[kMaxGroup][kKvBlock];
    __shared__ float red[8];
    __shared__ float mrow[kMaxGroup], corr[kMaxGroup], lrow[kMaxGroup];
    __shared__ int last_flag;

    const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.G;

    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch();
    if (p.pf && tid == 0) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        l2_prefetch_share(p.pf, p.pf_bytes, cta, gridDim.x * gridDim.y * gridDim.z);
    }
    pdl_wait();

    const int pos = p.pos[b];
    const int p0 = p.verify ? p.pos[0] : pos;  // first position this step writes (new k / v from p0 on)
    if (pos < 0 || pos >= p.max_pos || pos / kKvBlock >= p.max_pages || (p.verify && pos != p0 + b)) {
        if (tid == 0) atomicOr(p.err, kErrBounds);
        return;
    }
    const int L = pos + 1;
    const int npg = (L + kKvBlock - 1) / kKvBlock;
    const int ppc = (npg + p.nchunks - 1) / p.nchunks;
    const int pg0 = c * ppc, pg1 = min(pg0 + ppc, npg);
    // chunks that hold pages at this length: the others leave at once (no partial, no ticket), so a short
    // context costs what its pages do
    const int nce = (npg + ppc - 1) / ppc;
    if (c >= nce) return;
    const int* pt = p.page_table + (size_t)(p.verify ? 0 : b) * p.max_pages;
    const YIn yall{p.y, p.yacc};
    const YIn y = yall.at((size_t)b * p.ld_y);
    const float* cs = p.cos_tab + (size_t)pos * (kRot / 2);
    const float* sn = p.sin_tab + (size_t)pos * (kRot / 2);
    const size_t head_stride = (size_t)kKvBlock * kHD;  // elements per (page, head)

    // the first pages' bulk copies go out before the q / k math
    auto issue = [&](int i, int slot) {
        const int pg = pt[pg0 + i];
        const size_t off = ((size_t)pg * p.nkv + g) * head_stride;
        mbar_arrive_expect_tx(&full[slot], 2 * kPageBytes);
        bulk_g2s(ring + (size_t)slot * 2 * kPageBytes, p.kp + off, kPageBytes, &full[slot]);
        bulk_g2s(ring + (size_t)slot * 2 * kPageBytes + kPageBytes, p.vp + off, kPageBytes, &full[slot]);
    };
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
    if (tid == 0) {
        for (int i = 0; i < min(npages, 2); ++i) issue(i, i);
    }

    // q of the group's heads (fp32), all heads in one pass
    {
        __shared__ float redg[8][kMaxGroup];
        rms_rope_group(y.at((size_t)(g * G) * kHD), G, p.wq, cs, sn, qf, redg);
    }
    // k / v of the new positions p0 .. pos whose pages this CTA covers (row j's from its own y row)
    const int kbase = 2 * p.h * kHD;
    const int pg_lo = pg0 * kKvBlock, pg_hi = pg1 * kKvBlock;  // positions of this CTA's pages
    for (int t = max(p0, pg_lo); t <= pos && t < pg_hi; ++t) {
        const int j = t - p0;
        const YIn yj = yall.at((size_t)(p.verify ? j : b) * p.ld_y);
        rms_rope_head(yj.at(kbase + (size_t)g * kHD), p.wk, p.cos_tab + (size_t)t * (kRot / 2),
                      p.sin_tab + (size_t)t * (kRot / 2), knew[j], red, true);
        vnew[j][tid] = __uint_as_float((uint32_t)yj[kbase + p.nkv * kHD + g * kHD + tid] << 16);
    }
    const bool has_pos = pg0 <= pos / kKvBlock && pos / kKvBlock < pg1;
    if (has_pos) {
        __syncthreads();
        // append this row to the cache
        const int pg = pt[pos / kKvBlock];
        const size_t off = ((size_t)pg * p.nkv + g) * head_stride + (size_t)(pos % kKvBlock) * kHD + tid;
        p.kp[off] = __bfloat16_as_ushort(__float2bfloat16_rn(knew[pos - p0][tid]));
        p.vp[off] = __bfloat16_as_ushort(__float2bfloat16_rn(vnew[pos - p0][tid]));
    }
    __syncthreads();

    float qreg[kMaxGroup][8];
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) qreg[j][e] = j < G ? qf[j][lane * 8 + e] : 0.f;

    float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup];
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        o[j] = 0.f;
    }
    bool ok = true;
    for (int i = 0; i < npages; ++i) {
        const int slot = i & 1;
        if (ok) ok = mbar_wait(&full[slot], (i >> 1) & 1, p.err);
        const uint16_t* Ks = reinterpret_cast<const uint16_t*>(ring + (size_t)slot * 2 * kPageBytes);
        const uint16_t* Vs = Ks + kKvBlock * kHD;
        const int t0 = (pg0 + i) * kKvBlock;
        // scores: warp w takes rows w, w+8, ...; lane l dims 8l..8l+7
        for (int r = warp; r < kKvBlock; r += 8) {
            const int t = t0 + r;
            float dot[kMaxGroup];
            if (t >= p0 && t <= pos) {
                const float* kn = knew[t - p0];
#pragma unroll
                for (int j = 0; j < kMaxGroup; ++j) {
                    float a = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) a = fmaf(qreg[j][e], kn[lane * 8 + e], a);
                    dot[j] = a;
                }
            } else {
                const uint4 kv = lds128(Ks + r * kHD + lane * 8);
                const float kf[8] = {bf16lo(kv.x), bf16hi(kv.x), bf16lo(kv.y), bf16hi(kv.y),
                                     bf16lo(kv.z), bf16hi(kv.z), bf16lo(kv.w), bf16hi(kv.w)};
#pragma unroll
                for (int j = 0; j < kMaxGroup; ++j) {
                    float a = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) a = fmaf(qreg[j][e], kf[e], a);
                    dot[j] = a;
                }
            }
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j) {
                const float v = warp_sum(dot[j]);
                if (lane == 0 && j < G) sc[j][r] = t <= pos ? v : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax: warp j < G handles head j's 64 scores
        if (warp < G) {
            const int j = warp;
            const float s0 = sc[j][lane], s1 = sc[j][lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float mprev = i == 0 ? -INFINITY : mrow[j];
            const float mnew = fmaxf(mprev, mx);
            const float p0 = s0 == -INFINITY ? 0.f : expf(s0 - mnew);
            const float p1 = s1 == -INFINITY ? 0.f : expf(s1 - mnew);
            sc[j][lane] = p0;
            sc[j][lane + 32] = p1;
            const float ps = warp_sum(p0 + p1);
            if (lane == 0) {
                const float cr = i == 0 ? 0.f : expf(mrow[j] - mnew);
                corr[j] = cr;
                lrow[j] = (i == 0 ? 0.f : lrow[j] * cr) + ps;
                mrow[j] = mnew;
            }
        }
        __syncthreads();
        // o[j][d] = o * corr + sum_r p[j][r] * V[r][d]; thread = dim d
        {
            const int d = tid;
            float acc[kMaxGroup];
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j) acc[j] = 0.f;
            for (int r = 0; r < kKvBlock; ++r) {
                const int t = t0 + r;
                if (t > pos) break;
                const float vv = t >= p0 ? vnew[t - p0][d] : __uint_as_float((uint32_t)Vs[r * kHD + d] << 16);
#pragma unroll
                for (int j = 0; j < kMaxGroup; ++j) acc[j] = fmaf(sc[j][r], vv, acc[j]);
            }
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j) o[j] = o[j] * corr[j] + acc[j];
        }
        __syncthreads();  // the slot is free again
        if (tid == 0 && i + 2 < npages && ok) issue(i + 2, slot);
    }
#pragma unroll
    for (int j = 0; j < kMaxGroup; ++j) {
        m[j] = npages ? mrow[j < G ? j : 0] : -INFINITY;
        l[j] = npages ? lrow[j < G ? j : 0] : 0.f;
    }
    // partial of this chunk
    float* part = p.part + ((((size_t)b * p.nkv + g) * p.nchunks + c) * G) * (2 + kHD);
    for (int j = 0; j < G; ++j) {
        if (tid == 0) {
            part[j * (2 + kHD)] = m[j];
            part[j * (2 + kHD) + 1] = l[j];
        }
#pragma unroll
        for (int jj = 0; jj < kMaxGroup; ++jj)
            if (jj == j) part[j * (2 + kHD) + 2 + tid] = o[jj];
    }
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
    // combine the chunks in order: o = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, then the gate. The chunk
    // weights are computed once in shared memory; every thread then sums its dimension over the chunks with
    // independent loads.
    const float* base = p.part + (((size_t)b * p.nkv + g) * p.nchunks) * G * (2 + kHD);
    float* wch = reinterpret_cast<float*>(ring);  // [nchunks][G] chunk weights (the K/V ring is free now)
    for (int i = tid; i < nce * G; i += kAttnThreads) wch[i] = __ldcg(base + (size_t)i * (2 + kHD));
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int cc = 0; cc < nce; ++cc) M = fmaxf(M, wch[cc * G + tid]);
        float Lsum = 0.f;
        for (int cc = 0; cc < nce; ++cc) {
            const float mc = wch[cc * G + tid];
            const float w = mc == -INFINITY ? 0.f : expf(mc - M);
            wch[cc * G + tid] = w;
            Lsum = fmaf(w, __ldcg(base + ((size_t)cc * G + tid) * (2 + kHD) + 1), Lsum);
        }
        lrow[tid] = Lsum;
    }
    __syncthreads();
    for (int j = 0; j < G; ++j) {
        float O = 0.f;
#pragma unroll 8
        // chunk weights applied in chunk order; the loads of 4 chunks in flight at once
        for (int cc = 0; cc < nce; cc += 4) {
            float ov[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                ov[u] = cc + u < nce ? __ldcg(base + ((size_t)(cc + u) * G + j) * (2 + kHD) + 2 + tid) : 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float w = cc + u < nce ? wch[(cc + u) * G + j] : 0.f;
                if (w != 0.f) O = fmaf(w, ov[u], O);
            }
        }
        const int hq = g * G + j;
        const float gate = __uint_as_float((uint32_t)y[p.h * kHD + hq * kHD + tid] << 16);
        const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(O / lrow[j], sigmoid_f(gate)));
        const size_t idx = (size_t)b * p.h * kHD + hq * kHD + tid;
        reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
        if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
    }
    if (tid == 0) p.ticket[b * p.nkv + g] = 0;
}

size_t attn_workspace_bytes(int nranks, int rows, int nchunks) {
    const int h = 24 / nranks, nkv = nranks <= 4 ? 4 / nranks : 1, G = h / nkv;
    size_t part = (size_t)rows * nkv * nchunks * G * (2 + kHD) * 4;
    part = (part + 255) & ~size_t(255);
    return part + 256 + (size_t)rows * nkv * 4;
}

int attn_default_chunks(int nranks, int rows, int sm_count, int max_pages) {
    const int nkv = nranks <= 4 ? 4 / nranks : 1;
    int c = (sm_count + nkv * rows - 1) / (nkv * rows);
    if (c > max_pages) c = max_pages;
    return c < 1 ? 1 : c;
}

cudaError_t attn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const int32_t* page_table,
                        int max_pages, int num_pages, const float* wq, const float* wk, const float* cos_tab,
                        const float* sin_tab, int max_pos, uint16_t* kp, uint16_t* vp, uint16_t* o, uint16_t* mixer_copy,
                        void* work, size_t work_bytes, int nchunks, uint32_t* err, cudaStream_t st, bool pdl,
                        const void* pf, size_t pf_bytes, int verify, const long long* yacc) {
    if (nranks < 1 || 24 % nranks || rows < 1 || rows > kMaxRows || (verify && verify != rows)) return cudaErrorInvalidValue;
    if (work_bytes < attn_workspace_bytes(nranks, rows, nchunks)) return cudaErrorInvalidValue;
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
    size_t part = (size_t)rows * p.nkv * nchunks * p.G * (2 + kHD) * 4;
    part = (part + 255) & ~size_t(255);
    p.part = static_cast<float*>(work);
    p.ticket = reinterpret_cast<int*>(static_cast<uint8_t*>(work) + part + 256);
    p.nchunks = nchunks;
    p.verify = verify;
    p.pf = static_cast<const uint8_t*>(pf);
    p.pf_bytes = pf_bytes;
    p.err = err;
    const size_t smem = attn_smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nchunks, p.nkv, rows);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel, p);
}

}  // namespace qres
