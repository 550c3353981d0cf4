// Gated DeltaNet decode mixer for sm_100a: one 4-CTA cluster per (value head, user), CTA q owning value
// columns [32q, 32q + 32) of the head's state.
//
// Replaces the reference's conv1d + SiLU of the streamers (qwen36_resident/kernels/streamer_compute.cpp:279-370,
// history ring streamer_common.hpp:280-288) and its GDN head cores (gdn_head_reader.cpp / gdn_head_compute.cpp
// :180-347 / gdn_head_writer.cpp), i.e. the math of model.py:255-276:
//   conv  = bf16(silu(sum_j window[j] * tap[j]))          window = inputs at p-3, p-2, p-1, p (oldest first)
//   qn    = q * rsqrt(sum q^2 + 1e-6) * 128^-0.5;   kn = k * rsqrt(sum k^2 + 1e-6)
//   decay = exp(neg_a * softplus(a + dt));  beta = sigmoid(b)
//   delta = beta * (v - (decay * kn) @ S);  S <- decay * S + kn (x) delta;  o = qn @ S
//   out   = bf16(rmsnorm(o) * norm_w * silu(z))
// The fp32 state S [128 (k)][128 (v)] stays in HBM and is updated in place (64 KB read + 64 KB written per head
// and user). Its columns are independent, so a head splits into 4 CTAs of 32 columns (16 KB each way) for
// parallelism; the only cross-column quantity, the sum of o^2 of the gated RMSNorm, is reduced over the
// cluster through distributed shared memory in CTA order (deterministic). Each CTA recomputes the conv and the
// norms of the head's q and k (256 channels) and convolves its own 32 v channels.
//
// Conv history: a ring of QRES_HIST_SLOTS slots per user, position q's input in slot q % 8. A step at p reads
// the slots of p-3..p-1 and writes slot p (never a slot it reads), so the CTAs sharing a key head all read the q
// / k history while one of them writes it.
//
// Verify step (ResidentModel(verify=True), the reference's verify rows model.py:416-457, gdn_head_reader.cpp
// :367-370 / :523-537): the rows are R <= 5 consecutive positions p .. p+R-1 of one user, run as R consecutive
// steps inside one launch: the cluster keeps the head's state in registers from row to row, row r's conv window
// takes the inputs at p .. p+r from the step's own rows (and p+r-3 .. p-1 from the ring, which this step never
// writes since R + 3 <= 8), and row r's state goes to slot (slot0 + r) % R of the user's R state slots (slot0:
// the token state's slot, holding the state row 0 starts from). Continuing after accepting row k means slot0 +
// k and position p + k + 1: no rollback is needed.
#include <cooperative_groups.h>

#include "qres_common.cuh"

namespace cg = cooperative_groups;

namespace qres {

constexpr int kGdnThreads = 128;
constexpr int kGdnSplit = 4;               // CTAs (column quarters) per head
constexpr int kGdnCols = kDV / kGdnSplit;  // 32

struct GdnParams {
    int nk, nv;              // local key / value heads
    int ld_y;                // elements between users' y rows
    const uint16_t* y;       // [B][ld_y] bf16: q | k | v | z | a | b
    const long long* yacc;   // or the in-projection's fixed-point sums, same layout (y null)
    const int32_t* pos;      // [B]
    const uint16_t* taps;    // [conv][4] bf16
    const float* dt;         // [nv]
    const float* neg_a;      // [nv]
    const float* norm_w;     // [128]
    float* state;            // [B][nv][128][128]; verify: [R slots][nv][128][128] of the one user
    int rows;                // users (the batch kernel's groups)
    int verify;              // 0, or R: the rows are R consecutive positions of one user
    const int32_t* slot0;    // verify: the state slot row 0 starts from (device, the token state)
    uint16_t* hist;          // [B][8][conv]
    uint16_t* o;             // [B][nv * 128] bf16
    uint16_t* mixer_copy;    // optional second output
    const uint8_t* pf;       // the next projection's weights: prefetched into L2 while this kernel runs
    size_t pf_bytes;
    uint32_t* err;
};

__global__ void __cluster_dims__(1, 1, kGdnSplit) __launch_bounds__(kGdnThreads, 5) gdn_decode_kernel(const GdnParams p) {
    cg::cluster_group cluster = cg::this_cluster();
    const int hh = blockIdx.x;  // local value head
    const int b = blockIdx.y;   // user
    const int qtr = blockIdx.z; // column quarter (= rank in the cluster)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = p.nk * kDK, gv = p.nv * kDV;
    const int conv = 2 * gq + gv;
    const int group = p.nv / p.nk;
    const int kh = hh / group;
    const int c0 = qtr * kGdnCols;  // first column of this CTA

    __shared__ float qk[2][kDK];      // conv outputs q, k of the key head (bf16 values)
    __shared__ float vv[kGdnCols];    // conv output v of this CTA's columns
    __shared__ float red[16][kGdnCols];
    __shared__ float qs[kDK], ks[kDK], dl[kGdnCols];
    __shared__ float sc[8];
    __shared__ float osq;             // this CTA's sum of o^2, read by the whole cluster

    // thread layout over the CTA's 128 x 32 slice: column quad cq (4 columns), rows 8rp .. 8rp+7
    const int cq = tid & 7, rp = tid >> 3;
    const int R = p.verify;  // verify: rows of the one user, run in order in this cluster
    const int nrows = R ? R : 1;
    const size_t slot_stride = (size_t)p.nv * kDK * kDV;
    // Before griddepcontrol.wait only immutable data may be read (an earlier kernel of the stream may still be
    // running); an L2 prefetch of the state is safe (L2 is the point of coherence) and starts its 16 KB early.
    // The cluster's CTAs prefetch the head's 64 KB as four contiguous quarters (rows 32 q .. 32 q + 31), one bulk
    // prefetch each: a prefetch per 128-byte row of the CTA's own columns would queue 128 small operations.
    if (!R && tid == 0)
        bulk_prefetch_l2(p.state + ((((size_t)b * p.nv + hh) * kDK) + 32 * qtr) * kDV, 32 * kDV * 4);
    // the conv taps (immutable) and every slot of this CTA's conv-history channels (written only by this kernel,
    // a step earlier) into L2 as well: q and k of the key head (2 x 256 B per slot), v of the CTA's 32 columns
    if (tid >= kDK - 3 * 8 && tid < kDK) {
        const int i = tid - (kDK - 3 * 8);  // 24 threads: 8 slots x (q, k, v)
        const int slot = i / 3, part = i % 3;
        const uint16_t* h = p.hist + ((size_t)(R ? 0 : b) * QRES_HIST_SLOTS + slot) * conv;
        const size_t ch = part == 0 ? (size_t)kh * kDK : part == 1 ? (size_t)gq + kh * kDK : (size_t)2 * gq + hh * kDV + c0;
        const uint32_t bytes = part == 2 ? kGdnCols * 2 : kDK * 2;
        // 16-byte aligned starts and sizes (channel offsets are multiples of 32)
        bulk_prefetch_l2(h + ch, bytes);
    }
    if (tid == 0) {
        bulk_prefetch_l2(p.taps + (size_t)kh * kDK * 4, kDK * 8);
        bulk_prefetch_l2(p.taps + ((size_t)gq + kh * kDK) * 4, kDK * 8);
        bulk_prefetch_l2(p.taps + ((size_t)2 * gq + hh * kDV + c0) * 4, kGdnCols * 8);
    }
    // the following projection's weights (immutable) stream into L2 meanwhile: this kernel is latency-bound
    if (p.pf && tid == 0) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        l2_prefetch_share(p.pf, p.pf_bytes, cta, gridDim.x * gridDim.y * gridDim.z);
    }
    pdl_wait();
    const int s0slot = R ? *p.slot0 : 0;
    const int p0 = p.pos[R ? 0 : b];  // verify: row 0's position
    // the whole launch agrees on validity (uniform over the cluster): positions, and verify's rows / slot
    bool bad = p0 < 0 || (R && (s0slot < 0 || s0slot >= R));
    for (int r = 1; R && r < R; ++r) bad = bad || p.pos[r] != p0 + r;
    float4 s[8];
    if (!bad) {
        const float* Sin = p.state + (R ? (size_t)s0slot * slot_stride : (size_t)b * slot_stride) +
                           (size_t)hh * kDK * kDV + c0;
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i] = reinterpret_cast<const float4*>(Sin + (size_t)(rp * 8 + i) * kDV)[cq];
    }
    uint16_t* hist = p.hist + (size_t)(R ? 0 : b) * QRES_HIST_SLOTS * conv;
    // the head's per-layer parameters (immutable) and this CTA's gated-norm weights, loaded once
    const float dt_h = p.dt[hh], na_h = p.neg_a[hh];
    const float nw_c = p.norm_w[c0 + lane];
    for (int row = 0; row < nrows; ++row) {
        const int bb = R ? row : b;  // the row's index in y / o
        const int pos = p0 + (R ? row : 0);
        const YIn yall{p.y, p.yacc};
        const YIn y = yall.at((size_t)bb * p.ld_y);
        float* S = p.state + (R ? (size_t)((s0slot + row) % R) * slot_stride : (size_t)b * slot_stride) +
                   (size_t)hh * kDK * kDV + c0;
        // every in-projection value this row needs besides the conv inputs, issued with them: a, b of the head and
        // z of this CTA's columns (no load waits behind a barrier later)
        const int a_off = 2 * gq + 2 * gv;
        const uint16_t a_raw = bad ? 0 : y[a_off + hh];
        const uint16_t b_raw = bad ? 0 : y[a_off + p.nv + hh];
        const uint16_t z_raw = bad ? 0 : y[2 * gq + gv + hh * kDV + c0 + lane];
        if (!bad) {
            const int swr = pos % QRES_HIST_SLOTS;
            // ---- conv1d + SiLU: q, k of the key head (256 channels) and this CTA's 32 v channels; a thread's
            // (up to 3) channels have all their loads in flight before any arithmetic
            constexpr int kIt = (2 * kDK + kGdnCols + kGdnThreads - 1) / kGdnThreads;  // 3
            uint16_t yin[kIt], hw[kIt][3];
            uint2 tp[kIt];
            int chs[kIt];
#pragma unroll
            for (int it = 0; it < kIt; ++it) {
                const int i = tid + it * kGdnThreads;
                chs[it] = -1;
                if (i < 2 * kDK + kGdnCols) {
                    const int ch = i < kDK ? kh * kDK + i
                                           : i < 2 * kDK ? gq + kh * kDK + (i - kDK) : 2 * gq + hh * kDV + c0 + (i - 2 * kDK);
                    chs[it] = ch;
                    yin[it] = y[ch];
                    // window positions pos-3 .. pos-1: from the ring below p0, from this step's rows from p0 on
#pragma unroll
                    for (int jj = 0; jj < 3; ++jj) {
                        const int q = pos - 3 + jj;
                        hw[it][jj] = q >= p0 && R ? yall[(size_t)(q - p0) * p.ld_y + ch]
                                                  : hist[(size_t)((q + QRES_HIST_SLOTS) % QRES_HIST_SLOTS) * conv + ch];
                    }
                    tp[it] = *reinterpret_cast<const uint2*>(p.taps + (size_t)ch * 4);
                }
            }
#pragma unroll
            for (int it = 0; it < kIt; ++it) {
                const int i = tid + it * kGdnThreads;
                if (chs[it] < 0) continue;
                const int ch = chs[it];
                const int which = i < kDK ? 0 : i < 2 * kDK ? 1 : 2;
                float w[4];
#pragma unroll
                for (int jj = 0; jj < 3; ++jj) w[jj] = __uint_as_float((uint32_t)hw[it][jj] << 16);
                w[3] = __uint_as_float((uint32_t)yin[it] << 16);
                const float t0 = bf16lo(tp[it].x), t1 = bf16hi(tp[it].x), t2 = bf16lo(tp[it].y), t3 = bf16hi(tp[it].y);
                float acc = mul_rn(w[0], t0);
                acc = add_rn(acc, mul_rn(w[1], t1));
                acc = add_rn(acc, mul_rn(w[2], t2));
                acc = add_rn(acc, mul_rn(w[3], t3));
                const float c = bf16_round(silu_f(acc));
                if (which == 0) qk[0][i] = c;
                else if (which == 1) qk[1][i - kDK] = c;
                else vv[i - 2 * kDK] = c;
                // one writer per history element: the key head's first value head, quarter 0, for q / k; every
                // quarter for its v columns
                if (which == 2 || (hh % group == 0 && qtr == 0)) hist[swr * conv + ch] = yin[it];
            }
        }
        // the next launch may start its CTAs once this row's conv is done (earlier, their start-up work slowed
        // this latency-bound kernel)
        if (row == 0) pdl_launch();
        __syncthreads();
        if (!bad) {
            // ---- l2 norms of q (warps 0, 1) and k (warps 2, 3)
            const int which = warp >> 1;
            const float v0 = qk[which][(warp & 1) * 64 + lane], v1 = qk[which][(warp & 1) * 64 + 32 + lane];
            const float ss = warp_sum(v0 * v0 + v1 * v1);
            if (lane == 0) sc[warp] = ss;
        }
        __syncthreads();
        float decay = 0.f;
        if (!bad) {
            for (int i = tid; i < 2 * kDK; i += kGdnThreads) {
                const int which = i >> 7, e = i & 127;
                const float ssum = sc[2 * which] + sc[2 * which + 1];
                const float r = rsqrt_ieee(ssum + 1e-6f);
                const float v = mul_rn(qk[which][e], r);
                if (which == 0) qs[e] = mul_rn(v, 0.08838834764831845f);
                else ks[e] = v;
            }
            const float av = __uint_as_float((uint32_t)a_raw << 16);
            decay = expf(mul_rn(na_h, softplus_f(add_rn(av, dt_h))));
        }
        __syncthreads();
        float part[4] = {0.f, 0.f, 0.f, 0.f};
        if (!bad) {
            // ---- kS = (decay * kn) @ S over this CTA's columns
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float dk = mul_rn(decay, ks[rp * 8 + i]);
                part[0] = fmaf(dk, s[i].x, part[0]);
                part[1] = fmaf(dk, s[i].y, part[1]);
                part[2] = fmaf(dk, s[i].z, part[2]);
                part[3] = fmaf(dk, s[i].w, part[3]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) red[rp][4 * cq + j] = part[j];
        }
        __syncthreads();
        if (!bad && tid < kGdnCols) {
            const float beta = sigmoid_f(__uint_as_float((uint32_t)b_raw << 16));
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < 16; ++w) t += red[w][tid];
            dl[tid] = mul_rn(beta, vv[tid] - t);
        }
        __syncthreads();
        if (!bad) {
            // ---- S <- decay * S + kn (x) delta, o = qn @ S
            const float d0 = dl[4 * cq], d1 = dl[4 * cq + 1], d2 = dl[4 * cq + 2], d3 = dl[4 * cq + 3];
#pragma unroll
            for (int j = 0; j < 4; ++j) part[j] = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float kn = ks[rp * 8 + i], qn = qs[rp * 8 + i];
                float4 v = s[i];
                v.x = add_rn(mul_rn(decay, v.x), mul_rn(kn, d0));
                v.y = add_rn(mul_rn(decay, v.y), mul_rn(kn, d1));
                v.z = add_rn(mul_rn(decay, v.z), mul_rn(kn, d2));
                v.w = add_rn(mul_rn(decay, v.w), mul_rn(kn, d3));
                s[i] = v;  // the next row (verify) continues from it
                reinterpret_cast<float4*>(S + (size_t)(rp * 8 + i) * kDV)[cq] = v;
                part[0] = fmaf(qn, v.x, part[0]);
                part[1] = fmaf(qn, v.y, part[1]);
                part[2] = fmaf(qn, v.z, part[2]);
                part[3] = fmaf(qn, v.w, part[3]);
            }
        }
        __syncthreads();  // red reused
        if (!bad) {
#pragma unroll
            for (int j = 0; j < 4; ++j) red[rp][4 * cq + j] = part[j];
        }
        __syncthreads();
        float ov = 0.f;
        if (!bad && warp == 0) {
#pragma unroll
            for (int w = 0; w < 16; ++w) ov += red[w][lane];
            const float sq = warp_sum(ov * ov);
            if (lane == 0) osq = sq;
        }
        // ---- gated RMSNorm: the sum of o^2 over the head's 4 CTAs, read through distributed shared memory
        cluster.sync();
        if (!bad && warp == 0) {
            float tot = 0.f;
#pragma unroll
            for (int r = 0; r < kGdnSplit; ++r) tot += *cluster.map_shared_rank(&osq, r);
            const float mean = tot / (float)kDV;
            const float rr = rsqrt_ieee(mean + kEps);
            const int col = c0 + lane;
            const float on = mul_rn(mul_rn(ov, rr), nw_c);
            const float z = __uint_as_float((uint32_t)z_raw << 16);
            const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(on, silu_f(z)));
            const size_t idx = (size_t)bb * gv + hh * kDV + col;
            reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
            if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
        }
        cluster.sync();  // osq is rewritten by the next row; no CTA leaves while a peer may still read it
    }
    if (bad && tid == 0 && qtr == 0) atomicOr(p.err, kErrBounds);
}

// ---------------------------------------------------------------------------------------------------------
// The batch form (2 or more users, not verify): one 4-CTA cluster per (value head, group of UG users), CTA q
// owning the same 32 columns of every user's state in the group. At 8 users the one-user form needs 1,536 CTAs
// of which ~740 fit at once, so the launch ran in two waves of a latency-bound chain; here 384 CTAs of UG = 4
// users fit in one (three per SM: 64 KB of state in shared memory each). Each thread copies its own 8 x 4
// elements of every user's slice with 16-byte cp.async right after the dependency wait -- the group's 64 KB in
// flight at once -- and reads them back itself, so no barrier guards the copies. The passes run over all users
// of the group between the CTA's barriers (one set of barriers and two cluster barriers for the group instead of
// per user). Same arithmetic as the one-user form; the row sums of kS and o reduce a warp's 4 row groups by
// shuffles first, then the 4 warps in order.
template <int UG>
__global__ void __cluster_dims__(1, 1, kGdnSplit) __launch_bounds__(kGdnThreads, 3)
    gdn_batch_kernel(const GdnParams p) {
    cg::cluster_group cluster = cg::this_cluster();
    const int hh = blockIdx.x;       // local value head
    const int b0 = blockIdx.y * UG;  // first user of the group
    const int qtr = blockIdx.z;      // column quarter (= rank in the cluster)
    const int nu = min(UG, p.rows - b0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = p.nk * kDK, gv = p.nv * kDV;
    const int conv = 2 * gq + gv;
    const int group = p.nv / p.nk;
    const int kh = hh / group;
    const int c0 = qtr * kGdnCols;

    extern __shared__ __align__(16) float st[];  // [UG][128 rows][32 columns]: the users' state slices
    __shared__ float qk[UG][2][kDK];             // conv outputs q, k (then normalised in place)
    __shared__ float red[UG][4][kGdnCols];       // per warp row sums
    __shared__ float dl[UG][kGdnCols];
    __shared__ float sc[UG][4];
    __shared__ float osq[UG];  // this CTA's sum of o^2 per user, read by the whole cluster

    pdl_launch();
    const int cq = tid & 7, rp = tid >> 3;
    const size_t slot_stride = (size_t)p.nv * kDK * kDV;
    auto slice = [&](int u) { return p.state + (size_t)(b0 + u) * slot_stride + (size_t)hh * kDK * kDV + c0; };
    // immutable or L2-only work ahead of the dependency wait: the state, taps and history into L2 (the state as
    // the head's contiguous quarter q, one bulk prefetch per user: the cluster covers the head)
    if (tid < nu)
        bulk_prefetch_l2(p.state + (size_t)(b0 + tid) * slot_stride + ((size_t)hh * kDK + 32 * qtr) * kDV, 32 * kDV * 4);
    if (tid < 3 * UG) {
        const int u = tid / 3, part = tid % 3;
        if (u < nu) {
            const uint16_t* h = p.hist + (size_t)(b0 + u) * QRES_HIST_SLOTS * conv;
            const size_t ch = part == 0 ? (size_t)kh * kDK : part == 1 ? (size_t)gq + kh * kDK : (size_t)2 * gq + hh * kDV + c0;
            const uint32_t bytes = part == 2 ? kGdnCols * 2 : kDK * 2;
            for (int slot = 0; slot < QRES_HIST_SLOTS; ++slot) bulk_prefetch_l2(h + (size_t)slot * conv + ch, bytes);
        }
    }
    if (tid == 32) {
        bulk_prefetch_l2(p.taps + (size_t)kh * kDK * 4, kDK * 8);
        bulk_prefetch_l2(p.taps + ((size_t)gq + kh * kDK) * 4, kDK * 8);
        bulk_prefetch_l2(p.taps + ((size_t)2 * gq + hh * kDV + c0) * 4, kGdnCols * 8);
    }
    pdl_wait();

    int pos[UG];
    bool bad[UG];
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        pos[u] = u < nu ? p.pos[b0 + u] : -1;
        bad[u] = u >= nu || pos[u] < 0;
    }
    // ---- the state slices: this thread's rows rp*8 .. rp*8+7, columns 4cq .. 4cq+3 of each user
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        if (bad[u]) continue;
        const float* S = slice(u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = rp * 8 + i;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(st + (u * kDK + row) * kGdnCols + 4 * cq)),
                         "l"(S + (size_t)row * kDV + 4 * cq)
                         : "memory");
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");

    // ---- every other input of the group, issued together: a, b per user; z, conv inputs and history
    const YIn yall{p.y, p.yacc};
    const float dt_h = p.dt[hh], na_h = p.neg_a[hh];
    const float nw_c = p.norm_w[c0 + lane];
    const int vu = warp;  // this thread's v channel: column `lane` of user `warp`; the pass-4/5 user of the warp
    const int chq = kh * kDK + tid, chk = gq + kh * kDK + tid, chv = 2 * gq + hh * kDV + c0 + lane;
    const int a_off = 2 * gq + 2 * gv;
    uint16_t a_raw[UG], yq[UG], yk[UG], hq[UG][3], hk[UG][3];
    uint16_t b_raw = 0, z_raw = 0, yv = 0, hv[3] = {0, 0, 0};
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        a_raw[u] = yq[u] = yk[u] = 0;
        if (bad[u]) continue;
        const YIn y = yall.at((size_t)(b0 + u) * p.ld_y);
        const uint16_t* hist = p.hist + (size_t)(b0 + u) * QRES_HIST_SLOTS * conv;
        a_raw[u] = y[a_off + hh];
        yq[u] = y[chq];
        yk[u] = y[chk];
#pragma unroll
        for (int jj = 0; jj < 3; ++jj) {
            const size_t sl = (size_t)((pos[u] - 3 + jj + QRES_HIST_SLOTS) % QRES_HIST_SLOTS) * conv;
            hq[u][jj] = hist[sl + chq];
            hk[u][jj] = hist[sl + chk];
        }
    }
    const int posv = vu < nu ? p.pos[b0 + vu] : -1;  // the v user's position (no dynamic index into pos[])
    const bool vok = posv >= 0;
    if (vok) {
        const YIn y = yall.at((size_t)(b0 + vu) * p.ld_y);
        const uint16_t* hist = p.hist + (size_t)(b0 + vu) * QRES_HIST_SLOTS * conv;
        b_raw = y[a_off + p.nv + hh];
        z_raw = y[2 * gq + gv + hh * kDV + c0 + lane];
        yv = y[chv];
#pragma unroll
        for (int jj = 0; jj < 3; ++jj) hv[jj] = hist[(size_t)((posv - 3 + jj + QRES_HIST_SLOTS) % QRES_HIST_SLOTS) * conv + chv];
    }
    const uint2 tq = *reinterpret_cast<const uint2*>(p.taps + (size_t)chq * 4);
    const uint2 tk = *reinterpret_cast<const uint2*>(p.taps + (size_t)chk * 4);
    const uint2 tv = *reinterpret_cast<const uint2*>(p.taps + (size_t)chv * 4);

    // ---- conv1d + SiLU (bf16 window, round-to-nearest taps as the one-user form)
    auto conv4 = [](uint16_t h0, uint16_t h1, uint16_t h2, uint16_t x, uint2 t) {
        float acc = mul_rn(__uint_as_float((uint32_t)h0 << 16), bf16lo(t.x));
        acc = add_rn(acc, mul_rn(__uint_as_float((uint32_t)h1 << 16), bf16hi(t.x)));
        acc = add_rn(acc, mul_rn(__uint_as_float((uint32_t)h2 << 16), bf16lo(t.y)));
        acc = add_rn(acc, mul_rn(__uint_as_float((uint32_t)x << 16), bf16hi(t.y)));
        return bf16_round(silu_f(acc));
    };
    const bool qk_writer = hh % group == 0 && qtr == 0;  // one writer per q / k history element
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        if (bad[u]) continue;
        qk[u][0][tid] = conv4(hq[u][0], hq[u][1], hq[u][2], yq[u], tq);
        qk[u][1][tid] = conv4(hk[u][0], hk[u][1], hk[u][2], yk[u], tk);
        if (qk_writer) {
            uint16_t* hist = p.hist + ((size_t)(b0 + u) * QRES_HIST_SLOTS + pos[u] % QRES_HIST_SLOTS) * conv;
            hist[chq] = yq[u];
            hist[chk] = yk[u];
        }
    }
    const float vconv = vok ? conv4(hv[0], hv[1], hv[2], yv, tv) : 0.f;
    if (vok) p.hist[((size_t)(b0 + vu) * QRES_HIST_SLOTS + posv % QRES_HIST_SLOTS) * conv + chv] = yv;
    float decay[UG];
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        const float av = __uint_as_float((uint32_t)a_raw[u] << 16);
        decay[u] = bad[u] ? 0.f : expf(mul_rn(na_h, softplus_f(add_rn(av, dt_h))));
    }
    __syncthreads();
    // ---- l2 norms of q and k (the one-user form's pairing: warp w sums half w & 1 of q (w < 2) or k)
    {
        const int which = warp >> 1, h0 = (warp & 1) * 64;
#pragma unroll
        for (int u = 0; u < UG; ++u) {
            if (bad[u]) continue;
            const float v0 = qk[u][which][h0 + lane], v1 = qk[u][which][h0 + 32 + lane];
            const float ss = warp_sum(v0 * v0 + v1 * v1);
            if (lane == 0) sc[u][warp] = ss;
        }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        if (bad[u]) continue;
        const float rq = rsqrt_ieee(sc[u][0] + sc[u][1] + 1e-6f), rk = rsqrt_ieee(sc[u][2] + sc[u][3] + 1e-6f);
        qk[u][0][tid] = mul_rn(mul_rn(qk[u][0][tid], rq), 0.08838834764831845f);
        qk[u][1][tid] = mul_rn(qk[u][1][tid], rk);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's own copies: it alone reads them
    __syncthreads();
    // the following projection's weights into L2 while the passes run: issued once this kernel's own loads have
    // landed, so the prefetch does not queue ahead of them
    if (p.pf && tid == 64) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        l2_prefetch_share(p.pf, p.pf_bytes, cta, gridDim.x * gridDim.y * gridDim.z);
    }
    auto row_sums = [&](int u, float* part) {
        // the 4 row groups of the warp (lanes cq, cq + 8, cq + 16, cq + 24), then one word per warp
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            part[j] += __shfl_xor_sync(0xffffffffu, part[j], 8);
            part[j] += __shfl_xor_sync(0xffffffffu, part[j], 16);
        }
        if (lane < 8) {
#pragma unroll
            for (int j = 0; j < 4; ++j) red[u][warp][4 * cq + j] = part[j];
        }
    };
    // ---- pass 1: kS = (decay * kn) @ S
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        if (bad[u]) continue;
        float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 s = *reinterpret_cast<const float4*>(st + (u * kDK + rp * 8 + i) * kGdnCols + 4 * cq);
            const float dk = mul_rn(decay[u], qk[u][1][rp * 8 + i]);
            part[0] = fmaf(dk, s.x, part[0]);
            part[1] = fmaf(dk, s.y, part[1]);
            part[2] = fmaf(dk, s.z, part[2]);
            part[3] = fmaf(dk, s.w, part[3]);
        }
        row_sums(u, part);
    }
    __syncthreads();
    // ---- pass 2: delta = beta * (v - kS), thread (user warp, column lane)
    if (vok) {
        const float beta = sigmoid_f(__uint_as_float((uint32_t)b_raw << 16));
        const float t = ((red[vu][0][lane] + red[vu][1][lane]) + red[vu][2][lane]) + red[vu][3][lane];
        dl[vu][lane] = mul_rn(beta, vconv - t);
    }
    __syncthreads();
    // ---- pass 3: S <- decay * S + kn (x) delta (written back to HBM), o = qn @ S
#pragma unroll
    for (int u = 0; u < UG; ++u) {
        if (bad[u]) continue;
        float* S = slice(u);
        const float d0 = dl[u][4 * cq], d1 = dl[u][4 * cq + 1], d2 = dl[u][4 * cq + 2], d3 = dl[u][4 * cq + 3];
        const float dec = decay[u];
        float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = rp * 8 + i;
            const float kn = qk[u][1][row], qn = qk[u][0][row];
            float4 v = *reinterpret_cast<const float4*>(st + (u * kDK + row) * kGdnCols + 4 * cq);
            v.x = add_rn(mul_rn(dec, v.x), mul_rn(kn, d0));
            v.y = add_rn(mul_rn(dec, v.y), mul_rn(kn, d1));
            v.z = add_rn(mul_rn(dec, v.z), mul_rn(kn, d2));
            v.w = add_rn(mul_rn(dec, v.w), mul_rn(kn, d3));
            reinterpret_cast<float4*>(S + (size_t)row * kDV)[cq] = v;
            part[0] = fmaf(qn, v.x, part[0]);
            part[1] = fmaf(qn, v.y, part[1]);
            part[2] = fmaf(qn, v.z, part[2]);
            part[3] = fmaf(qn, v.w, part[3]);
        }
        __syncwarp();  // red[u][warp] of pass 1 was read in pass 2 behind the barrier; rewritten now
        row_sums(u, part);
    }
    __syncthreads();
    // ---- pass 4: o of (user warp, column lane) and the CTA's sum of o^2 per user
    float ov = 0.f;
    if (vok) {
        ov = ((red[vu][0][lane] + red[vu][1][lane]) + red[vu][2][lane]) + red[vu][3][lane];
        const float sq = warp_sum(ov * ov);
        if (lane == 0) osq[vu] = sq;
    }
    // ---- gated RMSNorm: the head's 4 CTAs' sums through distributed shared memory
    cluster.sync();
    if (vok) {
        float tot = 0.f;
#pragma unroll
        for (int r = 0; r < kGdnSplit; ++r) tot += *cluster.map_shared_rank(&osq[vu], r);
        const float rr = rsqrt_ieee(tot / (float)kDV + kEps);
        const float on = mul_rn(mul_rn(ov, rr), nw_c);
        const float z = __uint_as_float((uint32_t)z_raw << 16);
        const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(on, silu_f(z)));
        const size_t idx = (size_t)(b0 + vu) * gv + hh * kDV + c0 + lane;
        reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
        if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
    }
    cluster.sync();  // no CTA leaves while a peer may still read its osq
    if (tid == 0 && qtr == 0) {
        bool any = false;
#pragma unroll
        for (int u = 0; u < UG; ++u) any = any || (u < nu && pos[u] < 0);
        if (any) atomicOr(p.err, kErrBounds);
    }
}

cudaError_t gdn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const uint16_t* taps,
                       const float* dt, const float* neg_a, const float* norm_w, float* state, uint16_t* hist,
                       uint16_t* o, uint16_t* mixer_copy, uint32_t* err, cudaStream_t st, bool pdl,
                       const void* pf, size_t pf_bytes, int verify, const int32_t* slot0, const long long* yacc) {
    if (nranks < 1 || 16 % nranks || rows < 1 || rows > kMaxRows) return cudaErrorInvalidValue;
    if (verify && (verify != rows || rows + 3 > QRES_HIST_SLOTS || slot0 == nullptr)) return cudaErrorInvalidValue;
    GdnParams p;
    p.nk = 16 / nranks;
    p.nv = 48 / nranks;
    p.ld_y = ld_y;
    p.y = yacc ? nullptr : y;
    p.yacc = yacc;
    p.pos = pos;
    p.taps = taps;
    p.dt = dt;
    p.neg_a = neg_a;
    p.norm_w = norm_w;
    p.state = state;
    p.hist = hist;
    p.o = o;
    p.mixer_copy = mixer_copy;
    p.pf = static_cast<const uint8_t*>(pf);
    p.pf_bytes = pf_bytes;
    p.err = err;
    p.rows = rows;
    p.verify = verify;
    p.slot0 = slot0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nv, verify ? 1 : rows, kGdnSplit);
    cfg.blockDim = dim3(kGdnThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    if (!verify && rows > 1) {
        // the batch form: groups of 2 users up to 4 rows, of 4 above
        const int ug = rows <= 4 ? 2 : 4;
        cfg.gridDim = dim3(p.nv, (rows + ug - 1) / ug, kGdnSplit);
        cfg.dynamicSmemBytes = (size_t)ug * kDK * kGdnCols * sizeof(float);
        auto k = ug == 2 ? gdn_batch_kernel<2> : gdn_batch_kernel<4>;
        static bool smem_set[2] = {false, false};
        if (!smem_set[ug / 4]) {
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
            if (e != cudaSuccess) return e;
            smem_set[ug / 4] = true;
        }
        return cudaLaunchKernelEx(&cfg, k, p);
    }
    return cudaLaunchKernelEx(&cfg, gdn_decode_kernel, p);
}

}  // namespace qres
