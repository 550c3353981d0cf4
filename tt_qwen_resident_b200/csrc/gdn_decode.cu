// Gated DeltaNet decode mixer for sm_100a: one CTA per (value head, user).
//
// Replaces the reference's conv1d + SiLU of the streamers (qwen36_resident/kernels/streamer_compute.cpp:279-370,
// history ring streamer_common.hpp:280-288) and its GDN head cores (gdn_head_reader.cpp / gdn_head_compute.cpp
// :180-347 / gdn_head_writer.cpp), i.e. the math of model.py:255-276:
//   conv  = bf16(silu(sum_j window[j] * tap[j]))          window = inputs at p-3, p-2, p-1, p (oldest first)
//   qn    = q * rsqrt(sum q^2 + 1e-6) * 128^-0.5;   kn = k * rsqrt(sum k^2 + 1e-6)
//   decay = exp(neg_a * softplus(a + dt));  beta = sigmoid(b)
//   delta = beta * (v - (decay * kn) @ S);  S <- decay * S + kn (x) delta;  o = qn @ S
//   out   = bf16(rmsnorm(o) * norm_w * silu(z))
// The fp32 state S [128 (k)][128 (v)] of the head stays in HBM and is updated in place: 64 KB read + 64 KB
// written per (head, user) and step. Columns of S are independent, so a thread owns 4 columns x 16 rows in
// registers (coalesced float4 rows per warp); the two reductions over k go through shared memory in a fixed
// order (deterministic).
//
// Conv history: a ring of QRES_HIST_SLOTS slots per user, position q's input in slot q % 8. A step at p reads
// the slots of p-3..p-1 and writes slot p (never a slot it reads), so the three value heads that share a key
// head can all read the q / k history while the first of them writes it.
#include "qres_common.cuh"

namespace qres {

constexpr int kGdnThreads = 256;

struct GdnParams {
    int nk, nv;              // local key / value heads
    int ld_y;                // elements between users' y rows
    const uint16_t* y;       // [B][ld_y] bf16: q | k | v | z | a | b
    const int32_t* pos;      // [B]
    const uint16_t* taps;    // [conv][4] bf16
    const float* dt;         // [nv]
    const float* neg_a;      // [nv]
    const float* norm_w;     // [128]
    float* state;            // [B][nv][128][128]
    uint16_t* hist;          // [B][8][conv]
    uint16_t* o;             // [B][nv * 128] bf16
    uint16_t* mixer_copy;    // optional second output
    uint32_t* err;
};

__global__ void __launch_bounds__(kGdnThreads) gdn_decode_kernel(const GdnParams p) {
    const int hh = blockIdx.x;  // local value head
    const int b = blockIdx.y;   // user
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = p.nk * kDK, gv = p.nv * kDV;
    const int conv = 2 * gq + gv;
    const int kh = hh / (p.nv / p.nk);

    __shared__ float qk[2][kDK];   // conv outputs q, k of the key head (bf16 values)
    __shared__ float vv[kDV];      // conv output v of this value head
    __shared__ float red[8][kDV];
    __shared__ float qs[kDK], ks[kDK], dl[kDV];
    __shared__ float sc[8];

    pdl_launch();
    const int cq = lane;      // column quad: columns 4cq .. 4cq+3
    const int rp = warp;      // rows 16rp .. 16rp+15
    float* S = p.state + (((size_t)b * p.nv + hh) * kDK) * kDV;
    // Before griddepcontrol.wait only immutable data may be read (an earlier kernel of the stream may still be
    // running); an L2 prefetch of the state is safe (L2 is the point of coherence) and starts its 64 KB early.
    if (tid < 16) bulk_prefetch_l2(S + (size_t)tid * 8 * kDV, 8 * kDV * 4);
    pdl_wait();
    float4 s[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) s[i] = reinterpret_cast<const float4*>(S + (size_t)(rp * 16 + i) * kDV)[cq];
    const int pos = p.pos[b];
    if (pos < 0) {
        if (tid == 0) atomicOr(p.err, kErrBounds);
        return;
    }
    const uint16_t* y = p.y + (size_t)b * p.ld_y;
    uint16_t* hist = p.hist + (size_t)b * QRES_HIST_SLOTS * conv;
    const int s0 = (pos + QRES_HIST_SLOTS - 3) % QRES_HIST_SLOTS;
    const int s1 = (pos + QRES_HIST_SLOTS - 2) % QRES_HIST_SLOTS;
    const int s2 = (pos + QRES_HIST_SLOTS - 1) % QRES_HIST_SLOTS;
    const int sw = pos % QRES_HIST_SLOTS;
    // ---- conv1d + SiLU over the 384 channels of this head (q, k of the key head; v of the value head)
    for (int i = tid; i < 3 * kDK; i += kGdnThreads) {
        int ch, which;
        if (i < kDK) {
            ch = kh * kDK + i;
            which = 0;
        } else if (i < 2 * kDK) {
            ch = gq + kh * kDK + (i - kDK);
            which = 1;
        } else {
            ch = 2 * gq + hh * kDV + (i - 2 * kDK);
            which = 2;
        }
        const uint16_t yin = y[ch];
        const float w0 = __uint_as_float((uint32_t)hist[s0 * conv + ch] << 16);
        const float w1 = __uint_as_float((uint32_t)hist[s1 * conv + ch] << 16);
        const float w2 = __uint_as_float((uint32_t)hist[s2 * conv + ch] << 16);
        const float w3 = __uint_as_float((uint32_t)yin << 16);
        const uint2 tp = *reinterpret_cast<const uint2*>(p.taps + (size_t)ch * 4);
        const float t0 = bf16lo(tp.x), t1 = bf16hi(tp.x), t2 = bf16lo(tp.y), t3 = bf16hi(tp.y);
        float acc = mul_rn(w0, t0);
        acc = add_rn(acc, mul_rn(w1, t1));
        acc = add_rn(acc, mul_rn(w2, t2));
        acc = add_rn(acc, mul_rn(w3, t3));
        const float c = bf16_round(silu_f(acc));
        if (which == 0) qk[0][i] = c;
        else if (which == 1) qk[1][i - kDK] = c;
        else vv[i - 2 * kDK] = c;
        // the first value head of a key head writes the q / k history, every head its v history
        if (which == 2 || hh % (p.nv / p.nk) == 0) hist[sw * conv + ch] = yin;
    }
    __syncthreads();
    // ---- l2 norms of q and k (warps 0-3: q, 4-7: k), gates
    {
        const int which = warp >> 2;
        float v = qk[which][(warp & 3) * 32 + lane];
        float ss = warp_sum(v * v);
        if (lane == 0) sc[warp] = ss;
    }
    __syncthreads();
    if (tid < 2 * kDK) {
        const int which = tid >> 7, i = tid & 127;
        const float ssum = ((sc[4 * which] + sc[4 * which + 1]) + sc[4 * which + 2]) + sc[4 * which + 3];
        const float r = rsqrt_ieee(ssum + 1e-6f);
        float v = mul_rn(qk[which][i], r);
        if (which == 0) qs[i] = mul_rn(v, 0.08838834764831845f);
        else ks[i] = v;
    }
    __syncthreads();
    const int a_off = 2 * gq + 2 * gv;
    const float av = __uint_as_float((uint32_t)y[a_off + hh] << 16);
    const float bv = __uint_as_float((uint32_t)y[a_off + p.nv + hh] << 16);
    const float decay = expf(mul_rn(p.neg_a[hh], softplus_f(add_rn(av, p.dt[hh]))));
    const float beta = sigmoid_f(bv);
    // ---- kS = (decay * kn) @ S
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float dk = mul_rn(decay, ks[rp * 16 + i]);
        part[0] = fmaf(dk, s[i].x, part[0]);
        part[1] = fmaf(dk, s[i].y, part[1]);
        part[2] = fmaf(dk, s[i].z, part[2]);
        part[3] = fmaf(dk, s[i].w, part[3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rp][4 * cq + j] = part[j];
    __syncthreads();
    if (tid < kDV) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += red[w][tid];
        dl[tid] = mul_rn(beta, vv[tid] - t);
    }
    __syncthreads();
    // ---- S <- decay * S + kn (x) delta, o = qn @ S
    const float d0 = dl[4 * cq], d1 = dl[4 * cq + 1], d2 = dl[4 * cq + 2], d3 = dl[4 * cq + 3];
#pragma unroll
    for (int j = 0; j < 4; ++j) part[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float kn = ks[rp * 16 + i], qn = qs[rp * 16 + i];
        float4 v = s[i];
        v.x = add_rn(mul_rn(decay, v.x), mul_rn(kn, d0));
        v.y = add_rn(mul_rn(decay, v.y), mul_rn(kn, d1));
        v.z = add_rn(mul_rn(decay, v.z), mul_rn(kn, d2));
        v.w = add_rn(mul_rn(decay, v.w), mul_rn(kn, d3));
        reinterpret_cast<float4*>(S + (size_t)(rp * 16 + i) * kDV)[cq] = v;
        part[0] = fmaf(qn, v.x, part[0]);
        part[1] = fmaf(qn, v.y, part[1]);
        part[2] = fmaf(qn, v.z, part[2]);
        part[3] = fmaf(qn, v.w, part[3]);
    }
    __syncthreads();  // red reused
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rp][4 * cq + j] = part[j];
    __syncthreads();
    // ---- gated RMSNorm
    float ov = 0.f;
    if (tid < kDV) {
#pragma unroll
        for (int w = 0; w < 8; ++w) ov += red[w][tid];
    }
    {
        float sq = warp_sum(tid < kDV ? ov * ov : 0.f);
        if (lane == 0 && warp < 4) sc[warp] = sq;
    }
    __syncthreads();
    if (tid < kDV) {
        const float mean = (((sc[0] + sc[1]) + sc[2]) + sc[3]) / (float)kDV;
        const float r = rsqrt_ieee(mean + kEps);
        const float on = mul_rn(mul_rn(ov, r), p.norm_w[tid]);
        const float z = __uint_as_float((uint32_t)y[2 * gq + gv + hh * kDV + tid] << 16);
        const __nv_bfloat16 out = __float2bfloat16_rn(mul_rn(on, silu_f(z)));
        const size_t idx = (size_t)b * gv + hh * kDV + tid;
        reinterpret_cast<__nv_bfloat16*>(p.o)[idx] = out;
        if (p.mixer_copy) reinterpret_cast<__nv_bfloat16*>(p.mixer_copy)[idx] = out;
    }
}

cudaError_t gdn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const uint16_t* taps,
                       const float* dt, const float* neg_a, const float* norm_w, float* state, uint16_t* hist,
                       uint16_t* o, uint16_t* mixer_copy, uint32_t* err, cudaStream_t st, bool pdl) {
    if (nranks < 1 || 16 % nranks || rows < 1 || rows > kMaxRows) return cudaErrorInvalidValue;
    GdnParams p;
    p.nk = 16 / nranks;
    p.nv = 48 / nranks;
    p.ld_y = ld_y;
    p.y = y;
    p.pos = pos;
    p.taps = taps;
    p.dt = dt;
    p.neg_a = neg_a;
    p.norm_w = norm_w;
    p.state = state;
    p.hist = hist;
    p.o = o;
    p.mixer_copy = mixer_copy;
    p.err = err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nv, rows);
    cfg.blockDim = dim3(kGdnThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gdn_decode_kernel, p);
}

}  // namespace qres
