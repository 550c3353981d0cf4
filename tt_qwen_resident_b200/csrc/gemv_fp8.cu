// Block-scaled FP8 weight-streaming projection for 1..8 rows (users) on the sm_100a tensor cores (tcgen05).
//
// Replaces the reference's streamer cores (qwen36_resident/kernels/streamer_reader.cpp:45-89 weight ring,
// streamer_compute.cpp:60-92 M=1..8 matmul, :100-210 rmsnorm, :212-249 silu(g)*u, :252-273 residual fold).
//
// Math: out[u][n] = sum_kb scale[n][kb] * sum_{k in kb} q[n][k] * h[u][k], q the e4m3 weight, h the bf16
// activation, scale the fp32 scale of the 128 x 128 block holding (n, kb). Each 128-row x 128-K block ("unit")
// is one chain of 4 tcgen05.mma.kind::f8f6f4 (M = 128, N = 16, K = 32) with the weights as A, read by the tensor
// core straight from the shared-memory stage the bulk copy filled, and the activations as B. The activations
// enter as two e4m3 columns per user: with E the exponent of max|h| over the user's 128-K block, h * 2^(7-E) =
// hi + lo, hi = e4m3(h * 2^(7-E)), lo = e4m3(h * 2^(7-E) - hi). A bf16 carries 8 significant bits and each
// e4m3 term 4, so the split is exact for every element within 2^-10 of the block maximum; below that lo is
// rounded on the e4m3 subnormal grid, an absolute error of at most 2^-18 of the block maximum (far below the
// bf16 rounding of the result). The products accumulate in fp32 in tensor memory (TMEM); the epilogue warps
// read each unit's 16 x 128 accumulator, add hi + lo, and fold it into the row's fp32 result with the unit's
// weight scale times 2^(E-7).
//
// Layout (qres_tile_weight): rows in tiles of 128 (zero-padded), a tile's K in 128-wide units of 16 KB stored
// back to back; inside a unit the tensor core's 128-byte-swizzled K-major arrangement: row r's 128 bytes at
// r * 128, its 16-byte chunk c stored at chunk position c ^ (r % 8) (8-row groups 1024 bytes apart, the stride
// offset; bank-conflict-free reads of any 32-byte K slice). MMA m of a unit starts 32 * m bytes into the
// stage, inside the swizzle atom, as the hardware applies the XOR to the address bits. The scale table gives
// each tile 128 bytes of row selectors (which of the tile's <= 8 canonical 128-row blocks holds the row) and
// 8 fp32 scales per unit (the blocks' scales at that K block).
//
// CTA roles (256 threads, one CTA per SM, a second co-resident under programmatic dependent launch):
//   warp 0 lane 0   streams the CTA's contiguous run of units through a ring of 16 KB stages (cp.async.bulk,
//                   no multicast; the first stages before griddepcontrol.wait -- weights are immutable);
//   warp 1          owns the TMEM allocation; lane 0 issues the MMAs of a unit once its stage has landed and
//                   commits them to the stage's "empty" barrier and to the accumulator slot's "full" barrier;
//   warps 4..7      (TMEM lanes 0..127, one row each) drain accumulator slots, apply the scales, and finish
//                   tiles: a tile split between CTAs is completed by the last of them (an atomic ticket), which
//                   adds the parts in CTA order (deterministic);
//   all 8 warps     build the activations' hi / lo operand in shared memory first (rmsnorm or a bf16 input).
// Every wait is bounded (sets the error word and stops the pipeline).
#include "gemv_core.cuh"

namespace qres {

struct GemvParams {
    const uint8_t* w;
    const uint8_t* table;   // per tile: kSelBytes row selectors, then nkb x 8 fp32 scales
    int rows, tiles, K, nkb;
    int users;              // real users (<= template B)
    const float* x;         // PRO_RMSNORM(_ADD): fp32 [users][K] (two segments: [users][seg])
    const float* x2;        // PRO_RMSNORM over two segments: the second segment, fp32 [users][seg]
    int seg;                // 0, or the first segment's length (K = 2 seg; rows <= 4)
    const float* red;       // PRO_RMSNORM_ADD: partials [nsrc][users][K]; x_out = x + (sum of the sources in order)
    float* x_out;           // PRO_RMSNORM_ADD: written by CTA 0
    int nsrc;               // PRO_RMSNORM_ADD: 1 (all-reduced by NCCL) or one per rank (peer exchange)
    size_t src_stride;      // fp32 sources: floats between two sources
    // PRO_RMSNORM_ADD over the peer exchange: the sources are tagged words [nsrc][users][K], read until every word
    // carries this exchange's tag (*epoch * tag_mul + tag_add)
    const uint2* tagged;
    const uint32_t* epoch;
    uint32_t tag_mul, tag_add;
    // EPI_P2P: every finished row goes to each rank's window (this rank's region, [user][peer_ld]) as a tagged word
    int p2p_n;
    int peer_ld;
    uint2* peer_data[kMaxPeers];
    const uint16_t* in;     // PRO_BF16: bf16 [users][ld_in]
    int ld_in;
    void* out;              // EPI_BF16 / EPI_SILU_MUL: bf16 [users][ld_out]; EPI_RESID / EPI_F32: fp32
    int ld_out;
    int nstages;            // ring depth
    int nkw;                // K blocks in this CTA's activation window (the most any CTA needs)
    int nq;                 // unit order: K blocks per group (nkb = storage order; see unit_offset)
    float* part;            // [grid][2][8][128]: a CTA's split first / last tile
    int* ticket;            // [tiles]
    L2Heads next;           // the next projection of the step: the heads of its CTA runs are pulled into L2
    const long long* racc;  // PRO_RMSNORM_ADD: fixed-point partial source [users][K] (instead of red), or null
    const long long* gacc;  // PRO_SILU_ACC: fixed-point gate|up sums [users][ld_gacc]
    int ld_gacc;
    long long* acc_out;     // EPI_ACC: fixed-point target [users][ld_out]
    long long* zero;        // zeroed by this launch after its dependency wait (16-byte multiple)
    size_t zero_words;
    bool zero_sys;          // ... and fenced at system scope (other GPUs add into it later)
    // EPI_ACC, counted exchange: every rank's accumulator (xn > 0), else acc_out alone (plain)
    long long* xdst[kMaxPeers];
    int xn;
    // PRO_RMSNORM_ADD over counted racc: rc_ranks x (CTAs of the producing launch over the row's tile)
    // contributions per word; the producer split its units as base rc_base, remainder rc_rem, rc_nkb per tile
    int rc_ranks, rc_base, rc_rem, rc_nkb;
    uint32_t* err;
};

// walks a CTA's run of units in the launch's unit order: (K group, tile, K block in the group)
struct UnitWalk {
    int tiles, nq, kq, T, kbi;
    __device__ UnitWalk(int u, int tiles_, int nq_) : tiles(tiles_), nq(nq_) {
        const int per = tiles * nq;
        kq = u / per;
        const int r = u - kq * per;
        T = r / nq;
        kbi = r - T * nq;
    }
    __device__ int kb() const { return kq * nq + kbi; }
    __device__ void next() {
        if (++kbi == nq) {
            kbi = 0;
            if (++T == tiles) {
                T = 0;
                ++kq;
            }
        }
    }
};

template <int B, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_fp8_kernel(const GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kMaxStages] stage landed
    uint64_t* empty = full + kMaxStages;                 // [kMaxStages] stage consumed by its MMAs
    uint64_t* dfull = empty + kMaxStages;                // [kDSlots] accumulator slot written
    uint64_t* dempty = dfull + kDSlots;                  // [kDSlots] accumulator slot read (4 epilogue warps)
    uint64_t* drain = dempty + kDSlots;                  // every MMA of the CTA completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    int* tk_slot = reinterpret_cast<int*>(tmem_slot + 1);  // [2]
    float (*red)[8] = reinterpret_cast<float (*)[8]>(smem + 512);  // [8 warps][8 users]
    const int nkw = p.nkw;
    float* ainv = reinterpret_cast<float*>(smem + kHeadBytes);  // [nkw][8]: 2^(E-7) per K block and user
    uint8_t* act = smem + kHeadBytes + gemv_ainv_bytes(nkw);   // [group][nkw][8 chunks x LBO] (+ tail)
    constexpr int LBO = gemv_act_lbo(B);
    const size_t gstride = gemv_act_group(B, nkw);
    const size_t pre = kHeadBytes + gemv_ainv_bytes(nkw) + gemv_act_bytes(B, nkw);
    uint8_t* ring = smem + ((pre + 1023) & ~size_t(1023));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.K, nkb = p.nkb;
    const int U = p.tiles * nkb;
    const int G = gridDim.x;
    const int base = U / G, rem = U % G;
    const int u0 = blockIdx.x * base + min((int)blockIdx.x, rem);
    const int cnt = base + ((int)blockIdx.x < rem ? 1 : 0);
    const int NS = p.nstages;
    if (cnt == 0) return;
    // the K blocks this CTA touches (its activation window): in storage order (nq = nkb) a cyclic run from its
    // first unit's block; in grouped order the K groups its run spans
    const int nq = p.nq;
    int kb_start, nwin;
    if (nq == nkb) {
        kb_start = u0 % nkb;
        nwin = min(cnt, nkb);
    } else {
        const int per = p.tiles * nq, kq0 = u0 / per, kq1 = (u0 + cnt - 1) / per;
        kb_start = kq0 * nq;
        nwin = min((kq1 - kq0 + 1) * nq, nkb);
    }

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kDSlots; ++i) {
            mbar_init(&dfull[i], 1);
            mbar_init(&dempty[i], 4);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch();

    const uint64_t pol = policy_evict_first();  // every weight byte is read once per step
    auto issue = [&](int i) {
        const int slot = i % NS;
        mbar_arrive_expect_tx(&full[slot], kUnitBytes);
        bulk_g2s_hint(ring + (size_t)slot * kUnitBytes, p.w + unit_offset(u0 + i, p.tiles, nkb, nq) * kUnitBytes,
                      kUnitBytes, &full[slot], pol);
    };
    if (tid == 0)
        for (int i = 0; i < min(NS, cnt); ++i) issue(i);
    // and the ring's next fill into L2 (a prefetch, no shared destination): the stream keeps HBM busy while the
    // prologue waits for its dependency and builds the operand, and the refills after it come from L2
    if (tid == 0)
        for (int i = NS; i < min(2 * NS, cnt); ++i)
            bulk_prefetch_l2(p.w + unit_offset(u0 + i, p.tiles, nkb, nq) * kUnitBytes, kUnitBytes);

    pdl_wait();
    const int users = p.users;
    if (p.zero != nullptr) {
        // a fixed-point buffer of a later launch (its previous readers have completed before this launch's wait)
        uint4* z = reinterpret_cast<uint4*>(p.zero);
        bool wrote = false;
        for (size_t i = (size_t)blockIdx.x * kGemvThreads + tid; i < p.zero_words / 2; i += (size_t)G * kGemvThreads) {
            z[i] = make_uint4(0u, 0u, 0u, 0u);
            wrote = true;
        }
        // other GPUs add into this buffer only after they have seen this launch's own adds (which follow the
        // prologue's barrier): the zeros must be visible system-wide first
        if (p.zero_sys && wrote) __threadfence_system();
    }

    // ---- prologue: the activations' hi / lo operand for the K blocks of this CTA's window. Columns of users
    // past B (B < 4) are never written: an MMA column depends on its own operand column only.
    //
    // put_operand: the warp's 128 values h of user b, K block at window slot ws (lane: positions 4 lane .. + 3)
    // -> E = exponent of the block's max |h|, hi / lo e4m3 of h * 2^(7-E), 2^(E-7) for the epilogue
    auto put_operand = [&](int b, int ws, const float* h) {
        const float m = warp_max(fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3]))));
        int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127;
        e = max(e, -100);
        const float f = __uint_as_float((uint32_t)(127 + 7 - e) << 23);   // 2^(7-E): max|h| * f in [128, 256)
        const float fi = __uint_as_float((uint32_t)(127 - 7 + e) << 23);  // 2^(E-7)
        float lo[4];
        uint32_t hi_w = 0;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float y0 = h[j] * f, y1 = h[j + 1] * f;
            const uint32_t hb = e4m3x2(y0, y1);
            const float2 hf = e4m3x2_f32(hb);
            lo[j] = y0 - hf.x;  // exact
            lo[j + 1] = y1 - hf.y;
            hi_w |= hb << (8 * j);
        }
        const uint32_t lo_w = e4m3x2(lo[0], lo[1]) | (e4m3x2(lo[2], lo[3]) << 16);
        uint8_t* dst = act + (size_t)(b >> 2) * gstride + (size_t)ws * 8 * LBO + (lane >> 2) * LBO +
                       (2 * (b & 3)) * 16 + (lane & 3) * 4;
        *reinterpret_cast<uint32_t*>(dst) = hi_w;
        *reinterpret_cast<uint32_t*>(dst + 16) = lo_w;
        if (lane == 0) ainv[ws * 8 + b] = (b < users && m > 0.f) ? fi : 0.f;
    };
    // the tag of this launch's peer exchange (PRO_RMSNORM_ADD over tagged sources, or EPI_P2P)
    const uint32_t tag = (p.tagged != nullptr || EPI == EPI_P2P) ? *p.epoch * p.tag_mul + p.tag_add : 0u;
    // 4 consecutive tagged words of a source: re-read (bounded) until all carry the tag
    auto tagged4 = [&](const uint2* src) -> float4 {
        for (uint32_t it = 0;; ++it) {
            const uint4 a = ld_volatile128(src), c = ld_volatile128(src + 2);
            const bool fresh = a.y == tag && a.w == tag && c.y == tag && c.w == tag;
            if (fresh || it >= kPeerSpinLimit) {
                if (!fresh) atomicOr(p.err, kErrPeer | kErrTimeout);
                return make_float4(__uint_as_float(a.x), __uint_as_float(a.z), __uint_as_float(c.x), __uint_as_float(c.z));
            }
            __nanosleep(32);
        }
    };
    constexpr bool kAdd = PRO == PRO_RMSNORM_ADD || PRO == PRO_RMSNORM_XACC;  // residual + partial sums
    auto xload = [&](int b, int i) -> float4 {
        if (PRO == PRO_RMSNORM && p.seg) {
            const int s4 = p.seg / 4;
            return i < s4 ? reinterpret_cast<const float4*>(p.x + (size_t)b * p.seg)[i]
                          : reinterpret_cast<const float4*>(p.x2 + (size_t)b * p.seg)[i - s4];
        }
        float4 v = reinterpret_cast<const float4*>(p.x + (size_t)b * K)[i];
        if (kAdd) {
            // the sources summed in rank order first (n = 2: the same sum NCCL forms), then added to x
            float4 r;
            if (p.tagged != nullptr) {
                r = tagged4(p.tagged + (size_t)b * K + 4 * i);
                for (int s = 1; s < p.nsrc; ++s) {
                    const float4 q = tagged4(p.tagged + ((size_t)s * p.users + b) * K + 4 * i);
                    r.x += q.x;
                    r.y += q.y;
                    r.z += q.z;
                    r.w += q.w;
                }
            } else if (PRO == PRO_RMSNORM_XACC) {
                // counted words, complete (the sweep below)
                const longlong2* a = reinterpret_cast<const longlong2*>(p.racc + (size_t)b * K + 4 * i);
                const longlong2 a0 = __ldcg(a), a1 = __ldcg(a + 1);
                r = make_float4(acc_decode_cnt(a0.x), acc_decode_cnt(a0.y), acc_decode_cnt(a1.x), acc_decode_cnt(a1.y));
            } else if (p.racc != nullptr) {
                const longlong2* a = reinterpret_cast<const longlong2*>(p.racc + (size_t)b * K + 4 * i);
                const longlong2 a0 = __ldcg(a), a1 = __ldcg(a + 1);
                r = make_float4(acc_decode(a0.x), acc_decode(a0.y), acc_decode(a1.x), acc_decode(a1.y));
            } else {
                r = __ldcg(reinterpret_cast<const float4*>(p.red + (size_t)b * K) + i);
                for (int s = 1; s < p.nsrc; ++s) {
                    const float4 q = __ldcg(reinterpret_cast<const float4*>(p.red + s * p.src_stride + (size_t)b * K) + i);
                    r.x += q.x;
                    r.y += q.y;
                    r.z += q.z;
                    r.w += q.w;
                }
            }
            v.x += r.x;
            v.y += r.y;
            v.z += r.z;
            v.w += r.w;
        }
        return v;
    };
    // counted exchange over ranks: other GPUs' adds land at their own pace, so the CTA sweeps the accumulator words
    // (bounded) until every word holds rc_ranks x (the producer's CTAs over the word's tile) contributions; the
    // loads above then read complete words
    if (PRO == PRO_RMSNORM_XACC) {
        const int n4 = users * (K / 4), nk = p.rc_nkb;
        for (uint32_t it = 0;; ++it) {
            bool mine = true;
#pragma unroll 4
            for (int idx = tid; idx < n4; idx += kGemvThreads) {
                const int b = idx / (K / 4), i = idx - b * (K / 4);
                const long long* a = p.racc + (size_t)b * K + 4 * i;
                const uint4 v0 = ld_volatile128(a), v1 = ld_volatile128(a + 2);
                const int T = (4 * i) / kTileRows;
                const uint32_t want = (uint32_t)p.rc_ranks * (uint32_t)(cta_of_unit(T * nk + nk - 1, p.rc_base, p.rc_rem) -
                                                                        cta_of_unit(T * nk, p.rc_base, p.rc_rem) + 1);
                mine = mine && (v0.x & 255u) == want && (v0.z & 255u) == want && (v1.x & 255u) == want &&
                       (v1.z & 255u) == want;
            }
            if (__syncthreads_and(mine)) break;
            if (it >= kPeerSpinLimit / 64) {
                if (tid == 0) atomicOr(p.err, kErrPeer | kErrTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
    // rmsnorm with B <= 2 rows and K <= 8192 (the hidden size): one pass over x. Thread t's float4 j is
    // x[4 (t + 256 j) ..] -- K block warp + 8 j at lane -- so each warp writes the operand of the blocks it
    // holds, straight from registers.
    constexpr bool kRegs = (PRO == PRO_RMSNORM || kAdd) && B <= 2;
    constexpr int kXj = 8;
    const bool regs = kRegs && K <= kXj * 4 * kGemvThreads && p.seg == 0;
    float rn[B], rn2[B];  // rn2: the second segment's (two-segment prologue)
    if ((PRO == PRO_RMSNORM || kAdd) && !kRegs && p.seg == 0) {
        // more than 2 rows: the sums of squares with two users' loads in flight together (x_out by CTA 0)
#pragma unroll
        for (int b0 = 0; b0 < B; b0 += 2) {
            float ssa = 0.f, ssb = 0.f;
#pragma unroll 5
            for (int i = tid; i < K / 4; i += kGemvThreads) {
                float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
                if (b0 < users) va = xload(b0, i);
                if (b0 + 1 < users) vb = xload(b0 + 1, i);
                if (kAdd && blockIdx.x == 0) {
                    if (b0 < users) reinterpret_cast<float4*>(p.x_out + (size_t)b0 * K)[i] = va;
                    if (b0 + 1 < users) reinterpret_cast<float4*>(p.x_out + (size_t)(b0 + 1) * K)[i] = vb;
                }
                ssa += va.x * va.x + va.y * va.y + va.z * va.z + va.w * va.w;
                ssb += vb.x * vb.x + vb.y * vb.y + vb.z * vb.z + vb.w * vb.w;
            }
            ssa = warp_sum(ssa);
            ssb = warp_sum(ssb);
            if (lane == 0) {
                red[warp][b0] = ssa;
                if (b0 + 1 < B) red[warp][b0 + 1] = ssb;
            }
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float tsum = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) tsum += red[w][b];
            rn[b] = rsqrt_ieee(tsum / (float)K + kEps);
            rn2[b] = rn[b];
        }
    } else if (PRO == PRO_RMSNORM || kAdd) {
        float4 xr[kRegs ? B : 1][kXj];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float ss = 0.f;
            if (b < users) {
                // the hidden-size row plus fixed-point sums (the step's rmsnorm prologue): every load of the row issued
                // before any is used -- a load behind a per-iteration branch would cost one L2 round trip per
                // iteration (the operand build waits on this)
                constexpr int kXh = kHidden / (4 * kGemvThreads);  // 5
                if (regs && K == kHidden && kAdd && p.tagged == nullptr && p.racc != nullptr) {
                    longlong2 q[kXh][2];
#pragma unroll
                    for (int j = 0; j < kXh; ++j) {
                        const int i = tid + j * kGemvThreads;
                        xr[kRegs ? b : 0][j] = reinterpret_cast<const float4*>(p.x + (size_t)b * K)[i];
                        const longlong2* a = reinterpret_cast<const longlong2*>(p.racc + (size_t)b * K + 4 * i);
                        q[j][0] = __ldcg(a);
                        q[j][1] = __ldcg(a + 1);
                    }
#pragma unroll
                    for (int j = 0; j < kXh; ++j) {
                        const int i = tid + j * kGemvThreads;
                        float4 v = xr[kRegs ? b : 0][j];
                        if (PRO == PRO_RMSNORM_XACC) {
                            v.x += acc_decode_cnt(q[j][0].x);
                            v.y += acc_decode_cnt(q[j][0].y);
                            v.z += acc_decode_cnt(q[j][1].x);
                            v.w += acc_decode_cnt(q[j][1].y);
                        } else {
                            v.x += acc_decode(q[j][0].x);
                            v.y += acc_decode(q[j][0].y);
                            v.z += acc_decode(q[j][1].x);
                            v.w += acc_decode(q[j][1].y);
                        }
                        if (blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out + (size_t)b * K)[i] = v;
                        xr[kRegs ? b : 0][j] = v;
                        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    }
#pragma unroll
                    for (int j = kXh; j < kXj; ++j) xr[kRegs ? b : 0][j] = make_float4(0.f, 0.f, 0.f, 0.f);
                } else if (regs) {
#pragma unroll
                    for (int j = 0; j < kXj; ++j) {
                        const int i = tid + j * kGemvThreads;
                        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (i < K / 4) {
                            v = xload(b, i);
                            if (kAdd && blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out + (size_t)b * K)[i] = v;
                        }
                        xr[kRegs ? b : 0][j] = v;
                        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    }
                } else {
                    float ss2 = 0.f;
#pragma unroll 5
                    for (int i = tid; i < K / 4; i += kGemvThreads) {
                        const float4 v = xload(b, i);
                        if (kAdd && blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out + (size_t)b * K)[i] = v;
                        const float q = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                        if (p.seg && 4 * i >= p.seg) ss2 += q;
                        else ss += q;
                    }
                    if (B <= 4) {
                        ss2 = warp_sum(ss2);
                        if (lane == 0) red[warp][4 + (B <= 4 ? b : 0)] = ss2;
                    }
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp][b] = ss;
        }
        __syncthreads();
        const float klen = (float)(p.seg ? p.seg : K);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float tsum = 0.f, tsum2 = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                tsum += red[w][b];
                if (B <= 4) tsum2 += red[w][4 + (B <= 4 ? b : 0)];
            }
            rn[b] = rsqrt_ieee(tsum / klen + kEps);
            rn2[b] = rsqrt_ieee(tsum2 / klen + kEps);
        }
        if (regs) {
#pragma unroll
            for (int j = 0; j < kXj; ++j) {
                const int kb = warp + 8 * j;  // warp-uniform
                if (kb >= nkb) break;
                int ws = kb - kb_start;
                if (ws < 0) ws += nkb;
                if (ws >= nwin) continue;  // outside this CTA's window
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4 v = xr[kRegs ? b : 0][j];
                    // h = bf16(x * r)
                    const float h[4] = {bf16_round(v.x * rn[b]), bf16_round(v.y * rn[b]), bf16_round(v.z * rn[b]),
                                        bf16_round(v.w * rn[b])};
                    put_operand(b, ws, h);
                }
            }
        }
    } else {
#pragma unroll
        for (int b = 0; b < B; ++b) rn[b] = rn2[b] = 1.f;
    }
    // otherwise one warp per (user, K block) pair, 4 pairs in flight: lane holds K positions 4 * lane .. + 3
    const int npairs = regs ? 0 : B * nwin;
    for (int pr0 = warp; pr0 < npairs; pr0 += 32) {
        float hv[4][4];
        // PRO_SILU_ACC: a lane's 4 columns 4 lane .. + 3 of K block kb are the gate|up rows 256 kb + 8 lane .. + 7:
        // g(c), g(c+1), u(c), u(c+1), g(c+2), g(c+3), u(c+2), u(c+3) (quad-interleaved rows); all loads first
        longlong2 gq[PRO == PRO_SILU_ACC ? 4 : 1][4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int pr = pr0 + 8 * c;
            const int b = pr % B, ws = pr / B;
            int kb = kb_start + ws;
            if (kb >= nkb) kb -= nkb;
            hv[c][0] = hv[c][1] = hv[c][2] = hv[c][3] = 0.f;
            if (PRO == PRO_SILU_ACC) {
#pragma unroll
                for (int j = 0; j < 4; ++j) gq[PRO == PRO_SILU_ACC ? c : 0][j] = make_longlong2(0, 0);
            }
            if (pr < npairs && b < users) {
                if (PRO == PRO_BF16) {
                    const uint2 v = *reinterpret_cast<const uint2*>(p.in + (size_t)b * p.ld_in + kb * 128 + 4 * lane);
                    hv[c][0] = bf16lo(v.x);
                    hv[c][1] = bf16hi(v.x);
                    hv[c][2] = bf16lo(v.y);
                    hv[c][3] = bf16hi(v.y);
                } else if (PRO == PRO_SILU_ACC) {
                    const longlong2* g = reinterpret_cast<const longlong2*>(p.gacc + (size_t)b * p.ld_gacc + (size_t)kb * 256 + 8 * lane);
#pragma unroll
                    for (int j = 0; j < 4; ++j) gq[PRO == PRO_SILU_ACC ? c : 0][j] = __ldcg(g + j);
                } else {
                    const float4 v = xload(b, kb * 32 + lane);
                    hv[c][0] = v.x;
                    hv[c][1] = v.y;
                    hv[c][2] = v.z;
                    hv[c][3] = v.w;
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int pr = pr0 + 8 * c;
            if (pr >= npairs) break;  // warp-uniform
            const int b = pr % B, ws = pr / B;
            float h[4];
            if (PRO == PRO_BF16) {
#pragma unroll
                for (int j = 0; j < 4; ++j) h[j] = hv[c][j];
            } else if (PRO == PRO_SILU_ACC) {
                // h = bf16(silu(g) * u), the SwiGLU product the gate|up epilogue forms in the unfused path
                const longlong2* q = gq[PRO == PRO_SILU_ACC ? c : 0];
                const float g[4] = {acc_decode(q[0].x), acc_decode(q[0].y), acc_decode(q[2].x), acc_decode(q[2].y)};
                const float u[4] = {acc_decode(q[1].x), acc_decode(q[1].y), acc_decode(q[3].x), acc_decode(q[3].y)};
#pragma unroll
                for (int j = 0; j < 4; ++j) h[j] = __bfloat162float(__float2bfloat16_rn(silu_f(g[j]) * u[j]));
            } else {
                // h = bf16(x * r), r of the block's segment
                int kbq = kb_start + ws;
                if (kbq >= nkb) kbq -= nkb;
                const bool second = p.seg && kbq * 128 >= p.seg;
                float rb = 1.f;
#pragma unroll
                for (int bb = 0; bb < B; ++bb)
                    if (bb == b) rb = second ? rn2[bb] : rn[bb];
#pragma unroll
                for (int j = 0; j < 4; ++j) h[j] = bf16_round(hv[c][j] * rb);
            }
            put_operand(b, ws, h);
        }
    }
    fence_proxy_async();  // the operand written by generic stores, read by the tensor core (async proxy)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = min(NS, cnt);
    if (warp == 0) {
        // ---- producer
        if (lane == 0) {
            for (int i = NS; i < cnt; ++i) {
                if (!mbar_wait(&empty[i % NS], ((i / NS) - 1) & 1, p.err)) break;
                issue(i);
                issued = i + 1;
            }
            l2_prefetch_heads(p.next, blockIdx.x, G);
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t ring_a = smem_addr(ring), act_a = smem_addr(act);
            const uint32_t sbo_b = B > 4 ? (uint32_t)gstride : 0u;  // users 4..7 (columns 8..15)
            UnitWalk it(u0, p.tiles, nq);
            for (int i = 0; i < cnt; ++i) {
                const int slot = i % NS, d = i % kDSlots;
                int ws = it.kb() - kb_start;
                if (ws < 0) ws += nkb;
                it.next();
                if (!mbar_wait(&full[slot], (i / NS) & 1, p.err)) break;
                if (i >= kDSlots && !mbar_wait(&dempty[d], ((i / kDSlots) - 1) & 1, p.err)) break;
                tc_fence_after();
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const uint64_t ad = smem_desc(ring_a + slot * kUnitBytes + m * 32, 16, 1024, 2);
                    const uint64_t bd = smem_desc(act_a + ws * 8 * LBO + m * 2 * LBO, LBO, sbo_b);
                    tc_mma_f8(tmem + d * 16, ad, bd, m > 0 ? 1u : 0u);
                }
                tc_commit(&empty[slot]);
                tc_commit(&dfull[d]);
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.err);
        }
    } else if (warp >= 4) {
        // ---- epilogue: TMEM lanes 32q .. 32q + 31 (the warp's TMEM quarter), one tile row per thread
        const int q = warp & 3, row = 32 * q + lane;
        const size_t tstride = kSelBytes + (size_t)nkb * 32;
        bool ok = true;
        float acc[B], first_acc[B];
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b] = first_acc[b] = 0.f;
        int cur = -1, first_tile = -1;
        const int first_T = u0 / nkb;
        auto split_tile = [&](int T) { return cta_of_unit(T * nkb, base, rem) != cta_of_unit(T * nkb + nkb - 1, base, rem); };
        auto store = [&](int T, const float* v) {
            const int r = T * kTileRows + row;
            if (EPI == EPI_SILU_MUL) {
                // quads of rows are gate(j), gate(j+1), up(j), up(j+1): the up partner of row r is r + 2
                float up[B];
#pragma unroll
                for (int b = 0; b < B; ++b) up[b] = __shfl_down_sync(0xffffffffu, v[b], 2);
                if ((row & 3) < 2) {
                    const int col = 2 * (r >> 2) + (r & 3);
#pragma unroll
                    for (int b = 0; b < B; ++b)
                        if (b < users && 2 * col < p.rows)
                            reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)b * p.ld_out + col] =
                                __float2bfloat16_rn(silu_f(v[b]) * up[b]);
                }
            } else if (EPI == EPI_P2P) {
                // the row into every rank's window as a tagged word (one 8-byte store, remote over NVLink)
                if (r < p.rows) {
                    for (int d = 0; d < p.p2p_n; ++d) {
#pragma unroll
                        for (int b = 0; b < B; ++b)
                            if (b < users)
                                p.peer_data[d][(size_t)b * p.peer_ld + r] = make_uint2(__float_as_uint(v[b]), tag);
                    }
                }
            } else if (r < p.rows) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    if (b >= users) break;
                    if (EPI == EPI_BF16) {
                        reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)b * p.ld_out + r] = __float2bfloat16_rn(v[b]);
                    } else if (EPI == EPI_RESID) {
                        float* o = reinterpret_cast<float*>(p.out) + (size_t)b * p.ld_out + r;
                        *o = v[b] + *o;
                    } else {
                        reinterpret_cast<float*>(p.out)[(size_t)b * p.ld_out + r] = v[b];
                    }
                }
            }
        };
        // EPI_ACC: this CTA's part of a tile's rows into the fixed-point accumulators (split or not alike)
        auto red_tile = [&](int T, const float* v) {
            const int r = T * kTileRows + row;
            if (r < p.rows) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    if (b >= users) break;
                    const size_t off = (size_t)b * p.ld_out + r;
                    if (EPI == EPI_XACC) {
                        // the counted exchange: into every rank's accumulator (remote adds over NVLink)
                        const unsigned long long e = acc_encode_cnt(v[b]);
                        for (int d = 0; d < p.xn; ++d) atomicAdd(reinterpret_cast<unsigned long long*>(p.xdst[d] + off), e);
                    } else {
                        atomicAdd(reinterpret_cast<unsigned long long*>(p.acc_out + off), acc_encode(v[b]));
                    }
                }
            }
        };
        // the tiles of this CTA split with other CTAs (only its first and its last tile can be), finished
        // together in one round: parts out, one ticket each, the last CTA of a tile adds the parts in CTA order
        auto finish_split = [&](int n, int T0, float* v0, int T1, float* v1) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                if (t >= n) break;
                const int T = t ? T1 : T0;
                const float* v = t ? v1 : v0;
                float* dst = p.part + ((size_t)blockIdx.x * 2 + (T == first_T ? 0 : 1)) * 8 * 128;
#pragma unroll
                for (int b = 0; b < B; ++b) dst[b * 128 + row] = v[b];
            }
            // release / acquire through one thread per tile: the named barrier orders every epilogue thread's
            // part stores before that thread's (cumulative) fence and ticket; the last CTA of a tile fences again
            // before the barrier that releases its threads' reads (a fence in every thread costs microseconds)
            bar_sync(1, 128);
            if (row < n) {
                __threadfence();
                const int T = row ? T1 : T0;
                const int tk = atomicAdd(p.ticket + T, 1);
                tk_slot[row] = tk;
                if (tk == cta_of_unit(T * nkb + nkb - 1, base, rem) - cta_of_unit(T * nkb, base, rem)) __threadfence();
            }
            bar_sync(1, 128);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                if (t >= n) break;
                const int T = t ? T1 : T0;
                float* v = t ? v1 : v0;
                const int c0 = cta_of_unit(T * nkb, base, rem), c1 = cta_of_unit(T * nkb + nkb - 1, base, rem);
                if (tk_slot[t] != c1 - c0) continue;  // uniform over the epilogue warps
                // the parts of up to 16 CTAs in flight at once (one L2 round trip per batch: the loads are
                // unconditional, past-the-end ones re-read the last part), added in CTA order
                constexpr int kBatch = B <= 2 ? 16 : B <= 4 ? 8 : 4;
#pragma unroll
                for (int b = 0; b < B; ++b) v[b] = 0.f;
                for (int c = c0; c <= c1; c += kBatch) {
                    const float* src[kBatch];
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        const int cc = min(c + j, c1);
                        const int cu0 = cc * base + min(cc, rem);
                        src[j] = p.part + ((size_t)cc * 2 + ((T == cu0 / nkb) ? 0 : 1)) * 8 * 128 + row;
                    }
                    float q[kBatch][B];
#pragma unroll
                    for (int j = 0; j < kBatch; ++j)
#pragma unroll
                        for (int b = 0; b < B; ++b) q[j][b] = __ldcg(src[j] + b * 128);
#pragma unroll
                    for (int j = 0; j < kBatch; ++j)
                        if (c + j <= c1) {
#pragma unroll
                            for (int b = 0; b < B; ++b) v[b] += q[j][b];
                        }
                }
                if (row == 0) p.ticket[T] = 0;
                store(T, v);
            }
        };

        // the scale of the next unit is loaded one unit ahead
        UnitWalk it(u0, p.tiles, nq);
        int sel = p.table[(size_t)it.T * tstride + row];
        float s_next = __ldg(reinterpret_cast<const float*>(p.table + (size_t)it.T * tstride + kSelBytes) + it.kb() * 8 + sel);
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
        for (int i = 0; i < cnt; ++i) {
            const float s = s_next;
            const int Tc = it.T;
            int wsc = it.kb() - kb_start;
            if (wsc < 0) wsc += nkb;
            it.next();
            if (i + 1 < cnt) {
                if (it.T != Tc) sel = p.table[(size_t)it.T * tstride + row];
                s_next = __ldg(reinterpret_cast<const float*>(p.table + (size_t)it.T * tstride + kSelBytes) + it.kb() * 8 + sel);
            }
            // after a timeout the warp keeps its place in the loop without waiting (its results are void, the
            // error word is set): every epilogue warp reaches the same tile flushes and their named barriers
            const int d = i % kDSlots;
            if (ok && !mbar_wait(&dfull[d], (i / kDSlots) & 1, p.err)) ok = false;
            tc_fence_after();
            constexpr int NC = B <= 4 ? 2 * B : 16;
            float v[NC];
            tmem_load<NC>(taddr + d * 16, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dempty[d]);
            if (Tc != cur) {
                if (cur >= 0 && (EPI == EPI_ACC || EPI == EPI_XACC)) {
                    red_tile(cur, acc);
                } else if (cur >= 0) {
                    // a tile that ends inside the range: the first one may be split (held for the end), any
                    // later one lies wholly in this CTA
                    if (cur == first_T && split_tile(cur)) {
                        first_tile = cur;
#pragma unroll
                        for (int b = 0; b < B; ++b) first_acc[b] = acc[b];
                    } else {
                        store(cur, acc);
                    }
                }
#pragma unroll
                for (int b = 0; b < B; ++b) acc[b] = 0.f;
                cur = Tc;
            }
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] = fmaf(v[2 * b] + v[2 * b + 1], s * ainv[wsc * 8 + b], acc[b]);
        }
        if (EPI == EPI_ACC || EPI == EPI_XACC) {
            if (cur >= 0) red_tile(cur, acc);
        } else {
            if (cur >= 0 && !split_tile(cur)) {
                store(cur, acc);
                cur = -1;
            }
            if (cur >= 0 && first_tile >= 0) finish_split(2, first_tile, first_acc, cur, acc);
            else if (cur >= 0) finish_split(1, cur, acc, 0, acc);
            else if (first_tile >= 0) finish_split(1, first_tile, first_acc, 0, first_acc);
        }
    }
    if (warp == 0 && lane == 0) {
        // never release shared memory with a copy still landing in it
        for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------------------------

template <int B, int PRO, int EPI>
static cudaError_t launch_b(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
    auto k = gemv_fp8_kernel<B, PRO, EPI>;
    static size_t smem_set = 0;  // largest dynamic shared memory opted in so far for this instantiation
    if (smem > smem_set) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, p);
}

template <int PRO, int EPI>
static cudaError_t launch_pe(const GemvParams& p, int Bt, int grid, size_t smem, cudaStream_t st, bool pdl) {
    switch (Bt) {
        case 1: return launch_b<1, PRO, EPI>(p, grid, smem, st, pdl);
        case 2: return launch_b<2, PRO, EPI>(p, grid, smem, st, pdl);
        case 4: return launch_b<4, PRO, EPI>(p, grid, smem, st, pdl);
        default: return launch_b<8, PRO, EPI>(p, grid, smem, st, pdl);
    }
}

// ---------------------------------------------------------------------------------------------------------
// The rmsnorm input of a projection formed once per user (the step at 4 or more rows on one rank): x_out = x +
// the previous projection's fixed-point sums (or x alone), h = bf16(x_out * rsqrt(mean(x_out^2) + eps)). The
// projection then reads its activation window of h (PRO_BF16) instead of every CTA forming all of x_out and its
// norm for every user again (at 8 rows that is ~480 KB of reads per CTA before its first MMA). One CTA per user,
// 640 threads x 8 consecutive elements.
constexpr int kResidThreads = kHidden / 8;

// Over ranks (rc_ranks > 0) racc holds counted words -- (value << 8) + contributions, added by every rank's
// row-parallel epilogue -- and the CTA first sweeps its user's words (bounded) until each holds rc_ranks x (the
// producing launch's CTAs over the word's tile) contributions (the producer split its units as rc_base / rc_rem,
// rc_nkb K blocks per tile).
__global__ void __launch_bounds__(kResidThreads) resid_norm_kernel(const float* x, const long long* racc, float* x_out,
                                                                    uint16_t* h, int rc_ranks, int rc_base, int rc_rem,
                                                                    int rc_nkb, uint32_t* err) {
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float red[kResidThreads / 32];
    pdl_launch();
    pdl_wait();
    if (racc != nullptr && rc_ranks > 0) {
        // this thread's 8 words lie in one 128-row tile
        const int T = (8 * tid) / kTileRows;
        const uint32_t want = (uint32_t)rc_ranks * (uint32_t)(cta_of_unit(T * rc_nkb + rc_nkb - 1, rc_base, rc_rem) -
                                                              cta_of_unit(T * rc_nkb, rc_base, rc_rem) + 1);
        const long long* a = racc + (size_t)b * kHidden + 8 * tid;
        for (uint32_t it = 0;; ++it) {
            bool mine = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 v = ld_volatile128(a + 2 * j);
                mine = mine && (v.x & 255u) == want && (v.z & 255u) == want;
            }
            if (__syncthreads_and(mine)) break;
            if (it >= kPeerSpinLimit / 64) {
                if (tid == 0) atomicOr(err, kErrPeer | kErrTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
    const float4* xs = reinterpret_cast<const float4*>(x + (size_t)b * kHidden) + 2 * tid;
    float v[8];
    const float4 a0 = xs[0], a1 = xs[1];
    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
    v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    if (racc != nullptr) {
        const longlong2* ra = reinterpret_cast<const longlong2*>(racc + (size_t)b * kHidden) + 4 * tid;
        longlong2 q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = __ldcg(ra + j);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] += rc_ranks > 0 ? acc_decode_cnt(q[j].x) : acc_decode(q[j].x);
            v[2 * j + 1] += rc_ranks > 0 ? acc_decode_cnt(q[j].y) : acc_decode(q[j].y);
        }
        float4* xo = reinterpret_cast<float4*>(x_out + (size_t)b * kHidden) + 2 * tid;
        xo[0] = make_float4(v[0], v[1], v[2], v[3]);
        xo[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kResidThreads / 32; ++w) t += red[w];
    const float r = rsqrt_ieee(t / (float)kHidden + kEps);
    uint32_t hw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        hw[j] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j] * r)) |
                ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j + 1] * r)) << 16);
    reinterpret_cast<uint4*>(h + (size_t)b * kHidden)[tid] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
}

cudaError_t resid_norm_launch(int users, const float* x, const long long* racc, float* x_out, uint16_t* h,
                              cudaStream_t st, bool pdl, const GemvExchange* ex, uint32_t* err) {
    if (users < 1 || users > kMaxRows || (racc && !x_out)) return cudaErrorInvalidValue;
    int rc_ranks = 0, rc_base = 0, rc_rem = 0, rc_nkb = 0;
    if (ex != nullptr && ex->rc_ranks > 0) {
        // the counted words of a producer whose partition is given (as gemv_launch checks it)
        if (racc == nullptr || err == nullptr || ex->rc_grid < 1 || ex->rc_nkb < 1 || ex->rc_units < ex->rc_grid)
            return cudaErrorInvalidValue;
        rc_ranks = ex->rc_ranks;
        rc_base = ex->rc_units / ex->rc_grid;
        rc_rem = ex->rc_units % ex->rc_grid;
        rc_nkb = ex->rc_nkb;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(users);
    cfg.blockDim = dim3(kResidThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, resid_norm_kernel, x, racc, x_out, h, rc_ranks, rc_base, rc_rem, rc_nkb, err);
}

// The down-projection's input formed once per user (4 or more rows): h = bf16(silu(g) * u) from gate|up's
// fixed-point sums, whose rows come in quads per 4 columns c .. c+3 -- g(c), g(c+1), u(c), u(c+1), g(c+2), g(c+3),
// u(c+2), u(c+3) -- so column quad j reads the 8 words 8 j .. 8 j + 7. The down-projection then reads its window
// of h (PRO_BF16, 2 bytes per element and user) instead of every CTA decoding 16 bytes of sums per element and
// user of its window (~160 KB per CTA at 8 users). Same arithmetic as the PRO_SILU_ACC prologue.
__global__ void __launch_bounds__(256) silu_rows_kernel(const long long* acc, int ld_acc, int ic, int users, uint16_t* h) {
    pdl_launch();
    pdl_wait();
    const int nq = ic / 4;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < users * nq; i += gridDim.x * 256) {
        const int b = i / nq, j = i - b * nq;
        const longlong2* a = reinterpret_cast<const longlong2*>(acc + (size_t)b * ld_acc + 8 * (size_t)j);
        const longlong2 q0 = __ldcg(a), q1 = __ldcg(a + 1), q2 = __ldcg(a + 2), q3 = __ldcg(a + 3);
        const float g[4] = {acc_decode(q0.x), acc_decode(q0.y), acc_decode(q2.x), acc_decode(q2.y)};
        const float u[4] = {acc_decode(q1.x), acc_decode(q1.y), acc_decode(q3.x), acc_decode(q3.y)};
        uint32_t w[2];
#pragma unroll
        for (int t = 0; t < 2; ++t)
            w[t] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(silu_f(g[2 * t]) * u[2 * t])) |
                   ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(silu_f(g[2 * t + 1]) * u[2 * t + 1])) << 16);
        reinterpret_cast<uint2*>(h + (size_t)b * ic)[j] = make_uint2(w[0], w[1]);
    }
}

cudaError_t silu_rows_launch(int users, const long long* acc, int ld_acc, int ic, uint16_t* h, cudaStream_t st, bool pdl) {
    if (users < 1 || users > kMaxRows || ic % 4 || !acc || !h) return cudaErrorInvalidValue;
    const int total = users * (ic / 4);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min((total + 255) / 256, 2 * 148));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, silu_rows_kernel, acc, ld_acc, ic, users, h);
}

// shared memory of one GEMV CTA: half an SM's (a second CTA -- the next projection's, under programmatic
// dependent launch -- fits beside it and starts its weight stream during this one's tail); past that, up to
// the per-CTA maximum with a shallower ring
#ifndef QRES_GEMV_BUDGET_KB
#define QRES_GEMV_BUDGET_KB 113
#endif
constexpr size_t kGemvSmemBudget = QRES_GEMV_BUDGET_KB * 1024;
constexpr size_t kGemvSmemMax = 227 * 1024;
constexpr int kMinStages = 3;

static int bt_of(int users) { return users == 1 ? 1 : users == 2 ? 2 : users <= 4 ? 4 : 8; }

// K blocks per group of the launch's unit order (unit_offset): the plain fixed-point accumulators (EPI_ACC) take
// any number of partial sums per tile, so with 4 or more rows -- whose hi / lo operand costs 1 or 2 KB of shared
// memory per K block -- a CTA's run covers a few tiles of one K group (at most ~12 KB of operand per group)
// instead of one tile's whole K: a small activation window leaves room for a deep ring and two CTAs per SM and
// builds fewer operand blocks. Every other launch walks the storage order (nkb).
int gemv_group_blocks(int users, int epi, int K) {
    const int nkb = K / 128, Bt = bt_of(users);
    if (epi != EPI_ACC || Bt < 4) return nkb;
    const int per_kb = 8 * gemv_act_lbo(Bt) * (Bt > 4 ? 2 : 1) + 32;
    for (int d = nkb; d >= 2; --d)
        if (nkb % d == 0 && d * per_kb <= 12 * 1024) return d;
    return nkb;
}

// workspace: the tile tickets at a fixed place (they must read zero at every launch, whatever the grid or the
// weight: each launch leaves the ones it used at zero), then a [grid][2][8][128] fp32 part buffer per launch
constexpr int kGemvMaxTiles = 4096;  // 524,288 rows
size_t gemv_workspace_bytes(int grid) { return (size_t)kGemvMaxTiles * 4 + (size_t)grid * 2 * 8 * 128 * 4; }

// grid actually launched for a request of `grid` CTAs: at most one per unit, and enough that every CTA's
// activation window fits in shared memory
int gemv_grid(int users, int rows_pad, int K, int grid) {
    const int U = (rows_pad / kTileRows) * (K / 128);
    const int Bt = bt_of(users);
    int g = grid < 1 ? 1 : grid;
    if (g > U) g = U;
    for (;;) {
        const int nkw = std::min((U + g - 1) / g, K / 128);
        if (gemv_smem_bytes(Bt, nkw, kMinStages) <= kGemvSmemMax || g >= U) return g;
        g = std::min(U, g + g / 4 + 1);
    }
}

cudaError_t gemv_launch(const qres_weight& w, int users, int pro, const void* in, int ld_in, int epi, void* out,
                        int ld_out, int grid, uint32_t* err, cudaStream_t st, bool pdl, const float* red, float* x_out,
                        void* work, size_t work_bytes, const L2Heads* next, const GemvExchange* ex = nullptr) {
    if (users < 1 || users > kMaxRows || w.K % 128 != 0 || w.rows_pad % kTileRows != 0 || w.rows_pad < w.rows ||
        w.rows_pad > kGemvMaxTiles * kTileRows)
        return cudaErrorInvalidValue;
    const int Bt = bt_of(users);
    const int nkb = w.K / 128;
    const int tiles = w.rows_pad / kTileRows;
    grid = gemv_grid(users, w.rows_pad, w.K, grid);
    if (work == nullptr || work_bytes < gemv_workspace_bytes(grid)) return cudaErrorInvalidValue;
    GemvParams p;
    p.w = static_cast<const uint8_t*>(w.data);
    p.table = reinterpret_cast<const uint8_t*>(w.uscale);
    p.rows = w.rows;
    p.tiles = tiles;
    p.K = w.K;
    p.nkb = nkb;
    p.users = users;
    p.x = (pro == PRO_RMSNORM || pro == PRO_RMSNORM_ADD || pro == PRO_RMSNORM_XACC) ? static_cast<const float*>(in) : nullptr;
    p.in = pro == PRO_BF16 ? static_cast<const uint16_t*>(in) : nullptr;
    p.ld_in = ld_in;
    p.red = red;
    p.x_out = x_out;
    const GemvExchange none;
    const GemvExchange& e = ex ? *ex : none;
    if (pro == PRO_RMSNORM_ADD && ((red == nullptr && e.racc == nullptr) || x_out == nullptr)) return cudaErrorInvalidValue;
    if ((pro == PRO_SILU_ACC) != (e.gacc != nullptr) || (epi == EPI_ACC) != (e.acc_out != nullptr) ||
        (epi == EPI_XACC) != (e.xn > 0) || e.zero_words % 2 ||
        (e.racc != nullptr && pro == PRO_RMSNORM_ADD && (e.nsrc != 1 || e.rc_ranks != 0)) ||
        (e.racc != nullptr && pro != PRO_RMSNORM_ADD && pro != PRO_RMSNORM_XACC) ||
        (pro == PRO_RMSNORM_XACC && (e.racc == nullptr || e.rc_ranks < 1 || x_out == nullptr)))
        return cudaErrorInvalidValue;
    p.racc = e.racc;
    p.gacc = e.gacc;
    p.ld_gacc = e.ld_gacc;
    p.acc_out = e.acc_out;
    p.zero = e.zero;
    p.zero_words = e.zero ? e.zero_words : 0;
    p.zero_sys = e.zero_sys;
    if (e.xn < 0 || e.xn > kMaxPeers) return cudaErrorInvalidValue;
    p.xn = e.xn;
    for (int i = 0; i < kMaxPeers; ++i) p.xdst[i] = e.xdst[i];
    p.rc_ranks = e.rc_ranks;
    p.rc_nkb = e.rc_nkb;
    p.rc_base = p.rc_rem = 0;
    // the counted words keep their contribution count in the low 8 bits: ranks x (CTAs over one 128-row tile)
    // must stay below 256, for this launch's adds (EPI_XACC) and for the producer a prologue waits for
    auto max_ctas_per_tile = [](int units, int grid, int nkb) {
        const int b = units / grid, r = units % grid, big = r * (b + 1);
        auto cta = [&](int u) { return u < big ? u / (b + 1) : r + (u - big) / b; };
        int m = 0;
        for (int t = 0; t < units / nkb; ++t) m = std::max(m, cta(t * nkb + nkb - 1) - cta(t * nkb) + 1);
        return m;
    };
    if (e.rc_ranks > 0) {
        if (e.racc == nullptr || e.rc_grid < 1 || e.rc_nkb < 1 || e.rc_units < e.rc_grid) return cudaErrorInvalidValue;
        p.rc_base = e.rc_units / e.rc_grid;
        p.rc_rem = e.rc_units % e.rc_grid;
        if (e.rc_ranks * max_ctas_per_tile(e.rc_units, e.rc_grid, e.rc_nkb) >= 256) return cudaErrorInvalidValue;
    }
    if (epi == EPI_XACC && e.xn * max_ctas_per_tile(tiles * nkb, grid, nkb) >= 256) return cudaErrorInvalidValue;
    if (e.nsrc < 1 || e.nsrc > kMaxPeers || e.p2p_n < 0 || e.p2p_n > kMaxPeers) return cudaErrorInvalidValue;
    if ((epi == EPI_P2P) != (e.p2p_n > 0) || (e.tagged != nullptr && pro != PRO_RMSNORM_ADD) ||
        ((e.tagged != nullptr || e.p2p_n > 0) && e.epoch == nullptr))
        return cudaErrorInvalidValue;
    if (e.seg && (pro != PRO_RMSNORM || users > 4 || e.seg2 == nullptr || w.K != 2 * e.seg || e.seg % 128))
        return cudaErrorInvalidValue;
    p.x2 = e.seg2;
    p.seg = e.seg;
    p.nsrc = e.nsrc;
    p.src_stride = e.src_stride;
    p.tagged = e.tagged;
    p.epoch = e.epoch;
    p.tag_mul = e.tag_mul;
    p.tag_add = e.tag_add;
    p.p2p_n = e.p2p_n;
    p.peer_ld = e.peer_ld;
    for (int i = 0; i < kMaxPeers; ++i) p.peer_data[i] = e.peer_data[i];
    p.out = out;
    p.ld_out = ld_out;
    p.err = err;
    p.next = next ? *next : L2Heads{nullptr, 0, 0, 0, 0, 1, 1, 1};
    uint8_t* wk = static_cast<uint8_t*>(work);
    p.ticket = reinterpret_cast<int*>(wk);
    p.part = reinterpret_cast<float*>(wk + (size_t)kGemvMaxTiles * 4);
    const int U = tiles * nkb;
    p.nq = gemv_group_blocks(users, epi, w.K);
    if (p.nq == nkb) {
        p.nkw = std::min((U + grid - 1) / grid, nkb);
    } else {
        // the widest window: the K groups a CTA's run spans
        const int b = U / grid, r = U % grid, per = tiles * p.nq;
        p.nkw = 0;
        for (int c = 0; c < grid; ++c) {
            const int u0 = c * b + std::min(c, r), cnt = b + (c < r ? 1 : 0);
            p.nkw = std::max(p.nkw, std::min(((u0 + cnt - 1) / per - u0 / per + 1) * p.nq, nkb));
        }
    }
    // ring depth: as deep as half an SM allows, else as deep as the per-CTA maximum allows
    const size_t fixed = gemv_smem_bytes(Bt, p.nkw, 0);
    int ns = fixed < kGemvSmemBudget ? (int)((kGemvSmemBudget - fixed) / kUnitBytes) : 0;
    if (ns < kMinStages) ns = fixed < kGemvSmemMax ? (int)((kGemvSmemMax - fixed) / kUnitBytes) : 0;
    if (ns < kMinStages) return cudaErrorInvalidValue;
    ns = ns > kMaxStages ? kMaxStages : ns;
    p.nstages = ns;
    const size_t smem = gemv_smem_bytes(Bt, p.nkw, ns);
    if (pro == PRO_RMSNORM && epi == EPI_BF16) return launch_pe<PRO_RMSNORM, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_SILU_MUL) return launch_pe<PRO_RMSNORM, EPI_SILU_MUL>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_F32) return launch_pe<PRO_RMSNORM, EPI_F32>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_ACC) return launch_pe<PRO_RMSNORM, EPI_ACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_ADD && epi == EPI_BF16) return launch_pe<PRO_RMSNORM_ADD, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_ADD && epi == EPI_SILU_MUL) return launch_pe<PRO_RMSNORM_ADD, EPI_SILU_MUL>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_RESID) return launch_pe<PRO_BF16, EPI_RESID>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_F32) return launch_pe<PRO_BF16, EPI_F32>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_BF16) return launch_pe<PRO_BF16, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_P2P) return launch_pe<PRO_BF16, EPI_P2P>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_ACC) return launch_pe<PRO_BF16, EPI_ACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_ADD && epi == EPI_ACC) return launch_pe<PRO_RMSNORM_ADD, EPI_ACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_SILU_ACC && epi == EPI_ACC) return launch_pe<PRO_SILU_ACC, EPI_ACC>(p, Bt, grid, smem, st, pdl);
    // the counted exchange between ranks
    if (pro == PRO_BF16 && epi == EPI_XACC) return launch_pe<PRO_BF16, EPI_XACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_SILU_ACC && epi == EPI_XACC) return launch_pe<PRO_SILU_ACC, EPI_XACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_XACC && epi == EPI_ACC) return launch_pe<PRO_RMSNORM_XACC, EPI_ACC>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_XACC && epi == EPI_BF16) return launch_pe<PRO_RMSNORM_XACC, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace qres
