// The projections between two mixers as one persistent launch on the sm_100a tensor cores: the out-projection,
// gate|up, the down-projection and the next layer's in-projection (or the lm_head) of a decode step.
//
// Every phase is the FP8 weight-streaming GEMV of gemv_fp8.cu (same units, scale table, e4m3 hi / lo operand,
// tcgen05 MMAs into TMEM, split-tile finish by ticket), but the weight stream never stops at a phase boundary:
// warp 0 issues the CTA's units of all phases back to back through one ring, so HBM keeps streaming the next
// projection while the previous one's last tiles finish. The data dependencies between phases go through tagged
// words -- {32-bit value, tag} in one 8-byte store -- that the consumer re-reads (bounded) until they carry the
// producing phase's tag: the out- and down-projections' fp32 partials (into every rank's exchange window, so
// the same words carry the tensor-parallel all-reduce), and gate|up's SwiGLU output. A consumer thus waits
// exactly for the values it reads, and no grid-wide barrier exists.
//
// Roles (256 threads, two CTAs per SM; all CTAs of the launch are co-resident, which the grid size ensures):
//   warp 0 lane 0   streams units (never waits for data: weights are immutable);
//   warp 1          owns TMEM; lane 0 issues a phase's MMAs once the phase's operand is built;
//   warps 2..7      build each phase's activation operand (rmsnorm over the residual plus the exchanged
//                   partials, or the tagged / plain bf16 input) after the previous phase's epilogue is done;
//   warps 4..7      drain TMEM slots, apply the scales and finish tiles of each phase.
// Every wait is bounded (sets the error word and keeps going with void values, never hangs).
#include "gemv_chain.cuh"

namespace qres {

// unit range of CTA `cta` in a phase of U units over G CTAs
struct Range {
    int base, rem, u0, cnt;
};
__device__ __forceinline__ Range range_of(int U, int G, int cta) {
    Range r;
    r.base = U / G;
    r.rem = U % G;
    r.u0 = cta * r.base + min(cta, r.rem);
    r.cnt = r.base + (cta < r.rem ? 1 : 0);
    return r;
}

template <int B>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_chain_kernel(const __grid_constant__ ChainParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kMaxStages]
    uint64_t* empty = full + kMaxStages;                 // [kMaxStages]
    uint64_t* dfull = empty + kMaxStages;                // [kDSlots]
    uint64_t* dempty = dfull + kDSlots;                  // [kDSlots]
    uint64_t* drain = dempty + kDSlots;
    uint64_t* act_ready = drain + 1;                     // a phase's operand is built (phase parity)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(act_ready + 1);
    int* tk_slot = reinterpret_cast<int*>(tmem_slot + 1);  // [2]
    float (*red)[8] = reinterpret_cast<float (*)[8]>(smem + 512);  // [8 warps][8 users]
    const int nkw = p.nkw;
    float* ainv = reinterpret_cast<float*>(smem + kHeadBytes);
    uint8_t* act = smem + kHeadBytes + gemv_ainv_bytes(nkw);
    constexpr int LBO = gemv_act_lbo(B);
    const size_t gstride = gemv_act_group(B, nkw);
    const size_t pre = kHeadBytes + gemv_ainv_bytes(nkw) + gemv_act_bytes(B, nkw);
    uint8_t* ring = smem + ((pre + 1023) & ~size_t(1023));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, NS = p.nstages, users = p.users;

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
        mbar_init(act_ready, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- producer: every phase's units through one ring, no data waits
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int g = 0;
            bool ok = true;
            for (int k = 0; k < p.nphase && ok; ++k) {
                const ChainPhase& ph = p.ph[k];
                const Range r = range_of(ph.tiles * ph.nkb, G, blockIdx.x);
                for (int i = 0; i < r.cnt; ++i, ++g) {
                    const int slot = g % NS;
                    if (g >= NS && !mbar_wait(&empty[slot], ((g / NS) - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[slot], kUnitBytes);
                    bulk_g2s_hint(ring + (size_t)slot * kUnitBytes, ph.w + (size_t)(r.u0 + i) * kUnitBytes, kUnitBytes,
                                  &full[slot], pol);
                }
            }
            // never release shared memory with a copy still landing in it
            for (int i = max(0, g - NS); i < g; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t ring_a = smem_addr(ring), act_a = smem_addr(act);
            const uint32_t sbo_b = B > 4 ? (uint32_t)gstride : 0u;
            int g = 0;
            bool ok = true;
            for (int k = 0; k < p.nphase && ok; ++k) {
                const ChainPhase& ph = p.ph[k];
                const Range r = range_of(ph.tiles * ph.nkb, G, blockIdx.x);
                if (!mbar_wait(act_ready, k & 1, p.err)) break;
                tc_fence_after();
                int ws = 0;
                for (int i = 0; i < r.cnt; ++i, ++g) {
                    const int slot = g % NS, d = g % kDSlots;
                    if (!mbar_wait(&full[slot], (g / NS) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    if (g >= kDSlots && !mbar_wait(&dempty[d], ((g / kDSlots) - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const uint64_t ad = smem_desc(ring_a + slot * kUnitBytes + m * 32, 16, 1024, 2);
                        const uint64_t bd = smem_desc(act_a + ws * 8 * LBO + m * 2 * LBO, LBO, sbo_b);
                        tc_mma_f8(tmem + d * 16, ad, bd, m > 0 ? 1u : 0u);
                    }
                    tc_commit(&empty[slot]);
                    tc_commit(&dfull[d]);
                    if (++ws == ph.nkb) ws = 0;
                }
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.err);
        }
    } else {
        // ---- warps 2..7: each phase's operand, then (warps 4..7) its epilogue
        pdl_wait();  // the first phase's input is the previous kernel's output
        const uint32_t epoch = *p.epoch;
        const int pt = tid - 64;  // 0..191 over warps 2..7
        const int pw = warp - 2;  // 0..5
        bool ok = true;
        int g = 0;  // units drained so far (epilogue warps)
        // 4 consecutive tagged words: re-read (bounded) until all carry the tag
        auto tagged4 = [&](const uint2* src, uint32_t tag, uint4* lo, uint4* hi) {
            for (uint32_t it = 0;; ++it) {
                const uint4 a = ld_volatile128(src), c = ld_volatile128(src + 2);
                const bool fresh = a.y == tag && a.w == tag && c.y == tag && c.w == tag;
                if (fresh || !ok || it >= kPeerSpinLimit) {
                    if (!fresh && ok) {
                        atomicOr(p.err, kErrPeer | kErrTimeout);
                        ok = false;
                    }
                    *lo = a;
                    *hi = c;
                    return;
                }
                __nanosleep(32);
            }
        };
        for (int k = 0; k < p.nphase; ++k) {
            const ChainPhase& ph = p.ph[k];
            const int K = ph.K, nkb = ph.nkb;
            const Range r = range_of(ph.tiles * nkb, G, blockIdx.x);
            const int kb_start = r.cnt ? r.u0 % nkb : 0;
            const int nwin = min(r.cnt, nkb);
            // exchange slots / tags of this phase's input sets
            const uint2* set_src[2] = {nullptr, nullptr};
            uint32_t set_tag[2] = {0u, 0u};
            for (int s = 0; s < ph.nsets; ++s) {
                const uint32_t t = epoch * p.set_mul + ph.set_add[s];
                set_tag[s] = t;
                set_src[s] = p.xbase[p.rank] + (size_t)((t - 1) % 3) * p.slot_words;
            }
            // ---- operand of phase k (warps 2..7) once phase k-1's epilogue is done here (its MMAs read act)
            bar_sync(2, 192);
            // the warp's 128 values h of user b, K block at window slot ws -> e4m3 hi / lo operand and 2^(E-7)
            auto put_operand = [&](int b, int ws, const float* h) {
                const float m = warp_max(fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3]))));
                int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127;
                e = max(e, -100);
                const float f = __uint_as_float((uint32_t)(127 + 7 - e) << 23);
                const float fi = __uint_as_float((uint32_t)(127 - 7 + e) << 23);
                float lo[4];
                uint32_t hi_w = 0;
#pragma unroll
                for (int jj = 0; jj < 4; jj += 2) {
                    const float y0 = h[jj] * f, y1 = h[jj + 1] * f;
                    const uint32_t hb = e4m3x2(y0, y1);
                    const float2 hf = e4m3x2_f32(hb);
                    lo[jj] = y0 - hf.x;
                    lo[jj + 1] = y1 - hf.y;
                    hi_w |= hb << (8 * jj);
                }
                const uint32_t lo_w = e4m3x2(lo[0], lo[1]) | (e4m3x2(lo[2], lo[3]) << 16);
                uint8_t* dst = act + (size_t)(b >> 2) * gstride + (size_t)ws * 8 * LBO + (lane >> 2) * LBO +
                               (2 * (b & 3)) * 16 + (lane & 3) * 4;
                *reinterpret_cast<uint32_t*>(dst) = hi_w;
                *reinterpret_cast<uint32_t*>(dst + 16) = lo_w;
                if (lane == 0) ainv[ws * 8 + b] = (b < users && m > 0.f) ? fi : 0.f;
            };
            auto fresh = [](const uint4& a, const uint4& c, uint32_t tag) {
                return a.y == tag && a.w == tag && c.y == tag && c.w == tag;
            };
            if (r.cnt > 0 && ph.in_kind == CIN_NORM) {
                // per user: the residual rows with the exchanges added, in registers -- thread pt's float4 j is
                // x[4 (pt + 192 j)], i.e. K block pw + 6 j at lane -- all loads of a batch in flight before any tag
                // is checked; then the block's sum of squares and the operand straight from the registers
                constexpr int kCj = 7;  // K <= 7 x 192 x 4 = 5376 (the hidden size)
                for (int b = 0; b < B; ++b) {
                    float4 xv[kCj];
#pragma unroll
                    for (int jj = 0; jj < kCj; ++jj) {
                        const int i = pt + 192 * jj;
                        xv[jj] = (b < users && i < K / 4) ? reinterpret_cast<const float4*>(ph.x + (size_t)b * K)[i]
                                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    for (int s = 0; b < users && s < ph.nsets; ++s) {
                        // half by half (4 float4s): every rank's partial, summed in rank order, then added to x
#pragma unroll
                        for (int h0 = 0; h0 < kCj; h0 += 4) {
                            float4 es[4];
                            for (int q = 0; q < p.nsrc; ++q) {
                                const uint2* src = set_src[s] + (size_t)q * p.src_words + (size_t)b * K;
                                uint4 ra[4], rc[4];
#pragma unroll
                                for (int jj = 0; jj < 4; ++jj) {
                                    const int i = pt + 192 * (h0 + jj);
                                    if (h0 + jj < kCj && i < K / 4) {
                                        ra[jj] = ld_volatile128(src + 4 * i);
                                        rc[jj] = ld_volatile128(src + 4 * i + 2);
                                    }
                                }
#pragma unroll
                                for (int jj = 0; jj < 4; ++jj) {
                                    const int i = pt + 192 * (h0 + jj);
                                    if (h0 + jj < kCj && i < K / 4) {
                                        if (!fresh(ra[jj], rc[jj], set_tag[s])) tagged4(src + 4 * i, set_tag[s], &ra[jj], &rc[jj]);
                                        const float4 f = make_float4(__uint_as_float(ra[jj].x), __uint_as_float(ra[jj].z),
                                                                     __uint_as_float(rc[jj].x), __uint_as_float(rc[jj].z));
                                        if (q == 0) {
                                            es[jj] = f;
                                        } else {
                                            es[jj].x += f.x;
                                            es[jj].y += f.y;
                                            es[jj].z += f.z;
                                            es[jj].w += f.w;
                                        }
                                    }
                                }
                            }
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                if (h0 + jj < kCj && pt + 192 * (h0 + jj) < K / 4) {
                                    xv[h0 + jj].x += es[jj].x;
                                    xv[h0 + jj].y += es[jj].y;
                                    xv[h0 + jj].z += es[jj].z;
                                    xv[h0 + jj].w += es[jj].w;
                                }
                            }
                        }
                    }
                    float ss = 0.f;
#pragma unroll
                    for (int jj = 0; jj < kCj; ++jj) {
                        const int i = pt + 192 * jj;
                        if (i < K / 4) {
                            const float4 v = xv[jj];
                            if (ph.x_out && blockIdx.x == 0 && b < users)
                                reinterpret_cast<float4*>(ph.x_out + (size_t)b * K)[i] = v;
                            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                        }
                    }
                    ss = warp_sum(ss);
                    if (lane == 0) red[pw][b] = ss;
                    bar_sync(2, 192);
                    float tsum = 0.f;
                    for (int w = 0; w < 6; ++w) tsum += red[w][b];
                    const float rnb = rsqrt_ieee(tsum / (float)K + kEps);
#pragma unroll
                    for (int jj = 0; jj < kCj; ++jj) {
                        const int kb = pw + 6 * jj;  // warp-uniform
                        if (kb >= nkb) break;
                        int ws = kb - kb_start;
                        if (ws < 0) ws += nkb;
                        if (ws >= nwin) continue;  // outside this CTA's window
                        // h = bf16(x * r)
                        const float h[4] = {bf16_round(xv[jj].x * rnb), bf16_round(xv[jj].y * rnb),
                                            bf16_round(xv[jj].z * rnb), bf16_round(xv[jj].w * rnb)};
                        put_operand(b, ws, h);
                    }
                }
            } else if (r.cnt > 0) {
                // bf16 inputs: one warp per (user, K block) pair of the window, 4 pairs in flight
                const int npairs = B * nwin;
                for (int pr0 = pw; pr0 < npairs; pr0 += 24) {
                    uint4 ra[4], rc[4];
                    uint2 rv[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int pr = pr0 + 6 * c;
                        const int b = pr % B, ws = pr / B;
                        int kb = kb_start + ws;
                        if (kb >= nkb) kb -= nkb;
                        ra[c] = rc[c] = make_uint4(0, 0, 0, 0);
                        rv[c] = make_uint2(0, 0);
                        if (pr < npairs && b < users) {
                            if (ph.in_kind == CIN_BF16) {
                                rv[c] = *reinterpret_cast<const uint2*>(ph.in_bf16 + (size_t)b * K + kb * 128 + 4 * lane);
                            } else {
                                const uint2* src = ph.in_tagged + (size_t)b * K + kb * 128 + 4 * lane;
                                ra[c] = ld_volatile128(src);
                                rc[c] = ld_volatile128(src + 2);
                            }
                        }
                    }
                    const uint32_t itag = epoch * ph.in_mul + ph.in_add;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int pr = pr0 + 6 * c;
                        if (pr >= npairs) break;  // warp-uniform
                        const int b = pr % B, ws = pr / B;
                        float h[4] = {0.f, 0.f, 0.f, 0.f};
                        if (b < users) {
                            if (ph.in_kind == CIN_BF16) {
                                h[0] = bf16lo(rv[c].x);
                                h[1] = bf16hi(rv[c].x);
                                h[2] = bf16lo(rv[c].y);
                                h[3] = bf16hi(rv[c].y);
                            } else {
                                if (!fresh(ra[c], rc[c], itag)) {
                                    int kb = kb_start + ws;
                                    if (kb >= nkb) kb -= nkb;
                                    tagged4(ph.in_tagged + (size_t)b * K + kb * 128 + 4 * lane, itag, &ra[c], &rc[c]);
                                }
                                h[0] = bf16lo(ra[c].x);
                                h[1] = bf16lo(ra[c].z);
                                h[2] = bf16lo(rc[c].x);
                                h[3] = bf16lo(rc[c].z);
                            }
                        }
                        put_operand(b, ws, h);
                    }
                }
            }
            fence_proxy_async();
            tc_fence_before();
            bar_sync(2, 192);
            if (pt == 0) mbar_arrive(act_ready);
            if (warp < 4) continue;  // warps 2, 3: on to the next phase's operand barrier

            // ---- epilogue of phase k (warps 4..7, TMEM lanes 32q .. 32q + 31, one tile row per thread)
            const int q = warp & 3, row = 32 * q + lane;
            const size_t tstride = kSelBytes + (size_t)nkb * 32;
            const int first_T = r.cnt ? r.u0 / nkb : 0;
            float* part = p.part + (size_t)blockIdx.x * 2 * 2 * 8 * 128 + (size_t)(k & 1) * 2 * 8 * 128;
            int* ticket = p.ticket + (size_t)k * kChainTickets;
            const uint32_t out_tag = ph.out_kind == COUT_PARTIAL ? epoch * p.set_mul + ph.out_add : epoch * ph.out_mul + ph.out_add;
            auto cta_of = [&](int u) {
                const Range rr = range_of(ph.tiles * nkb, G, 0);
                return cta_of_unit(u, rr.base, rr.rem);
            };
            auto split_tile = [&](int T) { return cta_of(T * nkb) != cta_of(T * nkb + nkb - 1); };
            auto store = [&](int T, const float* v) {
                const int rg = T * kTileRows + row;
                if (ph.out_kind == COUT_SILU_TAGGED) {
                    float up[B];
#pragma unroll
                    for (int b = 0; b < B; ++b) up[b] = __shfl_down_sync(0xffffffffu, v[b], 2);
                    if ((row & 3) < 2) {
                        const int col = 2 * (rg >> 2) + (rg & 3);
#pragma unroll
                        for (int b = 0; b < B; ++b)
                            if (b < users && 2 * col < ph.rows) {
                                const __nv_bfloat16 a = __float2bfloat16_rn(silu_f(v[b]) * up[b]);
                                reinterpret_cast<uint2*>(ph.out)[(size_t)b * ph.ld_out + col] =
                                    make_uint2((uint32_t)__bfloat16_as_ushort(a), out_tag);
                            }
                    }
                } else if (rg < ph.rows) {
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        if (b >= users) break;
                        if (ph.out_kind == COUT_BF16) {
                            reinterpret_cast<__nv_bfloat16*>(ph.out)[(size_t)b * ph.ld_out + rg] = __float2bfloat16_rn(v[b]);
                        } else {
                            // this rank's partial into its region of every rank's window (remote over NVLink)
                            const size_t off = (size_t)((out_tag - 1) % 3) * p.slot_words + (size_t)p.rank * p.src_words +
                                               (size_t)b * ph.ld_out + rg;
                            for (int d = 0; d < p.nsrc; ++d) p.xbase[d][off] = make_uint2(__float_as_uint(v[b]), out_tag);
                        }
                    }
                }
            };
            auto finish_split = [&](int n, int T0, float* v0, int T1, float* v1) {
                const Range rr = range_of(ph.tiles * nkb, G, 0);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (t >= n) break;
                    const int T = t ? T1 : T0;
                    const float* v = t ? v1 : v0;
                    float* dst = part + (T == first_T ? 0 : 1) * 8 * 128;
#pragma unroll
                    for (int b = 0; b < B; ++b) dst[b * 128 + row] = v[b];
                }
                bar_sync(1, 128);
                if (row < n) {
                    __threadfence();
                    const int T = row ? T1 : T0;
                    const int tk = atomicAdd(ticket + T, 1);
                    tk_slot[row] = tk;
                    if (tk == cta_of_unit(T * nkb + nkb - 1, rr.base, rr.rem) - cta_of_unit(T * nkb, rr.base, rr.rem))
                        __threadfence();
                }
                bar_sync(1, 128);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (t >= n) break;
                    const int T = t ? T1 : T0;
                    float* v = t ? v1 : v0;
                    const int c0 = cta_of_unit(T * nkb, rr.base, rr.rem), c1 = cta_of_unit(T * nkb + nkb - 1, rr.base, rr.rem);
                    if (tk_slot[t] != c1 - c0) continue;  // uniform over the epilogue warps
                    constexpr int kBatch = B <= 2 ? 16 : B <= 4 ? 8 : 4;
#pragma unroll
                    for (int b = 0; b < B; ++b) v[b] = 0.f;
                    for (int c = c0; c <= c1; c += kBatch) {
                        const float* src[kBatch];
#pragma unroll
                        for (int j = 0; j < kBatch; ++j) {
                            const int cc = min(c + j, c1);
                            const int cu0 = cc * rr.base + min(cc, rr.rem);
                            src[j] = p.part + (size_t)cc * 2 * 2 * 8 * 128 + (size_t)(k & 1) * 2 * 8 * 128 +
                                     ((T == cu0 / nkb) ? 0 : 1) * 8 * 128 + row;
                        }
                        float qv[kBatch][B];
#pragma unroll
                        for (int j = 0; j < kBatch; ++j)
#pragma unroll
                            for (int b = 0; b < B; ++b) qv[j][b] = __ldcg(src[j] + b * 128);
#pragma unroll
                        for (int j = 0; j < kBatch; ++j)
                            if (c + j <= c1) {
#pragma unroll
                                for (int b = 0; b < B; ++b) v[b] += qv[j][b];
                            }
                    }
                    if (row == 0) ticket[T] = 0;
                    store(T, v);
                }
            };

            float acc[B], first_acc[B];
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] = first_acc[b] = 0.f;
            int cur = -1, first_tile = -1;
            int T = first_T, kb = kb_start, ws = 0;
            int sel = r.cnt ? __ldg(ph.table + (size_t)T * tstride + row) : 0;
            float s_next = r.cnt ? __ldg(reinterpret_cast<const float*>(ph.table + (size_t)T * tstride + kSelBytes) + kb * 8 + sel) : 0.f;
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
            for (int i = 0; i < r.cnt; ++i, ++g) {
                const float s = s_next;
                const int Tc = T, wsc = ws;
                if (++kb == nkb) {
                    kb = 0;
                    ++T;
                    if (i + 1 < r.cnt) sel = __ldg(ph.table + (size_t)T * tstride + row);
                }
                if (++ws == nkb) ws = 0;
                if (i + 1 < r.cnt)
                    s_next = __ldg(reinterpret_cast<const float*>(ph.table + (size_t)T * tstride + kSelBytes) + kb * 8 + sel);
                const int d = g % kDSlots;
                if (ok && !mbar_wait(&dfull[d], (g / kDSlots) & 1, p.err)) ok = false;
                tc_fence_after();
                constexpr int NC = B <= 4 ? 2 * B : 16;
                float v[NC];
                tmem_load<NC>(taddr + d * 16, v);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&dempty[d]);
                if (Tc != cur) {
                    if (cur >= 0) {
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
            if (cur >= 0 && !split_tile(cur)) {
                store(cur, acc);
                cur = -1;
            }
            if (cur >= 0 && first_tile >= 0) finish_split(2, first_tile, first_acc, cur, acc);
            else if (cur >= 0) finish_split(1, cur, acc, 0, acc);
            else if (first_tile >= 0) finish_split(1, first_tile, first_acc, 0, first_acc);
        }
        bar_sync(2, 192);  // the last phase's epilogue is done before warps 2, 3 leave
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

size_t chain_workspace_bytes(int grid) {
    return (size_t)kChainMaxPhases * kChainTickets * 4 + (size_t)grid * 2 * 2 * 8 * 128 * 4;
}

template <int B>
static cudaError_t chain_launch_b(const ChainParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
    auto k = gemv_chain_kernel<B>;
    static size_t smem_set = 0;
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

// Launch a chain: p's phases filled by the caller except the geometry fields computed here. grid must not exceed
// the CTAs that can be resident at once (two per SM at this shared-memory size): consumers wait for producers of
// the same launch.
cudaError_t chain_launch(ChainParams& p, int grid, int sm_count, void* work, size_t work_bytes, cudaStream_t st,
                         bool pdl) {
    if (p.nphase < 1 || p.nphase > kChainMaxPhases || p.users < 1 || p.users > kMaxRows || p.nsrc < 1 ||
        p.nsrc > kMaxPeers || grid < 1 || grid > 2 * sm_count || p.epoch == nullptr)
        return cudaErrorInvalidValue;
    if (work == nullptr || work_bytes < chain_workspace_bytes(grid)) return cudaErrorInvalidValue;
    const int Bt = p.users == 1 ? 1 : p.users == 2 ? 2 : p.users <= 4 ? 4 : 8;
    int nkw = 1;
    for (int k = 0; k < p.nphase; ++k) {
        ChainPhase& ph = p.ph[k];
        if (ph.K % 128 || ph.tiles < 1 || ph.tiles > kChainTickets || ph.nkb != ph.K / 128) return cudaErrorInvalidValue;
        const int U = ph.tiles * ph.nkb;
        nkw = std::max(nkw, std::min((U + grid - 1) / grid, ph.nkb));
    }
    uint8_t* wk = static_cast<uint8_t*>(work);
    p.ticket = reinterpret_cast<int*>(wk);
    p.part = reinterpret_cast<float*>(wk + (size_t)kChainMaxPhases * kChainTickets * 4);
    p.nkw = nkw;
    const size_t fixed = gemv_smem_bytes(Bt, nkw, 0);
    const size_t budget = 113 * 1024;
    if (fixed + 3 * (size_t)kUnitBytes > budget) return cudaErrorInvalidValue;  // two CTAs per SM or not at all
    int ns = (int)((budget - fixed) / kUnitBytes);
    ns = std::min(ns, kMaxStages);
    p.nstages = ns;
    const size_t smem = gemv_smem_bytes(Bt, nkw, ns);
    switch (Bt) {
        case 1: return chain_launch_b<1>(p, grid, smem, st, pdl);
        case 2: return chain_launch_b<2>(p, grid, smem, st, pdl);
        case 4: return chain_launch_b<4>(p, grid, smem, st, pdl);
        default: return chain_launch_b<8>(p, grid, smem, st, pdl);
    }
}

}  // namespace qres
