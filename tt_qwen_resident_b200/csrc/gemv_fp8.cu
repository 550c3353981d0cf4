// Block-scaled FP8 weight-streaming projection for 1..8 rows (users) on sm_100a tensor cores.
//
// Replaces the reference's streamer cores (qwen36_resident/kernels/streamer_reader.cpp:45-89 weight ring,
// streamer_compute.cpp:60-92 M=1..8 matmul, :100-210 rmsnorm, :212-249 silu(g)*u, :252-273 residual fold).
//
// Math: out[u][n] = sum_kb scale[sidx[n]][kb] * sum_{k in kb} h[u][k] * q[n][k], q the e4m3 weight, h the bf16
// activation; every product is exact (e4m3 -> f16 and bf16 -> f16 are exact conversions in the f16 range,
// f16 x f16 fits fp32) and accumulates in fp32. Each 16-row x 128-K block is one mma.sync.m16n8k16 chain of 8
// MMAs (weights as A, the rows' activations as B: one user per column, so 8 users cost what one does), then
// scaled by its block scale into the fp32 result.
//
// Layout (qres_tile_weight): rows in tiles of 16 (zero-padded); a tile's K in 128-wide blocks ("units", 2 KB
// each, a tile's units back to back); inside a unit row r's 128 bytes at r*128, its two 64-byte halves swapped
// when r is odd (conflict-free shared-memory reads). One fp32 scale per 128 x 128 block of the canonical
// matrix; the scales are streamed per unit (uscale: the scale of the unit's rows r % 4 < 2 and r % 4 >= 2,
// which is all a 16-row tile of these shards ever holds), loaded one stage ahead.
//
// Work split: the tiles x blocks units are divided evenly over every warp of the grid (148 CTAs x 8 warps);
// each warp streams its contiguous run of units through its own ring of shared-memory stages with
// cp.async.bulk (no multicast; its first stages are issued before griddepcontrol.wait, so under programmatic
// dependent launch the weight stream starts while the previous kernel finishes). A warp accumulates a tile in
// registers; a tile split between warps is finished by the last of them (an atomic ticket), which adds the
// parts in warp order (deterministic).
//
// MMA operand mapping: the 16 k-slots of an MMA may map to any 16 K positions as long as A and B agree. Lane
// (g, t) (g = lane / 4, t = lane % 4) takes the 4 bytes at K = 64*half + 16*t + 4*m of rows g and g + 8 for MMA
// m of a half-block. Words m = 0, 1 go through the conversion unit (bytes 0,1 -> k-slots 2t,2t+1; bytes 2,3 ->
// 2t+8,2t+9); words m = 2, 3 through integer ops (bytes 1,3 -> 2t,2t+1; bytes 0,2 -> 2t+8,2t+9, values scaled
// by 2^-8, undone once per block), which splits the conversion work between the XU and ALU pipes. The B
// fragment takes the same positions of user g's h, stored in shared memory in that order (h_slot). Each word m
// accumulates in its own fragment (short MMA dependency chains).
#include "qres_common.cuh"

namespace qres {

enum { PRO_RMSNORM = 0, PRO_BF16 = 1, PRO_RMSNORM_ADD = 2 };
enum { EPI_BF16 = 0, EPI_SILU_MUL = 1, EPI_RESID = 2, EPI_F32 = 3 };

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kUnitBytes = 2048;  // 16 rows x 128 K
constexpr int kStageUnits = 2;
constexpr int kStageBytes = kStageUnits * kUnitBytes;
constexpr int kMaxStages = 4;     // per warp
constexpr int kHPad = 8;          // f16 elements of padding per h row (bank spread between users)

struct GemvParams {
    const uint8_t* w;
    const float2* uscale;   // [tiles][nkb]: the block scale of each unit's rows r % 4 < 2 (.x) and r % 4 >= 2 (.y)
    int rows, tiles, K, nkb;
    int kb0, kb1;           // K blocks [kb0, kb1) of this launch (a K-split launch covers part of K)
    int users;              // real users (<= template B)
    const float* x;         // PRO_RMSNORM(_ADD): fp32 [users][K]
    const float* red;       // PRO_RMSNORM_ADD: all-reduced partials [users][K]; x_out = x + red
    float* x_out;           // PRO_RMSNORM_ADD: written by CTA 0
    const uint16_t* in;     // PRO_BF16: bf16 [users][ld_in]
    int ld_in;
    void* out;              // EPI_BF16 / EPI_SILU_MUL: bf16 [users][ld_out]; EPI_RESID / EPI_F32: fp32
    int ld_out;
    int nstages;            // ring depth per warp
    float* part;            // [grid * 8 warps][2][128]: a warp's split first / last tile
    int* ticket;            // [tiles]
    // the next weight-streaming projection of the step (same grid): once its own stream is done, every warp
    // prefetches the start of its range there into L2, so HBM keeps streaming through this kernel's tail
    const uint8_t* next_w;
    int next_units;         // units of the next launch
    int next_prefetch;      // units per warp to prefetch
    uint32_t* err;
};

__host__ __device__ inline size_t gemv_h_bytes(int B, int K) { return ((size_t)B * (K + kHPad) * 2 + 127) & ~size_t(127); }

__host__ __device__ inline size_t gemv_smem_bytes(int B, int K, int nstages) {
    return 512 /* barriers */ + gemv_h_bytes(B, K) + (size_t)kGemvWarps * nstages * kStageBytes;
}

// 4 e4m3 bytes (K positions P..P+3) -> two f16x2 by the conversion unit: lo = (P, P+1), hi = (P+2, P+3), exact
__device__ __forceinline__ void cvt_word_xu(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

// the same 4 bytes by integer ops, each as the f16 with bits (s << 15) | (low7 << 7): the e4m3 value times 2^-8,
// exact for normals and subnormals alike. odd = (P+1, P+3), even = (P, P+2) -- a different pairing, matched by
// the activations' layout in shared memory.
__device__ __forceinline__ void cvt_word_alu(uint32_t w, uint32_t& odd, uint32_t& even) {
    odd = (w & 0x80008000u) | ((w >> 1) & 0x3F803F80u);
    const uint32_t w8 = w << 8;
    even = (w8 & 0x80008000u) | ((w8 >> 1) & 0x3F803F80u);
}

// position of K index k of the activations in shared memory: inside every 16-group, the second 8 positions
// (the words converted by cvt_word_alu) are stored per 4-group as (1, 3, 0, 2)
__device__ __forceinline__ int h_slot(int k) {
    const int r = k & 15;
    if (r < 8) return k;
    const int q = r & 3;
    const int to = (q == 0) ? 2 : (q == 1) ? 0 : (q == 2) ? 3 : 1;
    return (k & ~3) + to;
}

__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// global warp owning unit u when U units are split over W warps (base = U / W, rem = U % W)
__device__ __forceinline__ int warp_of_unit(int u, int base, int rem) {
    const int big = rem * (base + 1);
    if (u < big) return u / (base + 1);
    return rem + (u - big) / base;
}

template <int B, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_fp8_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [8 warps][kMaxStages]
    __half* hs = reinterpret_cast<__half*>(smem + 512);
    const int hld = p.K + kHPad;
    uint8_t* ring = smem + 512 + gemv_h_bytes(B, p.K);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int K = p.K;
    const int nkbl = p.kb1 - p.kb0;  // blocks per tile in this launch
    const int U = p.tiles * nkbl;
    const int W = gridDim.x * kGemvWarps;
    const int gw = blockIdx.x * kGemvWarps + warp;
    const int base = U / W, rem = U % W;
    const int u0 = gw * base + min(gw, rem);
    const int cnt = base + (gw < rem ? 1 : 0);
    const int NS = p.nstages;
    const int nst = (cnt + kStageUnits - 1) / kStageUnits;
    uint64_t* bars = full + warp * kMaxStages;
    uint8_t* wring = ring + (size_t)warp * NS * kStageBytes;

    if (lane == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_launch();

    // stage s of this warp: units [u0 + 2s, min(u0 + 2s + 2, u0 + cnt)); a launch's units of one tile are
    // contiguous in memory, a stage crossing a tile boundary takes two copies
    auto unit_addr = [&](int u) -> const uint8_t* {
        const int T = u / nkbl, kb = p.kb0 + u % nkbl;
        return p.w + ((size_t)T * p.nkb + kb) * kUnitBytes;
    };
    const uint64_t pol = policy_evict_first();  // every weight byte is read once per step
    auto issue = [&](int s) {
        const int a = u0 + s * kStageUnits, n = min(kStageUnits, u0 + cnt - a);
        uint8_t* dst = wring + (size_t)(s % NS) * kStageBytes;
        mbar_arrive_expect_tx(&bars[s % NS], n * kUnitBytes);
        int i = 0;
        while (i < n) {
            int run = 1;
            while (i + run < n && (a + i + run) % nkbl != 0) ++run;
            bulk_g2s_hint(dst + i * kUnitBytes, unit_addr(a + i), run * kUnitBytes, &bars[s % NS], pol);
            i += run;
        }
    };
    if (lane == 0)
        for (int s = 0; s < min(NS, nst); ++s) issue(s);

    pdl_wait();
    const int users = p.users;
    // ---- prologue: h (f16 [B][K + pad]) in shared memory, from x (rmsnorm) or a bf16 input
    if (PRO == PRO_RMSNORM || PRO == PRO_RMSNORM_ADD) {
        __shared__ float red[kGemvWarps][B];
        auto xload = [&](int b, int i) -> float4 {
            float4 v = reinterpret_cast<const float4*>(p.x + (size_t)b * K)[i];
            if (PRO == PRO_RMSNORM_ADD) {
                const float4 r = reinterpret_cast<const float4*>(p.red + (size_t)b * K)[i];
                v.x += r.x;
                v.y += r.y;
                v.z += r.z;
                v.w += r.w;
            }
            return v;
        };
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float ss = 0.f;
            if (b < users) {
                for (int i = threadIdx.x; i < K / 4; i += kGemvThreads) {
                    const float4 v = xload(b, i);
                    if (PRO == PRO_RMSNORM_ADD && blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out + (size_t)b * K)[i] = v;
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp][b] = ss;
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float tsum = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) tsum += red[w][b];
            const float r = rsqrt_ieee(tsum / (float)K + kEps);
            __half* hv = hs + (size_t)b * hld;
            for (int i = threadIdx.x; i < K / 4; i += kGemvThreads) {
                float4 v = b < users ? xload(b, i) : make_float4(0.f, 0.f, 0.f, 0.f);
                // h = bf16(x * r), held exactly as f16, at its permuted slot
                hv[h_slot(4 * i)] = __float2half_rn(bf16_round(v.x * r));
                hv[h_slot(4 * i + 1)] = __float2half_rn(bf16_round(v.y * r));
                hv[h_slot(4 * i + 2)] = __float2half_rn(bf16_round(v.z * r));
                hv[h_slot(4 * i + 3)] = __float2half_rn(bf16_round(v.w * r));
            }
        }
    } else {
#pragma unroll
        for (int b = 0; b < B; ++b) {
            __half* hv = hs + (size_t)b * hld;
            const uint32_t* iv = reinterpret_cast<const uint32_t*>(p.in + (size_t)b * p.ld_in);
            for (int i = threadIdx.x; i < K / 2; i += kGemvThreads) {
                const uint32_t w2 = b < users ? iv[i] : 0u;
                hv[h_slot(2 * i)] = __float2half_rn(bf16lo(w2));
                hv[h_slot(2 * i + 1)] = __float2half_rn(bf16hi(w2));
            }
        }
    }
    __syncthreads();

    // ---- main loop: one 16 x 128 unit at a time
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int cur = -1;  // tile being accumulated
    bool ok = true;
    const bool rows_b = (g & 3) >= 2;  // rows g and g + 8 are both of a quad's second pair (the up rows of gate|up)
    const bool hrow = g < B;
    const __half* hg = hs + (size_t)(hrow ? g : 0) * hld;

    auto split_tile = [&](int T) {
        const int ufirst = T * nkbl, ulast = ufirst + nkbl - 1;
        return warp_of_unit(ufirst, base, rem) != warp_of_unit(ulast, base, rem);
    };
    auto flush = [&](int T, const float* a4) {
        // the tile's units may be spread over several warps: parts land in the workspace, the last writer sums
        const int ufirst = T * nkbl, ulast = ufirst + nkbl - 1;
        const int w0 = warp_of_unit(ufirst, base, rem), w1 = warp_of_unit(ulast, base, rem);
        float v[4] = {a4[0], a4[1], a4[2], a4[3]};
        bool mine = true;
        if (w0 != w1) {
            const int slot = (T == u0 / nkbl) ? 0 : 1;
            float* dst = p.part + ((size_t)gw * 2 + slot) * 128;
            reinterpret_cast<float4*>(dst)[lane] = make_float4(a4[0], a4[1], a4[2], a4[3]);
            __threadfence();
            __syncwarp();
            int tk = 0;
            if (lane == 0) tk = atomicAdd(p.ticket + T, 1);
            tk = __shfl_sync(0xffffffffu, tk, 0);
            mine = (tk == w1 - w0);
            if (mine) {
                __threadfence();
                v[0] = v[1] = v[2] = v[3] = 0.f;
                for (int ww = w0; ww <= w1; ++ww) {
                    const int wu0 = ww * base + min(ww, rem);
                    const int sl = (T == wu0 / nkbl) ? 0 : 1;
                    const float4 q = __ldcg(reinterpret_cast<const float4*>(p.part + ((size_t)ww * 2 + sl) * 128) + lane);
                    v[0] += q.x;
                    v[1] += q.y;
                    v[2] += q.z;
                    v[3] += q.w;
                }
                if (lane == 0) p.ticket[T] = 0;
            }
        }
        if (!mine) return;
        // epilogue from the fragment: v[0], v[1] = (row g, users 2t, 2t+1); v[2], v[3] = (row g + 8, same)
        const int r0 = T * 16 + g, r1 = r0 + 8;
        if (EPI == EPI_SILU_MUL) {
            // quads of rows are gate(j), gate(j+1), up(j), up(j+1): the up partner of row g is row g + 2 (lane + 8)
            float up[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) up[i] = __shfl_down_sync(0xffffffffu, v[i], 8);
            if ((g & 3) < 2) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int user = 2 * t + (i & 1);
                    const int quad = T * 4 + (g >> 2) + (i >= 2 ? 2 : 0);
                    const int col = 2 * quad + (g & 3);
                    if (user < users && 2 * col < p.rows)
                        reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)user * p.ld_out + col] =
                            __float2bfloat16_rn(silu_f(v[i]) * up[i]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int user = 2 * t + (i & 1);
                const int row = i >= 2 ? r1 : r0;
                if (user < users && row < p.rows) {
                    if (EPI == EPI_BF16) {
                        reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)user * p.ld_out + row] = __float2bfloat16_rn(v[i]);
                    } else if (EPI == EPI_RESID) {
                        float* o = reinterpret_cast<float*>(p.out) + (size_t)user * p.ld_out + row;
                        *o = v[i] + *o;
                    } else {
                        reinterpret_cast<float*>(p.out)[(size_t)user * p.ld_out + row] = v[i];
                    }
                }
            }
        }
    };

    // a split first tile is held back and flushed after the stream (its atomics never stall the ring)
    float first_acc[4] = {0.f, 0.f, 0.f, 0.f};
    int first_tile = -1;
    int tT = u0 / nkbl, tK = u0 % nkbl;  // (tile, block) of the next unit: a warp's units are consecutive
    // the unit scales of a stage are loaded one stage ahead (they never stall the stage's math)
    auto unit_scales = [&](int s2, float* out2) {
        const int a2 = u0 + s2 * kStageUnits;
#pragma unroll
        for (int i = 0; i < kStageUnits; ++i) {
            out2[i] = 0.f;
            if (s2 < nst && a2 + i < u0 + cnt) {
                const int uu = a2 + i, T2 = uu / nkbl, kb2 = p.kb0 + uu % nkbl;
                const float2 v = __ldg(p.uscale + (size_t)T2 * p.nkb + kb2);
                out2[i] = rows_b ? v.y : v.x;
            }
        }
    };
    float sc_cur[kStageUnits], sc_next[kStageUnits];
    unit_scales(0, sc_cur);
    for (int s = 0; s < nst; ++s) {
        unit_scales(s + 1, sc_next);
        const int slot = s % NS;
        if (ok) ok = mbar_wait(&bars[slot], (s / NS) & 1, p.err);
        const int a = u0 + s * kStageUnits, n = min(kStageUnits, u0 + cnt - a);
        // the stage's weights go to registers and its slot is refilled at once: every stage of the ring stays in
        // flight while this one is computed (the memory latency is covered by the whole ring, not all but one)
        uint4 wr[kStageUnits][2][2];
        if (ok) {
            const uint8_t* st = wring + (size_t)slot * kStageBytes;
#pragma unroll
            for (int i = 0; i < kStageUnits; ++i) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int sw = (half ^ (g & 1)) * 64 + 16 * t;  // rows g and g + 8 share the parity
                    if (i < n) {
                        wr[i][half][0] = lds128(st + i * kUnitBytes + g * 128 + sw);
                        wr[i][half][1] = lds128(st + i * kUnitBytes + (g + 8) * 128 + sw);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && ok && s + NS < nst) {
            fence_proxy_async();
            issue(s + NS);
        }
        if (ok) {
#pragma unroll
            for (int i = 0; i < kStageUnits; ++i) {
                if (i >= n) break;
                const int T = tT, kb = p.kb0 + tK;
                if (++tK == nkbl) {
                    tK = 0;
                    ++tT;
                }
                if (T != cur) {
                    if (cur >= 0) {
                        if (first_tile < 0 && cur == u0 / nkbl && split_tile(cur)) {
                            first_tile = cur;
                            first_acc[0] = acc[0];
                            first_acc[1] = acc[1];
                            first_acc[2] = acc[2];
                            first_acc[3] = acc[3];
                        } else {
                            flush(cur, acc);
                        }
                    }
                    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
                    cur = T;
                }
                const float sc = sc_cur[i];
                // 4 independent accumulators (one per word m): short dependency chains
                float d[4][4];
#pragma unroll
                for (int m = 0; m < 4; ++m) d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint4 wa = wr[i][half][0], wb = wr[i][half][1];
                    uint4 h0 = make_uint4(0, 0, 0, 0), h1 = make_uint4(0, 0, 0, 0);
                    if (hrow) {
                        const __half* hp = hg + (kb - p.kb0) * 128 + half * 64 + 16 * t;
                        h0 = lds128(hp);
                        h1 = lds128(hp + 8);
                    }
                    uint32_t a0, a1, a2, a3;
                    // words 0, 1: the conversion unit; words 2, 3: integer ops (values x 2^-8)
                    cvt_word_xu(wa.x, a0, a2);
                    cvt_word_xu(wb.x, a1, a3);
                    mma_f16(d[0], a0, a1, a2, a3, h0.x, h0.y);
                    cvt_word_xu(wa.y, a0, a2);
                    cvt_word_xu(wb.y, a1, a3);
                    mma_f16(d[1], a0, a1, a2, a3, h0.z, h0.w);
                    cvt_word_alu(wa.z, a0, a2);
                    cvt_word_alu(wb.z, a1, a3);
                    mma_f16(d[2], a0, a1, a2, a3, h1.x, h1.y);
                    cvt_word_alu(wa.w, a0, a2);
                    cvt_word_alu(wb.w, a1, a3);
                    mma_f16(d[3], a0, a1, a2, a3, h1.z, h1.w);
                }
#pragma unroll
                for (int i2 = 0; i2 < 4; ++i2) {
                    const float v = (d[0][i2] + d[1][i2]) + 256.f * (d[2][i2] + d[3][i2]);
                    acc[i2] = fmaf(v, sc, acc[i2]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kStageUnits; ++i) sc_cur[i] = sc_next[i];
    }
    if (!ok && lane == 0) {
        // never leave a copy in flight into shared memory that is about to be released
        for (int s = max(0, nst - NS); s < nst; ++s) mbar_wait(&bars[s % NS], (s / NS) & 1, nullptr);
    }
    // the stream is done: pull the start of this warp's range of the next projection into L2
    if (lane == 0 && p.next_w != nullptr && p.next_prefetch > 0) {
        const int nb = p.next_units / W, nr = p.next_units % W;
        const int nu0 = gw * nb + min(gw, nr), ncnt = nb + (gw < nr ? 1 : 0);
        const int pre = min(ncnt, p.next_prefetch);
        if (pre > 0) l2_prefetch_share(p.next_w + (size_t)nu0 * kUnitBytes, (size_t)pre * kUnitBytes, 0, 1);
    }
    if (ok) {
        if (cur >= 0) flush(cur, acc);
        if (first_tile >= 0) flush(first_tile, first_acc);
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

// smem budget of one GEMV CTA: two CTAs (the finishing kernel's and the next one's) share an SM under PDL
constexpr size_t kGemvSmemBudget = 112 * 1024;
constexpr size_t kGemvSmemMax = 220 * 1024;

static int bt_of(int users) { return users == 1 ? 1 : users == 2 ? 2 : users <= 4 ? 4 : 8; }

// K blocks one launch may cover at this row count (the f16 activations of the covered K sit in shared memory)
int gemv_max_kb(int users) {
    const int Bt = bt_of(users);
    for (int kb = 160; kb >= 1; --kb)
        if (gemv_smem_bytes(Bt, kb * 128, 2) <= kGemvSmemMax) return kb;
    return 1;
}

size_t gemv_workspace_bytes(int grid, int max_tiles) {
    return (size_t)grid * kGemvWarps * 2 * 128 * 4 + 256 + (size_t)max_tiles * 4;
}

cudaError_t gemv_launch(const qres_weight& w, int users, int pro, const void* in, int ld_in, int epi, void* out,
                        int ld_out, int grid, uint32_t* err, cudaStream_t st, bool pdl, const float* red, float* x_out,
                        void* work, size_t work_bytes, int kb0, int kb1, const qres_weight* next, int next_prefetch) {
    if (users < 1 || users > kMaxRows || w.K % 128 != 0 || w.rows_pad % 16 != 0) return cudaErrorInvalidValue;
    const int Bt = bt_of(users);
    const int nkb = w.K / 128;
    if (kb1 <= 0) kb1 = nkb;
    if (kb0 < 0 || kb0 >= kb1 || kb1 > nkb) return cudaErrorInvalidValue;
    if (kb0 != 0 && pro != PRO_BF16) return cudaErrorInvalidValue;  // rmsnorm needs the whole row
    const int tiles = w.rows_pad / 16;
    if (grid < 1) grid = 1;
    if (work == nullptr || work_bytes < gemv_workspace_bytes(grid, tiles)) return cudaErrorInvalidValue;
    GemvParams p;
    p.w = static_cast<const uint8_t*>(w.data);
    p.uscale = reinterpret_cast<const float2*>(w.uscale);
    p.rows = w.rows;
    p.tiles = tiles;
    p.K = (kb1 - kb0) * 128;  // the activations this launch reads
    p.nkb = nkb;
    p.kb0 = kb0;
    p.kb1 = kb1;
    p.users = users;
    p.x = pro != PRO_BF16 ? static_cast<const float*>(in) : nullptr;
    p.in = pro == PRO_BF16 ? static_cast<const uint16_t*>(in) + (size_t)kb0 * 128 : nullptr;
    p.ld_in = ld_in;
    p.red = red;
    p.x_out = x_out;
    if (pro == PRO_RMSNORM_ADD && (red == nullptr || x_out == nullptr)) return cudaErrorInvalidValue;
    p.out = out;
    p.ld_out = ld_out;
    p.err = err;
    p.next_w = next ? static_cast<const uint8_t*>(next->data) : nullptr;
    p.next_units = next ? (next->rows_pad / 16) * (next->K / 128) : 0;
    p.next_prefetch = next ? next_prefetch : 0;
    uint8_t* wk = static_cast<uint8_t*>(work);
    p.part = reinterpret_cast<float*>(wk);
    p.ticket = reinterpret_cast<int*>(wk + (size_t)grid * kGemvWarps * 2 * 128 * 4 + 256);
    // ring depth: as deep as the budget allows (two CTAs per SM), at least 2 stages per warp
    const size_t hb = gemv_h_bytes(Bt, p.K);
    int ns = hb + 512 < kGemvSmemBudget ? (int)((kGemvSmemBudget - 512 - hb) / ((size_t)kGemvWarps * kStageBytes)) : 0;
    if (ns < 2) ns = hb + 512 < kGemvSmemMax ? (int)((kGemvSmemMax - 512 - hb) / ((size_t)kGemvWarps * kStageBytes)) : 0;
    if (ns < 2) return cudaErrorInvalidValue;
    ns = ns > kMaxStages ? kMaxStages : ns;
    p.nstages = ns;
    const size_t smem = gemv_smem_bytes(Bt, p.K, ns);
    if (pro == PRO_RMSNORM && epi == EPI_BF16) return launch_pe<PRO_RMSNORM, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_SILU_MUL) return launch_pe<PRO_RMSNORM, EPI_SILU_MUL>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_ADD && epi == EPI_BF16) return launch_pe<PRO_RMSNORM_ADD, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_RMSNORM_ADD && epi == EPI_SILU_MUL) return launch_pe<PRO_RMSNORM_ADD, EPI_SILU_MUL>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_RESID) return launch_pe<PRO_BF16, EPI_RESID>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_F32) return launch_pe<PRO_BF16, EPI_F32>(p, Bt, grid, smem, st, pdl);
    if (pro == PRO_BF16 && epi == EPI_BF16) return launch_pe<PRO_BF16, EPI_BF16>(p, Bt, grid, smem, st, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace qres
