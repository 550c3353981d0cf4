// Block-scaled FP8 weight-streaming projection (batch-1..8 GEMV) for sm_100a.
//
// Replaces the reference's streamer cores (qwen36_resident/kernels/streamer_reader.cpp:45-89 weight ring,
// streamer_compute.cpp:60-92 M=1..8 matmul, :100-210 rmsnorm, :212-249 silu(g)*u, :252-273 residual fold).
//
// Layout (qres_tile_weight): rows in quads of 4; a quad's K in chunks of 512 bytes; chunk c of quad q holds its
// 4 rows back to back at byte q*4K + c*2048 (the last chunk may be 128/256/384 wide). One fp32 scale per
// 128 x 128 block of the canonical matrix, reached through sidx[row].
//
// Work split: CTA i streams a contiguous, balanced range of quads. Its quads are taken 8 at a time (a
// "group"); stage (group, chunk) = the chunk of each of the group's quads, fetched with one cp.async.bulk per
// quad (no multicast) into a ring of 16 KB stages by a producer warp, and consumed by 8 consumer warps, warp j
// owning quad j of the group for all of its chunks (its accumulators stay in registers across chunks). The
// producer issues the first stages before griddepcontrol.wait, so under programmatic dependent launch the
// weight stream of this kernel starts while the previous kernel is still finishing.
//
// Per chunk a lane holds 16 consecutive K of one 128-block: it dots them with the 4 rows and folds the block
// scale in once (acc += scale * sum_16(h * q)), fp32 throughout; q is decoded exactly through e4m3x2->f16x2.
#include "qres_common.cuh"

namespace qres {

enum { PRO_RMSNORM = 0, PRO_BF16 = 1, PRO_RMSNORM_ADD = 2 };
enum { EPI_BF16 = 0, EPI_SILU_MUL = 1, EPI_RESID = 2, EPI_F32 = 3 };

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kChunk = 512;                       // K bytes per chunk
constexpr int kStageBytes = kGemvConsumerWarps * 4 * kChunk;  // 16 KB
constexpr int kMaxStages = 12;

struct GemvParams {
    const uint8_t* w;
    const float* scales;
    const int32_t* sidx;
    int rows, rows_pad, K, nkb;
    int users;              // real users (<= template B)
    const float* x;         // PRO_RMSNORM(_ADD): fp32 [users][K]
    const float* red;       // PRO_RMSNORM_ADD: all-reduced partials [users][K]; x_out = x + red
    float* x_out;           // PRO_RMSNORM_ADD: written by CTA 0
    const uint16_t* in;     // PRO_BF16: bf16 [users][K]
    void* out;              // EPI_BF16 / EPI_SILU_MUL: bf16 [users][ld_out]; EPI_RESID / EPI_F32: fp32
    int ld_out;
    int nstages;            // ring depth
    uint32_t* err;
};

__host__ __device__ inline size_t gemv_smem_bytes(int B, int K, int nstages) {
    size_t h = (size_t)B * K * 2;
    h = (h + 127) & ~size_t(127);
    return 256 /* barriers */ + h + (size_t)nstages * kStageBytes;
}

template <int B, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_fp8_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    uint16_t* hs = reinterpret_cast<uint16_t*>(smem + 256);
    size_t hbytes = ((size_t)B * p.K * 2 + 127) & ~size_t(127);
    uint8_t* ring = smem + 256 + hbytes;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.K;
    const int nc = (K + kChunk - 1) / kChunk;
    const int nq_all = p.rows_pad >> 2;
    const int G = gridDim.x;
    const int base = nq_all / G, rem = nq_all % G;
    const int cta = blockIdx.x;
    const int nq = base + (cta < rem ? 1 : 0);
    const int q0 = cta * base + min(cta, rem);
    const int ngroups = (nq + kGemvConsumerWarps - 1) / kGemvConsumerWarps;
    const int total = ngroups * nc;
    const int NS = p.nstages;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGemvConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch();

    if (warp == kGemvConsumerWarps) {
        // ---------------- producer: stream the CTA's quads stage by stage ----------------
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int s = 0; s < total && ok; ++s) {
                const int slot = s % NS;
                if (s >= NS) {
                    ok = mbar_wait(&empty[slot], ((s / NS) - 1) & 1, p.err);
                    if (!ok) break;
                }
                const int g = s / nc, c = s % nc;
                const int gq0 = q0 + g * kGemvConsumerWarps;
                const int gn = min(kGemvConsumerWarps, q0 + nq - gq0);
                const int wc = min(kChunk, K - c * kChunk);
                const uint32_t bytes = 4u * wc;
                mbar_arrive_expect_tx(&full[slot], bytes * gn);
                uint8_t* dst = ring + (size_t)slot * kStageBytes;
                for (int j = 0; j < gn; ++j) {
                    const uint8_t* src = p.w + (size_t)(gq0 + j) * 4 * K + (size_t)c * 4 * kChunk;
                    bulk_g2s(dst + j * 4 * kChunk, src, bytes, &full[slot]);
                }
                issued = s + 1;
            }
            if (!ok) {
                // never leave a copy in flight into shared memory that is about to be released
                for (int s = max(0, issued - NS); s < issued; ++s) mbar_wait(&full[s % NS], (s / NS) & 1, p.err);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();
    const int users = p.users;
    // prologue: h (bf16, [B][K]) in shared memory
    if (PRO == PRO_RMSNORM || PRO == PRO_RMSNORM_ADD) {
        __shared__ float red[kGemvConsumerWarps][B];
        float ss[B];
        // x (+ the all-reduced partials: x_out = x + red, the residual update of a row-parallel projection)
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
            ss[b] = 0.f;
            if (b < users) {
                for (int i = threadIdx.x; i < K / 4; i += kGemvConsumerWarps * 32) {
                    float4 v = xload(b, i);
                    if (PRO == PRO_RMSNORM_ADD && blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out + (size_t)b * K)[i] = v;
                    ss[b] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
            }
            ss[b] = warp_sum(ss[b]);
            if (lane == 0) red[warp][b] = ss[b];
        }
        bar_sync(1, kGemvConsumerWarps * 32);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvConsumerWarps; ++w) t += red[w][b];
            const float r = rsqrt_ieee(t / (float)K + kEps);
            if (b < users) {
                uint2* hv = reinterpret_cast<uint2*>(hs + (size_t)b * K);
                for (int i = threadIdx.x; i < K / 4; i += kGemvConsumerWarps * 32) {
                    float4 v = xload(b, i);
                    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x * r, v.y * r);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(v.z * r, v.w * r);
                    uint2 o;
                    o.x = *reinterpret_cast<uint32_t*>(&lo);
                    o.y = *reinterpret_cast<uint32_t*>(&hi);
                    hv[i] = o;
                }
            } else {
                uint2* hv = reinterpret_cast<uint2*>(hs + (size_t)b * K);
                for (int i = threadIdx.x; i < K / 4; i += kGemvConsumerWarps * 32) hv[i] = make_uint2(0, 0);
            }
        }
    } else {
#pragma unroll
        for (int b = 0; b < B; ++b) {
            uint4* hv = reinterpret_cast<uint4*>(hs + (size_t)b * K);
            const uint4* iv = reinterpret_cast<const uint4*>(p.in + (size_t)b * K);
            for (int i = threadIdx.x; i < K / 8; i += kGemvConsumerWarps * 32)
                hv[i] = b < users ? iv[i] : make_uint4(0, 0, 0, 0);
        }
    }
    bar_sync(1, kGemvConsumerWarps * 32);

    float acc[4][B];
    int sr[4];
    bool ok = true;
    for (int s = 0; s < total; ++s) {
        const int slot = s % NS;
        const int g = s / nc, c = s % nc;
        const int gq0 = q0 + g * kGemvConsumerWarps;
        const int gn = min(kGemvConsumerWarps, q0 + nq - gq0);
        const bool mine = warp < gn;
        if (c == 0) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
#pragma unroll
                for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
                sr[r] = mine ? __ldg(p.sidx + (gq0 + warp) * 4 + r) : 0;
            }
        }
        if (ok) ok = mbar_wait(&full[slot], (s / NS) & 1, p.err);
        const int wc = min(kChunk, K - c * kChunk);
        if (ok && mine && lane * 16 < wc) {
            const uint8_t* st = ring + (size_t)slot * kStageBytes + warp * 4 * kChunk + lane * 16;
            const int k0 = c * kChunk + lane * 16;
            const int kb = k0 >> 7;
            float sc[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) sc[r] = __ldg(p.scales + (size_t)sr[r] * p.nkb + kb);
            uint4 wv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) wv[r] = lds128(st + r * wc);
            float wf[4][16];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                fp8x4_to_f32(wv[r].x, &wf[r][0]);
                fp8x4_to_f32(wv[r].y, &wf[r][4]);
                fp8x4_to_f32(wv[r].z, &wf[r][8]);
                fp8x4_to_f32(wv[r].w, &wf[r][12]);
            }
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const uint4 h0 = lds128(hs + (size_t)b * K + k0);
                const uint4 h1 = lds128(hs + (size_t)b * K + k0 + 8);
                const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                float hf[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    hf[2 * i] = bf16lo(hw[i]);
                    hf[2 * i + 1] = bf16hi(hw[i]);
                }
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    float d0 = 0.f, d1 = 0.f;
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        d0 = fmaf(hf[i], wf[r][i], d0);
                        d1 = fmaf(hf[i + 1], wf[r][i + 1], d1);
                    }
                    acc[r][b] = fmaf(d0 + d1, sc[r], acc[r][b]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (c == nc - 1 && mine) {
            // reduce the quad's 4 x B sums over the lanes, then write the epilogue
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);
            const int row0 = (gq0 + warp) * 4;
            if (EPI == EPI_SILU_MUL) {
                // quad rows = gate(j), gate(j+1), up(j), up(j+1) of output pair j = 2 * quad
                if (lane < 2 * B) {
                    const int b = lane >> 1, i = lane & 1;
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int bb = 0; bb < B; ++bb)
                        if (bb == b) {
                            gv = i ? acc[1][bb] : acc[0][bb];
                            uv = i ? acc[3][bb] : acc[2][bb];
                        }
                    const int col = (row0 >> 1) + i;
                    if (b < users && 2 * col < p.rows) {
                        const float a = silu_f(gv) * uv;
                        reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)b * p.ld_out + col] = __float2bfloat16_rn(a);
                    }
                }
            } else {
                if (lane < 4 * B) {
                    const int r = lane & 3, b = lane >> 2;
                    float v = 0.f;
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
                        for (int bb = 0; bb < B; ++bb)
                            if (rr == r && bb == b) v = acc[rr][bb];
                    const int row = row0 + r;
                    if (b < users && row < p.rows) {
                        if (EPI == EPI_BF16) {
                            reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)b * p.ld_out + row] = __float2bfloat16_rn(v);
                        } else if (EPI == EPI_RESID) {
                            float* o = reinterpret_cast<float*>(p.out) + (size_t)b * p.ld_out + row;
                            *o = v + *o;
                        } else {
                            reinterpret_cast<float*>(p.out)[(size_t)b * p.ld_out + row] = v;
                        }
                    }
                }
            }
        }
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
constexpr size_t kGemvSmemBudget = 110 * 1024;

cudaError_t gemv_launch(const qres_weight& w, int users, int pro, const void* in, int epi, void* out, int ld_out,
                        int grid, uint32_t* err, cudaStream_t st, bool pdl, const float* red, float* x_out) {
    if (users < 1 || users > kMaxRows || w.K % 128 != 0 || w.rows_pad % 4 != 0) return cudaErrorInvalidValue;
    const int Bt = users == 1 ? 1 : users == 2 ? 2 : users <= 4 ? 4 : 8;
    GemvParams p;
    p.w = static_cast<const uint8_t*>(w.data);
    p.scales = w.scales;
    p.sidx = w.sidx;
    p.rows = w.rows;
    p.rows_pad = w.rows_pad;
    p.K = w.K;
    p.nkb = w.K / 128;
    p.users = users;
    p.x = pro != PRO_BF16 ? static_cast<const float*>(in) : nullptr;
    p.red = red;
    p.x_out = x_out;
    if (pro == PRO_RMSNORM_ADD && (red == nullptr || x_out == nullptr)) return cudaErrorInvalidValue;
    p.in = pro == PRO_BF16 ? static_cast<const uint16_t*>(in) : nullptr;
    p.out = out;
    p.ld_out = ld_out;
    p.err = err;
    size_t hb = ((size_t)Bt * w.K * 2 + 127) & ~size_t(127);
    int ns = (int)((kGemvSmemBudget - 256 - hb) / kStageBytes);
    if (ns < 2) {
        // large B * K: one CTA per SM, more shared memory
        ns = (int)((200 * 1024 - 256 - hb) / kStageBytes);
    }
    if (ns < 2) return cudaErrorInvalidValue;
    ns = ns > kMaxStages ? kMaxStages : ns;
    p.nstages = ns;
    size_t smem = gemv_smem_bytes(Bt, w.K, ns);
    const int nq = w.rows_pad / 4;
    if (grid > nq) grid = nq;
    if (grid < 1) grid = 1;
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
