// The persistent chain of projections between two mixers (gemv_chain.cu): its launch parameters.
#pragma once

#include "gemv_core.cuh"

namespace qres {

enum { CIN_BF16 = 0, CIN_TAGGED_BF16 = 1, CIN_NORM = 2 };
enum { COUT_BF16 = 0, COUT_SILU_TAGGED = 1, COUT_PARTIAL = 2 };
constexpr int kChainMaxPhases = 4;
constexpr int kChainTickets = 4096;  // per phase

struct ChainPhase {
    const uint8_t* w;
    const uint8_t* table;
    int rows, tiles, K, nkb;
    int in_kind, out_kind;
    // CIN_BF16: bf16 [users][K] written before the launch (griddepcontrol.wait orders it)
    const uint16_t* in_bf16;
    // CIN_TAGGED_BF16: tagged bf16 words [users][K] of an earlier phase, tag (*epoch * in_mul + in_add)
    const uint2* in_tagged;
    uint32_t in_mul, in_add;
    // CIN_NORM: h = bf16(rmsnorm(x + e_0 + e_1)), e_s = the sum in rank order of exchange s's tagged partials
    // [nsrc][users][K] in the slot (*epoch * set_mul + set_add[s] - 1) % 3 of set_base (slot stride slot_words),
    // tag (*epoch * set_mul + set_add[s]); CTA 0 writes x + e_0 + e_1 to x_out when set
    const float* x;
    int nsets;
    uint32_t set_add[2];
    float* x_out;
    // COUT_BF16: bf16 [users][ld_out]; COUT_SILU_TAGGED: tagged bf16 [users][ld_out] with tag
    // (*epoch * out_mul + out_add); COUT_PARTIAL: tagged fp32 words into this rank's region of every rank's
    // exchange slot (*epoch * set_mul + out_add - 1) % 3, tag (*epoch * set_mul + out_add)
    void* out;
    int ld_out;
    uint32_t out_mul, out_add;
};

struct ChainParams {
    int nphase;
    int users;
    int nsrc;                   // ranks (sources of an exchange)
    const uint32_t* epoch;      // steps completed (device)
    // exchange windows: rank r's base (its slot 0, source 0), slot stride and source stride in tagged words
    uint2* xbase[kMaxPeers];
    size_t slot_words, src_words;
    uint32_t set_mul;           // exchanges per step
    int rank;
    ChainPhase ph[kChainMaxPhases];
    float* part;                // [grid][2 phase parities][2][8][128]
    int* ticket;                // [kChainMaxPhases][kChainTickets]
    int nstages;
    int nkw;                    // activation window capacity (K blocks)
    uint32_t* err;
};

size_t chain_workspace_bytes(int grid);
cudaError_t chain_launch(ChainParams& p, int grid, int sm_count, void* work, size_t work_bytes, cudaStream_t st,
                         bool pdl);

}  // namespace qres
