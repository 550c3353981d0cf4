/*
 * libqres -- the resident decode step of a Qwen3.6-27B-shaped hybrid model (48 Gated DeltaNet + 16 gated
 * full-attention layers) as hand-written sm_100a CUDA kernels behind a plain C ABI.
 *
 * It replaces the device side of sott0n/tt-qwen-resident's decode path: the per-chip resident program that
 * ``ResidentModel`` builds (qwen36_resident/model.py:403-1299) and launches with ``ttnn.generic_op`` /
 * ``ttnn.execute_trace`` (model.py:1485-1508), and the kernels under qwen36_resident/kernels/.
 *
 * Conventions: every function returns a qres_status (0 = ok) and never throws; on failure the context keeps a
 * message for qres_last_error. Device memory is allocated by the caller (e.g. torch) and passed as raw
 * pointers; the library never frees caller memory. Work is stream-ordered on the caller's stream (a
 * cudaStream_t passed as void*). One context per rank (process).
 */
#ifndef QRES_H_
#define QRES_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QRES_API __attribute__((visibility("default")))
#else
#define QRES_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    QRES_OK = 0,
    QRES_ERR_ARG = 1,    /* bad argument / shape / unbound buffer */
    QRES_ERR_CUDA = 2,   /* a CUDA runtime call failed */
    QRES_ERR_DEVICE = 3, /* a kernel reported an error word (bounded wait ran out, index out of range) */
    QRES_ERR_STATE = 4,  /* call out of order (e.g. replay without a captured graph) */
    QRES_ERR_COMM = 5    /* the tensor-parallel exchange failed */
} qres_status;

/* projection kinds (the weight entries of model.py:582-589) */
typedef enum {
    QRES_W_GDN_IN = 0,  /* [q|k|v|z|a|b] rows of the rank's GDN heads, K = 5120 */
    QRES_W_ATTN_IN = 1, /* [q|gate|k|v] rows of the rank's attention heads, K = 5120 */
    QRES_W_OUT = 2,     /* out-projection, 5120 rows, K = 6144 / nranks (row-parallel) */
    QRES_W_GATEUP = 3,  /* gate|up rows interleaved in pairs (g0 g1 u0 u1 ...), K = 5120 */
    QRES_W_DOWN = 4,    /* down-projection, 5120 rows, K = 17408 / nranks (row-parallel) */
    QRES_W_HEAD = 5,    /* lm_head rows of the rank's vocab slice, K = 5120 */
    QRES_W_FC = 6       /* MTP draft layer fc (mtp.py:54-60): 5120 rows, K = 10240 = [embedding | hidden] columns
                         * with the pre-fc norm weights (1 + w) folded in; layer ignored; one rank. A context
                         * with an fc forms layer 0's residual as fc([rmsnorm(e) | rmsnorm(h)]) (e = the token's
                         * embedding row, h = io.h_in), not from x0 / the embedding directly */
} qres_weight_kind;

#define QRES_MAX_ROWS 8    /* users (or verify rows) per step */
#define QRES_HIST_SLOTS 8  /* conv-history ring slots per user: position p lives in slot p % 8 */
#define QRES_KV_BLOCK 64   /* positions per KV page */
#define QRES_TOPK 32       /* candidates per list (sampling.hpp kTopK) */

/* model / launch configuration (the shape arguments of ResidentModel, model.py:404-420) */
typedef struct {
    int32_t layers;        /* decoder layers per step */
    int32_t attn_interval; /* layer l is full attention when interval > 0 && (l + 1) % interval == 0 */
    int32_t vocab;         /* lm_head rows over all ranks; 0 = no lm_head */
    int32_t rows;          /* users per step, 1..QRES_MAX_ROWS */
    int32_t max_pages;     /* page-table entries per user */
    int32_t num_pages;     /* pages in each attention layer's K (and V) pool */
    int32_t sm_count;      /* SMs to use; 0 = the device's (the weight-streaming kernels run 2 CTAs per SM) */
    int32_t flags;         /* QRES_FLAG_VERIFY | QRES_FLAG_TILE_FINISH, or 0 */
} qres_config;

/* qres_config.flags: the verify step (ResidentModel(verify=True), model.py:416-457): the `rows` rows (2..5) are
 * consecutive positions p .. p+rows-1 of ONE user, run as consecutive steps inside one step (row r sees rows
 * < r). Each GDN layer's state holds `rows` slots; row r leaves its state in slot (tok.slot + r) % rows, so
 * continuing after accepting row k uses position p + k + 1 and slot (tok.slot + k) % rows (no rollback). The
 * conv history and the KV cache are position-keyed and need nothing. */
#define QRES_FLAG_VERIFY 1
/* qres_config.flags: with an lm_head (one rank, or ranks with the peer window of qres_p2p_open
 * and native peer atomics), the in-, out-, gate|up and down-projections add each CTA's partial sums into 64-bit
 * fixed-point accumulators (2^-30 units) with one atomic add per row, and the consumer reads the sums: the next
 * prologue (the residual add, or silu(g) * u) or the mixer (rounding them to bf16). The row-parallel out- and
 * down-projections add counted words ((value << 8) + 1) into every rank's accumulator over NVLink, and the next
 * prologue reads a word once it holds every rank's contributions. Integer addition makes the result independent
 * of the order of the adds and identical on every rank. This flag turns that off: split 128-row tiles are
 * finished instead by the last of their CTAs (an atomic ticket, the parts added in CTA order) and ranks exchange
 * tagged words, as with more rows. On B200 at one rank and one row the accumulators measured 6.51 ms per step
 * against 7.39 ms with tile finishing. */
#define QRES_FLAG_TILE_FINISH 4

/* one FP8-e4m3 projection, block-scaled (one fp32 scale per 128 x 128 block of the canonical matrix), in the
 * GEMV layout made by qres_tile_weight: rows in tiles of 128 (zero-padded), a tile's K in 128-wide units of
 * 16 KB stored back to back, inside a unit the tensor core's 128-byte-swizzled K-major arrangement (byte (r, c)
 * at r * 128 + ((c / 16) ^ (r % 8)) * 16 + c % 16). uscale points at the scale table: per tile, 128
 * bytes of row selectors (row r's canonical 128-row block is the tile's slot sel[r], 0..7), then for each
 * 128-K block the 8 slots' fp32 scales -- (128 + (K / 128) * 32) bytes per tile. */
typedef struct {
    const void* data;      /* rows_pad * K bytes */
    const float* uscale;   /* the scale table, rows_pad / 128 tiles */
    int32_t rows;          /* real rows */
    int32_t rows_pad;      /* rows rounded up to a multiple of 128 (at most 524,288) */
    int32_t K;             /* multiple of 128 */
    int32_t reserved;
} qres_weight;

/* per-layer decode state (State, model.py:151-174), laid out for this rank */
typedef struct {
    float* gdn_state;     /* GDN layer: [rows][48/n][128][128] fp32, updated in place (verify: [rows slots]) */
    uint16_t* conv_hist;  /* GDN layer: [rows][QRES_HIST_SLOTS][conv_ch/n] bf16 */
    uint16_t* k_pool;     /* attention layer: [num_pages][kv_heads_local][64][256] bf16 */
    uint16_t* v_pool;     /* attention layer: same */
} qres_layer_state;

/* the token state of a step (model.py:1314-1351 / streamer_common.hpp:227-230), in device memory */
typedef struct {
    int32_t pos[QRES_MAX_ROWS];   /* position of each row */
    int32_t token[QRES_MAX_ROWS]; /* token id of each row (embedding gather); < 0: take the row of x0 */
    int32_t feed;                 /* 1: the step writes its greedy token and pos + 1 back here */
    int32_t step;                 /* incremented by every step (device side) */
    int32_t slot;                 /* verify: the GDN state slot row 0 starts from (model.py:79 TOK_SLOT) */
    int32_t reserved[13];
} qres_tok;

/* per-step inputs and outputs (device pointers) */
typedef struct {
    qres_tok* tok;
    const float* x0;        /* [rows][5120] fp32 (bf16 values), used where tok.token < 0 */
    const uint16_t* embed;  /* [vocab][5120] bf16, or NULL */
    const int32_t* page_table; /* [rows][max_pages] */
    float* x;               /* [rows][5120] residual stream; x after the last layer when the step ends */
    uint16_t* logits;       /* [rows][vocab / n] bf16 (lm_head) */
    uint32_t* topk;         /* [rows][2 * QRES_TOPK] this rank's list: keys, then vocab indices (lm_head) */
    int32_t* out;           /* [rows][4]: greedy token, position, 0, 0 (lm_head) */
    uint16_t* mixer_out;    /* [rows][6144 / n] bf16 copy of the last layer's mixer output, or NULL */
    const float* h_in;      /* with an fc (QRES_W_FC): [rows][5120] fp32, the hidden rows h, else NULL */
} qres_io;

typedef struct qres_ctx qres_ctx;

/* ---- context ---- */
/* Replaces ResidentModel.__init__'s program build (model.py:403-1299) for one rank of nranks. */
QRES_API qres_status qres_create(const qres_config* cfg, int32_t rank, int32_t nranks, qres_ctx** out);
QRES_API qres_status qres_destroy(qres_ctx* ctx);
/* The last error message of the context (or of the library when ctx is NULL). */
QRES_API qres_status qres_last_error(const qres_ctx* ctx, char* buf, size_t len);

/* ---- binding (the DRAM tensors ResidentModel places: weights model.py:574-605, state :623-760) ---- */
/* Projection `kind` of `layer` (QRES_W_HEAD: layer ignored). Binds pointers; nothing is copied. */
QRES_API qres_status qres_load_weights(qres_ctx* ctx, int32_t layer, int32_t kind, const qres_weight* w);
/* GDN layer parameters: conv taps [conv_ch/n][4] bf16 (tap 0 = oldest), dt_bias and neg_A [48/n] fp32,
 * gated-norm weight [128] fp32 (weights.py:162-189). */
QRES_API qres_status qres_load_gdn_params(qres_ctx* ctx, int32_t layer, const uint16_t* taps, const float* dt,
                                 const float* neg_a, const float* norm_w);
/* Attention layer parameters: q-norm weight already divided by sqrt(256), k-norm weight, [256] fp32 each
 * (model.py:237-238). */
QRES_API qres_status qres_load_attn_params(qres_ctx* ctx, int32_t layer, const float* wq, const float* wk);
/* Per-layer decode state buffers (State, model.py:151-174; load_state :1447-1470 writes their contents). */
QRES_API qres_status qres_bind_state(qres_ctx* ctx, int32_t layer, const qres_layer_state* st);
/* Write user `user`'s decode state of GDN layer `layer` into the bound buffers (ResidentModel.load_state,
 * model.py:1447-1470): `state` = this rank's heads' fp32 state [48/n][128][128]; `hist3` = the layer's conv inputs
 * at positions pos-3 .. pos-1 (oldest first), bf16 [3][conv_ch/n], stored into their history-ring slots (position
 * p in slot p % QRES_HIST_SLOTS); hist3 may be NULL. Device pointers, copied on `stream`. A verify context takes
 * `user` as the state slot. Layers that share a state buffer share what is written. */
QRES_API qres_status qres_load_gdn_state(qres_ctx* ctx, int32_t layer, int32_t user, const float* state,
                                         const uint16_t* hist3, int32_t pos, void* stream);
/* Read user `user`'s fp32 state [48/n][128][128] of GDN layer `layer` (the reference reads State back with its
 * ttnn.to_torch of the state tensors, model.py:1447-1470). */
QRES_API qres_status qres_dump_gdn_state(qres_ctx* ctx, int32_t layer, int32_t user, float* state, void* stream);
/* Write user `user`'s K and V rows of attention layer `layer` for positions 0 .. npos-1 (bf16 [kv_heads_local]
 * [npos][256] each, device pointers) into the pages its page table names (io.page_table; position p in page
 * page_table[user][p / 64], row p % 64). Other positions' rows are untouched. A page index outside the pool sets
 * the device error word (qres_check). */
QRES_API qres_status qres_load_kv(qres_ctx* ctx, int32_t layer, int32_t user, const uint16_t* k, const uint16_t* v,
                                  int32_t npos, void* stream);
/* Read positions 0 .. npos-1 of user `user`'s K and V rows of attention layer `layer` back, same layout. */
QRES_API qres_status qres_dump_kv(qres_ctx* ctx, int32_t layer, int32_t user, uint16_t* k, uint16_t* v, int32_t npos,
                                  void* stream);
/* Rope tables [max_pos][32] fp32 cos and sin of model.py:128-131 (fp64 angles rounded to fp32). */
QRES_API qres_status qres_bind_rope(qres_ctx* ctx, const float* cos_tab, const float* sin_tab, int32_t max_pos);
QRES_API qres_status qres_bind_io(qres_ctx* ctx, const qres_io* io);
/* The sampling parameters of the fed token (ResidentModel.set_sampling, model.py:1528-1551; the hub's draw,
 * sampling.hpp:113-143 over the final top-32 list): `words` = device [rows][4] uint32 -- 1 / temperature in Q16
 * (0 = greedy), top-k (<= 1 greedy, at most 32), top-p in Q16 (65536 = off), seed -- read by every step until
 * bound again; NULL (the default) = greedy. The step then writes out[row] = {drawn token, position + 1, greedy
 * argmax, 0} and, in feed mode, feeds the drawn token. The draw's random number hashes (seed, position). */
QRES_API qres_status qres_bind_sampling(qres_ctx* ctx, const uint32_t* words);
/* Scratch the step needs (activations, split-K partials, counters, the error word). */
QRES_API qres_status qres_workspace_size(const qres_ctx* ctx, size_t* bytes);
QRES_API qres_status qres_bind_workspace(qres_ctx* ctx, void* dev, size_t bytes);

/* ---- tensor parallelism ---- */
/* The row-parallel all-reduces after the out- and down-projections (mlp_hub.cpp:309-364) and the top-k
 * exchange after the lm_head (mlp_hub.cpp:366-411) run over NCCL for nranks > 1. Rank 0 makes an id
 * (128 bytes) with qres_nccl_unique_id, the caller broadcasts it, every rank calls qres_nccl_init. libpath: the
 * libnccl.so.2 to load (NULL: the one already loaded in the process, else the default search). */
QRES_API qres_status qres_nccl_unique_id(const char* libpath, void* id128);
QRES_API qres_status qres_nccl_init(qres_ctx* ctx, const char* libpath, const void* id128);

/* ---- fused tensor-parallel exchange over NVLink peer memory ----
 * Replaces the NCCL path above inside the step (mlp_hub.cpp:309-364 all-reduce, :366-411 list exchange): the
 * row-parallel out- / down-projection stores each finished 128-row tile of its fp32 partial straight into every
 * rank's window from its epilogue (peer stores) and advances a counter there; the next projection's rmsnorm
 * prologue waits for all ranks' counters (bounded; a timeout sets the device error word) and adds the partials in
 * rank order, so every rank holds the same residual bit for bit. The lm_head's top-32 lists travel the same way.
 * Bytes of this rank's window: */
QRES_API qres_status qres_p2p_window_size(const qres_ctx* ctx, size_t* bytes);
/* Allocate this rank's window (cudaMalloc, zeroed -- the one device allocation the library makes itself, since
 * CUDA IPC maps whole allocations; freed by qres_destroy) and write its CUDA IPC handle (64 bytes). */
QRES_API qres_status qres_p2p_alloc(qres_ctx* ctx, void* handle64);
/* Map every rank's window (nranks handles of 64 bytes in rank order, as all-gathered by the caller) and switch
 * the step to the peer exchange. Needs the workspace bound; resets the device step count the exchange counters
 * derive from, so every rank opens before any rank's first step (a barrier after the call). */
QRES_API qres_status qres_p2p_open(qres_ctx* ctx, const void* handles);

/* The exchange the step uses between ranks, as the context is configured now: QRES_XCHG_NONE (one rank),
 * QRES_XCHG_NCCL (qres_nccl_init), QRES_XCHG_TAGGED (peer window, tagged words), QRES_XCHG_COUNTED (peer window,
 * counted fixed-point words; needs native 64-bit peer atomics between every pair of ranks' GPUs, checked at
 * qres_p2p_open where the process sees those GPUs -- otherwise the tagged exchange runs). Negative: bad context. */
typedef enum { QRES_XCHG_NONE = 0, QRES_XCHG_NCCL = 1, QRES_XCHG_TAGGED = 2, QRES_XCHG_COUNTED = 3 } qres_exchange;
QRES_API int32_t qres_exchange_mode(const qres_ctx* ctx);

/* ---- the step (ResidentModel.step, model.py:1499-1508) ---- */
/* Enqueue one decode step on `stream`. */
QRES_API qres_status qres_decode_step(qres_ctx* ctx, void* stream);
/* capture_trace / step-with-trace / release_trace (model.py:1485-1505) as a CUDA graph of one step. */
QRES_API qres_status qres_capture(qres_ctx* ctx, void* stream);
QRES_API qres_status qres_replay(qres_ctx* ctx, void* stream);
QRES_API qres_status qres_release_graph(qres_ctx* ctx);
/* Synchronise `stream` and read the device error word; QRES_ERR_DEVICE (with a message) when a kernel of the
 * step reported a timeout or an out-of-range index. The word is cleared. */
QRES_API qres_status qres_check(qres_ctx* ctx, void* stream);
/* One bounded wait of the kind the peer exchange runs on a peer's counter (the next projection waiting for the
 * other ranks' partial sums, mlp_hub.cpp:309-364): poll the device word `flag` until it reaches `want`, at most
 * `polls` times (each with a short sleep); if it does not, set the context's error word (timeout and peer bits),
 * which the next qres_check reports as QRES_ERR_DEVICE. The kernel returns either way and the context stays
 * usable. It exercises the lost-peer path on one GPU with a word that nothing advances; it has no counterpart in
 * the reference, whose device waits have no limit. */
QRES_API qres_status qres_wait_probe(qres_ctx* ctx, const uint32_t* flag, uint32_t want, uint32_t polls, void* stream);
/* Kernel launches enqueued by the last qres_decode_step. */
QRES_API int32_t qres_step_launches(const qres_ctx* ctx);

/* ---- single kernels (the building blocks of a step, for tests and microbenchmarks) ---- */
/* y = act(h @ W^T) for `rows` users: pro 0 = h = bf16(rmsnorm(x)) from fp32 x [rows][K]; pro 1 = h = bf16
 * input [rows][K]. epi 0 = bf16 out [rows][w.rows]; 1 = SwiGLU over interleaved gate|up pairs, bf16 out
 * [rows][w.rows / 2]; 2 = fp32 out[r] += acc (residual); 3 = fp32 out = acc; 4 = the step's fixed-point
 * accumulation: out int64 [rows][w.rows] += round(acc * 2^30) with one atomic add per CTA and row (out zeroed by
 * the caller; value = out * 2^-30; with 4 or more rows the units are walked in K groups as in the step). grid: CTAs requested (0 = twice
 * the SM count; fewer are launched when the weight has fewer 128 x 128 units). work: qres_gemv_workspace_size
 * bytes for that grid (split-tile tickets and partials), zeroed once before first use (every launch leaves it
 * reusable). */
QRES_API qres_status qres_gemv_workspace_size(int32_t grid, int32_t rows_pad, size_t* bytes);
QRES_API qres_status qres_gemv(const qres_weight* w, int32_t rows, int32_t pro, const void* in, int32_t epi, void* out,
                      int32_t grid, uint32_t* err, void* work, size_t work_bytes, void* stream);
/* One GDN mixer (streamer conv1d+SiLU model.py:255-258 and gdn_head_compute.cpp) for `rows` users at the
 * positions in pos[] (device): y [rows][ld_y] in-projection rows -> o [rows][6144/n] bf16. */
QRES_API qres_status qres_gdn_mixer(int32_t nranks, int32_t rows, const uint16_t* y, int32_t ld_y, const int32_t* pos,
                           const uint16_t* taps, const float* dt, const float* neg_a, const float* norm_w,
                           float* state, uint16_t* conv_hist, uint16_t* o, uint32_t* err, void* stream);
/* One gated-attention mixer (model.py:233-247) over the paged KV cache: y [rows][ld_y] -> o [rows][6144/n]
 * bf16; appends each row's k / v at its position. work: qres_attn_workspace_size bytes, zeroed once before
 * first use (the kernel leaves it reusable). */
QRES_API qres_status qres_attn_workspace_size(int32_t nranks, int32_t rows, int32_t max_pos, size_t* bytes);
QRES_API qres_status qres_attn_mixer(int32_t nranks, int32_t rows, const uint16_t* y, int32_t ld_y, const int32_t* pos,
                            const int32_t* page_table, int32_t max_pages, const float* wq, const float* wk,
                            const float* cos_tab, const float* sin_tab, uint16_t* k_pool, uint16_t* v_pool,
                            uint16_t* o, void* work, size_t work_bytes, uint32_t* err, void* stream);
/* Per-row top-32 list (keys, then indices; sampling.hpp:24-74 order and tie rule) and argmax of bf16 logits
 * [rows][n_logits] whose first element is vocab index `base` (streamer_writer.cpp:451-500 + the hub's merge).
 * work: qres_topk_workspace_size bytes, zeroed once before first use (the kernel leaves it reusable). */
QRES_API qres_status qres_topk_workspace_size(int32_t rows, int32_t n_logits, size_t* bytes);
QRES_API qres_status qres_topk(int32_t rows, const uint16_t* logits, int32_t n_logits, int32_t base, uint32_t* lists,
                      int32_t* argmax, void* work, size_t work_bytes, void* stream);

/* The sampling draw alone (sampling.hpp:113-143): for each of `rows` rows, the token drawn from its top-32 list
 * (lists [rows][64]: keys descending then indices, as qres_topk writes them) with its parameter words
 * (words [rows][4], see qres_bind_sampling) at its position (pos [rows]) into token [rows]. Device pointers. */
QRES_API qres_status qres_sample(int32_t rows, const uint32_t* lists, const uint32_t* words, const int32_t* pos,
                                 int32_t* token, void* stream);

/* The same top-32 / argmax as qres_topk without a workspace argument: it allocates nothing. It has no
 * counterpart in the reference. It is for callers that cannot allocate device memory -- a host framework that
 * owns every device byte through its own pool and hands a plugin only its inputs and outputs. Its scratch (the
 * per-block candidate lists and per-row tickets) is a fixed 256 KiB device array inside the library, held by
 * every GPU that loads it until exit; requests larger than that (more than 8 rows of 260,096 logits) are
 * rejected with QRES_ERR_ARG. The first call on a device looks up the array's device address with
 * cudaGetSymbolAddress (make that first call before any stream capture). All calls share the array: calls that
 * overlap on the GPU (other streams, other threads) race and must be serialised by the caller. Each call clears
 * the tickets it needs before its kernel. */
QRES_API qres_status qres_topk_noalloc(int32_t rows, const uint16_t* logits, int32_t n_logits, int32_t base,
                                       uint32_t* lists, int32_t* argmax, void* stream);

/* ---- weight preparation ---- */
/* fp32 [N][K] -> e4m3 bytes [N][K] + scales [ceil(N/128)][K/128] (amax / 448 per 128 x 128 block). */
QRES_API qres_status qres_quantize_fp8(const float* w, int32_t N, int32_t K, uint8_t* q, float* scales, void* stream);
/* row-major e4m3 [rows][K] -> the GEMV layout of qres_weight (rows_pad = rows rounded up to 128, zero rows). */
QRES_API qres_status qres_tile_weight(const uint8_t* src, int32_t rows, int32_t K, uint8_t* dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QRES_H_ */
