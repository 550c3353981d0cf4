// libqres C ABI: context, buffer binding, the decode step as a sequence of programmatic-dependent launches,
// its CUDA-graph capture, NCCL for tensor parallelism, and the single-kernel entry points.
//
// The step (ResidentModel.step, qwen36_resident/model.py:1499-1508, one launch of the per-chip program) is,
// per rank:
//   rows in (x0 or embed[token])
//   per layer: in-proj GEMV (rmsnorm prologue)  -> GDN or attention mixer -> out-proj GEMV (+ residual)
//              gate|up GEMV (rmsnorm prologue, SwiGLU epilogue) -> down GEMV (+ residual)
//   lm_head GEMV -> top-32 / argmax (-> cross-rank merge) -> next-token feed
// With nranks > 1 the out / down GEMVs write fp32 partials, NCCL all-reduces them, and the next GEMV's
// prologue adds them to the residual (x_out = x + sum of partials), alternating two residual buffers.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gemv_core.cuh"

namespace qres {
cudaError_t gemv_launch(const qres_weight& w, int users, int pro, const void* in, int ld_in, int epi, void* out,
                        int ld_out, int grid, uint32_t* err, cudaStream_t st, bool pdl, const float* red, float* x_out,
                        void* work, size_t work_bytes, const L2Heads* next, const GemvExchange* ex = nullptr);
size_t gemv_workspace_bytes(int grid);
int gemv_grid(int users, int rows_pad, int K, int grid);
int gemv_group_blocks(int users, int epi, int K);
cudaError_t silu_rows_launch(int users, const long long* acc, int ld_acc, int ic, uint16_t* h, cudaStream_t st, bool pdl);
cudaError_t resid_norm_launch(int users, const float* x, const long long* racc, float* x_out, uint16_t* h,
                              cudaStream_t st, bool pdl, const GemvExchange* ex, uint32_t* err);
cudaError_t gdn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const uint16_t* taps,
                       const float* dt, const float* neg_a, const float* norm_w, float* state, uint16_t* hist,
                       uint16_t* o, uint16_t* mixer_copy, uint32_t* err, cudaStream_t st, bool pdl,
                       const void* pf, size_t pf_bytes, int verify = 0, const int32_t* slot0 = nullptr,
                       const long long* yacc = nullptr);
size_t attn_workspace_bytes(int nranks, int rows, int nchunks);
int attn_default_chunks(int nranks, int rows, int sm_count, int max_pages);
cudaError_t attn_launch(int nranks, int rows, const uint16_t* y, int ld_y, const int32_t* pos, const int32_t* page_table,
                        int max_pages, int num_pages, const float* wq, const float* wk, const float* cos_tab,
                        const float* sin_tab, int max_pos, uint16_t* kp, uint16_t* vp, uint16_t* o, uint16_t* mixer_copy,
                        void* work, size_t work_bytes, int nchunks, uint32_t* err, cudaStream_t st, bool pdl,
                        const void* pf, size_t pf_bytes, int verify = 0, const long long* yacc = nullptr);
cudaError_t tile_weight_launch(const uint8_t* src, int rows, int K, uint8_t* dst, cudaStream_t st);
cudaError_t quantize_fp8_launch(const float* w, int N, int K, uint8_t* q, float* scales, cudaStream_t st);
int topk_default_blocks(int n);
size_t topk_workspace_bytes(int rows, int nblk);
cudaError_t topk_launch(int rows, const uint16_t* logits, int n, int ld, int base, uint32_t* lists, int32_t* argmax,
                        void* work, int nblk, cudaStream_t st, bool pdl);
cudaError_t merge_lists_launch(const uint32_t* lists, int nlists, int rows, uint32_t* out, int32_t* argmax,
                               cudaStream_t st, bool pdl, const uint32_t* wait_cnt = nullptr,
                               const uint32_t* epoch = nullptr, uint32_t* err = nullptr);
cudaError_t publish_lists_launch(const uint32_t* list, int words, const P2PDest& dst, const uint32_t* epoch,
                                 cudaStream_t st, bool pdl);
cudaError_t topk_static_scratch(void** out, size_t* bytes);
size_t topk_ticket_offset(int rows, int nblk);
cudaError_t embed_rows_launch(const qres_tok* tok, const float* x0, const uint16_t* embed, int vocab, float* x, int rows,
                              uint32_t* err, cudaStream_t st, bool pdl);
cudaError_t feed_launch(qres_tok* tok, const int32_t* argmax, int32_t* out, int rows, cudaStream_t st, bool pdl,
                        uint32_t* epoch, const uint32_t* lists, const uint32_t* words);
cudaError_t sample_launch(int rows, const uint32_t* lists, const uint32_t* words, const int32_t* pos, int32_t* token,
                          cudaStream_t st);
cudaError_t kv_rows_launch(uint16_t* kp, uint16_t* vp, uint16_t* k, uint16_t* v, const int32_t* page_table, int npos,
                           int nkv, int num_pages, bool to_pages, uint32_t* err, cudaStream_t st);
cudaError_t wait_probe_launch(const uint32_t* flag, uint32_t want, uint32_t limit, uint32_t* err, cudaStream_t st);
}  // namespace qres

using namespace qres;

namespace {

std::mutex g_err_mu;
std::string g_err;  // errors without a context

// NCCL entry points, resolved at run time from the libnccl.so.2 the process uses
struct Nccl {
    void* h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char* (*errStr)(ncclResult_t) = nullptr;
};
Nccl g_nccl;
std::mutex g_nccl_mu;

bool load_nccl(const char* libpath, std::string* why) {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.h) return true;
    void* h = nullptr;
    if (libpath && *libpath) h = dlopen(libpath, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        *why = std::string("cannot load libnccl.so.2: ") + dlerror();
        return false;
    }
    g_nccl.h = h;
    g_nccl.getUniqueId = (decltype(g_nccl.getUniqueId))dlsym(h, "ncclGetUniqueId");
    g_nccl.commInitRank = (decltype(g_nccl.commInitRank))dlsym(h, "ncclCommInitRank");
    g_nccl.allReduce = (decltype(g_nccl.allReduce))dlsym(h, "ncclAllReduce");
    g_nccl.allGather = (decltype(g_nccl.allGather))dlsym(h, "ncclAllGather");
    g_nccl.commDestroy = (decltype(g_nccl.commDestroy))dlsym(h, "ncclCommDestroy");
    g_nccl.errStr = (decltype(g_nccl.errStr))dlsym(h, "ncclGetErrorString");
    if (!g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allReduce || !g_nccl.allGather || !g_nccl.commDestroy) {
        *why = "libnccl.so.2 lacks an entry point";
        g_nccl.h = nullptr;
        return false;
    }
    return true;
}

// A rank's peer-exchange window (qres_p2p_*): one cudaMalloc allocation, mapped into every other rank with
// CUDA IPC. Layout: list counters [2 slots][8 source ranks] (uint32, 256-byte header), then the row-parallel
// partials [3 slots][8 sources][rows][5120] as tagged words {fp32 bits, tag}, then the top-32 lists
// [2 slots][8 sources][rows][64] uint32. Row-parallel exchange j of step s uses slot j % 2 and tag
// s * 2L + j + 1 (L layers; never 0, so the zeroed window holds no valid word); step s's lists use slot s % 2 and
// their counters only grow (the k-th use of a slot completes at k).
struct P2PLayout {
    size_t lcnt = 0, data = 256, lists = 0, xa = 0, xc = 0, total = 0;
    explicit P2PLayout(int rows) {
        lists = data + (size_t)3 * 8 * rows * kHidden * 8;
        // the counted accumulators of the out- and down-projection exchanges (every rank adds into them)
        xa = lists + (size_t)2 * 8 * rows * 2 * QRES_TOPK * 4;
        xc = xa + (size_t)rows * kHidden * 8;
        total = xc + (size_t)rows * kHidden * 8;
    }
};

struct Layer {
    qres_weight w[5] = {};
    bool has[5] = {false, false, false, false, false};
    const uint16_t* taps = nullptr;
    const float *dt = nullptr, *neg_a = nullptr, *norm_w = nullptr;
    const float *wq = nullptr, *wk = nullptr;
    qres_layer_state st = {};
    bool has_st = false;
};

}  // namespace

struct qres_ctx {
    qres_config cfg;
    int rank = 0, nranks = 1, device = 0, sm_count = 148;
    // per-rank dims
    int nk = 16, nv = 48, h = 24, nkv = 4, ic = 17408, vocab_local = 0, ld_y = 0, gv = 6144;
    std::vector<Layer> layers;
    qres_weight head = {};
    bool has_head = false;
    qres_weight fc = {};  // the MTP draft layer's fc (QRES_W_FC)
    bool has_fc = false;
    const float *cos_tab = nullptr, *sin_tab = nullptr;
    const uint32_t* sampling = nullptr;  // [rows][4] words of the fed token's draw (qres_bind_sampling), or greedy
    int max_pos = 0;
    qres_io io = {};
    bool has_io = false;
    // workspace carve
    uint8_t* ws = nullptr;
    size_t ws_bytes = 0;
    uint32_t* err = nullptr;
    float *xb = nullptr, *xe = nullptr, *partial = nullptr;
    uint16_t *y = nullptr, *o = nullptr, *a = nullptr;
    uint16_t* hbuf = nullptr;  // [rows][5120] bf16: a projection's rmsnorm input formed once (resid_norm)
    int32_t* argmax = nullptr;
    uint32_t* gathered = nullptr;
    void* attn_work = nullptr;
    size_t attn_work_bytes = 0;
    int attn_chunks = 1;
    void* topk_work = nullptr;
    int topk_blk = 1;
    void* gemv_work = nullptr;
    size_t gemv_work_bytes = 0;
    // one rank: the out-projection's, gate|up's and the down-projection's fixed-point sums (EPI_ACC), and the
    // in-projection's (read by the mixers), which follows the out-projection's in memory
    long long* acc[4] = {};
    ncclComm_t comm = nullptr;
    // peer exchange (qres_p2p_alloc / qres_p2p_open): this rank's window and every rank's window as mapped here
    uint8_t* p2p_local = nullptr;
    uint8_t* p2p_peer[8] = {};
    bool p2p_on = false;
    bool p2p_atomics = false;  // 64-bit atomic adds to the peers' windows (native over NVLink)
    uint32_t* epoch = nullptr;  // steps completed (workspace), advanced by the feed kernel
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    std::string last_error;
};

namespace {

qres_status fail(qres_ctx* c, qres_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) {
        c->last_error = buf;
    } else {
        std::lock_guard<std::mutex> lk(g_err_mu);
        g_err = buf;
    }
    return s;
}

#define CU(ctx, call)                                                                                      \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess) return fail(ctx, QRES_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                            \
    } while (0)

bool is_attn(const qres_ctx* c, int l) {
    return c->cfg.attn_interval > 0 && (l + 1) % c->cfg.attn_interval == 0;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// workspace layout: offsets of each scratch region
struct Carve {
    size_t err, epoch, xb, xe, partial, y, o, a, hbuf, argmax, gathered, attn, topk, gemv, gemv_bytes, acc[4], total;
};

Carve carve(const qres_ctx* c) {
    Carve k;
    const int R = c->cfg.rows;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    k.err = take(256);
    k.epoch = take(256);
    k.xb = take((size_t)R * kHidden * 4);
    k.xe = take((size_t)R * kHidden * 4);
    k.partial = take((size_t)R * kHidden * 4);
    k.y = take((size_t)R * c->ld_y * 2);
    k.o = take((size_t)R * c->gv * 2);
    k.a = take((size_t)R * c->ic * 2);
    k.hbuf = take((size_t)R * kHidden * 2);
    k.argmax = take((size_t)R * 4);
    k.gathered = take((size_t)c->nranks * R * 2 * QRES_TOPK * 4);
    k.attn = take(attn_workspace_bytes(c->nranks, R, c->attn_chunks));
    k.topk = take(c->vocab_local ? topk_workspace_bytes(R, c->topk_blk) : 0);
    k.gemv_bytes = gemv_workspace_bytes(2 * c->sm_count);
    k.gemv = take(k.gemv_bytes);
    // fixed-point accumulators of the one-rank step (int64): out-projection [rows][5120] and right behind it the
    // in-projection [rows][ld_y] (one range for the launch that zeroes both), gate|up [rows][2 x 17408],
    // down-projection [rows][5120]
    k.acc[0] = take((size_t)R * kHidden * 8 + (size_t)R * c->ld_y * 8);
    k.acc[3] = k.acc[0] + (size_t)R * kHidden * 8;
    k.acc[1] = take((size_t)R * 2 * c->ic * 8);
    k.acc[2] = take((size_t)R * kHidden * 8);
    k.total = off;
    return k;
}

qres_status check_weight(qres_ctx* c, const qres_weight* w, int rows, int K, const char* what) {
    if (!w || !w->data || !w->uscale) return fail(c, QRES_ERR_ARG, "%s: null pointer", what);
    if (w->rows != rows || w->K != K || w->rows_pad != ((rows + 127) & ~127))
        return fail(c, QRES_ERR_ARG, "%s: shape rows=%d K=%d rows_pad=%d (want rows=%d K=%d)", what, w->rows, w->K,
                    w->rows_pad, rows, K);
    return QRES_OK;
}

}  // namespace

// =============================================================================================== C ABI
extern "C" {

qres_status qres_last_error(const qres_ctx* ctx, char* buf, size_t len) {
    if (!buf || !len) return QRES_ERR_ARG;
    std::string s;
    if (ctx) {
        s = ctx->last_error;
    } else {
        std::lock_guard<std::mutex> lk(g_err_mu);
        s = g_err;
    }
    snprintf(buf, len, "%s", s.c_str());
    return QRES_OK;
}

qres_status qres_create(const qres_config* cfg, int32_t rank, int32_t nranks, qres_ctx** out) {
    if (!cfg || !out) return fail(nullptr, QRES_ERR_ARG, "qres_create: null argument");
    if (!(nranks == 1 || nranks == 2 || nranks == 4 || nranks == 8) || rank < 0 || rank >= nranks)
        return fail(nullptr, QRES_ERR_ARG, "qres_create: rank %d of %d (nranks must be 1, 2, 4 or 8)", rank, nranks);
    if (cfg->rows < 1 || cfg->rows > QRES_MAX_ROWS || cfg->layers < 1)
        return fail(nullptr, QRES_ERR_ARG, "qres_create: rows %d, layers %d", cfg->rows, cfg->layers);
    if (cfg->vocab % nranks) return fail(nullptr, QRES_ERR_ARG, "qres_create: vocab %d not divisible by %d", cfg->vocab, nranks);
    if (cfg->flags & ~(QRES_FLAG_VERIFY | QRES_FLAG_TILE_FINISH))
        return fail(nullptr, QRES_ERR_ARG, "qres_create: unknown flags %#x", cfg->flags);
    if ((cfg->flags & QRES_FLAG_VERIFY) && (cfg->rows < 2 || cfg->rows + 3 > QRES_HIST_SLOTS))
        return fail(nullptr, QRES_ERR_ARG, "qres_create: a verify step has 2..%d rows, not %d", QRES_HIST_SLOTS - 3,
                    cfg->rows);
    qres_ctx* c = new qres_ctx();
    c->cfg = *cfg;
    c->rank = rank;
    c->nranks = nranks;
    cudaGetDevice(&c->device);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device);
    c->sm_count = cfg->sm_count > 0 ? cfg->sm_count : sms;
    c->nk = 16 / nranks;
    c->nv = 48 / nranks;
    c->h = 24 / nranks;
    c->nkv = nranks <= 4 ? 4 / nranks : 1;
    c->ic = 17408 / nranks;
    c->gv = 6144 / nranks;
    c->vocab_local = cfg->vocab / nranks;
    const int n_gdn = 2 * c->nk * kDK + 2 * c->nv * kDV + 2 * c->nv;
    const int n_attn = 2 * c->h * kHD + 2 * c->nkv * kHD;
    c->ld_y = ((n_gdn > n_attn ? n_gdn : n_attn) + 7) & ~7;
    c->layers.resize(cfg->layers);
    c->attn_chunks = attn_default_chunks(nranks, cfg->rows, c->sm_count, cfg->max_pages > 0 ? cfg->max_pages : 1);
    c->topk_blk = c->vocab_local ? topk_default_blocks(c->vocab_local) : 1;
    *out = c;
    return QRES_OK;
}

qres_status qres_destroy(qres_ctx* ctx) {
    if (!ctx) return QRES_OK;
    if (ctx->exec) cudaGraphExecDestroy(ctx->exec);
    if (ctx->graph) cudaGraphDestroy(ctx->graph);
    if (ctx->comm && g_nccl.commDestroy) g_nccl.commDestroy(ctx->comm);
    for (int r = 0; r < ctx->nranks; ++r)
        if (ctx->p2p_peer[r] && ctx->p2p_peer[r] != ctx->p2p_local) cudaIpcCloseMemHandle(ctx->p2p_peer[r]);
    if (ctx->p2p_local) cudaFree(ctx->p2p_local);
    delete ctx;
    return QRES_OK;
}

qres_status qres_load_weights(qres_ctx* c, int32_t layer, int32_t kind, const qres_weight* w) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    if (kind == QRES_W_FC) {
        // the MTP draft layer's fc (K = the embedding row | the hidden row); one rank only
        if (c->nranks != 1) return fail(c, QRES_ERR_ARG, "the fc (MTP draft layer) runs on one rank");
        qres_status s = check_weight(c, w, kHidden, 2 * kHidden, "fc");
        if (s) return s;
        c->fc = *w;
        c->has_fc = true;
        return QRES_OK;
    }
    if (kind == QRES_W_HEAD) {
        if (!c->vocab_local) return fail(c, QRES_ERR_ARG, "lm_head bound but vocab is 0");
        qres_status s = check_weight(c, w, c->vocab_local, kHidden, "lm_head");
        if (s) return s;
        c->head = *w;
        c->has_head = true;
        return QRES_OK;
    }
    if (layer < 0 || layer >= c->cfg.layers || kind < 0 || kind > QRES_W_DOWN)
        return fail(c, QRES_ERR_ARG, "qres_load_weights: layer %d kind %d", layer, kind);
    int rows = 0, K = kHidden;
    switch (kind) {
        case QRES_W_GDN_IN: rows = 2 * c->nk * kDK + 2 * c->nv * kDV + 2 * c->nv; break;
        case QRES_W_ATTN_IN: rows = 2 * c->h * kHD + 2 * c->nkv * kHD; break;
        case QRES_W_OUT: rows = kHidden; K = c->gv; break;
        case QRES_W_GATEUP: rows = 2 * c->ic; break;
        case QRES_W_DOWN: rows = kHidden; K = c->ic; break;
    }
    if (kind == QRES_W_GDN_IN && is_attn(c, layer)) return fail(c, QRES_ERR_ARG, "layer %d is attention", layer);
    if (kind == QRES_W_ATTN_IN && !is_attn(c, layer)) return fail(c, QRES_ERR_ARG, "layer %d is GDN", layer);
    qres_status s = check_weight(c, w, rows, K, "projection");
    if (s) return s;
    c->layers[layer].w[kind] = *w;
    c->layers[layer].has[kind] = true;
    return QRES_OK;
}

qres_status qres_load_gdn_params(qres_ctx* c, int32_t layer, const uint16_t* taps, const float* dt, const float* neg_a,
                                 const float* norm_w) {
    if (!c || layer < 0 || layer >= c->cfg.layers || !taps || !dt || !neg_a || !norm_w)
        return fail(c, QRES_ERR_ARG, "qres_load_gdn_params: bad argument");
    Layer& L = c->layers[layer];
    L.taps = taps;
    L.dt = dt;
    L.neg_a = neg_a;
    L.norm_w = norm_w;
    return QRES_OK;
}

qres_status qres_load_attn_params(qres_ctx* c, int32_t layer, const float* wq, const float* wk) {
    if (!c || layer < 0 || layer >= c->cfg.layers || !wq || !wk)
        return fail(c, QRES_ERR_ARG, "qres_load_attn_params: bad argument");
    c->layers[layer].wq = wq;
    c->layers[layer].wk = wk;
    return QRES_OK;
}

qres_status qres_bind_state(qres_ctx* c, int32_t layer, const qres_layer_state* st) {
    if (!c || !st || layer < 0 || layer >= c->cfg.layers) return fail(c, QRES_ERR_ARG, "qres_bind_state: bad argument");
    if (is_attn(c, layer) ? (!st->k_pool || !st->v_pool) : (!st->gdn_state || !st->conv_hist))
        return fail(c, QRES_ERR_ARG, "qres_bind_state: layer %d lacks its buffers", layer);
    c->layers[layer].st = *st;
    c->layers[layer].has_st = true;
    return QRES_OK;
}

// ---- decode state in and out (State / load_state, model.py:151-174, 1447-1470) ----

static qres_status gdn_layer_state(qres_ctx* c, int32_t layer, int32_t user, const char* what, float** st,
                                   size_t* bytes) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "%s: null context", what);
    if (layer < 0 || layer >= c->cfg.layers || is_attn(c, layer) || !c->layers[layer].has_st)
        return fail(c, QRES_ERR_ARG, "%s: layer %d is not a bound GDN layer", what, layer);
    if (user < 0 || user >= c->cfg.rows) return fail(c, QRES_ERR_ARG, "%s: user %d of %d", what, user, c->cfg.rows);
    *bytes = (size_t)c->nv * kDK * kDV * 4;
    *st = c->layers[layer].st.gdn_state + (size_t)user * c->nv * kDK * kDV;
    return QRES_OK;
}

qres_status qres_load_gdn_state(qres_ctx* c, int32_t layer, int32_t user, const float* state, const uint16_t* hist3,
                                int32_t pos, void* stream) {
    float* dst = nullptr;
    size_t bytes = 0;
    qres_status s = gdn_layer_state(c, layer, user, "qres_load_gdn_state", &dst, &bytes);
    if (s) return s;
    if (!state || pos < 0) return fail(c, QRES_ERR_ARG, "qres_load_gdn_state: state null or pos %d", pos);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CU(c, cudaMemcpyAsync(dst, state, bytes, cudaMemcpyDeviceToDevice, st));
    if (hist3) {
        // the history ring of this user (a verify context's single user); position q in slot q % QRES_HIST_SLOTS
        const int conv = 2 * c->nk * kDK + c->nv * kDV;
        const int hu = (c->cfg.flags & QRES_FLAG_VERIFY) ? 0 : user;
        uint16_t* ring = c->layers[layer].st.conv_hist + (size_t)hu * QRES_HIST_SLOTS * conv;
        for (int age = 0; age < 3; ++age) {
            const int slot = ((pos - 3 + age) % QRES_HIST_SLOTS + QRES_HIST_SLOTS) % QRES_HIST_SLOTS;
            CU(c, cudaMemcpyAsync(ring + (size_t)slot * conv, hist3 + (size_t)age * conv, (size_t)conv * 2,
                                  cudaMemcpyDeviceToDevice, st));
        }
    }
    return QRES_OK;
}

qres_status qres_dump_gdn_state(qres_ctx* c, int32_t layer, int32_t user, float* state, void* stream) {
    float* src = nullptr;
    size_t bytes = 0;
    qres_status s = gdn_layer_state(c, layer, user, "qres_dump_gdn_state", &src, &bytes);
    if (s) return s;
    if (!state) return fail(c, QRES_ERR_ARG, "qres_dump_gdn_state: null destination");
    CU(c, cudaMemcpyAsync(state, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
    return QRES_OK;
}

static qres_status kv_rows(qres_ctx* c, int32_t layer, int32_t user, uint16_t* k, uint16_t* v, int32_t npos,
                           void* stream, bool load) {
    const char* what = load ? "qres_load_kv" : "qres_dump_kv";
    if (!c) return fail(nullptr, QRES_ERR_ARG, "%s: null context", what);
    if (layer < 0 || layer >= c->cfg.layers || !is_attn(c, layer) || !c->layers[layer].has_st)
        return fail(c, QRES_ERR_ARG, "%s: layer %d is not a bound attention layer", what, layer);
    if (user < 0 || user >= c->cfg.rows || !k || !v || npos < 1 || npos > c->cfg.max_pages * kKvBlock)
        return fail(c, QRES_ERR_ARG, "%s: user %d, %d positions (at most %d)", what, user, npos,
                    c->cfg.max_pages * kKvBlock);
    if (!c->has_io || !c->io.page_table || !c->err) return fail(c, QRES_ERR_STATE, "%s before bind_io / bind_workspace", what);
    const Layer& L = c->layers[layer];
    const int32_t* pt = c->io.page_table + (size_t)((c->cfg.flags & QRES_FLAG_VERIFY) ? 0 : user) * c->cfg.max_pages;
    CU(c, kv_rows_launch(L.st.k_pool, L.st.v_pool, k, v, pt, npos, c->nkv, c->cfg.num_pages, load, c->err,
                         static_cast<cudaStream_t>(stream)));
    return QRES_OK;
}

qres_status qres_load_kv(qres_ctx* c, int32_t layer, int32_t user, const uint16_t* k, const uint16_t* v, int32_t npos,
                         void* stream) {
    return kv_rows(c, layer, user, const_cast<uint16_t*>(k), const_cast<uint16_t*>(v), npos, stream, true);
}

qres_status qres_dump_kv(qres_ctx* c, int32_t layer, int32_t user, uint16_t* k, uint16_t* v, int32_t npos,
                         void* stream) {
    return kv_rows(c, layer, user, k, v, npos, stream, false);
}

qres_status qres_bind_rope(qres_ctx* c, const float* cos_tab, const float* sin_tab, int32_t max_pos) {
    if (!c || !cos_tab || !sin_tab || max_pos < 1) return fail(c, QRES_ERR_ARG, "qres_bind_rope: bad argument");
    c->cos_tab = cos_tab;
    c->sin_tab = sin_tab;
    c->max_pos = max_pos;
    return QRES_OK;
}

qres_status qres_bind_io(qres_ctx* c, const qres_io* io) {
    if (!c || !io || !io->tok || !io->x) return fail(c, QRES_ERR_ARG, "qres_bind_io: tok and x are required");
    if (c->vocab_local && (!io->logits || !io->topk || !io->out))
        return fail(c, QRES_ERR_ARG, "qres_bind_io: the lm_head needs logits, topk and out");
    c->io = *io;
    c->has_io = true;
    return QRES_OK;
}

qres_status qres_bind_sampling(qres_ctx* c, const uint32_t* words) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    if (words && !c->cfg.vocab) return fail(c, QRES_ERR_ARG, "qres_bind_sampling: sampling needs an lm_head");
    c->sampling = words;  // a captured graph holds the pointer it was captured with: bind before qres_capture
    return QRES_OK;
}

qres_status qres_workspace_size(const qres_ctx* c, size_t* bytes) {
    if (!c || !bytes) return QRES_ERR_ARG;
    *bytes = carve(c).total;
    return QRES_OK;
}

qres_status qres_bind_workspace(qres_ctx* c, void* dev, size_t bytes) {
    if (!c || !dev) return fail(c, QRES_ERR_ARG, "qres_bind_workspace: null");
    Carve k = carve(c);
    if (bytes < k.total) return fail(c, QRES_ERR_ARG, "qres_bind_workspace: %zu bytes, need %zu", bytes, k.total);
    uint8_t* w = static_cast<uint8_t*>(dev);
    CU(c, cudaMemset(w, 0, k.total));
    CU(c, cudaDeviceSynchronize());
    c->ws = w;
    c->ws_bytes = bytes;
    c->err = reinterpret_cast<uint32_t*>(w + k.err);
    c->epoch = reinterpret_cast<uint32_t*>(w + k.epoch);
    c->xb = reinterpret_cast<float*>(w + k.xb);
    c->xe = reinterpret_cast<float*>(w + k.xe);
    c->partial = reinterpret_cast<float*>(w + k.partial);
    c->y = reinterpret_cast<uint16_t*>(w + k.y);
    c->o = reinterpret_cast<uint16_t*>(w + k.o);
    c->a = reinterpret_cast<uint16_t*>(w + k.a);
    c->hbuf = reinterpret_cast<uint16_t*>(w + k.hbuf);
    c->argmax = reinterpret_cast<int32_t*>(w + k.argmax);
    c->gathered = reinterpret_cast<uint32_t*>(w + k.gathered);
    c->attn_work = w + k.attn;
    c->attn_work_bytes = attn_workspace_bytes(c->nranks, c->cfg.rows, c->attn_chunks);
    c->topk_work = c->vocab_local ? (void*)(w + k.topk) : nullptr;
    c->gemv_work = w + k.gemv;
    c->gemv_work_bytes = k.gemv_bytes;
    for (int i = 0; i < 4; ++i) c->acc[i] = reinterpret_cast<long long*>(w + k.acc[i]);
    return QRES_OK;
}

qres_status qres_p2p_window_size(const qres_ctx* c, size_t* bytes) {
    if (!c || !bytes) return QRES_ERR_ARG;
    *bytes = P2PLayout(c->cfg.rows).total;
    return QRES_OK;
}

qres_status qres_p2p_alloc(qres_ctx* c, void* handle64) {
    if (!c || !handle64) return fail(c, QRES_ERR_ARG, "qres_p2p_alloc: null argument");
    if (c->nranks < 2) return fail(c, QRES_ERR_ARG, "qres_p2p_alloc: one rank has no peers");
    if (c->p2p_local) return fail(c, QRES_ERR_STATE, "qres_p2p_alloc: window already allocated");
    const size_t bytes = P2PLayout(c->cfg.rows).total;
    void* p = nullptr;
    CU(c, cudaMalloc(&p, bytes));
    c->p2p_local = static_cast<uint8_t*>(p);
    CU(c, cudaMemset(p, 0, bytes));
    CU(c, cudaDeviceSynchronize());
    cudaIpcMemHandle_t h;
    CU(c, cudaIpcGetMemHandle(&h, p));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(handle64, &h, 64);
    return QRES_OK;
}

qres_status qres_p2p_open(qres_ctx* c, const void* handles) {
    if (!c || !handles) return fail(c, QRES_ERR_ARG, "qres_p2p_open: null argument");
    if (!c->p2p_local) return fail(c, QRES_ERR_STATE, "qres_p2p_open before qres_p2p_alloc");
    if (!c->ws) return fail(c, QRES_ERR_STATE, "qres_p2p_open before qres_bind_workspace");
    if (c->p2p_on) return fail(c, QRES_ERR_STATE, "qres_p2p_open: already open");
    const uint8_t* hs = static_cast<const uint8_t*>(handles);
    for (int r = 0; r < c->nranks; ++r) {
        if (r == c->rank) {
            c->p2p_peer[r] = c->p2p_local;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)r * 64, 64);
        void* p = nullptr;
        CU(c, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        c->p2p_peer[r] = static_cast<uint8_t*>(p);
    }
    CU(c, cudaMemset(c->epoch, 0, 4));
    CU(c, cudaDeviceSynchronize());
    // the counted exchange adds into the peers' windows with 64-bit atomics: only where every other visible GPU
    // has native peer atomics with this one
    int ndev = 0;
    CU(c, cudaGetDeviceCount(&ndev));
    bool atomics = ndev >= c->nranks;
    for (int d = 0; d < ndev && atomics; ++d) {
        if (d == c->device) continue;
        int v = 0;
        if (cudaDeviceGetP2PAttribute(&v, cudaDevP2PAttrNativeAtomicSupported, c->device, d) != cudaSuccess || !v)
            atomics = false;
    }
    c->p2p_atomics = atomics;
    c->p2p_on = true;
    return QRES_OK;
}

qres_status qres_nccl_unique_id(const char* libpath, void* id128) {
    std::string why;
    if (!id128) return fail(nullptr, QRES_ERR_ARG, "null id");
    if (!load_nccl(libpath, &why)) return fail(nullptr, QRES_ERR_COMM, "%s", why.c_str());
    ncclUniqueId id;
    ncclResult_t r = g_nccl.getUniqueId(&id);
    if (r != ncclSuccess) return fail(nullptr, QRES_ERR_COMM, "ncclGetUniqueId: %d", (int)r);
    memcpy(id128, &id, sizeof id);
    return QRES_OK;
}

qres_status qres_nccl_init(qres_ctx* c, const char* libpath, const void* id128) {
    std::string why;
    if (!c || !id128) return fail(c, QRES_ERR_ARG, "null argument");
    if (!load_nccl(libpath, &why)) return fail(c, QRES_ERR_COMM, "%s", why.c_str());
    ncclUniqueId id;
    memcpy(&id, id128, sizeof id);
    ncclResult_t r = g_nccl.commInitRank(&c->comm, c->nranks, id, c->rank);
    if (r != ncclSuccess)
        return fail(c, QRES_ERR_COMM, "ncclCommInitRank: %s", g_nccl.errStr ? g_nccl.errStr(r) : "error");
    return QRES_OK;
}

// the fixed-point accumulators (EPI_ACC; between ranks the counted exchange): with an lm_head, any row count, not
// switched off by QRES_FLAG_TILE_FINISH, and across ranks only over the peer window with native peer atomics
static bool uses_accumulators(const qres_ctx* c) {
    const bool tp = c->nranks > 1;
    return !(c->cfg.flags & QRES_FLAG_TILE_FINISH) && c->cfg.vocab > 0 &&
           (!tp || (c->p2p_on && c->p2p_atomics));
}

static qres_status enqueue_step(qres_ctx* c, cudaStream_t st) {
    const int R = c->cfg.rows, n = c->nranks;
    const bool tp = n > 1;
    if (!c->has_io || !c->ws) return fail(c, QRES_ERR_STATE, "decode step before bind_io / bind_workspace");
    if (tp && !c->comm && !c->p2p_on) return fail(c, QRES_ERR_STATE, "nranks > 1 needs qres_p2p_open or qres_nccl_init");
    const bool p2p = tp && c->p2p_on;
    const int verify = (c->cfg.flags & QRES_FLAG_VERIFY) ? R : 0;
    const P2PLayout pl(R);
    if (c->cfg.vocab && !c->has_head) return fail(c, QRES_ERR_STATE, "lm_head not loaded");
    if (c->has_fc && (!c->io.h_in || R > 4)) return fail(c, QRES_ERR_STATE, "the fc needs io.h_in (and at most 4 rows)");
    for (int l = 0; l < c->cfg.layers; ++l) {
        const Layer& L = c->layers[l];
        const bool at = is_attn(c, l);
        if (!L.has[at ? QRES_W_ATTN_IN : QRES_W_GDN_IN] || !L.has[QRES_W_OUT] || !L.has[QRES_W_GATEUP] ||
            !L.has[QRES_W_DOWN] || !L.has_st)
            return fail(c, QRES_ERR_STATE, "layer %d: weights or state not bound", l);
        if (at ? (!L.wq || !c->cos_tab || !c->io.page_table) : (!L.taps))
            return fail(c, QRES_ERR_STATE, "layer %d: parameters not bound", l);
    }
    // weight-streaming CTAs per projection: two per SM, fewer for a small one (a tensor-parallel shard) so that
    // each CTA streams at least ~4 units of 16 KB -- every CTA pays a fixed prologue (reading the whole
    // residual, with the peer exchange one copy per rank), which the small shards' few units do not amortise
    auto grid_of = [&](const qres_weight& w) {
        const int units = (w.rows_pad / 128) * (w.K / 128);
        return std::max(c->sm_count / 2, std::min(2 * c->sm_count, units / 4));
    };
    const int32_t* pos = c->io.tok->pos;
    int launches = 0;
    auto K = [&](cudaError_t e, const char* what) -> qres_status {
        if (e != cudaSuccess) return fail(c, QRES_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
        ++launches;
        return QRES_OK;
    };
#define STEP(call, what)                       \
    do {                                       \
        qres_status s_ = K((call), what);      \
        if (s_) return s_;                     \
    } while (0)
    float* cur = c->io.x;  // residual stream
    float* other = c->xb;
    if (!c->has_fc) {
        STEP(embed_rows_launch(c->io.tok, c->io.x0, c->io.embed, c->cfg.vocab, cur, R, c->err, st, true), "rows in");
    }
    bool pending = false;  // all-reduced partials waiting to be added to cur
    int xchg = 0;          // row-parallel exchanges issued so far in this step (peer exchange: slot xchg % 2)
    auto allreduce = [&]() -> qres_status {
        ncclResult_t r = g_nccl.allReduce(c->partial, c->partial, (size_t)R * kHidden, ncclFloat32, ncclSum, c->comm, st);
        if (r != ncclSuccess) return fail(c, QRES_ERR_COMM, "ncclAllReduce: %d", (int)r);
        return QRES_OK;
    };
    // a GEMV with the rmsnorm prologue over the residual (adding pending partials first when TP)
    // the weight-streaming projections in step order: each launch prefetches the start of the next one into
    // L2 once its own stream is done (the lm_head's next is layer 0's in-projection of the following step)
    std::vector<const qres_weight*> order;
    for (int l = 0; l < c->cfg.layers; ++l) {
        const Layer& L = c->layers[l];
        order.push_back(&L.w[is_attn(c, l) ? QRES_W_ATTN_IN : QRES_W_GDN_IN]);
        order.push_back(&L.w[QRES_W_OUT]);
        order.push_back(&L.w[QRES_W_GATEUP]);
        order.push_back(&L.w[QRES_W_DOWN]);
    }
    if (c->cfg.vocab) order.push_back(&c->head);
    // units k0 .. k0 + k - 1 of every CTA run of projection w as that launch will split it
    const bool accm = uses_accumulators(c);
    auto heads_of = [&](const qres_weight& w, int k0, int k) -> L2Heads {
        const int units = (w.rows_pad / 128) * (w.K / 128);
        // the unit order of that launch: grouped only for the accumulating projections (not the lm_head)
        const int nq = gemv_group_blocks(R, (accm && &w != &c->head) ? EPI_ACC : EPI_BF16, w.K);
        return L2Heads{static_cast<const uint8_t*>(w.data), units, gemv_grid(R, w.rows_pad, w.K, grid_of(w)), k0, k,
                       w.rows_pad / 128, w.K / 128, nq};
    };
    // (deeper prefetch, here or from the mixers, measured slower: it competes with the stream it precedes)
    const int kPrefetchUnits = 2;  // 32 KB per CTA run
    std::vector<L2Heads> next_heads(order.size());
    for (size_t i = 0; i < order.size(); ++i) next_heads[i] = heads_of(*order[(i + 1) % order.size()], 0, kPrefetchUnits);
    auto next_of = [&](const qres_weight* w) -> const L2Heads* {
        for (size_t i = 0; i < order.size(); ++i)
            if (order[i] == w) return &next_heads[i];
        return nullptr;
    };
    auto gemv = [&](const qres_weight& w, int pro, const void* in, int ld_in, int epi, void* out, int ld_out,
                    const float* red, float* x_out, const char* what) -> qres_status {
        return K(gemv_launch(w, R, pro, in, ld_in, epi, out, ld_out, grid_of(w), c->err, st, true, red, x_out, c->gemv_work,
                             c->gemv_work_bytes, next_of(&w)),
                 what);
    };
    // Fixed-point accumulators (EPI_ACC, with an lm_head; over ranks with the peer exchange and native
    // peer atomics). The in-projection and gate|up add into this rank's buffers (accD, read by the mixer; accB,
    // read by the down prologue as silu(g) * u). The row-parallel out- and down-projections add into XA and XC,
    // which the next rmsnorm prologue adds to the residual. Each launch zeroes a buffer whose last reader finished
    // before it started and whose next writer starts after it.
    // - One rank: plain sums, read after the producing launch has completed. Out-proj zeroes accB, gate|up XC,
    //   down XA and accD (one range).
    // - n ranks (EPI_XACC / PRO_RMSNORM_XACC): the out- and down-projections add counted words into every rank's
    //   XA / XC (in the peer window), and the next prologue reads them once each word holds all contributions.
    //   In-proj zeroes accB, out-proj XC, gate|up accD, down XA -- the exchange buffers with a system-scope fence:
    //   peers add into them only after this rank's next contributions, which follow the fence.
    long long* const accB = c->acc[1];
    long long* const accD = c->acc[3];
    long long* xa_at[8] = {};
    long long* xc_at[8] = {};
    for (int r = 0; r < n; ++r) {
        xa_at[r] = tp ? reinterpret_cast<long long*>(c->p2p_peer[r] + pl.xa) : c->acc[0];
        xc_at[r] = tp ? reinterpret_cast<long long*>(c->p2p_peer[r] + pl.xc) : c->acc[2];
    }
    long long* const XA = xa_at[c->rank];
    long long* const XC = xc_at[c->rank];
    struct Pending {
        const long long* acc = nullptr;
        int units = 0, grid = 0, nkb = 0;  // the producing launch's partition (its per-tile contribution count)
    } pending_acc;
    auto producer_of = [&](const qres_weight& w, const long long* acc) {
        Pending q;
        q.acc = acc;
        q.nkb = w.K / 128;
        q.units = (w.rows_pad / 128) * q.nkb;
        q.grid = gemv_grid(R, w.rows_pad, w.K, grid_of(w));
        return q;
    };
    auto take_pending = [&](GemvExchange& ex) {
        ex.racc = pending_acc.acc;
        ex.rc_ranks = tp ? n : 0;
        ex.rc_units = pending_acc.units;
        ex.rc_grid = pending_acc.grid;
        ex.rc_nkb = pending_acc.nkb;
        pending_acc = Pending();
    };
    // 4 or more rows: a projection's rmsnorm input is formed once per user (resid_norm: x + the pending sums -- over
    // ranks the counted words, once complete -> the other residual buffer, h = bf16(rmsnorm) -> hbuf) and the
    // projection reads its window of h, instead of each of its CTAs re-reading every user's residual and sums
    // (~480 KB per CTA at 8 rows).
    const bool split = accm && R >= 4;
    auto resid_norm = [&](bool add) -> qres_status {
        GemvExchange ex;
        if (add) take_pending(ex);
        pending_acc = Pending();
        qres_status s = K(resid_norm_launch(R, cur, ex.racc, add ? other : nullptr, c->hbuf, st, true, &ex, c->err),
                          "resid-norm");
        if (add) std::swap(cur, other);
        return s;
    };
    auto norm_gemv = [&](const qres_weight& w, int epi, void* out, int ld_out, const char* what) -> qres_status {
        if (split && pending_acc.acc) {
            qres_status s = resid_norm(true);
            if (s) return s;
            return K(gemv_launch(w, R, PRO_BF16, c->hbuf, kHidden, epi, out, ld_out, grid_of(w), c->err, st, true, nullptr,
                                 nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&w)),
                     what);
        }
        if (pending_acc.acc) {
            GemvExchange ex;
            take_pending(ex);
            qres_status s = K(gemv_launch(w, R, tp ? 4 : 2, cur, kHidden, epi, out, ld_out, grid_of(w), c->err, st, true, nullptr,
                                          other, c->gemv_work, c->gemv_work_bytes, next_of(&w), &ex),
                              what);
            std::swap(cur, other);
            return s;
        }
        if (pending && p2p) {
            // the peer exchange xchg - 1: every rank's tagged partial, added in rank order
            const int j = xchg - 1, slot = j & 1;
            GemvExchange ex;
            ex.nsrc = n;
            ex.tagged = reinterpret_cast<const uint2*>(c->p2p_local + pl.data) + (size_t)slot * 8 * R * kHidden;
            ex.epoch = c->epoch;
            ex.tag_mul = 2u * (uint32_t)c->cfg.layers;
            ex.tag_add = (uint32_t)j + 1u;
            qres_status s = K(gemv_launch(w, R, 2, cur, kHidden, epi, out, ld_out, grid_of(w), c->err, st, true,
                                          reinterpret_cast<const float*>(ex.tagged), other, c->gemv_work,
                                          c->gemv_work_bytes, next_of(&w), &ex),
                              what);
            std::swap(cur, other);
            pending = false;
            return s;
        }
        if (pending) {
            qres_status s = gemv(w, 2, cur, kHidden, epi, out, ld_out, c->partial, other, what);
            std::swap(cur, other);
            pending = false;
            return s;
        }
        return gemv(w, 0, cur, kHidden, epi, out, ld_out, nullptr, nullptr, what);
    };
    // a row-parallel projection: residual update (one rank) or fp32 partial + all-reduce (TP)
    auto row_parallel = [&](const qres_weight& w, const uint16_t* in, const char* what) -> qres_status {
        if (p2p) {
            // fused exchange: the epilogue stores each finished tile into every rank's window (slot xchg % 2)
            const int slot = xchg & 1;
            GemvExchange ex;
            ex.p2p_n = n;
            ex.peer_ld = kHidden;
            ex.epoch = c->epoch;
            ex.tag_mul = 2u * (uint32_t)c->cfg.layers;
            ex.tag_add = (uint32_t)xchg + 1u;
            for (int r = 0; r < n; ++r)
                ex.peer_data[r] = reinterpret_cast<uint2*>(c->p2p_peer[r] + pl.data) + ((size_t)slot * 8 + c->rank) * R * kHidden;
            qres_status s = K(gemv_launch(w, R, 1, in, w.K, 4, nullptr, kHidden, grid_of(w), c->err, st, true, nullptr,
                                          nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&w), &ex),
                              what);
            ++xchg;
            pending = true;
            return s;
        }
        qres_status s = gemv(w, 1, in, w.K, tp ? 3 : 2, tp ? c->partial : cur, kHidden, nullptr, nullptr, what);
        if (s || !tp) return s;
        s = allreduce();
        pending = true;
        return s;
    };
    if (c->has_fc) {
        // the MTP draft layer's input (mtp.py:1-14, streamer_compute.cpp:424-435): x = fc([rmsnorm(e) |
        // rmsnorm(h)]) for e = the token's embedding row and h = io.h_in (a previous step's last x); the pre-fc
        // norm weights are folded into the fc's columns; no residual
        STEP(embed_rows_launch(c->io.tok, c->io.x0, c->io.embed, c->cfg.vocab, c->xe, R, c->err, st, true), "rows in");
        GemvExchange ex;
        ex.seg = kHidden;
        ex.seg2 = c->io.h_in;
        STEP(gemv_launch(c->fc, R, 0, c->xe, kHidden, 3, cur, kHidden, grid_of(c->fc), c->err, st, true, nullptr, nullptr,
                         c->gemv_work, c->gemv_work_bytes, nullptr, &ex),
             "fc");
    }
    for (int l = 0; l < c->cfg.layers; ++l) {
        const Layer& L = c->layers[l];
        const bool at = is_attn(c, l);
        uint16_t* mcopy = (l == c->cfg.layers - 1) ? c->io.mixer_out : nullptr;
        qres_status s = QRES_OK;
        if (accm) {
            // into the in-projection's accumulators (the mixer rounds the sums to bf16 as it reads them)
            const qres_weight& wi = L.w[at ? QRES_W_ATTN_IN : QRES_W_GDN_IN];
            GemvExchange ei;
            const bool add = pending_acc.acc != nullptr;
            ei.acc_out = accD;
            if (tp) {
                ei.zero = accB;
                ei.zero_words = (size_t)R * 2 * c->ic;
            }
            if (split) {
                s = resid_norm(add);
                if (s) return s;
                STEP(gemv_launch(wi, R, PRO_BF16, c->hbuf, kHidden, 5, nullptr, c->ld_y, grid_of(wi), c->err, st, true,
                                 nullptr, nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&wi), &ei),
                     "in-proj");
            } else {
                if (add) take_pending(ei);
                STEP(gemv_launch(wi, R, add ? (tp ? 4 : 2) : 0, cur, kHidden, 5, nullptr, c->ld_y, grid_of(wi), c->err, st,
                                 true, nullptr, add ? other : nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&wi), &ei),
                     "in-proj");
                if (add) std::swap(cur, other);
            }
        } else {
            s = norm_gemv(L.w[at ? QRES_W_ATTN_IN : QRES_W_GDN_IN], 0, c->y, c->ld_y, "in-proj");
            if (s) return s;
        }
        // the mixer is latency-bound: it pulls the whole out-projection into L2 meanwhile
        const void* pf = L.w[QRES_W_OUT].data;
        const size_t pf_bytes = (size_t)L.w[QRES_W_OUT].rows_pad * L.w[QRES_W_OUT].K;
        if (at) {
            STEP(attn_launch(n, R, c->y, c->ld_y, pos, c->io.page_table, c->cfg.max_pages, c->cfg.num_pages, L.wq, L.wk,
                             c->cos_tab, c->sin_tab, c->max_pos, L.st.k_pool, L.st.v_pool, c->o, mcopy, c->attn_work,
                             c->attn_work_bytes, c->attn_chunks, c->err, st, true, pf, pf_bytes, verify, accm ? accD : nullptr),
                 "attention");
        } else {
            STEP(gdn_launch(n, R, c->y, c->ld_y, pos, L.taps, L.dt, L.neg_a, L.norm_w, L.st.gdn_state, L.st.conv_hist,
                            c->o, mcopy, c->err, st, true, pf, pf_bytes, verify, &c->io.tok->slot, accm ? accD : nullptr),
                 "gdn");
        }
        if (accm) {
            const qres_weight& wo = L.w[QRES_W_OUT];
            const qres_weight& wg = L.w[QRES_W_GATEUP];
            const qres_weight& wd = L.w[QRES_W_DOWN];
            GemvExchange eo;
            if (tp) {
                eo.xn = n;
                for (int r = 0; r < n; ++r) eo.xdst[r] = xa_at[r];
                eo.zero = XC;
                eo.zero_words = (size_t)R * kHidden;
                eo.zero_sys = true;
            } else {
                eo.acc_out = XA;
                eo.zero = accB;
                eo.zero_words = (size_t)R * 2 * c->ic;
            }
            STEP(gemv_launch(wo, R, 1, c->o, wo.K, tp ? 6 : 5, nullptr, kHidden, grid_of(wo), c->err, st, true, nullptr, nullptr,
                             c->gemv_work, c->gemv_work_bytes, next_of(&wo), &eo),
                 "out-proj");
            GemvExchange eg;
            pending_acc = producer_of(wo, XA);
            eg.acc_out = accB;
            eg.zero = tp ? accD : XC;
            eg.zero_words = tp ? (size_t)R * c->ld_y : (size_t)R * kHidden;
            if (split) {
                s = resid_norm(true);
                if (s) return s;
                STEP(gemv_launch(wg, R, PRO_BF16, c->hbuf, kHidden, 5, nullptr, 2 * c->ic, grid_of(wg), c->err, st, true,
                                 nullptr, nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&wg), &eg),
                     "gate-up");
            } else {
                take_pending(eg);
                STEP(gemv_launch(wg, R, tp ? 4 : 2, cur, kHidden, 5, nullptr, 2 * c->ic, grid_of(wg), c->err, st, true, nullptr,
                                 other, c->gemv_work, c->gemv_work_bytes, next_of(&wg), &eg),
                     "gate-up");
                std::swap(cur, other);
            }
            GemvExchange ed;
            if (split) {
                // silu(g) * u formed once per user into `a` (unused on the accumulator path), read as bf16
                STEP(silu_rows_launch(R, accB, 2 * c->ic, c->ic, c->a, st, true), "silu-mul");
            } else {
                ed.gacc = accB;
                ed.ld_gacc = 2 * c->ic;
            }
            ed.zero = XA;  // one rank: and accD, right behind it
            ed.zero_words = (size_t)R * kHidden + (tp ? 0 : (size_t)R * c->ld_y);
            if (tp) {
                ed.xn = n;
                for (int r = 0; r < n; ++r) ed.xdst[r] = xc_at[r];
                ed.zero_sys = true;
            } else {
                ed.acc_out = XC;
            }
            STEP(gemv_launch(wd, R, split ? PRO_BF16 : PRO_SILU_ACC, split ? c->a : nullptr, wd.K, tp ? 6 : 5, nullptr, kHidden,
                             grid_of(wd), c->err, st, true, nullptr, nullptr, c->gemv_work, c->gemv_work_bytes, next_of(&wd), &ed),
                 "down");
            pending_acc = producer_of(wd, XC);
            continue;
        }
        s = row_parallel(L.w[QRES_W_OUT], c->o, "out-proj");
        if (s) return s;
        s = norm_gemv(L.w[QRES_W_GATEUP], 1, c->a, c->ic, "gate-up");
        if (s) return s;
        s = row_parallel(L.w[QRES_W_DOWN], c->a, "down");
        if (s) return s;
    }
    if (c->cfg.vocab) {
        qres_status s = norm_gemv(c->head, 0, c->io.logits, c->vocab_local, "lm_head");
        if (s) return s;
        const int base = c->rank * c->vocab_local;
        if (!tp) {
            STEP(topk_launch(R, c->io.logits, c->vocab_local, c->vocab_local, base, c->io.topk, c->argmax, c->topk_work,
                             c->topk_blk, st, true),
                 "top-k");
        } else if (p2p) {
            STEP(topk_launch(R, c->io.logits, c->vocab_local, c->vocab_local, base, c->io.topk, nullptr, c->topk_work,
                             c->topk_blk, st, true),
                 "top-k");
            P2PDest dst;
            dst.n = n;
            dst.slot_words = (size_t)8 * R * 2 * QRES_TOPK;
            for (int r = 0; r < n; ++r) {
                dst.data[r] = reinterpret_cast<uint32_t*>(c->p2p_peer[r] + pl.lists) + (size_t)c->rank * R * 2 * QRES_TOPK;
                dst.cnt[r] = reinterpret_cast<uint32_t*>(c->p2p_peer[r] + pl.lcnt) + c->rank;
            }
            STEP(publish_lists_launch(c->io.topk, R * 2 * QRES_TOPK, dst, c->epoch, st, true), "list exchange");
            STEP(merge_lists_launch(reinterpret_cast<const uint32_t*>(c->p2p_local + pl.lists), n, R, c->io.topk,
                                    c->argmax, st, true, reinterpret_cast<const uint32_t*>(c->p2p_local + pl.lcnt),
                                    c->epoch, c->err),
                 "merge");
        } else {
            STEP(topk_launch(R, c->io.logits, c->vocab_local, c->vocab_local, base, c->io.topk, nullptr, c->topk_work,
                             c->topk_blk, st, true),
                 "top-k");
            ncclResult_t r = g_nccl.allGather(c->io.topk, c->gathered, (size_t)R * 2 * QRES_TOPK, ncclUint32, c->comm, st);
            if (r != ncclSuccess) return fail(c, QRES_ERR_COMM, "ncclAllGather: %d", (int)r);
            STEP(merge_lists_launch(c->gathered, n, R, c->io.topk, c->argmax, st, true), "merge");
        }
        STEP(feed_launch(c->io.tok, c->argmax, c->io.out, R, st, true, c->epoch, c->io.topk, c->sampling), "feed");
    } else {
        STEP(feed_launch(c->io.tok, nullptr, nullptr, R, st, true, c->epoch, nullptr, nullptr), "feed");
    }
    if (cur != c->io.x) CU(c, cudaMemcpyAsync(c->io.x, cur, (size_t)R * kHidden * 4, cudaMemcpyDeviceToDevice, st));
#undef STEP
    c->launches = launches;
    return QRES_OK;
}

qres_status qres_decode_step(qres_ctx* c, void* stream) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    if (c->nranks > 1 && !c->cfg.vocab)
        return fail(c, QRES_ERR_ARG, "nranks > 1 without an lm_head is not supported");
    return enqueue_step(c, static_cast<cudaStream_t>(stream));
}

qres_status qres_capture(qres_ctx* c, void* stream) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    qres_release_graph(c);
    CU(c, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    qres_status s = qres_decode_step(c, stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
    }
    if (e != cudaSuccess) return fail(c, QRES_ERR_CUDA, "end capture: %s", cudaGetErrorString(e));
    c->graph = g;
    CU(c, cudaGraphInstantiate(&c->exec, g, 0));
    return QRES_OK;
}

qres_status qres_replay(qres_ctx* c, void* stream) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    if (!c->exec) return fail(c, QRES_ERR_STATE, "replay without a captured graph");
    CU(c, cudaGraphLaunch(c->exec, static_cast<cudaStream_t>(stream)));
    return QRES_OK;
}

qres_status qres_release_graph(qres_ctx* c) {
    if (!c) return QRES_ERR_ARG;
    if (c->exec) cudaGraphExecDestroy(c->exec);
    if (c->graph) cudaGraphDestroy(c->graph);
    c->exec = nullptr;
    c->graph = nullptr;
    return QRES_OK;
}

qres_status qres_check(qres_ctx* c, void* stream) {
    if (!c) return fail(nullptr, QRES_ERR_ARG, "null context");
    CU(c, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    if (!c->err) return QRES_OK;
    uint32_t w = 0;
    CU(c, cudaMemcpy(&w, c->err, 4, cudaMemcpyDeviceToHost));
    if (!w) return QRES_OK;
    CU(c, cudaMemset(c->err, 0, 4));
    return fail(c, QRES_ERR_DEVICE, "device error word 0x%x:%s%s%s", w, (w & kErrTimeout) ? " bounded wait ran out;" : "",
                (w & kErrBounds) ? " index out of range (position / page / token);" : "",
                (w & kErrPeer) ? " peer epoch mismatch;" : "");
}

int32_t qres_step_launches(const qres_ctx* c) { return c ? c->launches : 0; }

qres_status qres_wait_probe(qres_ctx* c, const uint32_t* flag, uint32_t want, uint32_t polls, void* stream) {
    if (!c || !flag || polls == 0) return fail(c, QRES_ERR_ARG, "qres_wait_probe: bad argument");
    if (!c->err) return fail(c, QRES_ERR_STATE, "qres_wait_probe before qres_bind_workspace");
    CU(c, wait_probe_launch(flag, want, polls, c->err, static_cast<cudaStream_t>(stream)));
    return QRES_OK;
}

int32_t qres_exchange_mode(const qres_ctx* c) {
    if (!c) return -1;
    if (c->nranks == 1) return QRES_XCHG_NONE;
    if (c->p2p_on) return uses_accumulators(c) ? QRES_XCHG_COUNTED : QRES_XCHG_TAGGED;
    return c->comm ? QRES_XCHG_NCCL : QRES_XCHG_NONE;
}

// ---- single kernels ----

qres_status qres_gemv_workspace_size(int32_t grid, int32_t rows_pad, size_t* bytes) {
    if (!bytes || rows_pad < 128 || rows_pad % 128 || rows_pad > 4096 * 128)
        return fail(nullptr, QRES_ERR_ARG, "qres_gemv_workspace_size: bad argument");
    if (grid <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&grid, cudaDevAttrMultiProcessorCount, dev);
        grid *= 2;
    }
    *bytes = gemv_workspace_bytes(grid);
    return QRES_OK;
}

qres_status qres_gemv(const qres_weight* w, int32_t rows, int32_t pro, const void* in, int32_t epi, void* out,
                      int32_t grid, uint32_t* err, void* work, size_t work_bytes, void* stream) {
    if (!w || !in || !out || !work || pro < 0 || pro > 1 || epi < 0 || epi > 4)
        return fail(nullptr, QRES_ERR_ARG, "qres_gemv: bad argument");
    if (grid <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&grid, cudaDevAttrMultiProcessorCount, dev);
        grid *= 2;  // two CTAs per SM
    }
    const int ld_out = epi == 1 ? w->rows / 2 : w->rows;
    GemvExchange ex;
    if (epi == 4) ex.acc_out = static_cast<long long*>(out);  // the step's accumulators (EPI_ACC)
    cudaError_t ce = gemv_launch(*w, rows, pro, in, w->K, epi == 4 ? EPI_ACC : epi, epi == 4 ? nullptr : out, ld_out, grid,
                                 err, static_cast<cudaStream_t>(stream), false, nullptr, nullptr, work, work_bytes,
                                 nullptr, &ex);
    if (ce != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_gemv: %s", cudaGetErrorString(ce));
    return QRES_OK;
}

qres_status qres_gdn_mixer(int32_t nranks, int32_t rows, const uint16_t* y, int32_t ld_y, const int32_t* pos,
                           const uint16_t* taps, const float* dt, const float* neg_a, const float* norm_w, float* state,
                           uint16_t* conv_hist, uint16_t* o, uint32_t* err, void* stream) {
    if (!y || !pos || !taps || !dt || !neg_a || !norm_w || !state || !conv_hist || !o)
        return fail(nullptr, QRES_ERR_ARG, "qres_gdn_mixer: null argument");
    cudaError_t e = gdn_launch(nranks, rows, y, ld_y, pos, taps, dt, neg_a, norm_w, state, conv_hist, o, nullptr, err,
                               static_cast<cudaStream_t>(stream), false, nullptr, 0);
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_gdn_mixer: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_attn_workspace_size(int32_t nranks, int32_t rows, int32_t max_pos, size_t* bytes) {
    if (!bytes || nranks < 1 || rows < 1) return fail(nullptr, QRES_ERR_ARG, "qres_attn_workspace_size: bad argument");
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int pages = (max_pos + kKvBlock - 1) / kKvBlock;
    *bytes = attn_workspace_bytes(nranks, rows, attn_default_chunks(nranks, rows, sms, pages));
    return QRES_OK;
}

qres_status qres_attn_mixer(int32_t nranks, int32_t rows, const uint16_t* y, int32_t ld_y, const int32_t* pos,
                            const int32_t* page_table, int32_t max_pages, const float* wq, const float* wk,
                            const float* cos_tab, const float* sin_tab, uint16_t* k_pool, uint16_t* v_pool, uint16_t* o,
                            void* work, size_t work_bytes, uint32_t* err, void* stream) {
    if (!y || !pos || !page_table || !wq || !wk || !cos_tab || !sin_tab || !k_pool || !v_pool || !o || !work)
        return fail(nullptr, QRES_ERR_ARG, "qres_attn_mixer: null argument");
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int chunks = attn_default_chunks(nranks, rows, sms, max_pages);
    // num_pages / max_pos bounds: the caller's pool holds max_pages * rows pages at most in this entry point
    cudaError_t e = attn_launch(nranks, rows, y, ld_y, pos, page_table, max_pages, max_pages * rows, wq, wk, cos_tab,
                                sin_tab, max_pages * kKvBlock, k_pool, v_pool, o, nullptr, work, work_bytes, chunks, err,
                                static_cast<cudaStream_t>(stream), false, nullptr, 0);
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_attn_mixer: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_topk_workspace_size(int32_t rows, int32_t n_logits, size_t* bytes) {
    if (!bytes || rows < 1 || n_logits < 1) return QRES_ERR_ARG;
    *bytes = topk_workspace_bytes(rows, topk_default_blocks(n_logits));
    return QRES_OK;
}

qres_status qres_topk(int32_t rows, const uint16_t* logits, int32_t n_logits, int32_t base, uint32_t* lists,
                      int32_t* argmax, void* work, size_t work_bytes, void* stream) {
    if (!logits || !lists || !work || rows < 1 || n_logits < 1) return fail(nullptr, QRES_ERR_ARG, "qres_topk: bad argument");
    const int nblk = topk_default_blocks(n_logits);
    if (work_bytes < topk_workspace_bytes(rows, nblk)) return fail(nullptr, QRES_ERR_ARG, "qres_topk: workspace too small");
    cudaError_t e = topk_launch(rows, logits, n_logits, n_logits, base, lists, argmax, work, nblk,
                                static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_topk: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_sample(int32_t rows, const uint32_t* lists, const uint32_t* words, const int32_t* pos, int32_t* token,
                        void* stream) {
    if (!lists || !words || !pos || !token || rows < 1) return fail(nullptr, QRES_ERR_ARG, "qres_sample: bad argument");
    cudaError_t e = sample_launch(rows, lists, words, pos, token, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_sample: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_topk_noalloc(int32_t rows, const uint16_t* logits, int32_t n_logits, int32_t base, uint32_t* lists,
                              int32_t* argmax, void* stream) {
    if (!logits || !lists || rows < 1 || rows > QRES_MAX_ROWS || n_logits < 1)
        return fail(nullptr, QRES_ERR_ARG, "qres_topk_noalloc: bad argument");
    const int nblk = topk_default_blocks(n_logits);
    void* scratch = nullptr;
    size_t cap = 0;
    cudaError_t e = topk_static_scratch(&scratch, &cap);
    if (e != cudaSuccess)
        return fail(nullptr, QRES_ERR_CUDA, "qres_topk_noalloc: scratch address: %s", cudaGetErrorString(e));
    const size_t need = topk_workspace_bytes(rows, nblk);
    if (need > cap)
        return fail(nullptr, QRES_ERR_ARG,
                    "qres_topk_noalloc: %d rows x %d logits need %zu bytes of scratch, the fixed array holds %zu "
                    "(at most 8 rows of 260,096 logits); use qres_topk with a workspace",
                    rows, n_logits, need, cap);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the tickets must start at zero: a call that stopped early (an error) may have left them set
    e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + topk_ticket_offset(rows, nblk), 0, (size_t)rows * 4, st);
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_topk_noalloc: %s", cudaGetErrorString(e));
    e = topk_launch(rows, logits, n_logits, n_logits, base, lists, argmax, scratch, nblk, st, false);
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_topk_noalloc: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_quantize_fp8(const float* w, int32_t N, int32_t K, uint8_t* q, float* scales, void* stream) {
    if (!w || !q || !scales || N < 1 || K < 1) return fail(nullptr, QRES_ERR_ARG, "qres_quantize_fp8: bad argument");
    cudaError_t e = quantize_fp8_launch(w, N, K, q, scales, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_quantize_fp8: %s", cudaGetErrorString(e));
    return QRES_OK;
}

qres_status qres_tile_weight(const uint8_t* src, int32_t rows, int32_t K, uint8_t* dst, void* stream) {
    if (!src || !dst || rows < 1 || K % 128) return fail(nullptr, QRES_ERR_ARG, "qres_tile_weight: bad argument");
    cudaError_t e = tile_weight_launch(src, rows, K, dst, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(nullptr, QRES_ERR_CUDA, "qres_tile_weight: %s", cudaGetErrorString(e));
    return QRES_OK;
}

}  // extern "C"
