"""The resident decode model on B200: the host object of sott0n/tt-qwen-resident's ``ResidentModel``
(qwen36_resident/model.py:403-1598) over libqres.

Same method names and meaning: ``token_state`` builds a step's input (x0 rows or tokens, positions), ``step``
runs one decode step (asynchronously, on the current stream), ``x`` / ``mixer_output`` / ``logits`` /
``argmax`` / ``fed_token`` read its results, ``reset`` / ``load_state`` write the decode state,
``capture_trace`` / ``release_trace`` record / drop the step as a CUDA graph. Weights, state and activations
live in torch-allocated device memory; every kernel runs in libqres (no torch math on the step's path).

Differences by design: weights are FP8-e4m3 with one fp32 scale per 128x128 block (the reference: Tenstorrent
bf8/bf4); the KV cache is paged (64 positions per page) in bf16; tensor parallelism is 1, 2, 4 or 8 ranks
(KV heads replicated on 2 ranks at 8), one process per GPU.
"""
import ctypes
import math

import numpy as np
import torch

from . import _lib, ops
from .weights import CONV_CH, DK, DV, HD, HIDDEN, NKV, NV, RankDims, shard, stack_matrices

ROPE_THETA = 10_000_000.0
ROT = 64
TOP_K = _lib.QRES_TOPK


def is_attn(l, interval):
    return interval > 0 and (l + 1) % interval == 0


def rope_table(max_pos):
    """cos / sin [max_pos, 32] of model.py:128-131: fp64 angles pos * theta^(-2i/64), rounded to fp32"""
    inv = 1.0 / ROPE_THETA ** (torch.arange(0, ROT, 2, dtype=torch.float64) / ROT)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv
    return torch.cos(ang).float(), torch.sin(ang).float()


class ResidentModel:
    def __init__(
        self,
        w,
        layers,
        interval,
        batch=1,
        max_pos=4096,
        lm_head=False,
        embed=None,
        rank=0,
        nranks=1,
        state_copies=None,
        page_table=None,
        device="cuda",
        sm_count=0,
        nccl_id=None,
        p2p=False,
        verify=False,
        fc=None,
        tile_finish=False,
        share=None,
    ):
        """w: canonical FP8 weights (weights.random_canonical / canonical_from_*): lists per kind; layer l of a
        kind uses copy (k-th layer of that kind) % copies (mlp / out: l % copies), as the reference's
        random_weights copies. state_copies: (gdn, attn) decode states (default one per layer; fewer share a
        state between layers like the reference's State copies). embed: [vocab, 5120] bf16 table for token
        rows (device-fed decode). page_table: [batch, max_pages] int32 (default: user b's pages contiguous).
        share: another ResidentModel of the same layers, rank and vocab whose device weights this one uses (w is
        then ignored; e.g. a batch-8 model beside a batch-1 one without a second copy of the weights)."""
        self.device = torch.device(device)
        self.layers, self.interval, self.batch = layers, interval, batch
        # verify (model.py:416-457): the batch rows are consecutive positions of ONE user (row r sees rows < r);
        # each GDN state holds `batch` slots (row r leaves its state in slot (slot + r) % batch)
        self.verify = bool(verify)
        if self.verify:
            assert 2 <= batch <= _lib.QRES_HIST_SLOTS - 3, "a verify step has 2..5 rows"
            assert state_copies is None, "verify: one GDN state / KV cache per layer"
        self.users = batch
        self.rank, self.nranks = rank, nranks
        if share is not None:
            self.lm_head = lm_head and share.lm_head
            vocab = share.vocab if self.lm_head else 0
        else:
            self.lm_head = lm_head and w.get("head") is not None
            vocab = w["head"].shape[0] if self.lm_head else 0
        self.vocab = vocab
        self.d = d = RankDims(rank, nranks, vocab)
        self.max_pos = max_pos
        self.max_pages = -(-max_pos // _lib.QRES_KV_BLOCK)
        self.n_attn = sum(is_attn(l, interval) for l in range(layers))
        self.n_gdn = layers - self.n_attn
        gc, ac = state_copies or (self.n_gdn, self.n_attn)
        self.state_copies = (max(gc, 1) if self.n_gdn else 0, max(ac, 1) if self.n_attn else 0)
        L = _lib.lib()
        # tile_finish: split projection tiles finished by their last CTA (ticket) rather than summed in the
        # fixed-point accumulators the library uses by default (with an lm_head)
        flags = (
            (_lib.QRES_FLAG_VERIFY if self.verify else 0)
            | (_lib.QRES_FLAG_TILE_FINISH if tile_finish else 0)
        )
        cfg = _lib.Config(layers, interval, vocab, batch, self.max_pages, batch * self.max_pages, sm_count, flags)
        h = ctypes.c_void_p()
        _lib.check(L.qres_create(ctypes.byref(cfg), rank, nranks, ctypes.byref(h)), None, "qres_create")
        self.ctx = h
        self._keep = []
        dev = self.device
        # ---- weights: the rank's slices, re-laid for the GEMV (or another model's, same layers / rank / vocab)
        if share is not None:
            assert (share.layers, share.interval, share.rank, share.nranks, share.vocab) == (layers, interval, rank,
                                                                                           nranks, vocab)
            assert fc is None and share.device == self.device
            w = None
        self._init_weights(w, share, fc)
        self.weight_bytes = self._count_weight_bytes()
        self._init_buffers(page_table, embed)
        # ---- bind
        self._bind()
        sz = ctypes.c_size_t()
        _lib.check(L.qres_workspace_size(self.ctx, ctypes.byref(sz)), self.ctx, "workspace size")
        self.ws = torch.zeros(sz.value, dtype=torch.uint8, device=dev)
        _lib.check(L.qres_bind_workspace(self.ctx, _lib.ptr(self.ws), sz.value), self.ctx, "bind workspace")
        if nranks > 1 and nccl_id is not None:
            buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
            _lib.check(L.qres_nccl_init(self.ctx, None, buf), self.ctx, "nccl init")
        if nranks > 1 and p2p:
            self._open_p2p()
        elif nranks > 1 and nccl_id is None:
            raise ValueError("nranks > 1 needs p2p=True (fused peer exchange) or the NCCL id (see nccl_unique_id)")
        self.trace = False
        self._initial = None

    def _init_weights(self, w, share, fc):
        d, dev = self.d, self.device
        if share is not None:
            for k in ("w_gdn", "gdn_params", "w_attn", "attn_params", "w_out", "w_gu", "w_down", "w_head"):
                setattr(self, k, getattr(share, k))
            self.w_fc = None
            return
        self.w_gdn = [shard(g["Win"], d.gdn_rows()) for g in w["gdn"]] if self.n_gdn else []
        self.gdn_params = [
            dict(
                taps=g["taps"][d.conv_channels().to(g["taps"].device)].contiguous().to(dev),
                dt=g["dt"][d.r * d.nv : (d.r + 1) * d.nv].contiguous().to(dev),
                neg_a=g["neg_a"][d.r * d.nv : (d.r + 1) * d.nv].contiguous().to(dev),
                norm_w=g["norm_w"].float().contiguous().to(dev),
            )
            for g in (w["gdn"] if self.n_gdn else [])
        ]
        self.w_attn = [shard(a["Win"], d.attn_rows()) for a in w["attn"]] if self.n_attn else []
        self.attn_params = [
            dict(wq=(a["wq"].float() / math.sqrt(HD)).contiguous().to(dev), wk=a["wk"].float().contiguous().to(dev))
            for a in (w["attn"] if self.n_attn else [])
        ]
        self.w_out = [shard(o, None, d.mixer_k()) for o in w["out"]]
        self.w_gu = [shard(stack_matrices(m["G"], m["U"]), d.gateup_rows()) for m in w["mlp"]]
        self.w_down = [shard(m["D"], None, d.mlp_k()) for m in w["mlp"]]
        self.w_head = shard(w["head"], d.vocab_rows()) if self.lm_head else None
        # the MTP draft layer (mtp.py:1-14): layer 0's residual is fc([rmsnorm(e) | rmsnorm(h)]), e the token's
        # embedding row, h the rows of h_d (set_hidden: a previous step's last x); fc canonical [5120, 10240]
        # FP8 with the pre-fc norm weights folded into its columns
        if fc is not None:
            assert self.nranks == 1, "the fc (MTP draft layer) runs on one rank"
            self.w_fc = shard(fc)
        else:
            self.w_fc = None

    def _init_buffers(self, page_table, embed):
        d, dev, max_pos = self.d, self.device, self.max_pos
        # ---- decode state (per state copy)
        R = self.batch
        self.gdn_state = [torch.zeros(R, d.nv, DK, DV, device=dev) for _ in range(self.state_copies[0])]
        self.conv_hist = [
            torch.zeros(R, _lib.QRES_HIST_SLOTS, d.conv, dtype=torch.bfloat16, device=dev)
            for _ in range(self.state_copies[0])
        ]
        npages = R * self.max_pages
        self.k_pool = [torch.zeros(npages, d.nkv, 64, HD, dtype=torch.bfloat16, device=dev) for _ in range(self.state_copies[1])]
        self.v_pool = [torch.zeros(npages, d.nkv, 64, HD, dtype=torch.bfloat16, device=dev) for _ in range(self.state_copies[1])]
        if page_table is None:
            page_table = torch.arange(npages, dtype=torch.int32).view(R, self.max_pages)
        self.page_table = page_table.to(torch.int32).to(dev).contiguous()
        # ---- io
        self.tok_d = torch.zeros(_lib.TOK_WORDS, dtype=torch.int32, device=dev)
        self.x0_d = torch.zeros(R, HIDDEN, device=dev)
        self.x_d = torch.zeros(R, HIDDEN, device=dev)
        self.logits_d = torch.zeros(R, max(d.vocab, 1), dtype=torch.bfloat16, device=dev)
        self.topk_d = torch.zeros(R, 2 * TOP_K, dtype=torch.int32, device=dev)
        self.out_d = torch.zeros(R, 4, dtype=torch.int32, device=dev)
        self.mixer_d = torch.zeros(R, d.gv, dtype=torch.bfloat16, device=dev)
        self.h_d = torch.zeros(R, HIDDEN, device=dev)  # the fc's hidden rows (MTP draft layer)
        self.sampling_d = torch.zeros(R, 4, dtype=torch.int32, device=dev)  # the draw's words (greedy: all 0)
        self.embed = embed.to(dev).bfloat16().contiguous() if embed is not None else None
        cos, sin = rope_table(max_pos)
        self.cos_d, self.sin_d = cos.to(dev), sin.to(dev)

    def _open_p2p(self):
        """the fused peer exchange: allocate this rank's window, all-gather the CUDA IPC handles over the default
        torch.distributed group (every rank constructs its model collectively), map them, then a barrier so no
        rank steps before every window is open"""
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("p2p=True needs an initialised torch.distributed process group (for the handle exchange)")
        L = _lib.lib()
        h = ctypes.create_string_buffer(64)
        _lib.check(L.qres_p2p_alloc(self.ctx, h), self.ctx, "p2p alloc")
        handles = [None] * self.nranks
        dist.all_gather_object(handles, bytes(h.raw))
        allh = ctypes.create_string_buffer(b"".join(handles), 64 * self.nranks)
        _lib.check(L.qres_p2p_open(self.ctx, allh), self.ctx, "p2p open")
        dist.barrier()

    # ------------------------------------------------------------------------------------------ binding
    def _layer_copy(self, l):
        """(kind copy, state copy) of layer l: the k-th layer of its kind uses copy k % copies"""
        k = sum(is_attn(j, self.interval) == is_attn(l, self.interval) for j in range(l))
        if is_attn(l, self.interval):
            return k % len(self.w_attn), k % self.state_copies[1]
        return k % len(self.w_gdn), k % self.state_copies[0]

    def _bind(self):
        L, c = _lib.lib(), self.ctx
        self._state_layer = {}  # (kind, state copy) -> the first layer bound to it (the state entry points' layer)
        for l in range(self.layers):
            wc, sc = self._layer_copy(l)
            self._state_layer.setdefault(("attn" if is_attn(l, self.interval) else "gdn", sc), l)
            m = l % len(self.w_out)
            if is_attn(l, self.interval):
                _lib.check(L.qres_load_weights(c, l, _lib.W_ATTN_IN, ctypes.byref(self.w_attn[wc].cstruct())), c, "w")
                p = self.attn_params[wc]
                _lib.check(L.qres_load_attn_params(c, l, _lib.ptr(p["wq"]), _lib.ptr(p["wk"])), c, "attn params")
                st = _lib.LayerState(0, 0, self.k_pool[sc].data_ptr(), self.v_pool[sc].data_ptr())
            else:
                _lib.check(L.qres_load_weights(c, l, _lib.W_GDN_IN, ctypes.byref(self.w_gdn[wc].cstruct())), c, "w")
                p = self.gdn_params[wc]
                _lib.check(
                    L.qres_load_gdn_params(c, l, _lib.ptr(p["taps"]), _lib.ptr(p["dt"]), _lib.ptr(p["neg_a"]), _lib.ptr(p["norm_w"])),
                    c,
                    "gdn params",
                )
                st = _lib.LayerState(self.gdn_state[sc].data_ptr(), self.conv_hist[sc].data_ptr(), 0, 0)
            _lib.check(L.qres_bind_state(c, l, ctypes.byref(st)), c, "state")
            _lib.check(L.qres_load_weights(c, l, _lib.W_OUT, ctypes.byref(self.w_out[m].cstruct())), c, "w out")
            _lib.check(L.qres_load_weights(c, l, _lib.W_GATEUP, ctypes.byref(self.w_gu[m].cstruct())), c, "w gu")
            _lib.check(L.qres_load_weights(c, l, _lib.W_DOWN, ctypes.byref(self.w_down[m].cstruct())), c, "w down")
        if self.lm_head:
            _lib.check(L.qres_load_weights(c, -1, _lib.W_HEAD, ctypes.byref(self.w_head.cstruct())), c, "w head")
        if self.w_fc is not None:
            _lib.check(L.qres_load_weights(c, -1, _lib.W_FC, ctypes.byref(self.w_fc.cstruct())), c, "w fc")
        _lib.check(L.qres_bind_rope(c, _lib.ptr(self.cos_d), _lib.ptr(self.sin_d), self.max_pos), c, "rope")
        io = _lib.Io(
            self.tok_d.data_ptr(),
            self.x0_d.data_ptr(),
            self.embed.data_ptr() if self.embed is not None else 0,
            self.page_table.data_ptr(),
            self.x_d.data_ptr(),
            self.logits_d.data_ptr() if self.lm_head else 0,
            self.topk_d.data_ptr() if self.lm_head else 0,
            self.out_d.data_ptr() if self.lm_head else 0,
            self.mixer_d.data_ptr(),
            self.h_d.data_ptr() if self.w_fc is not None else 0,
        )
        _lib.check(L.qres_bind_io(c, ctypes.byref(io)), c, "io")
        ops.bind_context(c, self.tok_d, self.x_d, self.out_d)
        if self.lm_head:
            _lib.check(L.qres_bind_sampling(c, _lib.ptr(self.sampling_d)), c, "sampling")

    def set_hidden(self, h, stream=None):
        """the hidden rows the next step's fc reads (MTP draft layer): a [rows, 5120] fp32 device tensor, e.g.
        the main model's x_d or this model's own (copied, so the step may overwrite its source)"""
        s = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(s):
            self.h_d.copy_(h.reshape(self.batch, HIDDEN), non_blocking=True)

    def _count_weight_bytes(self):
        """algorithmic weight bytes one step streams on this rank (FP8 + 4 B per 128x128 block)"""
        b = 0
        for l in range(self.layers):
            wc, _ = self._layer_copy(l)
            m = l % len(self.w_out)
            b += (self.w_attn[wc] if is_attn(l, self.interval) else self.w_gdn[wc]).nbytes
            b += self.w_out[m].nbytes + self.w_gu[m].nbytes + self.w_down[m].nbytes
        if self.lm_head:
            b += self.w_head.nbytes
        return b

    def state_bytes_per_step(self, ctx=None):
        """algorithmic decode-state bytes of one step on this rank: GDN states read + written, conv history
        (3 rows read, 1 written), KV rows read (ctx positions per attention layer) -- per user"""
        d = self.d
        ctx = ctx if ctx is not None else self.max_pos // 2
        gdn = self.n_gdn * (2 * d.nv * DK * DV * 4 + 4 * d.conv * 2)
        kv = self.n_attn * (ctx + 1) * d.nkv * HD * 2 * 2
        return self.batch * (gdn + kv)

    # ------------------------------------------------------------------------------------------ token state
    def token_state(self, x0=None, pos=0, tokens=None, feed=False, slot=0):
        """host token state (model.py:1314-1351): x0 [HIDDEN] or [batch, HIDDEN] rows (bf16 values) or token ids
        (gathered from the embedding on device), at position(s) pos. Verify: pos is row 0's position (rows at
        pos .. pos + batch - 1) and slot the GDN state slot row 0 starts from; after a step at (p, s), continuing
        from row k is (p + k + 1, (s + k) % batch). Returns (words int32 [32], x0 or None)."""
        B = self.batch
        if self.verify:
            p0 = pos[0] if isinstance(pos, (list, tuple)) else pos
            pos = [p0 + r for r in range(B)]
            assert 0 <= slot < B, slot
        pos = [pos] * B if not isinstance(pos, (list, tuple)) else list(pos)
        assert len(pos) == B and all(0 <= p < self.max_pos for p in pos), pos
        words = torch.zeros(_lib.TOK_WORDS, dtype=torch.int32)
        words[_lib.TOK_POS : _lib.TOK_POS + B] = torch.tensor(pos, dtype=torch.int32)
        if tokens is not None:
            tokens = [tokens] * B if not isinstance(tokens, (list, tuple)) else list(tokens)
            assert self.embed is not None, "token rows need the embedding table"
            words[_lib.TOK_TOKEN : _lib.TOK_TOKEN + B] = torch.tensor(tokens, dtype=torch.int32)
            xr = None
        else:
            words[_lib.TOK_TOKEN : _lib.TOK_TOKEN + B] = -1
            xr = x0.reshape(B, HIDDEN).float()
        words[_lib.TOK_FEED] = int(feed)
        words[_lib.TOK_SLOT] = int(slot)
        return words, xr

    def write_token_state(self, tok):
        words, xr = tok
        self.tok_d.copy_(words, non_blocking=True)
        if xr is not None:
            self.x0_d.copy_(xr, non_blocking=True)

    def step(self, tok=None, stream=None):
        """one decode step (async); tok None: continue from the token state the previous step fed (feed mode)"""
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            if tok is not None:
                self.write_token_state(tok)
            torch.ops.qres.decode_step(self.ctx.value, self.tok_d, self.x_d, self.out_d, self.trace)

    def check(self, stream=None):
        """synchronise and raise if a kernel of the step reported an error (timeout / index out of range)"""
        _lib.check(_lib.lib().qres_check(self.ctx, _lib.stream_ptr(stream)), self.ctx, "device")

    @property
    def launches(self):
        """kernels of libqres one step launches"""
        return _lib.lib().qres_step_launches(self.ctx)

    @property
    def exchange(self):
        """the exchange between ranks the step uses: "none" (one rank), "nccl", "tagged" or "counted" words"""
        return _lib.XCHG_NAMES[_lib.lib().qres_exchange_mode(self.ctx)]

    def capture_trace(self, stream=None):
        """record one step as a CUDA graph (model.py:1485-1492); step() then replays it"""
        s = stream or torch.cuda.Stream(device=self.device)
        torch.cuda.synchronize(self.device)
        _lib.check(_lib.lib().qres_capture(self.ctx, _lib.stream_ptr(s)), self.ctx, "capture")
        torch.cuda.synchronize(self.device)
        self.trace = True

    def release_trace(self):
        if self.trace:
            _lib.lib().qres_release_graph(self.ctx)
            self.trace = False

    # ------------------------------------------------------------------------------------------ results
    def x(self):
        """x after the step: [HIDDEN] or [batch, HIDDEN]"""
        x = self.x_d.float().cpu()
        return x[0] if self.batch == 1 else x

    def mixer_output(self):
        """the last layer's mixer output (the out-projection's bf16 input) of this rank: [gv] or [batch, gv]"""
        o = self.mixer_d.float().cpu()
        return o[0] if self.batch == 1 else o

    def logits(self):
        """this rank's logits [vocab / n] (bf16 values) or [batch, vocab / n]"""
        lg = self.logits_d.float().cpu()
        return lg[0] if self.batch == 1 else lg

    def topk(self):
        """the merged top-32 list per row: (keys [batch, 32], vocab indices [batch, 32])"""
        t = self.topk_d.cpu().to(torch.int64) & 0xFFFFFFFF
        return t[:, :TOP_K], t[:, TOP_K:]

    def argmax(self):
        """vocab index of the largest logit, the smallest index on ties (model.py:1558-1573); a list for batch > 1"""
        a = self.out_d[:, 2].cpu().tolist()
        return a[0] if self.batch == 1 else a

    def fed_token(self, user=0):
        """(token, position) the last step fed into the next one: the greedy pick, or the draw when sampling is set"""
        o = self.out_d[user].cpu().tolist()
        return int(o[0]), int(o[1])

    # ------------------------------------------------------------------------------------------ sampling
    @staticmethod
    def sampling_words(temperature=0.0, top_k=1, top_p=1.0, seed=0):
        """the draw's 4 parameter words (model.py:1528-1536): 1 / temperature in Q16 (0 = greedy), top_k (< 1: all
        32; 1 = greedy), top_p in Q16, seed"""
        top_k = TOP_K if top_k < 1 else min(int(top_k), TOP_K)
        inv = min(round(65536 / temperature), 2**31 - 1) if temperature > 0 else 0
        return [inv, top_k, min(max(round(top_p * 65536), 1), 65536), int(seed) & 0xFFFFFFFF]

    def set_sampling(self, temperature=0.0, top_k=1, top_p=1.0, seed=None, user=None):
        """the parameters of the fed token's draw (model.py:1538-1551), read by every later step until set again
        (also a captured graph's replays: the words live in a bound device buffer); user None sets every row.
        seed None picks one."""
        assert self.lm_head, "sampling draws from the lm_head's top-32 list"
        if seed is None:
            seed = int(np.random.randint(0, 2**32, dtype=np.uint64))
        w = torch.from_numpy(np.array(self.sampling_words(temperature, top_k, top_p, seed), dtype=np.uint32).view(np.int32))
        rows = range(self.batch) if user is None else [user]
        for r in rows:
            self.sampling_d[r].copy_(w, non_blocking=False)

    # ------------------------------------------------------------------------------------------ state
    def load_state(self, st, user=0, slot=0):
        """write a decode state (attributes pos, gdn [copies][48,128,128], hist [copies][3, 10240] for positions
        pos-3..pos-1, K / V [copies][4, max_pos, 256]) as user `user`'s (model.py:1447-1470); verify: the one
        user's, its GDN states into state slot `slot`"""
        d, dev = self.d, self.device
        ch = d.conv_channels()
        if self.verify:
            assert user == 0
        L, s = _lib.lib(), _lib.stream_ptr()
        keep = []  # sources stay alive until the copies have run
        for c in range(self.state_copies[0]):
            if c < len(st.gdn):
                S = st.gdn[c][d.r * d.nv : (d.r + 1) * d.nv].to(dev).contiguous()
                h = st.hist[c][:, ch].to(dev).bfloat16().contiguous()
                keep += [S, h]
                _lib.check(L.qres_load_gdn_state(self.ctx, self._state_layer[("gdn", c)], slot if self.verify else user,
                                                 _lib.ptr(S), _lib.ptr(h), st.pos, s), self.ctx, "load gdn state")
        for c in range(self.state_copies[1]):
            P = min(st.pos, st.K[c].shape[1]) if c < len(st.K) else 0
            if P > 0:
                k = st.K[c][d.kv0 : d.kv0 + d.nkv, :P].to(dev).bfloat16().contiguous()  # [nkv, P, 256]
                v = st.V[c][d.kv0 : d.kv0 + d.nkv, :P].to(dev).bfloat16().contiguous()
                keep += [k, v]
                _lib.check(L.qres_load_kv(self.ctx, self._state_layer[("attn", c)], user, _lib.ptr(k), _lib.ptr(v), P, s),
                           self.ctx, "load kv")
        self.check()

    def dump_gdn_state(self, copy=0, user=0):
        """GDN state [48/n, 128, 128] of state copy `copy`: user `user`'s, or (verify) state slot `user`"""
        out = torch.empty(self.d.nv, DK, DV, device=self.device)
        _lib.check(_lib.lib().qres_dump_gdn_state(self.ctx, self._state_layer[("gdn", copy)], user, _lib.ptr(out),
                                                   _lib.stream_ptr()), self.ctx, "dump gdn state")
        return out.cpu()

    def dump_kv(self, copy, npos, user=0):
        """(K, V) rows of positions 0 .. npos-1 of attention state copy `copy`, user `user`: bf16 [nkv, npos, 256]"""
        k = torch.empty(self.d.nkv, npos, HD, dtype=torch.bfloat16, device=self.device)
        v = torch.empty_like(k)
        _lib.check(_lib.lib().qres_dump_kv(self.ctx, self._state_layer[("attn", copy)], user, _lib.ptr(k), _lib.ptr(v),
                                           npos, _lib.stream_ptr()), self.ctx, "dump kv")
        self.check()
        return k.cpu(), v.cpu()

    def kv_rows(self, copy, positions, user=0, which="K"):
        """rows of the paged cache at positions: [nkv, len, 256] float"""
        pool = (self.k_pool if which == "K" else self.v_pool)[copy]
        pt = self.page_table[user].cpu()
        out = [pool[int(pt[p // 64]), :, p % 64].float().cpu() for p in positions]
        return torch.stack(out, 1)

    def reset(self):
        """zero the decode state (GDN states, conv histories, KV pools)"""
        for t in self.gdn_state + self.conv_hist + self.k_pool + self.v_pool:
            t.zero_()

    def close(self):
        if getattr(self, "ctx", None):
            self.release_trace()
            ops.unbind_context(self.ctx)
            _lib.lib().qres_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id():
    """128-byte NCCL id for the ranks' communicator (rank 0 makes it; the caller broadcasts it)"""
    buf = ctypes.create_string_buffer(128)
    _lib.check(_lib.lib().qres_nccl_unique_id(None, buf), None, "nccl id")
    return bytes(buf.raw)
