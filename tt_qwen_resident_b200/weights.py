"""Canonical FP8 weights -> the per-rank GEMV layout of libqres.

Mirrors the reference's checkpoint-to-shard step (qwen36_resident/weights.py): chip c of n holds GDN key heads
[16c/n, ...), value heads [48c/n, ...), attention query heads [24c/n, ...) and their KV head(s), MLP columns
[17408c/n, ...) and lm_head vocab rows [Vc/n, ...); the out- and down-projections are row-parallel (their K is
split). Norm weights are folded into the following projection before quantisation (weights.py:162-164), so
the GPU applies a plain rmsnorm.

Canonical layout (projection weights [out_features, in_features], FP8-e4m3 + one fp32 scale per 128x128 block):
  GDN in-proj  [16480, 5120]  rows q(16x128) | k(16x128) | v(48x128) | z(48x128) | a(48) | b(48)
  attn in-proj [14336, 5120]  rows q(24x256) | gate(24x256) | k(4x256) | v(4x256)
  out-proj [5120, 6144], gate / up [17408, 5120], down [5120, 17408], lm_head [vocab, 5120]
A rank's projection keeps the canonical quantisation: its rows (and K range) are gathered, every row keeps
the scale of its canonical 128-row block, and the bytes are re-laid into the GEMV's layout (128-row tiles of
16 KB units, see ``scale_table`` for the scales).
"""
import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib

HIDDEN, INTER = 5120, 17408
NK, NV, DK, DV = 16, 48, 128, 128
NQ, NKV, HD = 24, 4, 256
GQ, GV = NK * DK, NV * DV
CONV_CH = 2 * GQ + GV
GDN_ROWS = 2 * GQ + 2 * GV + 2 * NV
ATTN_ROWS = 2 * NQ * HD + 2 * NKV * HD


@dataclass
class FP8Matrix:
    """canonical block-scaled FP8 matrix: q uint8 [N, K] (e4m3 bits), scales fp32 [ceil(N/128), K/128]"""

    q: torch.Tensor
    scales: torch.Tensor

    @property
    def shape(self):
        return tuple(self.q.shape)


@dataclass
class GemvWeight:
    """one rank's projection in the GEMV layout (device tensors)"""

    data: torch.Tensor  # uint8 [rows_pad * K]
    uscale: torch.Tensor  # uint8 [rows_pad / 128, 128 + (K / 128) * 32]: the scale table (scale_table)
    rows: int
    K: int

    @property
    def rows_pad(self):
        return (self.rows + 127) // 128 * 128

    def cstruct(self):
        return _lib.Weight(self.data.data_ptr(), self.uscale.data_ptr(), self.rows, self.rows_pad, self.K, 0)

    @property
    def nbytes(self):
        """algorithmic bytes: 1 per weight plus 4 per 128 x 128 block"""
        return self.rows * self.K + 4 * math.ceil(self.rows / 128) * (self.K // 128)


class RankDims:
    """the slices of rank r of n (heads, columns, vocab) in the canonical layout"""

    def __init__(self, r, n, vocab=0):
        assert n in (1, 2, 4, 8) and 0 <= r < n
        self.r, self.n = r, n
        self.nk, self.nv = NK // n, NV // n
        self.gq, self.gv = self.nk * DK, self.nv * DV
        self.conv = 2 * self.gq + self.gv
        self.h = NQ // n
        self.nkv = max(NKV // n, 1)
        self.kv0 = (r * NKV) // n if n <= NKV else r // (n // NKV)
        self.ic = INTER // n
        self.vocab = vocab // n if vocab else 0
        self.gdn_rows_n = 2 * self.gq + 2 * self.gv + 2 * self.nv
        self.attn_rows_n = 2 * self.h * HD + 2 * self.nkv * HD

    def gdn_rows(self):
        r, gq, gv, nv = self.r, self.gq, self.gv, self.nv
        a0 = 2 * GQ + 2 * GV
        ar = torch.arange
        return torch.cat(
            [
                ar(r * gq, (r + 1) * gq),
                GQ + ar(r * gq, (r + 1) * gq),
                2 * GQ + ar(r * gv, (r + 1) * gv),
                2 * GQ + GV + ar(r * gv, (r + 1) * gv),
                a0 + ar(r * nv, (r + 1) * nv),
                a0 + NV + ar(r * nv, (r + 1) * nv),
            ]
        )

    def conv_channels(self):
        r, gq, gv = self.r, self.gq, self.gv
        ar = torch.arange
        return torch.cat([ar(r * gq, (r + 1) * gq), GQ + ar(r * gq, (r + 1) * gq), 2 * GQ + ar(r * gv, (r + 1) * gv)])

    def attn_rows(self):
        r, aq = self.r, self.h * HD
        k0, v0 = 2 * NQ * HD, 2 * NQ * HD + NKV * HD
        kv = torch.arange(self.kv0 * HD, (self.kv0 + self.nkv) * HD)
        ar = torch.arange
        return torch.cat([ar(r * aq, (r + 1) * aq), NQ * HD + ar(r * aq, (r + 1) * aq), k0 + kv, v0 + kv])

    def mixer_k(self):
        return self.r * GV // self.n, (self.r + 1) * GV // self.n

    def mlp_k(self):
        return self.r * self.ic, (self.r + 1) * self.ic

    def gateup_rows(self):
        """rows of cat(G, U) interleaved in pairs: G[2j], G[2j+1], U[2j], U[2j+1] (the SwiGLU epilogue's quads)"""
        g = torch.arange(self.r * self.ic, (self.r + 1) * self.ic).view(-1, 2)
        return torch.cat([g, INTER + g], 1).reshape(-1)

    def vocab_rows(self):
        return torch.arange(self.r * self.vocab, (self.r + 1) * self.vocab)


def quantize(w):
    """fp32 [N, K] -> FP8Matrix, on the GPU (libqres) when w is a CUDA tensor"""
    assert w.is_cuda, "quantize runs on the GPU (qres_quantize_fp8)"
    q, s = _lib.quantize_fp8(w.float().contiguous())
    return FP8Matrix(q, s)


def scale_table(blk, scales, kb0, kb1):
    """The GEMV's scale table of one projection: blk = canonical 128-row block of every local row (LongTensor,
    length rows), scales = the canonical fp32 block scales [row blocks][K / 128], K blocks [kb0, kb1) kept.
    Per 128-row tile: 128 bytes of row selectors (row r's block is the tile's slot sel[r] of at most 8), then for
    every K block the 8 slots' scales (fp32; unused slots 0). uint8 [tiles, 128 + (kb1 - kb0) * 32]."""
    n = blk.numel()
    tiles = -(-n // 128)
    b = torch.empty(tiles * 128, dtype=torch.long, device=blk.device)
    b[:n] = blk
    b[n:] = blk[n - 1]  # padding rows reuse a slot of the tile
    b = b.view(tiles, 128)
    srt = b.sort(dim=1).values
    new = torch.ones_like(srt, dtype=torch.long)
    new[:, 1:] = (srt[:, 1:] != srt[:, :-1]).long()
    rank = new.cumsum(1) - 1  # slot of each distinct block, in ascending block order
    sel = torch.gather(rank, 1, torch.searchsorted(srt, b))
    if int(sel.max()) >= 8:
        raise ValueError("a 128-row tile holds rows of more than 8 canonical scale blocks")
    slot_blk = b[:, :1].repeat(1, 8)
    slot_blk.scatter_(1, sel, b)
    used = torch.zeros(tiles, 8, dtype=torch.bool, device=blk.device)
    used.scatter_(1, sel, True)
    sc = scales.to(blk.device, torch.float32)[:, kb0:kb1]
    tab = sc[slot_blk] * used.unsqueeze(-1)  # [tiles, 8, nkb]
    tab = tab.transpose(1, 2).contiguous()  # [tiles, nkb, 8]
    return torch.cat([sel.to(torch.uint8), tab.view(tiles, -1).view(torch.uint8)], dim=1).contiguous()


def shard(m, rows=None, k=None, device="cuda"):
    """rank projection of canonical m: rows (LongTensor of canonical rows; None = all), k = (k0, k1) K range.
    Every 128-row tile may hold rows of at most 8 canonical 128-row scale blocks (the shards of this model hold
    at most 4: head / column slices, gate|up interleaved pairs)."""
    q, sc = m.q, m.scales
    N, K = q.shape
    rows = torch.arange(N) if rows is None else rows
    k0, k1 = k if k is not None else (0, K)
    assert k0 % 128 == 0 and k1 % 128 == 0
    rows_d = rows.to(q.device)
    ql = q.index_select(0, rows_d)[:, k0:k1].contiguous().to(device)
    table = scale_table(rows.to(device) // 128, sc, k0 // 128, k1 // 128)
    data = _lib.tile_weight(ql)
    return GemvWeight(data=data, uscale=table, rows=len(rows), K=k1 - k0)


def stack_matrices(a, b):
    """canonical cat(a, b) along rows (for gate | up): scales stacked by 128-row blocks (a's rows a multiple of
    128)"""
    assert a.q.shape[0] % 128 == 0
    return FP8Matrix(torch.cat([a.q, b.q]), torch.cat([a.scales, b.scales]))


def random_canonical(layers, interval, vocab, seed=0, device="cuda", copies=None, std=None):
    """random-init canonical weights of the named shape on the GPU (bench / large tests), quantised with libqres.
    Scales follow the reference's random_weights (model.py:177-216); std (e.g. 0.02) overrides the projections'.
    copies: (gdn, attn, mlp) distinct layers per kind (None: every layer distinct)."""
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, device=device)
    n_attn = sum(interval > 0 and (l + 1) % interval == 0 for l in range(layers))
    n_gdn = layers - n_attn
    cg, ca, cm = copies or (n_gdn, n_attn, layers)
    s = (lambda d: std) if std else (lambda d: d)
    w = dict(gdn=[], attn=[], mlp=[], out=[], head=None)
    for _ in range(cg):
        Win = rn(GDN_ROWS, HIDDEN) * s(1 / math.sqrt(HIDDEN))
        w["gdn"].append(
            dict(
                Win=quantize(Win),
                taps=(0.5 * rn(CONV_CH, 4)).bfloat16(),
                dt=0.5 * rn(NV),
                neg_a=-torch.exp(torch.rand(NV, generator=g, device=device) * 2 - 1),
                norm_w=(1 + 0.1 * rn(DV)).bfloat16().float(),
            )
        )
        del Win
    for _ in range(ca):
        Win = rn(ATTN_ROWS, HIDDEN) * s(1 / math.sqrt(HIDDEN))
        w["attn"].append(
            dict(Win=quantize(Win), wq=(1 + 0.1 * rn(HD)).bfloat16().float(), wk=(1 + 0.1 * rn(HD)).bfloat16().float())
        )
        del Win
    for _ in range(cm):
        w["out"].append(quantize(rn(HIDDEN, GV) * s(0.5 / math.sqrt(GV))))
        G = quantize(rn(INTER, HIDDEN) * s(1 / math.sqrt(HIDDEN)))
        U = quantize(rn(INTER, HIDDEN) * s(1 / math.sqrt(HIDDEN)))
        D = quantize(rn(HIDDEN, INTER) * s(0.5 / math.sqrt(INTER)))
        w["mlp"].append(dict(G=G, U=U, D=D))
    if vocab:
        head = torch.empty(vocab, HIDDEN, dtype=torch.uint8, device=device)
        nb = -(-vocab // 128)
        scales = torch.empty(nb, HIDDEN // 128, dtype=torch.float32, device=device)
        step = 128 * 256  # quantise in slabs (fp32 of the whole head is 5 GB)
        for r0 in range(0, vocab, step):
            r1 = min(vocab, r0 + step)
            m = quantize(rn(r1 - r0, HIDDEN) * s(1 / math.sqrt(HIDDEN)))
            head[r0:r1] = m.q
            scales[r0 // 128 : r0 // 128 + m.scales.shape[0]] = m.scales
        w["head"] = FP8Matrix(head, scales)
    return w


def canonical_from_fp32(w32, device="cuda"):
    """canonical FP8 weights from an fp32 canonical weight set (attributes gdn / attn / out / mlp / head, the
    layout above), quantised on the GPU"""
    Q = lambda t: quantize(t.to(device))
    return dict(
        gdn=[
            dict(
                Win=Q(g["Win"]),
                taps=g["taps"].to(device).bfloat16(),
                dt=g["dt"].to(device).float(),
                neg_a=g["neg_a"].to(device).float(),
                norm_w=g["norm_w"].to(device).float(),
            )
            for g in w32.gdn
        ],
        attn=[dict(Win=Q(a["Win"]), wq=a["wq"].to(device).float(), wk=a["wk"].to(device).float()) for a in w32.attn],
        out=[Q(o) for o in w32.out],
        mlp=[dict(G=Q(m["G"]), U=Q(m["U"]), D=Q(m["D"])) for m in w32.mlp],
        head=Q(w32.head) if w32.head is not None else None,
    )


def canonical_from_fp8(w8, device="cuda"):
    """canonical FP8 weights from (q uint8, scales) pairs quantised elsewhere (same structure, each projection a
    (q, scales) tuple)"""
    M = lambda t: FP8Matrix(t[0].to(device), t[1].to(device).float())
    return dict(
        gdn=[
            dict(
                Win=M(g["Win"]),
                taps=g["taps"].to(device).bfloat16(),
                dt=g["dt"].to(device).float(),
                neg_a=g["neg_a"].to(device).float(),
                norm_w=g["norm_w"].to(device).float(),
            )
            for g in w8["gdn"]
        ],
        attn=[dict(Win=M(a["Win"]), wq=a["wq"].to(device).float(), wk=a["wk"].to(device).float()) for a in w8["attn"]],
        out=[M(o) for o in w8["out"]],
        mlp=[dict(G=M(m["G"]), U=M(m["U"]), D=M(m["D"])) for m in w8["mlp"]],
        head=M(w8["head"]) if w8.get("head") is not None else None,
    )
