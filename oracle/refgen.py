"""Seeded random weights and decode state, in the reference's RNG order (TEST INFRASTRUCTURE ONLY).

Restates ``qwen36_resident/model.py:151-174`` (``State``) and ``model.py:177-216`` (``random_weights``): the
reference draws every tensor per chip of a 4-chip tensor-parallel split, in a fixed order, from one CPU
``torch.Generator``. Drawing the same numbers in the same order here gives the reference's exact weights and
state without importing it; they are then re-assembled into the canonical unsharded layout below, which the
oracle (``oracle/step.py``) and the GPU path both consume.

Canonical layout (all projection weights [out_features, in_features]):
  GDN in-proj  [16480, 5120]  rows q(16x128) | k(16x128) | v(48x128) | z(48x128) | a(48) | b(48)
  conv taps    [10240, 4]     channels q | k | v, tap 0 = oldest input
  attn in-proj [14336, 5120]  rows q(24x256) | gate(24x256) | k(4x256) | v(4x256)
  out-proj     [5120, 6144]   in-features = value heads (GDN) or q heads (attention)
  gate / up    [17408, 5120]; down [5120, 17408]; lm_head [vocab, 5120]
State per user: gdn [48, 128, 128] fp32 per GDN copy; hist [3, 10240] (oldest first) per GDN copy;
K, V [4, max_pos, 256] per attention copy (bf16 values, rows >= pos zero).
"""
import math
from dataclasses import dataclass, field

import torch

HIDDEN, INTER = 5120, 17408
NK, NV, DK, DV, CONV_K = 16, 48, 128, 128, 4
NQ, NKV, HD, ROT = 24, 4, 256, 64
REF_CHIPS = 4  # the reference's random_weights / State are drawn per chip of a 4-chip split
GQ, GV = NK * DK, NV * DV  # 2048, 6144
CONV_CH = 2 * GQ + GV  # 10240
GDN_ROWS = 2 * GQ + 2 * GV + 2 * NV  # 16480
ATTN_ROWS = 2 * NQ * HD + 2 * NKV * HD  # 14336


def bf16(t):
    return t.bfloat16().float()


@dataclass
class Canon:
    """canonical (unsharded) fp32 weights; layer l of a kind uses copy (k-th layer of that kind) % copies"""

    gdn: list = field(default_factory=list)  # dict(Win, taps, dt, neg_a, norm_w)
    attn: list = field(default_factory=list)  # dict(Win, wq, wk)
    out: list = field(default_factory=list)  # Wout [5120, 6144]
    mlp: list = field(default_factory=list)  # dict(G, U, D)
    head: torch.Tensor = None  # [vocab, 5120]


@dataclass
class CanonState:
    pos: int
    max_pos: int
    gdn: list  # [48, 128, 128] per GDN copy
    hist: list  # [3, 10240] per GDN copy
    K: list  # [4, max_pos, 256] per attention copy
    V: list


def _chip_dims(n=REF_CHIPS):
    nk, nv = NK // n, NV // n
    gq, gv = nk * DK, nv * DV
    conv = 2 * gq + gv
    return nk, nv, gq, gv, conv


def random_weights(gdn_copies, attn_copies, mlp_copies, vocab=0, seed=0, quant=None):
    """model.py:177-216 drawn per chip (n=4) and assembled canonically; quant (e.g. oracle.fp8.fake_quant) is
    applied to each canonical projection matrix, the stand-in for the reference's per-chip ``quantize``"""
    q_ = quant or (lambda t: t)
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)
    n = REF_CHIPS
    nk, nv, gq, gv, conv = _chip_dims(n)
    b0 = conv + gv + nv
    ic = INTER // n
    w = Canon()
    for _ in range(gdn_copies):
        Win = torch.zeros(GDN_ROWS, HIDDEN)
        taps = torch.zeros(CONV_CH, CONV_K)
        dt, neg_a = torch.zeros(NV), torch.zeros(NV)
        for c in range(n):
            blk = rn(HIDDEN, b0 + nv) / math.sqrt(HIDDEN)  # columns q | k | v | z | a | b of chip c
            t = bf16(0.5 * rn(conv, CONV_K))
            dt[c * nv : (c + 1) * nv] = 0.5 * rn(nv)
            neg_a[c * nv : (c + 1) * nv] = -torch.exp(torch.rand(nv, generator=g) * 2 - 1)
            cols = blk.T  # [rows, HIDDEN]
            Win[c * gq : (c + 1) * gq] = cols[0:gq]
            Win[GQ + c * gq : GQ + (c + 1) * gq] = cols[gq : 2 * gq]
            Win[2 * GQ + c * gv : 2 * GQ + (c + 1) * gv] = cols[2 * gq : conv]
            Win[2 * GQ + GV + c * gv : 2 * GQ + GV + (c + 1) * gv] = cols[conv : conv + gv]
            a0 = 2 * GQ + 2 * GV
            Win[a0 + c * nv : a0 + (c + 1) * nv] = cols[conv + gv : conv + gv + nv]
            Win[a0 + NV + c * nv : a0 + NV + (c + 1) * nv] = cols[conv + gv + nv : conv + gv + 2 * nv]
            taps[c * gq : (c + 1) * gq] = t[0:gq]
            taps[GQ + c * gq : GQ + (c + 1) * gq] = t[gq : 2 * gq]
            taps[2 * GQ + c * gv : 2 * GQ + (c + 1) * gv] = t[2 * gq : conv]
        norm_w = bf16(1 + 0.1 * rn(DV))
        w.gdn.append(dict(Win=q_(Win), taps=taps, dt=dt, neg_a=neg_a, norm_w=norm_w))
    h = NQ // n
    aq = h * HD
    for _ in range(attn_copies):
        Win = torch.zeros(ATTN_ROWS, HIDDEN)
        for c in range(n):
            cols = (rn(HIDDEN, 2 * aq + 2 * HD) / math.sqrt(HIDDEN)).T
            Win[c * aq : (c + 1) * aq] = cols[0:aq]
            Win[NQ * HD + c * aq : NQ * HD + (c + 1) * aq] = cols[aq : 2 * aq]
            Win[2 * NQ * HD + c * HD : 2 * NQ * HD + (c + 1) * HD] = cols[2 * aq : 2 * aq + HD]
            Win[2 * NQ * HD + NKV * HD + c * HD : 2 * NQ * HD + NKV * HD + (c + 1) * HD] = cols[2 * aq + HD :]
        wq, wk = bf16(1 + 0.1 * rn(HD)), bf16(1 + 0.1 * rn(HD))
        w.attn.append(dict(Win=q_(Win), wq=wq, wk=wk))
    for _ in range(mlp_copies):
        Wout = torch.zeros(HIDDEN, GV)
        for c in range(n):
            Wout[:, c * gv : (c + 1) * gv] = (rn(gv, HIDDEN) * (0.5 / math.sqrt(gv))).T
        w.out.append(q_(Wout))
        G, U, D = torch.zeros(INTER, HIDDEN), torch.zeros(INTER, HIDDEN), torch.zeros(HIDDEN, INTER)
        for c in range(n):
            G[c * ic : (c + 1) * ic] = (rn(HIDDEN, ic) / math.sqrt(HIDDEN)).T
            U[c * ic : (c + 1) * ic] = (rn(HIDDEN, ic) / math.sqrt(HIDDEN)).T
            D[:, c * ic : (c + 1) * ic] = (rn(ic, HIDDEN) * (0.5 / math.sqrt(ic))).T
        w.mlp.append(dict(G=q_(G), U=q_(U), D=q_(D)))
    if vocab:
        assert vocab % n == 0
        per = vocab // n
        head = torch.zeros(vocab, HIDDEN)
        for c in range(n):
            head[c * per : (c + 1) * per] = (rn(HIDDEN, per) / math.sqrt(HIDDEN)).T
        w.head = q_(head)
    return w


def random_state(gdn_copies, attn_copies, pos, max_pos, seed=1, zero=False):
    """model.py:151-174 drawn per chip (n=4) and assembled canonically (KV rows rounded to bf16, the GPU's KV
    dtype, in place of the reference's bf8)"""
    g = torch.Generator().manual_seed(seed)
    rn = (lambda *s: torch.zeros(*s)) if zero else (lambda *s: torch.randn(*s, generator=g))
    n = REF_CHIPS
    nk, nv, gq, gv, conv = _chip_dims(n)
    gdn = []
    for _ in range(gdn_copies):
        gdn.append(torch.cat([0.05 * rn(nv, DK, DV) for _ in range(n)]))
    hist = []
    for _ in range(gdn_copies):
        hh = torch.zeros(CONV_K - 1, CONV_CH)
        for c in range(n):
            t = bf16(rn(CONV_K - 1, conv))
            hh[:, c * gq : (c + 1) * gq] = t[:, 0:gq]
            hh[:, GQ + c * gq : GQ + (c + 1) * gq] = t[:, gq : 2 * gq]
            hh[:, 2 * GQ + c * gv : 2 * GQ + (c + 1) * gv] = t[:, 2 * gq :]
        hist.append(hh)
    K, V = [], []
    for _ in range(attn_copies):
        ks, vs = [], []
        for _ in range(n):  # chip c holds KV head c
            k, v = bf16(rn(max_pos, HD)), bf16(rn(max_pos, HD))
            k[pos:], v[pos:] = 0, 0
            ks.append(k)
            vs.append(v)
        K.append(torch.stack(ks))
        V.append(torch.stack(vs))
    return CanonState(pos=pos, max_pos=max_pos, gdn=gdn, hist=hist, K=K, V=V)


def clone_state(st):
    return CanonState(
        pos=st.pos,
        max_pos=st.max_pos,
        gdn=[t.clone() for t in st.gdn],
        hist=[t.clone() for t in st.hist],
        K=[t.clone() for t in st.K],
        V=[t.clone() for t in st.V],
    )
