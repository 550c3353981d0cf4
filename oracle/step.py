"""One resident decode step in fp32 torch on the CPU (TEST INFRASTRUCTURE ONLY).

Restates ``qwen36_resident/model.py:219-292`` (``torch_step``) over the canonical weights of
``oracle/refgen.py``, tensor-parallel over ``n`` ranks exactly as the reference splits chips: every rank
projects its own heads / MLP columns, the row-parallel out- and down-projections give per-rank partials
(rank 0's includes the residual) and x is their sum in rank order (``model.py:279-287``). At n=4 the per-rank
matrices are the reference's per-chip matrices, so the arithmetic is the reference's op for op; any n gives
the same math up to fp32 summation order. bf16 rounding points follow the reference: projections, conv
output, GDN / attention outputs, k rows, SwiGLU product; x, q, the softmax and the logits stay fp32.

Helpers restated: ``rmsnorm``/``bf16`` (model.py:84-90), ``is_attn`` (:93-94), ``rope_tables``/``rope``
(:128-140).
"""
import math

import torch
import torch.nn.functional as F

from oracle.refgen import CONV_CH, DK, DV, GQ, GV, HD, HIDDEN, INTER, NK, NKV, NQ, NV, ROT, bf16

EPS = 1e-6
ROPE_THETA = 10_000_000.0


def rmsnorm(x, w=None):
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS)
    return y if w is None else y * w


def is_attn(l, interval):
    return interval > 0 and (l + 1) % interval == 0


def rope_tables(pos):
    inv = 1.0 / ROPE_THETA ** (torch.arange(0, ROT, 2, dtype=torch.float64) / ROT)
    ang = pos * inv
    return torch.cos(ang).float(), torch.sin(ang).float()


def rope(t, cos, sin):
    h = ROT // 2
    t = t.clone()
    a, b = t[..., :h].clone(), t[..., h:ROT].clone()
    t[..., :h] = a * cos - b * sin
    t[..., h:ROT] = b * cos + a * sin
    return t


class Shard:
    """row / column ranges of rank r of n in the canonical layout (GDN heads, attention heads, MLP columns,
    vocab); KV heads are replicated on 2 ranks when n = 8"""

    def __init__(self, r, n):
        assert n in (1, 2, 4, 8) and 0 <= r < n
        self.r, self.n = r, n
        self.nk, self.nv = NK // n, NV // n
        self.gq, self.gv = self.nk * DK, self.nv * DV
        self.h = NQ // n
        self.nkv = max(NKV // n, 1)
        self.kv0 = (r * NKV) // n if n <= NKV else r // (n // NKV)
        self.ic = INTER // n

    def gdn_rows(self):
        r, gq, gv, nv = self.r, self.gq, self.gv, self.nv
        a0 = 2 * GQ + 2 * GV
        return torch.cat(
            [
                torch.arange(r * gq, (r + 1) * gq),
                GQ + torch.arange(r * gq, (r + 1) * gq),
                2 * GQ + torch.arange(r * gv, (r + 1) * gv),
                2 * GQ + GV + torch.arange(r * gv, (r + 1) * gv),
                a0 + torch.arange(r * nv, (r + 1) * nv),
                a0 + NV + torch.arange(r * nv, (r + 1) * nv),
            ]
        )

    def conv_channels(self):
        r, gq, gv = self.r, self.gq, self.gv
        return torch.cat(
            [
                torch.arange(r * gq, (r + 1) * gq),
                GQ + torch.arange(r * gq, (r + 1) * gq),
                2 * GQ + torch.arange(r * gv, (r + 1) * gv),
            ]
        )

    def attn_rows(self):
        r, aq = self.r, self.h * HD
        k0, v0 = 2 * NQ * HD, 2 * NQ * HD + NKV * HD
        kv = torch.arange(self.kv0 * HD, (self.kv0 + self.nkv) * HD)
        return torch.cat(
            [torch.arange(r * aq, (r + 1) * aq), NQ * HD + torch.arange(r * aq, (r + 1) * aq), k0 + kv, v0 + kv]
        )

    def mixer_cols(self):
        """in-features of the out-projection on this rank (value heads / q heads, both 6144 / n)"""
        return torch.arange(self.r * GV // self.n, (self.r + 1) * GV // self.n)

    def mlp_cols(self):
        return torch.arange(self.r * self.ic, (self.r + 1) * self.ic)

    def vocab_rows(self, vocab):
        per = vocab // self.n
        return torch.arange(self.r * per, (self.r + 1) * per)


class Prepared:
    """per-rank contiguous [in, out] fp32 matrices of the canonical weights (the reference's per-chip weight
    orientation, so that h @ W runs the same matmul as ``torch_step``)"""

    def __init__(self, w, n):
        self.n, self.w = n, w
        self.sh = [Shard(r, n) for r in range(n)]
        T = lambda m: m.T.contiguous()
        self.gdn = [[dict(Win=T(g["Win"][s.gdn_rows()]), taps=g["taps"][s.conv_channels()]) for s in self.sh] for g in w.gdn]
        self.attn = [[T(a["Win"][s.attn_rows()]) for s in self.sh] for a in w.attn]
        self.out = [[T(o[:, s.mixer_cols()]) for s in self.sh] for o in w.out]
        self.mlp = [
            [dict(G=T(m["G"][s.mlp_cols()]), U=T(m["U"][s.mlp_cols()]), D=T(m["D"][:, s.mlp_cols()])) for s in self.sh]
            for m in w.mlp
        ]
        self.head = None
        if w.head is not None:
            V = w.head.shape[0]
            self.head = [T(w.head[s.vocab_rows(V)]) for s in self.sh]


def gdn_mixer(y, s, taps, wg, hist, S_all):
    """the GDN mixer of rank s (model.py:255-276): y the rank's bf16 in-projection row [q|k|v|z|a|b], taps its
    conv taps [conv, 4], wg the layer's dt / neg_a [48] and norm_w, hist [3, conv] (inputs at pos-3..pos-1),
    S_all the layer's states [48, 128, 128] (the rank's heads updated in place). Returns (o, new hist)."""
    conv_l = 2 * s.gq + s.gv
    window = torch.cat([hist, y[:conv_l][None]], 0)  # oldest first
    conv = bf16(F.silu((window * taps.T).sum(0)))
    q, k, v = conv[: s.gq], conv[s.gq : 2 * s.gq], conv[2 * s.gq : conv_l]
    z0 = conv_l
    a0 = z0 + s.gv
    b0 = a0 + s.nv
    z, a, b = y[z0:a0], y[a0:b0], y[b0 : b0 + s.nv]
    scale = DK**-0.5
    outs = []
    for hh in range(s.nv):
        g_h = s.r * s.nv + hh  # global value head
        kh = hh // (s.nv // s.nk)
        qn = q[kh * DK : (kh + 1) * DK]
        qn = qn * torch.rsqrt(qn.pow(2).sum() + 1e-6) * scale
        kn = k[kh * DK : (kh + 1) * DK]
        kn = kn * torch.rsqrt(kn.pow(2).sum() + 1e-6)
        decay = torch.exp(wg["neg_a"][g_h] * F.softplus(a[hh] + wg["dt"][g_h]))
        beta = torch.sigmoid(b[hh])
        S = S_all[g_h]
        delta = beta * (v[hh * DV : (hh + 1) * DV] - (decay * kn) @ S)
        S = decay * S + torch.outer(kn, delta)
        S_all[g_h] = S
        on = rmsnorm(qn @ S, wg["norm_w"])
        outs.append(bf16(on * F.silu(z[hh * DV : (hh + 1) * DV])))
    return torch.cat(outs), window[1:]


def attn_mixer(y, s, wq, wk, K_all, V_all, pos, cos, sin):
    """the gated-attention mixer of rank s (model.py:233-247): y the rank's bf16 row [q|gate|k|v], K_all /
    V_all the layer's caches [4, max_pos, 256] (row pos of the rank's KV heads written). Returns o (bf16)."""
    aq = s.h * HD
    q = y[:aq].view(s.h, HD)
    gate = y[aq : 2 * aq].view(s.h, HD)
    k = y[2 * aq : 2 * aq + s.nkv * HD].view(s.nkv, HD)
    v = y[2 * aq + s.nkv * HD :].view(s.nkv, HD)
    qn = rope(rmsnorm(q, wq / math.sqrt(HD)), cos, sin)
    kn = bf16(rope(rmsnorm(k, wk), cos, sin))
    group = s.h // s.nkv
    outs = []
    for j in range(s.nkv):
        kvh = s.kv0 + j
        K = torch.cat([K_all[kvh][:pos], kn[j][None]])
        V = torch.cat([V_all[kvh][:pos], v[j][None]])
        qj = qn[j * group : (j + 1) * group]
        p = torch.softmax(qj @ K.T, dim=-1)
        outs.append(bf16((p @ V) * torch.sigmoid(gate[j * group : (j + 1) * group])).flatten())
        K_all[kvh][pos] = kn[j]
        V_all[kvh][pos] = v[j]
    return torch.cat(outs)


def torch_step(x0, P, st, layers, interval, lm_head=False, mixer_out=None):
    """one decode step of one user at st.pos over Prepared weights P; updates st (GDN states, conv histories,
    KV rows at pos) in place and returns x (and the per-rank logits with lm_head). mixer_out: a list that
    receives (layer, rank, o) per mixer, o the bf16 input of the out-projection. The k-th layer of a kind uses
    weight copy k % len(weights) and state copy k % len(states) (the reference uses one count for both)."""
    pos = st.pos
    cos, sin = rope_tables(pos)
    x = x0.clone()
    w = P.w
    g_i = a_i = 0
    for l in range(layers):
        h = bf16(rmsnorm(x))
        parts = []
        if is_attn(l, interval):
            c = a_i % len(w.attn)
            cs = a_i % len(st.K)  # the state copy (= the weight copy when their counts match, as in the reference)
            wa = w.attn[c]
            for r, s in enumerate(P.sh):
                y = bf16(h @ P.attn[c][r])
                o = attn_mixer(y, s, wa["wq"], wa["wk"], st.K[cs], st.V[cs], pos, cos, sin)
                if mixer_out is not None:
                    mixer_out.append((l, r, o))
                parts.append(o @ P.out[l % len(w.out)][r] + (x if r == 0 else 0))
            a_i += 1
        else:
            c = g_i % len(w.gdn)
            cs = g_i % len(st.gdn)
            wg = w.gdn[c]
            for r, s in enumerate(P.sh):
                y = bf16(h @ P.gdn[c][r]["Win"])
                ch = s.conv_channels()
                hist = st.hist[cs][:, ch]
                o, st.hist[cs][:, ch] = gdn_mixer(y, s, P.gdn[c][r]["taps"], wg, hist, st.gdn[cs])
                if mixer_out is not None:
                    mixer_out.append((l, r, o))
                parts.append(o @ P.out[l % len(w.out)][r] + (x if r == 0 else 0))
            g_i += 1
        x = sum(parts)
        h = bf16(rmsnorm(x))
        m = P.mlp[l % len(w.mlp)]
        x = sum(
            bf16(F.silu(h @ cm["G"]) * (h @ cm["U"])) @ cm["D"] + (x if r == 0 else 0) for r, cm in enumerate(m)
        )
    st.pos += 1
    if lm_head:
        h = bf16(rmsnorm(x))
        return x, [h @ wh for wh in P.head]
    return x


def logits_bf16(per_rank):
    """concatenated logits in vocab order, rounded to bf16 as the GPU writes them"""
    return bf16(torch.cat(list(per_rank)))
