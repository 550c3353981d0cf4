"""A Qwen3.6-27B Hugging Face checkpoint -> the canonical FP8 weights ResidentModel shards (weights.py).

The reference's loader (qwen36_resident/weights.py:46-257, and the MTP layer's in mtp.py:33-69) reads the
safetensors checkpoint and cuts it per chip; here the loader keeps the canonical unsharded layout and
``ResidentModel`` / ``weights.shard`` cut the rank's rows, so one conversion serves every tensor-parallel size.
The same foldings: every (1 + w) RMSNorm weight goes into the columns of the projection that follows it (the
input norm into the in-projection, the post-attention norm into gate and up, the final norm into the lm_head, the
MTP layer's pre-fc norms into the fc's embedding / hidden halves and its own norm into its copy of the lm_head);
the q / k head norms become (1 + w) in bf16; neg_A = -exp(A_log); the GDN gated norm weight is used as is.
Projections are folded in fp32 and then quantised to FP8-e4m3 with one fp32 scale per 128 x 128 block on the
GPU (qres_quantize_fp8).

Canonical rows (weights.py): GDN in-proj q | k | v | z | a | b from in_proj_qkv (q | k | v), in_proj_z, in_proj_a,
in_proj_b; attention in-proj q | gate | k | v, q and gate de-interleaved from q_proj's per-head [q | gate] rows.
"""
import json
import os

import torch

from . import weights as W

PREFIX = "model.language_model."
MTP = "mtp."


class Checkpoint:
    """a local safetensors checkpoint directory (model.safetensors.index.json + config.json)"""

    def __init__(self, path):
        from safetensors import safe_open

        self.path = path
        self._open = safe_open
        self.index = json.load(open(os.path.join(path, "model.safetensors.index.json")))["weight_map"]
        cfg = json.load(open(os.path.join(path, "config.json")))
        self.config = cfg.get("text_config", cfg)
        self._files = {}

    def get(self, name):
        f = self.index[name]
        if f not in self._files:
            self._files[f] = self._open(os.path.join(self.path, f), framework="pt")
        return self._files[f].get_tensor(name)

    def layer(self, i, name, prefix=PREFIX):
        return self.get(f"{prefix}layers.{i}.{name}")


def _fold(norm_w, w):
    """w [N, K] with its columns scaled by (1 + norm_w) [K], fp32"""
    return w.float() * (1.0 + norm_w.float())[None, :]


def gdn_layer(ck, i, prefix=PREFIX):
    """fp32 canonical GDN mixer of layer i: in-proj (input norm folded), conv taps, dt, neg_a, gated-norm weight"""
    L = lambda n: ck.layer(i, n, prefix)
    ln = L("input_layernorm.weight")
    win = torch.cat([L("linear_attn.in_proj_qkv.weight"), L("linear_attn.in_proj_z.weight"),
                     L("linear_attn.in_proj_a.weight"), L("linear_attn.in_proj_b.weight")])
    assert win.shape == (W.GDN_ROWS, W.HIDDEN), win.shape
    return dict(
        Win=_fold(ln, win),
        taps=L("linear_attn.conv1d.weight")[:, 0].float().bfloat16().float(),  # [10240, 4], tap 0 = oldest
        dt=L("linear_attn.dt_bias").float(),
        neg_a=-L("linear_attn.A_log").float().exp(),
        norm_w=L("linear_attn.norm.weight").float().bfloat16().float(),
    )


def attn_layer(ck, i, prefix=PREFIX):
    """fp32 canonical attention mixer of layer i: in-proj q | gate | k | v (input norm folded), (1 + q / k norm)"""
    L = lambda n: ck.layer(i, n, prefix)
    ln = L("input_layernorm.weight")
    qg = L("self_attn.q_proj.weight").reshape(W.NQ, 2, W.HD, -1)  # per head [q | gate]
    win = torch.cat([qg[:, 0].reshape(W.NQ * W.HD, -1), qg[:, 1].reshape(W.NQ * W.HD, -1), L("self_attn.k_proj.weight"),
                     L("self_attn.v_proj.weight")])
    assert win.shape == (W.ATTN_ROWS, W.HIDDEN), win.shape
    return dict(Win=_fold(ln, win), wq=(1.0 + L("self_attn.q_norm.weight").float()).bfloat16().float(),
                wk=(1.0 + L("self_attn.k_norm.weight").float()).bfloat16().float())


def out_proj(ck, i, attn, prefix=PREFIX):
    return ck.layer(i, "self_attn.o_proj.weight" if attn else "linear_attn.out_proj.weight", prefix).float()


def mlp(ck, i, prefix=PREFIX):
    L = lambda n: ck.layer(i, n, prefix)
    ln = L("post_attention_layernorm.weight")
    return dict(G=_fold(ln, L("mlp.gate_proj.weight")), U=_fold(ln, L("mlp.up_proj.weight")),
                D=L("mlp.down_proj.weight").float())


def lm_head(ck, norm_name=f"{PREFIX}norm.weight"):
    return _fold(ck.get(norm_name), ck.get("lm_head.weight"))


def embedding(ck):
    """the token embedding table [vocab, 5120] bf16"""
    return ck.get(f"{PREFIX}embed_tokens.weight").bfloat16()


def _quantize_all(fp32, device):
    Q = lambda t: W.quantize(t.to(device))
    out = dict(gdn=[], attn=[], out=[], mlp=[], head=None)
    for g in fp32["gdn"]:
        out["gdn"].append(dict(Win=Q(g["Win"]), taps=g["taps"].to(device).bfloat16(), dt=g["dt"].to(device),
                               neg_a=g["neg_a"].to(device), norm_w=g["norm_w"].to(device)))
    for a in fp32["attn"]:
        out["attn"].append(dict(Win=Q(a["Win"]), wq=a["wq"].to(device), wk=a["wk"].to(device)))
    out["out"] = [Q(o) for o in fp32["out"]]
    out["mlp"] = [dict(G=Q(m["G"]), U=Q(m["U"]), D=Q(m["D"])) for m in fp32["mlp"]]
    if fp32.get("head") is not None:
        out["head"] = Q(fp32["head"])
    return out


def canonical_fp32(ck, layers=None, with_head=True):
    """the first `layers` layers (default all) in the canonical layout, fp32 (every layer its own copy)"""
    layers = layers or int(ck.config["num_hidden_layers"])
    interval = int(ck.config["full_attention_interval"])
    w = dict(gdn=[], attn=[], out=[], mlp=[], head=None)
    for i in range(layers):
        attn = interval > 0 and (i + 1) % interval == 0
        (w["attn"] if attn else w["gdn"]).append(attn_layer(ck, i) if attn else gdn_layer(ck, i))
        w["out"].append(out_proj(ck, i, attn))
        w["mlp"].append(mlp(ck, i))
    if with_head:
        w["head"] = lm_head(ck)
    return w


def load(ck, layers=None, device="cuda", with_head=True):
    """canonical FP8 weights for ResidentModel(w, layers, full_attention_interval, ...), quantised on the GPU one
    layer at a time (the fp32 copy of one layer at a time on the host)"""
    layers = layers or int(ck.config["num_hidden_layers"])
    interval = int(ck.config["full_attention_interval"])
    out = dict(gdn=[], attn=[], out=[], mlp=[], head=None)
    for i in range(layers):
        attn = interval > 0 and (i + 1) % interval == 0
        one = dict(gdn=[] if attn else [gdn_layer(ck, i)], attn=[attn_layer(ck, i)] if attn else [],
                   out=[out_proj(ck, i, attn)], mlp=[mlp(ck, i)], head=None)
        q = _quantize_all(one, device)
        for k in ("gdn", "attn", "out", "mlp"):
            out[k] += q[k]
    if with_head:
        out["head"] = W.quantize(lm_head(ck).to(device))
    return out


def mtp_fp32(ck):
    """the MTP draft layer (mtp.py:33-69): one attention decoder layer under mtp.layers.0, its copy of the lm_head
    folded with mtp.norm, and the fc [5120, 10240] over [embedding | hidden] with the pre-fc norms folded"""
    w = dict(gdn=[], attn=[attn_layer(ck, 0, MTP)], out=[out_proj(ck, 0, True, MTP)], mlp=[mlp(ck, 0, MTP)],
             head=lm_head(ck, f"{MTP}norm.weight"))
    scale = 1.0 + torch.cat([ck.get(f"{MTP}pre_fc_norm_embedding.weight").float(),
                             ck.get(f"{MTP}pre_fc_norm_hidden.weight").float()])
    fc = ck.get(f"{MTP}fc.weight").float() * scale[None, :]
    return w, fc


def load_mtp(ck, device="cuda"):
    """(canonical FP8 weights of the draft model, the fc as an FP8Matrix) for ResidentModel(..., fc=fc)"""
    w, fc = mtp_fp32(ck)
    return _quantize_all(w, device), W.quantize(fc.to(device))
