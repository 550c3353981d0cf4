"""A synthetic Qwen3.6-27B-named checkpoint in memory (test helper): the Hugging Face tensor names and shapes the
loader reads (tt_qwen_resident_b200/checkpoint.py), random bf16 values, and a config; any MLP width."""
import torch

from tt_qwen_resident_b200 import checkpoint as C
from tt_qwen_resident_b200 import weights as W


class DictCheckpoint:
    def __init__(self, tensors, config):
        self.t, self.config = tensors, config

    def get(self, name):
        return self.t[name]

    def layer(self, i, name, prefix=C.PREFIX):
        return self.get(f"{prefix}layers.{i}.{name}")


def fake(layers=2, interval=2, vocab=256, inter=W.INTER, seed=0, mtp=True):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).bfloat16()
    H = W.HIDDEN
    t = {}

    def attn(pre, i):
        t[f"{pre}layers.{i}.input_layernorm.weight"] = rn(H, sc=0.1)
        t[f"{pre}layers.{i}.self_attn.q_proj.weight"] = rn(2 * W.NQ * W.HD, H, sc=H**-0.5)
        t[f"{pre}layers.{i}.self_attn.k_proj.weight"] = rn(W.NKV * W.HD, H, sc=H**-0.5)
        t[f"{pre}layers.{i}.self_attn.v_proj.weight"] = rn(W.NKV * W.HD, H, sc=H**-0.5)
        t[f"{pre}layers.{i}.self_attn.q_norm.weight"] = rn(W.HD, sc=0.1)
        t[f"{pre}layers.{i}.self_attn.k_norm.weight"] = rn(W.HD, sc=0.1)
        t[f"{pre}layers.{i}.self_attn.o_proj.weight"] = rn(H, W.NQ * W.HD, sc=0.5 * (W.NQ * W.HD) ** -0.5)

    def mlp(pre, i):
        t[f"{pre}layers.{i}.post_attention_layernorm.weight"] = rn(H, sc=0.1)
        t[f"{pre}layers.{i}.mlp.gate_proj.weight"] = rn(inter, H, sc=H**-0.5)
        t[f"{pre}layers.{i}.mlp.up_proj.weight"] = rn(inter, H, sc=H**-0.5)
        t[f"{pre}layers.{i}.mlp.down_proj.weight"] = rn(H, inter, sc=0.5 * inter**-0.5)

    for i in range(layers):
        p = C.PREFIX
        if interval > 0 and (i + 1) % interval == 0:
            attn(p, i)
        else:
            t[f"{p}layers.{i}.input_layernorm.weight"] = rn(H, sc=0.1)
            t[f"{p}layers.{i}.linear_attn.in_proj_qkv.weight"] = rn(W.CONV_CH, H, sc=H**-0.5)
            t[f"{p}layers.{i}.linear_attn.in_proj_z.weight"] = rn(W.GV, H, sc=H**-0.5)
            t[f"{p}layers.{i}.linear_attn.in_proj_a.weight"] = rn(W.NV, H, sc=H**-0.5)
            t[f"{p}layers.{i}.linear_attn.in_proj_b.weight"] = rn(W.NV, H, sc=H**-0.5)
            t[f"{p}layers.{i}.linear_attn.conv1d.weight"] = rn(W.CONV_CH, 1, 4, sc=0.5)
            t[f"{p}layers.{i}.linear_attn.dt_bias"] = rn(W.NV, sc=0.5)
            t[f"{p}layers.{i}.linear_attn.A_log"] = (torch.rand(W.NV, generator=g) * 2 - 1).bfloat16()
            t[f"{p}layers.{i}.linear_attn.norm.weight"] = (1 + rn(W.DV, sc=0.1).float()).bfloat16()
            t[f"{p}layers.{i}.linear_attn.out_proj.weight"] = rn(H, W.GV, sc=0.5 * W.GV**-0.5)
        mlp(p, i)
    t[f"{C.PREFIX}norm.weight"] = rn(H, sc=0.1)
    t[f"{C.PREFIX}embed_tokens.weight"] = rn(vocab, H)
    t["lm_head.weight"] = rn(vocab, H, sc=H**-0.5)
    if mtp:
        attn(C.MTP, 0)
        mlp(C.MTP, 0)
        t[f"{C.MTP}norm.weight"] = rn(H, sc=0.1)
        t[f"{C.MTP}pre_fc_norm_embedding.weight"] = rn(H, sc=0.1)
        t[f"{C.MTP}pre_fc_norm_hidden.weight"] = rn(H, sc=0.1)
        t[f"{C.MTP}fc.weight"] = rn(H, 2 * H, sc=(2 * H) ** -0.5)
    cfg = dict(num_hidden_layers=layers, full_attention_interval=interval, vocab_size=vocab, hidden_size=H)
    return DictCheckpoint(t, cfg)
