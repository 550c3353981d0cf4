"""The checkpoint loader's name mapping and foldings on the CPU (tt_qwen_resident_b200/checkpoint.py, after the
reference's qwen36_resident/weights.py:46-257 and mtp.py:33-69): canonical rows assembled from the Hugging Face
tensors, (1 + w) norm weights folded into the following projection's columns, q / gate de-interleaved per head,
neg_A = -exp(A_log), the MTP fc's pre-fc norms; and the safetensors-backed Checkpoint reading a directory."""
import json

import torch
from safetensors.torch import save_file

from ckpt_fake import fake
from tt_qwen_resident_b200 import checkpoint as C
from tt_qwen_resident_b200 import weights as W


def test_mapping_and_folding():
    ck = fake(layers=2, interval=2, vocab=64, inter=256)
    w = C.canonical_fp32(ck)
    assert len(w["gdn"]) == 1 and len(w["attn"]) == 1 and len(w["out"]) == 2 and len(w["mlp"]) == 2
    f = lambda n: ck.t[n].float()
    p = C.PREFIX + "layers.0."
    ln = 1 + f(p + "input_layernorm.weight")
    g = w["gdn"][0]
    qkv = f(p + "linear_attn.in_proj_qkv.weight")
    assert torch.equal(g["Win"][: W.CONV_CH], qkv * ln)  # q | k | v
    assert torch.equal(g["Win"][W.CONV_CH : W.CONV_CH + W.GV], f(p + "linear_attn.in_proj_z.weight") * ln)
    assert torch.equal(g["Win"][-2 * W.NV : -W.NV], f(p + "linear_attn.in_proj_a.weight") * ln)
    assert torch.equal(g["Win"][-W.NV :], f(p + "linear_attn.in_proj_b.weight") * ln)
    assert torch.equal(g["taps"], f(p + "linear_attn.conv1d.weight")[:, 0])
    assert torch.equal(g["neg_a"], -f(p + "linear_attn.A_log").exp())
    assert torch.equal(g["norm_w"], f(p + "linear_attn.norm.weight"))  # the gated norm takes w as is
    p1 = C.PREFIX + "layers.1."
    ln1 = 1 + f(p1 + "input_layernorm.weight")
    a = w["attn"][0]
    qg = f(p1 + "self_attn.q_proj.weight").view(W.NQ, 2, W.HD, W.HIDDEN)
    h = 5  # query head 5: its q rows, then (after all q heads) its gate rows
    assert torch.equal(a["Win"][h * W.HD : (h + 1) * W.HD], qg[h, 0] * ln1)
    assert torch.equal(a["Win"][(W.NQ + h) * W.HD : (W.NQ + h + 1) * W.HD], qg[h, 1] * ln1)
    assert torch.equal(a["Win"][2 * W.NQ * W.HD : 2 * W.NQ * W.HD + W.NKV * W.HD], f(p1 + "self_attn.k_proj.weight") * ln1)
    assert torch.equal(a["wq"], (1 + f(p1 + "self_attn.q_norm.weight")).bfloat16().float())
    assert torch.equal(w["out"][1], f(p1 + "self_attn.o_proj.weight"))
    assert torch.equal(w["out"][0], f(p + "linear_attn.out_proj.weight"))
    pa = 1 + f(p1 + "post_attention_layernorm.weight")
    assert torch.equal(w["mlp"][1]["G"], f(p1 + "mlp.gate_proj.weight") * pa)
    assert torch.equal(w["mlp"][1]["D"], f(p1 + "mlp.down_proj.weight"))
    assert torch.equal(w["head"], f("lm_head.weight") * (1 + f(C.PREFIX + "norm.weight")))
    wm, fc = C.mtp_fp32(ck)
    sc = 1 + torch.cat([f(C.MTP + "pre_fc_norm_embedding.weight"), f(C.MTP + "pre_fc_norm_hidden.weight")])
    assert torch.equal(fc, f(C.MTP + "fc.weight") * sc)
    assert torch.equal(wm["head"], f("lm_head.weight") * (1 + f(C.MTP + "norm.weight")))


def test_safetensors_directory(tmp_path):
    t = {"a.weight": torch.randn(4, 8).bfloat16(), "b.weight": torch.randn(3).bfloat16()}
    save_file({"a.weight": t["a.weight"]}, str(tmp_path / "model-00001.safetensors"))
    save_file({"b.weight": t["b.weight"]}, str(tmp_path / "model-00002.safetensors"))
    json.dump({"weight_map": {"a.weight": "model-00001.safetensors", "b.weight": "model-00002.safetensors"}},
              open(tmp_path / "model.safetensors.index.json", "w"))
    json.dump({"text_config": {"num_hidden_layers": 64, "full_attention_interval": 4}}, open(tmp_path / "config.json", "w"))
    ck = C.Checkpoint(str(tmp_path))
    assert ck.config["full_attention_interval"] == 4
    assert torch.equal(ck.get("a.weight"), t["a.weight"]) and torch.equal(ck.get("b.weight"), t["b.weight"])
