"""A model built from a (synthetic) Qwen3.6-27B-named checkpoint through the loader (checkpoint.load: name mapping,
norm folding, FP8 quantisation on the GPU) steps like the oracle on the same weights: one G A step with the lm_head,
x and logits within 2e-2 relative (test_model_gpu's tolerances), from the same random decode state."""
import types

import pytest
import torch

from ckpt_fake import fake
from oracle import fp8, refgen, step
from tt_qwen_resident_b200 import checkpoint as C
from tt_qwen_resident_b200.model import ResidentModel

pytestmark = pytest.mark.gpu


def test_model_from_checkpoint_matches_oracle(cuda):
    torch.set_num_threads(8)
    ck = fake(layers=2, interval=2, vocab=1024, mtp=False)
    w8 = C.load(ck, device=cuda)
    f32 = C.canonical_fp32(ck)
    # the oracle multiplies with the dequantised FP8 values the GPU streams
    D = lambda m: fp8.dequantize_blocks(m.q.cpu(), m.scales.cpu())
    w = types.SimpleNamespace(
        gdn=[dict(g, Win=D(q["Win"])) for g, q in zip(f32["gdn"], w8["gdn"])],
        attn=[dict(a, Win=D(q["Win"])) for a, q in zip(f32["attn"], w8["attn"])],
        out=[D(o) for o in w8["out"]],
        mlp=[dict(G=D(m["G"]), U=D(m["U"]), D=D(m["D"])) for m in w8["mlp"]],
        head=D(w8["head"]),
    )
    P = step.Prepared(w, 1)
    st = refgen.random_state(1, 1, 40, 104, seed=1)
    model = ResidentModel(w8, 2, 2, batch=1, max_pos=104, lm_head=True, embed=C.embedding(ck))
    model.load_state(st)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(3)).bfloat16().float()
    model.step(model.token_state(x0, 40))
    model.check()
    x_ref, lg = step.torch_step(x0, P, st, 2, 2, lm_head=True)
    rel = lambda a, b: float((a - b).norm() / b.norm())
    assert rel(model.x(), x_ref) < 2e-2
    assert rel(model.logits(), step.logits_bf16(lg)) < 2e-2
    model.close()
