"""256 free-running greedy decode steps on the GPU against the oracle's own greedy chain (the build's gate:
identical greedy argmax over 256 random-weight decode steps).

Schedule G G G A G G G A (8 layers at the full widths, every layer with its own decode state) + an lm_head of
16,384 rows, a random start state at position 32 (random GDN states and conv histories, random KV for the first
32 positions), first token 17, token rows from a seeded bf16 embedding table. The device runs device-fed: one
token state, then back-to-back replays of the captured step, each step's token picked and fed on the device
(the reference's feed, mlp_hub.cpp:414-458); the oracle runs torch_step (model.py:219-292) on its own carried
state with its own greedy picks (model.py:1558-1573 argmax rule). Neither side is ever reloaded from the other.

The two sides round differently (fp32 summation order; bf16 rounding points then flip), so the logits differ by
a small amount that the carried state keeps. The chains must pick the same token at every step. Where they do
not, the swap must be explained by the measured errors at exactly those two logits: the oracle's margin of its
pick o over the device's pick d, ref[o] - ref[d], must be at most |dev[o] - ref[o]| + |dev[d] - ref[d]| (a near
tie at bf16 resolution; the test prints it). The device is then re-fed the oracle's token (a host write of the
token state) and both chains continue. Any other mismatch fails, as does a drift of the logits beyond 5e-2
relative at any step.
"""
import pytest
import torch

from oracle import refgen, sampling, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import setup8  # noqa: F401

pytestmark = pytest.mark.gpu

STEPS, POS0, TOK0, VOCAB = 256, 32, 17, 16384


def test_free_running_greedy_256_steps(cuda, setup8):
    w8, P = setup8
    layers, interval = 8, 4
    emb = torch.randn(VOCAB, 5120, generator=torch.Generator().manual_seed(9)).bfloat16()
    st = refgen.random_state(6, 2, POS0, POS0 + STEPS + 8, seed=1)
    # the oracle's greedy chain (its own picks, its own carried state)
    ref_st = refgen.clone_state(st)
    ref_logits, ref_tok = [], []
    tok = TOK0
    for _ in range(STEPS):
        _, lg = step.torch_step(emb[tok].float(), P, ref_st, layers, interval, lm_head=True)
        lr = step.logits_bf16(lg)
        tok = sampling.argmax_rule(lr)
        ref_logits.append(lr)
        ref_tok.append(tok)
    # the device chain
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=1, max_pos=POS0 + STEPS + 8,
                          lm_head=True, embed=emb)
    model.load_state(st)
    model.capture_trace()
    model.step(model.token_state(tokens=TOK0, pos=POS0, feed=True))
    swaps, worst = [], 0.0
    for i in range(STEPS):
        if i:
            model.step(None)
        model.check()
        d, np_ = model.fed_token()
        assert np_ == POS0 + i + 1
        dev = model.logits()
        lr = ref_logits[i]
        rel = float((dev - lr).norm() / lr.norm())
        worst = max(worst, rel)
        assert rel < 5e-2, (i, rel)
        assert d == sampling.argmax_rule(dev), i  # the device pick follows the rule on its own logits
        o = ref_tok[i]
        if d != o:
            margin = float(lr[o] - lr[d])
            err = float((dev[o] - lr[o]).abs() + (dev[d] - lr[d]).abs())
            print(f"step {i}: device {d} oracle {o}: oracle margin {margin:.4g}, measured logit error {err:.4g}")
            assert margin <= err, (i, d, o, margin, err)
            swaps.append(i)
            # both chains continue from the oracle's token: the next replay reads this token state
            model.write_token_state(model.token_state(tokens=o, pos=POS0 + i + 1, feed=True))
    model.release_trace()
    print(f"256 free-running greedy steps: {STEPS - len(swaps)} identical picks, near-tie swaps at {swaps}, "
          f"worst logit rel err {worst:.2e}")
    assert len(swaps) <= STEPS // 16
