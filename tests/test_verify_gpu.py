"""The verify step (ResidentModel(verify=True)): R rows of ONE user at positions p .. p+R-1 in one step,
against the oracle run as R consecutive batch-1 steps (the reference's tests/test_resident_verify.py:1-78:
row r continues each layer's state from row r - 1; after a step the next one continues from the accepted row
k, so the conv history ring, the GDN state slots and the shared KV cache are exercised both ways).

Each verify step starts the device from the oracle's state (loaded into the state slot the step reads, as
the reference's test restarts its torch reference) so errors do not compound; continuation is still the
device's: position p + k + 1, state slot (slot + k) % R, the KV rows and conv history the device wrote. Per
row: x and the logits within 2e-2 relative of the oracle's (test_model_gpu's tolerances); the R GDN state
slots the step wrote match the oracle's state after each row; the K rows appended at p .. p+R-1 match.
"""
import pytest
import torch

from oracle import refgen, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import rel, setup8  # noqa: F401  (module fixture)

pytestmark = pytest.mark.gpu

ACCEPT = [0, 1, 3, 2, 1]  # per step: the accepted row (clipped to R - 1)


@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("layers,interval", [(4, 0), (4, 4)], ids=["gdn", "mixed"])
def test_verify_matches_consecutive_steps(cuda, setup8, R, layers, interval):
    w8, P = setup8
    pos = 61  # the rows straddle a KV page boundary (63 | 64)
    n_attn = sum(step.is_attn(l, interval) for l in range(layers))
    st = refgen.random_state(layers - n_attn, n_attn, pos, pos + 64, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=R, max_pos=pos + 64,
                          lm_head=True, verify=True)
    g = torch.Generator().manual_seed(7)
    ref, p, slot = refgen.clone_state(st), pos, 0
    model.load_state(ref, slot=slot)
    for s, acc in enumerate(ACCEPT):
        k = min(acc, R - 1)
        x0 = torch.randn(R, 5120, generator=g).bfloat16().float()
        model.step(model.token_state(x0, p, slot=slot))
        model.check()
        got_x, got_l = model.x(), model.logits()
        cur, after = refgen.clone_state(ref), []
        for r in range(R):
            assert cur.pos == p + r
            xr, lg = step.torch_step(x0[r], P, cur, layers, interval, lm_head=True)
            assert rel(got_x[r], xr) < 2e-2, (s, r)
            assert rel(got_l[r], step.logits_bf16(lg)) < 2e-2, (s, r)
            after.append(refgen.clone_state(cur))
        for r in range(R):  # row r's state in slot (slot + r) % R
            for c in range(layers - n_attn):
                assert rel(model.dump_gdn_state(c, (slot + r) % R), after[r].gdn[c]) < 2e-2, (s, r, c)
        if n_attn:
            k_dev = model.kv_rows(0, list(range(p, p + R)))
            assert rel(k_dev, after[-1].K[0][:, p : p + R]) < 2e-2, s
        # continue from row k: the device keeps its own conv ring and KV rows; the oracle's state after row k
        # is loaded into the slot the next step reads (same values the device holds there, up to rounding)
        ref, p, slot = after[k], p + k + 1, (slot + k) % R
        model.load_state(ref, slot=slot)
    model.close()


def test_verify_continuation_without_reload(cuda, setup8):
    """three verify steps back to back with no state reload (rows accepted 1, 0, 3 of 4): the device's own
    slots, ring and cache carry the state; x of every row within 3e-2 of the oracle's consecutive steps"""
    w8, P = setup8
    layers, interval, R, pos = 4, 4, 4, 126
    st = refgen.random_state(3, 1, pos, pos + 64, seed=2)
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=R, max_pos=pos + 64,
                          lm_head=True, verify=True)
    model.load_state(st)
    g = torch.Generator().manual_seed(11)
    ref, p, slot = refgen.clone_state(st), pos, 0
    for k in (1, 0, 3):
        x0 = torch.randn(R, 5120, generator=g).bfloat16().float()
        model.step(model.token_state(x0, p, slot=slot))
        model.check()
        got = model.x()
        cur, after = refgen.clone_state(ref), []
        for r in range(R):
            xr, _ = step.torch_step(x0[r], P, cur, layers, interval, lm_head=True)
            assert rel(got[r], xr) < 3e-2, (p, r)
            after.append(refgen.clone_state(cur))
        ref, p, slot = after[k], p + k + 1, (slot + k) % R
    model.close()
