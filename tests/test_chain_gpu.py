"""The chained projections (gemv_chain.cu: out-proj, gate|up, down and the next in-proj or the lm_head as one
persistent launch, dependencies through tagged words) against the per-projection launches and the oracle.

The two paths compute the same math; they sum the rmsnorm's squares over different thread groupings, so an
element's bf16 rounding may flip: the chained step's x and logits stay within 2e-2 relative of the oracle
(test_model_gpu's tolerance) and within 1e-2 of the per-projection step, over three consecutive steps of the
G G G A x2 + lm_head schedule from the same state, eager and replayed from a CUDA graph (bit-identical)."""
import pytest
import torch

from oracle import refgen, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import rel, setup8  # noqa: F401

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows", [1, 3])
def test_chain_matches_per_projection_and_oracle(cuda, setup8, rows):
    w8, P = setup8
    layers, interval, pos = 8, 4, 100
    st = refgen.random_state(6, 2, pos, pos + 64, seed=1)
    g = torch.Generator().manual_seed(7)
    xs = [torch.randn(rows, 5120, generator=g).bfloat16().float() for _ in range(3)]
    out = {}
    for chain in (True, False):
        model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=rows, max_pos=pos + 64,
                              lm_head=True, chain=chain)
        for trace in (False, True):
            for u in range(rows):
                model.load_state(st, user=u)
            if trace:
                model.capture_trace()
            res = []
            for k, x0 in enumerate(xs):
                model.step(model.token_state(x0, [pos + k] * rows))
                model.check()
                res.append((model.x().clone(), model.logits().clone()))
            model.release_trace()
            out[(chain, trace)] = res
        model.close()
    for k in range(3):
        xc, lc = out[(True, False)][k]
        xp, lp = out[(False, False)][k]
        assert torch.equal(xc, out[(True, True)][k][0]) and torch.equal(lc, out[(True, True)][k][1])  # graph == eager
        assert rel(xc, xp) < 1e-2 and rel(lc, lp) < 1e-2, k
    # the first step against the oracle, per row
    ref = refgen.clone_state(st)
    x_ref, lg = step.torch_step(xs[0][0], P, ref, layers, interval, lm_head=True)
    xc, lc = out[(True, False)][0]
    xc, lc = (xc[0], lc[0]) if rows > 1 else (xc, lc)
    assert rel(xc, x_ref) < 2e-2
    assert rel(lc, step.logits_bf16(lg)) < 2e-2
