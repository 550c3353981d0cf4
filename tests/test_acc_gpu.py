"""The fixed-point accumulators of the one-rank step (EPI_ACC: each CTA's partial sums of the out-, gate|up and
down-projections added as 64-bit integers in 2^-30 units; the next prologue forms the residual add or
silu(g) * u from them) against the tile-finishing path (split tiles summed in CTA order by their last CTA) and
the oracle.

Integer addition is associative, so the accumulated step must be bit-identical from run to run however the
CTAs' atomic adds interleave: eager and CUDA-graph replays of the same inputs agree bit for bit. The two paths
round differently (one float rounding of the exact sum of 2^-30-rounded parts, against fp32 additions in CTA
order); a flipped bf16 rounding of an activation carries on through the recurrent state, so by the third step
the two agree to ~5e-3 relative (asserted: 1e-2), and each stays within test_model_gpu's 2e-2 of the oracle at
every one of three consecutive steps of the G G G A x2 + lm_head schedule, at 1, 2 and 8 rows (at 8 rows the
accumulating projections walk their units in K groups, several CTAs adding into every tile)."""
import pytest
import torch

from oracle import refgen, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import rel, setup8  # noqa: F401

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows", [1, 2, 8])
def test_accumulators_match_tile_finish_and_oracle(cuda, setup8, rows):
    w8, P = setup8
    layers, interval, pos = 8, 4, 100
    st = refgen.random_state(6, 2, pos, pos + 64, seed=1)
    g = torch.Generator().manual_seed(11)
    xs = [torch.randn(rows, 5120, generator=g).bfloat16().float() for _ in range(3)]
    out = {}
    for tile_finish in (False, True):
        model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=rows, max_pos=pos + 64,
                              lm_head=True, tile_finish=tile_finish)
        for run in ("eager", "graph", "graph2"):
            for u in range(rows):
                model.load_state(st, user=u)
            if run == "graph":
                model.capture_trace()
            res = []
            for k, x0 in enumerate(xs):
                model.step(model.token_state(x0, [pos + k] * rows))
                model.check()
                res.append((model.x().clone(), model.logits().clone(), model.argmax()))
            if run == "graph2":
                model.release_trace()
            out[(tile_finish, run)] = res
        model.close()
    # the oracle over the same three steps (row 0), both paths
    ref = refgen.clone_state(st)
    for k in range(3):
        x_ref, lg = step.torch_step(xs[k][0], P, ref, layers, interval, lm_head=True)
        for tf in (False, True):
            xk, lk, _ = out[(tf, "eager")][k]
            xk, lk = (xk[0], lk[0]) if rows > 1 else (xk, lk)
            assert rel(xk, x_ref) < 2e-2 and rel(lk, step.logits_bf16(lg)) < 2e-2, (k, tf)
    for k in range(3):
        xa, la, aa = out[(False, "eager")][k]
        for run in ("graph", "graph2"):  # bit-reproducible whatever order the adds land in
            xg, lg_, ag = out[(False, run)][k]
            assert torch.equal(xa, xg) and torch.equal(la, lg_) and aa == ag, (k, run)
        xt, lt, _ = out[(True, "eager")][k]
        assert rel(xa, xt) < 1e-2 and rel(la, lt) < 1e-2, k
