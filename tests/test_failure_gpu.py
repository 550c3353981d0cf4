"""Failure detection on one GPU without a GPU fault: a bounded wait of the peer exchange's kind
(qres_wait_probe: the poll loop the next projection runs on a peer's counter) on a device word that nothing
advances runs out of its budget, sets the context's error word, and returns; qres_check then reports
QRES_ERR_DEVICE with the timeout, the word is cleared, and the same context runs a normal step. A word that holds
the wanted count passes without an error."""
import pytest
import torch

from oracle import refgen
from tt_qwen_resident_b200 import _lib, weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import setup8  # noqa: F401

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(cuda, setup8):
    w8, _ = setup8
    model = ResidentModel(weights.canonical_from_fp8(w8), 2, 2, batch=1, max_pos=64, lm_head=True)
    model.load_state(refgen.random_state(1, 1, 8, 64, seed=1))
    flag = torch.zeros(4, dtype=torch.int32, device=cuda)
    L, s = _lib.lib(), _lib.stream_ptr()
    # a word that already holds the count: no error
    flag[0] = 3
    _lib.check(L.qres_wait_probe(model.ctx, _lib.ptr(flag), 3, 1000, s), model.ctx, "probe")
    model.check()
    # a word nothing advances: the wait runs out (~20k polls), the kernel returns, the error is reported
    _lib.check(L.qres_wait_probe(model.ctx, _lib.ptr(flag[1:]), 1, 20000, s), model.ctx, "probe")
    with pytest.raises(_lib.QresError, match="bounded wait ran out"):
        model.check()
    # the word was cleared and the context is usable: a normal step runs and checks clean
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(2)).bfloat16().float()
    model.step(model.token_state(x0, 8))
    model.check()
    assert model.fed_token()[1] == 9
    model.close()
