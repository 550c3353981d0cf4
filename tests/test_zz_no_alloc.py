"""qres_topk_noalloc, the top-32 / argmax entry point that allocates nothing, against qres_topk.

Some callers cannot allocate device memory: a host framework that owns every device byte through its own pool
and hands a plugin only its inputs and outputs. qres_topk_noalloc serves them from a fixed 256 KiB array inside
the library instead of a caller workspace. This test calls it twice in a row through the C ABI, on different
logits (so a stale result left in the shared array would show), and requires the same lists and argmax as
qres_topk with its own workspace: top-k is bit-exact. It also checks that a request too large for the array is
refused with an argument error before any GPU work. The file is named to be collected last and keeps no state
between its calls and the rest of the suite, so it passes alone in a fresh process as well as after the others.
"""
import ctypes

import pytest
import torch

from tt_qwen_resident_b200 import _lib

pytestmark = pytest.mark.gpu


def _noalloc(logits, base):
    rows, n = logits.shape
    lists = torch.full((rows, 2 * _lib.QRES_TOPK), -1, dtype=torch.int32, device=logits.device)
    am = torch.full((rows,), -1, dtype=torch.int32, device=logits.device)
    st = _lib.lib().qres_topk_noalloc(rows, _lib.ptr(logits), n, base, _lib.ptr(lists), _lib.ptr(am), _lib.stream_ptr())
    _lib.check(st, None, "qres_topk_noalloc")
    return lists, am


def test_topk_noalloc_matches_workspace_entry_point_twice(cuda):
    g = torch.Generator().manual_seed(2024)
    cases = [(8, 248320, 0), (3, 31040, 31040 * 5)]  # full vocabulary x 8 rows, then an n=8 shard at its base
    for rows, n, base in cases:
        lg = (torch.randn(rows, n, generator=g) * 3).bfloat16()
        for b in range(rows):  # ties at the maximum and at the 32nd place
            top = int(lg[b].float().argmax())
            lg[b, (7 * b + 11) % n] = lg[b, top]
            lg[b, n - 1 - b] = lg[b, top]
        lg_d = lg.to(cuda)
        want_lists, want_am = _lib.topk(lg_d, base=base)
        got_lists, got_am = _noalloc(lg_d, base)
        torch.cuda.synchronize()
        assert torch.equal(got_lists.cpu(), want_lists.cpu()), (rows, n)
        assert torch.equal(got_am.cpu(), want_am.cpu()), (rows, n)


def test_topk_noalloc_rejects_requests_beyond_its_array(cuda):
    rows, n = 8, 300000  # 8 x 128 blocks of candidates: more than the 256 KiB array holds
    logits = torch.zeros(rows, n, dtype=torch.bfloat16, device=cuda)
    lists = torch.zeros(rows, 2 * _lib.QRES_TOPK, dtype=torch.int32, device=cuda)
    am = torch.zeros(rows, dtype=torch.int32, device=cuda)
    st = _lib.lib().qres_topk_noalloc(rows, _lib.ptr(logits), n, 0, _lib.ptr(lists), _lib.ptr(am), _lib.stream_ptr())
    assert st == 1  # QRES_ERR_ARG
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
