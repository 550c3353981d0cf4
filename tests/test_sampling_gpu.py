"""On-device sampling of the fed token (the hub's draw, qwen36_resident/kernels/sampling.hpp:77-143) on the GPU.

1. Known answers: the 135 draws of tests/golden/sampling.json (the reference test's own integer draw,
   tests/test_resident_sampling.py:37-95, over its 5 parameter cases) reproduced bit-exactly by the device: the
   top-32 lists from qres_topk on the fixture's logits, then qres_sample with each record's words and position.
2. In the step, after the reference's test_resident_sampling.py:97-160: with set_sampling, a host-fed run (the host
   writes every token state; the device's list must equal the oracle's list of the device logits and the device's
   draw the oracle's draw from it) and a device-fed run (captured step replayed back to back, the draw fed on the
   device) give the same tokens, and some draw leaves the argmax (the sampler is not greedy).
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import refgen, sampling
from tt_qwen_resident_b200 import _lib, weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import setup8  # noqa: F401

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampling.json")


def words_i32(words):
    return torch.from_numpy(np.array(words, dtype=np.uint32).view(np.int32))


def test_draws_match_reference_fixture(cuda):
    g = json.load(open(GOLD))
    vecs = [torch.tensor(v, dtype=torch.int32).to(torch.int16).view(torch.bfloat16) for v in g["vectors"]]
    n = min(v.numel() for v in vecs)
    lists = [_lib.topk(v.view(1, -1).to(cuda))[0][0] for v in vecs]  # the vectors differ in length
    torch.cuda.synchronize()
    recs = g["draws"]
    L = torch.stack([lists[r["vec"]] for r in recs]).contiguous()
    W = torch.stack([words_i32(r["words"]) for r in recs]).to(cuda)
    P = torch.tensor([r["pos"] for r in recs], dtype=torch.int32, device=cuda)
    tok = torch.full((len(recs),), -1, dtype=torch.int32, device=cuda)
    _lib.check(_lib.lib().qres_sample(len(recs), _lib.ptr(L), _lib.ptr(W), _lib.ptr(P), _lib.ptr(tok),
                                      _lib.stream_ptr()), None, "sample")
    got = tok.cpu().tolist()
    want = [r["token"] for r in recs]
    assert got == want
    assert n > 32 and any(t != sampling.argmax_rule(vecs[r["vec"]].float()) for t, r in zip(got, recs))


@pytest.mark.parametrize("case", [(1.0, 20, 0.95, 1234), (3.0, 32, 1.0, 5)])
def test_sampled_decode_fed_equals_host_fed(cuda, setup8, case):
    w8, _ = setup8
    vocab, steps, pos0 = 16384, 16, 24
    emb = torch.randn(vocab, 5120, generator=torch.Generator().manual_seed(9)).bfloat16()
    st = refgen.random_state(6, 2, pos0, pos0 + steps + 8, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8), 8, 4, batch=1, max_pos=pos0 + steps + 8, lm_head=True,
                          embed=emb)
    model.set_sampling(*case)
    words = ResidentModel.sampling_words(*case)
    # host-fed: the host writes every token state; the device draws, the oracle checks the draw
    model.load_state(st)
    tok, host, left_argmax = 17, [], 0
    for i in range(steps):
        p = pos0 + i
        model.step(model.token_state(tokens=tok, pos=p))
        model.check()
        ks, ix = model.topk()
        lk, li = sampling.topk_list(model.logits())
        assert ks[0].tolist() == lk and ix[0].tolist() == li, i  # the device list of its own logits
        d, np_ = model.fed_token()
        assert np_ == p + 1 and d == sampling.draw(lk, li, words, p), i
        left_argmax += d != model.argmax()
        tok = d
        host.append(d)
    assert left_argmax > 0
    # device-fed: one token state, then replays of the captured step
    model.load_state(st)
    model.capture_trace()
    model.step(model.token_state(tokens=17, pos=pos0, feed=True))
    fed = []
    for i in range(steps):
        if i:
            model.step(None)
        model.check()
        fed.append(model.fed_token()[0])
    model.release_trace()
    assert fed == host
