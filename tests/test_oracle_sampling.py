"""Integer sampling / top-k / argmax rules of the oracle against the reference test's own draw
(tests/golden/sampling.json, made from sott0n/tt-qwen-resident tests/test_resident_sampling.py:37-95)."""
import json
import os

import torch

from oracle import sampling as S

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampling.json")


def test_draw_matches_reference_fixture():
    g = json.load(open(GOLD))
    vecs = [torch.tensor(v, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float() for v in g["vectors"]]
    assert len(g["draws"]) == 135
    for r in g["draws"]:
        ks, ix = S.topk_list(vecs[r["vec"]])
        assert S.draw(ks, ix, r["words"], r["pos"]) == r["token"], r


def test_sampling_words_cases():
    g = json.load(open(GOLD))
    for i, (t, k, p, seed) in enumerate(g["cases"]):
        r = g["draws"][3 * i]  # the first vector: 3 positions per case
        assert S.sampling_words(t, k, p, seed) == r["words"]


def test_argmax_tie_rule_and_merge():
    lg = torch.tensor([1.0, 3.0, -2.0, 3.0, 0.5, 3.0]).bfloat16().float()
    assert S.argmax_rule(lg) == 1
    ks, ix = S.topk_list(lg, k=4)
    assert ix == [1, 3, 5, 0]
    # merging per-slice lists equals the list of the whole vector
    g = torch.Generator().manual_seed(0)
    v = (torch.randn(5000, generator=g) * 0.3).bfloat16().float()
    v[4000] = v[17] = v.max()
    lists = [S.topk_list(v[i : i + 1000], base=i) for i in range(0, 5000, 1000)]
    assert S.merge(lists) == S.topk_list(v)
    assert S.merge(lists)[1][0] == S.argmax_rule(v) == 17


def test_key_order():
    vals = torch.tensor([-3.0, -0.0, 0.0, 1e-3, 2.0, -1e-3]).bfloat16()
    keys = S.keys_of(vals.float())
    order = sorted(range(6), key=lambda i: int(keys[i]))
    assert [float(vals[i]) for i in order][0] == -3.0
    for b in range(0, 0x10000, 97):
        assert S.bf16_of(S.key_of(b)) == b
