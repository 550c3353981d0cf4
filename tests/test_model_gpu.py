"""Decode-step parity of ResidentModel (libqres) against the oracle, after the reference's own tests:
consecutive steps of G G G A G G G A + lm_head (tests/bench_resident_model.py:483-549), carried state, graph
replay bit-identical to eager steps (test_resident_accuracy.py:223-258), device-fed greedy == host-fed greedy
(test_resident_feed.py:370-436).

Every layer has its own decode state here (weights may be shared copies): the reference's shared state copies
shift one conv history several times per step, a test economy that a position-keyed history ring does not
model.

Tolerances: per step the device and the oracle start from the same state (the oracle state is reloaded into the
model before every step), so errors do not compound: x and the logits within 2e-2 relative (BASELINE atol 2e-2
on bf16 activations; the oracle itself moves by ~0.5% between equally valid fp32 orders, see
test_oracle_golden), argmax equal unless the oracle's top-2 bf16 logits are within the measured logit error.
"""
import copy

import pytest
import torch

from oracle import fp8, refgen, sampling, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel

pytestmark = pytest.mark.gpu


def quantized(w32):
    Q = lambda t: fp8.quantize_blocks(t)
    return dict(
        gdn=[dict(g, Win=Q(g["Win"])) for g in w32.gdn],
        attn=[dict(a, Win=Q(a["Win"])) for a in w32.attn],
        out=[Q(o) for o in w32.out],
        mlp=[dict(G=Q(m["G"]), U=Q(m["U"]), D=Q(m["D"])) for m in w32.mlp],
        head=Q(w32.head) if w32.head is not None else None,
    )


def dequantized(w8, w32):
    D = lambda t: fp8.dequantize_blocks(*t)
    w = copy.copy(w32)
    w.gdn = [dict(g, Win=D(q["Win"])) for g, q in zip(w32.gdn, w8["gdn"])]
    w.attn = [dict(a, Win=D(q["Win"])) for a, q in zip(w32.attn, w8["attn"])]
    w.out = [D(o) for o in w8["out"]]
    w.mlp = [dict(G=D(m["G"]), U=D(m["U"]), D=D(m["D"])) for m in w8["mlp"]]
    w.head = D(w8["head"]) if w8["head"] is not None else None
    return w


@pytest.fixture(scope="module")
def setup8():
    torch.set_num_threads(8)
    w32 = refgen.random_weights(2, 1, 2, vocab=16384, seed=0)
    w8 = quantized(w32)
    P = step.Prepared(dequantized(w8, w32), 1)
    return w8, P


def rel(a, b):
    return float((a - b).norm() / b.norm())


def test_decode_steps_parity(cuda, setup8):
    w8, P = setup8
    layers, interval, pos = 8, 4, 100
    st = refgen.random_state(6, 2, pos, pos + 64, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=1, max_pos=pos + 64, lm_head=True)
    g = torch.Generator().manual_seed(7)
    for s in range(3):
        model.load_state(st)
        x0 = torch.randn(5120, generator=g).bfloat16().float()
        model.step(model.token_state(x0, st.pos))
        model.check()
        mix = []
        x_ref, lg = step.torch_step(x0, P, st, layers, interval, lm_head=True, mixer_out=mix)
        o_ref = torch.cat([o for l, _, o in mix if l == layers - 1])
        assert rel(model.x(), x_ref) < 2e-2
        assert rel(model.mixer_output(), o_ref) < 2e-2
        lr = step.logits_bf16(lg)
        got = model.logits()
        assert rel(got, lr) < 2e-2
        am, am_ref = model.argmax(), sampling.argmax_rule(lr)
        assert am == sampling.argmax_rule(got)  # the device pick follows the rule on its own logits
        if am != am_ref:
            top2 = lr.topk(2).values
            assert float(top2[0] - top2[1]) <= 2 * float((got - lr).abs().max()), (am, am_ref)
    # the GDN states and the KV rows the device wrote (this step from the same start state)
    model.load_state(st)
    ref = refgen.clone_state(st)
    x0 = torch.randn(5120, generator=g).bfloat16().float()
    model.step(model.token_state(x0, ref.pos))
    model.check()
    step.torch_step(x0, P, ref, layers, interval, lm_head=True)
    for c in range(6):
        assert rel(model.dump_gdn_state(c), ref.gdn[c]) < 2e-2
    k = model.kv_rows(0, [st.pos])[:, 0]
    assert rel(k, ref.K[0][:, st.pos]) < 2e-2


def test_graph_replay_bitidentical_and_deterministic(cuda, setup8):
    w8, _ = setup8
    pos = 40
    st = refgen.random_state(6, 2, pos, pos + 64, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8), 8, 4, batch=1, max_pos=pos + 64, lm_head=True)
    g = torch.Generator().manual_seed(5)
    xs = [torch.randn(5120, generator=g).bfloat16().float() for _ in range(4)]

    def run(trace):
        model.load_state(st)
        if trace:
            model.capture_trace()
            model.load_state(st)  # capture does not run the step, but be explicit
        out = []
        for i, x0 in enumerate(xs):
            model.step(model.token_state(x0, pos + i))
            model.check()
            out.append((model.x().clone(), model.logits().clone()))
        model.release_trace()
        return out

    a, b, c = run(False), run(True), run(False)
    for (xa, la), (xb, lb), (xc, lc) in zip(a, b, c):
        assert torch.equal(xa, xb) and torch.equal(la, lb)
        assert torch.equal(xa, xc) and torch.equal(la, lc)


def test_device_fed_greedy_equals_host_fed(cuda, setup8):
    w8, _ = setup8
    vocab = 16384
    emb = (torch.randn(vocab, 5120, generator=torch.Generator().manual_seed(9))).bfloat16()
    st = refgen.random_state(6, 2, 0, 64, seed=1, zero=True)
    model = ResidentModel(weights.canonical_from_fp8(w8), 8, 4, batch=1, max_pos=64, lm_head=True, embed=emb)
    # host-fed: the host reads each argmax and writes the next token state
    model.load_state(st)
    tok, host = 17, []
    for p in range(12):
        model.step(model.token_state(tokens=tok, pos=p))
        model.check()
        tok = model.argmax()
        host.append(tok)
    # device-fed: one token state, then steps back to back (captured graph)
    model.load_state(st)
    model.capture_trace()
    model.step(model.token_state(tokens=17, pos=0, feed=True))
    fed = []
    for p in range(12):
        if p:
            model.step(None)
        model.check()
        t, np_ = model.fed_token()
        assert np_ == p + 1
        fed.append(t)
    model.release_trace()
    assert fed == host


@pytest.mark.parametrize("layers,interval", [(1, 0), (1, 1), (2, 2), (4, 4)])
def test_layer_schedules_parity(cuda, setup8, layers, interval):
    """short schedules (one GDN layer, one attention layer, G A, G G G A) from the same start state: localises a
    mismatch to a layer kind"""
    w8, P = setup8
    pos = 70
    n_attn = sum(step.is_attn(l, interval) for l in range(layers))
    st = refgen.random_state(layers - n_attn, n_attn, pos, pos + 64, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=1, max_pos=pos + 64, lm_head=True)
    model.load_state(st)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(3)).bfloat16().float()
    model.step(model.token_state(x0, st.pos))
    model.check()
    mix = []
    x_ref, lg = step.torch_step(x0, P, st, layers, interval, lm_head=True, mixer_out=mix)
    o_ref = torch.cat([o for l, _, o in mix if l == layers - 1])
    errs = (rel(model.mixer_output(), o_ref), rel(model.x(), x_ref), rel(model.logits(), step.logits_bf16(lg)))
    assert max(errs) < 2e-2, errs


def test_batch8_decode_steps_parity(cuda, setup8):
    """BASELINE config 4's shape at 8 layers: 8 users per step, each with its own decode state (GDN states, conv
    histories, KV cache behind a shuffled page table) at its own position, two consecutive steps carried on both
    sides (model.py:421-446 users as rows, :780-823 per-user state). Every user's x, logits, greedy pick, GDN
    states and appended KV row against its own oracle chain."""
    w8, P = setup8
    layers, interval, B, max_pos = 8, 4, 8, 384
    pos = [40 + 37 * u for u in range(B)]
    sts = [refgen.random_state(6, 2, pos[u], max_pos, seed=100 + u) for u in range(B)]
    max_pages = max_pos // 64
    pt = torch.randperm(B * max_pages, generator=torch.Generator().manual_seed(5)).to(torch.int32).view(B, max_pages)
    model = ResidentModel(weights.canonical_from_fp8(w8), layers, interval, batch=B, max_pos=max_pos, lm_head=True,
                          page_table=pt)
    for u in range(B):
        model.load_state(sts[u], user=u)
    refs = [refgen.clone_state(s) for s in sts]
    g = torch.Generator().manual_seed(21)
    for k in range(2):
        x0 = torch.randn(B, 5120, generator=g).bfloat16().float()
        model.step(model.token_state(x0, [p + k for p in pos]))
        model.check()
        X, LG, AM = model.x(), model.logits(), model.argmax()
        for u in range(B):
            x_ref, lg = step.torch_step(x0[u], P, refs[u], layers, interval, lm_head=True)
            lr = step.logits_bf16(lg)
            assert rel(X[u], x_ref) < 2e-2, (k, u)
            assert rel(LG[u], lr) < 2e-2, (k, u)
            d, o = AM[u], sampling.argmax_rule(lr)
            assert d == sampling.argmax_rule(LG[u]), (k, u)
            if d != o:
                assert float(lr[o] - lr[d]) <= float((LG[u][o] - lr[o]).abs() + (LG[u][d] - lr[d]).abs()), (k, u)
    for u in range(B):
        for c in range(6):
            assert rel(model.gdn_state[c][u].cpu(), refs[u].gdn[c]) < 2e-2, (u, c)
        k_dev = model.kv_rows(1, [pos[u], pos[u] + 1], user=u)
        assert rel(k_dev, refs[u].K[1][:, pos[u] : pos[u] + 2]) < 2e-2, u
