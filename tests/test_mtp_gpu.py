"""The MTP draft layer (ResidentModel(fc=...)): a chain of three drafts after a main step, against the oracle's
draft entries (oracle/mtp.py, after the reference's mtp.py:1-14 / mtp_acceptance.py:70-81). The draft model
is one attention layer with its own KV cache and the main model's lm_head; draft k's fc reads the token of the
step before and that step's last x (the main model's for the first draft, then the previous draft's).

Each draft's oracle entry takes the device's token and hidden rows (so a near-tie in one pick does not move
the rest of the chain) and the oracle's own draft state: x and logits within 2e-2 relative
(test_model_gpu's tolerances), the pick by the argmax rule unless the oracle's top-2 logits are within the
measured logit error."""
import pytest
import torch

from oracle import fp8, mtp, refgen, sampling, step
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import dequantized, quantized, rel, setup8  # noqa: F401

pytestmark = pytest.mark.gpu


def test_mtp_draft_chain_matches_oracle(cuda, setup8):
    w8, P = setup8
    vocab, pos = 16384, 90
    emb = (torch.randn(vocab, 5120, generator=torch.Generator().manual_seed(9))).bfloat16()
    # the draft layer: random attention + MLP weights, the main model's head; the fc with folded norm weights
    wd32 = refgen.random_weights(0, 1, 1, vocab=0, seed=5)
    wd8 = quantized(wd32)
    wd8["head"] = w8["head"]
    g = torch.Generator().manual_seed(6)
    fc32 = torch.randn(5120, 10240, generator=g) / 10240**0.5 * (1 + 0.1 * torch.randn(10240, generator=g))
    fq, fs = fp8.quantize_blocks(fc32)
    fc = fp8.dequantize_blocks(fq, fs)
    wd32.head = P.w.head
    Pd = step.Prepared(dequantized(wd8, wd32), 1)

    main = ResidentModel(weights.canonical_from_fp8(w8), 4, 4, batch=1, max_pos=pos + 64, lm_head=True, embed=emb)
    draft = ResidentModel(weights.canonical_from_fp8(wd8), 1, 1, batch=1, max_pos=pos + 64, lm_head=True, embed=emb,
                          fc=weights.FP8Matrix(fq.cuda(), fs.cuda()))
    st = refgen.random_state(3, 1, pos, pos + 64, seed=1)
    st_d = refgen.random_state(0, 1, pos, pos + 64, seed=3)
    main.load_state(st)
    draft.load_state(st_d)
    x0 = torch.randn(5120, generator=g).bfloat16().float()
    main.step(main.token_state(x0, pos))
    main.check()
    tok, h = main.argmax(), main.x()
    draft.set_hidden(main.x_d)
    ref = refgen.clone_state(st_d)
    for k in range(3):
        draft.step(draft.token_state(tokens=tok, pos=pos + k))
        draft.check()
        x_ref, lg = mtp.draft_step(tok, h, emb, fc, Pd, ref)
        assert rel(draft.x(), x_ref) < 2e-2, k
        lr, got = step.logits_bf16(lg), draft.logits()
        assert rel(got, lr) < 2e-2, k
        am, am_ref = draft.argmax(), sampling.argmax_rule(lr)
        assert am == sampling.argmax_rule(got), k
        if am != am_ref:
            top2 = lr.topk(2).values
            assert float(top2[0] - top2[1]) <= 2 * float((got - lr).abs().max()), (k, am, am_ref)
        # the next draft: this draft's token and last x
        tok, h = am, draft.x()
        draft.set_hidden(draft.x_d)
    main.close()
    draft.close()
