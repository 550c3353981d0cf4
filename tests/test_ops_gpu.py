"""The PyTorch custom ops (torch.ops.qres.*) and the vLLM adapter on the GPU.

- torch.ops.qres.quantize_fp8 / topk / sample against the oracle (bit-exact contracts);
- torch.ops.qres.decode_step is the step ResidentModel.step runs, and refuses buffers not bound to the context;
- Qwen36ResidentForCausalLM (generator_vllm.py:34-160 contract): prefill through the decode step, then device-
  sampled greedy decode with reload_inputs only on the first step, read_from_device every step, gives the same
  tokens as the model driven host-fed; host-sampled steps return the logits.
"""
from types import SimpleNamespace

import pytest
import torch

import tt_qwen_resident_b200  # noqa: F401  (registers torch.ops.qres)
from oracle import fp8, refgen, sampling
from tt_qwen_resident_b200 import _lib, weights
from tt_qwen_resident_b200.generator_vllm import Qwen36ResidentForCausalLM
from tt_qwen_resident_b200.model import ResidentModel
from test_model_gpu import setup8  # noqa: F401

pytestmark = pytest.mark.gpu


def test_torch_ops_match_oracle(cuda):
    g = torch.Generator().manual_seed(3)
    w = torch.randn(300, 640, generator=g) * 0.02
    q, s = torch.ops.qres.quantize_fp8(w.to(cuda))
    q_ref, s_ref = fp8.quantize_blocks(w)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)
    lg = (torch.randn(3, 31040, generator=g) * 2).bfloat16()
    lists, am = torch.ops.qres.topk(lg.to(cuda), 77)
    lists = lists.cpu().to(torch.int64) & 0xFFFFFFFF
    for b in range(3):
        ks, ix = sampling.topk_list(lg[b].float(), base=77)
        assert lists[b, :32].tolist() == ks and lists[b, 32:].tolist() == ix
        assert int(am[b]) == 77 + sampling.argmax_rule(lg[b].float())
    words = [ResidentModel.sampling_words(1.0, 20, 0.95, 1234), ResidentModel.sampling_words(0.3, 5, 0.5, 99),
             ResidentModel.sampling_words(0.0, 1, 1.0, 0)]
    import numpy as np

    W = torch.from_numpy(np.array(words, dtype=np.uint32).view(np.int32)).to(cuda)
    pos = torch.tensor([5, 6, 7], dtype=torch.int32, device=cuda)
    lists_d, _ = torch.ops.qres.topk(lg.to(cuda), 0)
    tok = torch.ops.qres.sample(lists_d, W, pos).cpu().tolist()
    for b in range(3):
        ks, ix = sampling.topk_list(lg[b].float())
        assert tok[b] == sampling.draw(ks, ix, words[b], 5 + b)


def test_decode_step_op_refuses_unbound_buffers(cuda, setup8):
    w8, _ = setup8
    model = ResidentModel(weights.canonical_from_fp8(w8), 2, 2, batch=1, max_pos=64, lm_head=True)
    model.load_state(refgen.random_state(1, 1, 8, 64, seed=1))
    other = torch.zeros_like(model.x_d)
    with pytest.raises(_lib.QresError):
        torch.ops.qres.decode_step(model.ctx.value, model.tok_d, other, model.out_d, False)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(2)).bfloat16().float()
    model.write_token_state(model.token_state(x0, 8))
    torch.ops.qres.decode_step(model.ctx.value, model.tok_d, model.x_d, model.out_d, False)
    model.check()
    assert model.fed_token()[1] == 9


def test_vllm_adapter_device_sampled_greedy_equals_host_fed(cuda, setup8):
    w8, _ = setup8
    vocab = 16384
    emb = torch.randn(vocab, 5120, generator=torch.Generator().manual_seed(9)).bfloat16()
    prompt = [17, 400, 9, 1234, 5]
    steps = 12
    # the model driven directly, host-fed greedy
    ref = ResidentModel(weights.canonical_from_fp8(w8), 8, 4, batch=1, max_pos=64, lm_head=True, embed=emb)
    for p, t in enumerate(prompt):
        ref.step(ref.token_state(tokens=t, pos=p))
    ref.check()
    want, tok = [], ref.argmax()
    for i in range(steps):
        want.append(tok)
        ref.step(ref.token_state(tokens=tok, pos=len(prompt) + i))
        ref.check()
        tok = ref.argmax()
    ref.close()
    # the adapter: prefill, then device sampling (greedy words) with inputs written once
    model = ResidentModel(weights.canonical_from_fp8(w8), 8, 4, batch=1, max_pos=72, lm_head=True, embed=emb)
    a = Qwen36ResidentForCausalLM(model, max_seq_len=64)
    logits = a.prefill_forward(torch.tensor([prompt]), None, None, torch.tensor([len(prompt)]))
    assert logits.shape == (1, 1, vocab)
    first = sampling.argmax_rule(logits.view(-1))
    assert first == want[0]
    sp = SimpleNamespace(temperature=[0.0], top_k=[1], top_p=[1.0], seed=[0])
    got = [first]
    tok, pos = first, len(prompt)
    for i in range(steps - 1):
        t = a.decode_forward(torch.tensor([[tok]]), torch.tensor([pos]), reload_inputs=i == 0,
                             reload_sampling_params=i == 0, read_from_device=True, sampling_params=sp)
        tok, pos = int(t), pos + 1
        got.append(tok)
    assert got == want
    # a host-sampled step returns the logits of the step
    lg = a.decode_forward(torch.tensor([[tok]]), torch.tensor([pos]))
    assert lg.shape == (1, 1, vocab)
