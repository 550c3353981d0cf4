"""The MTP speculative-decode loop (tt_qwen_resident_b200.mtp.SpecDecoder, after the reference's
qwen36_resident/mtp.py:292-591, generalised to 3 drafts and a 4-row verify step) on the GPU.

Speculative decode must reproduce plain greedy decode token for token (every committed token is the main model's
greedy pick at its position; the verify step's row r equals the step at its position): checked with the random
draft layer (which rarely guesses right), with planted drafts that are right up to a varying first mistake (every
accept length 0..3 occurs), and through the streaming interface the vLLM block adapter uses (start / next_block).
"""
import pytest
import torch

from oracle import fp8, refgen
from tt_qwen_resident_b200 import weights
from tt_qwen_resident_b200.generator_vllm import Qwen36ResidentMTPForCausalLM
from tt_qwen_resident_b200.model import ResidentModel
from tt_qwen_resident_b200.mtp import SpecDecoder
from test_model_gpu import quantized, setup8  # noqa: F401

pytestmark = pytest.mark.gpu

VOCAB, N_NEW, K = 16384, 24, 3


@pytest.fixture(scope="module")
def spec(cuda, setup8):
    w8, _ = setup8
    emb = torch.randn(VOCAB, 5120, generator=torch.Generator().manual_seed(9)).bfloat16()
    wd8 = quantized(refgen.random_weights(0, 1, 1, vocab=0, seed=5))
    wd8["head"] = w8["head"]
    g = torch.Generator().manual_seed(6)
    fc32 = torch.randn(5120, 10240, generator=g) / 10240**0.5
    fq, fs = fp8.quantize_blocks(fc32)
    max_pos = 128
    main = ResidentModel(weights.canonical_from_fp8(w8), 4, 4, batch=K + 1, max_pos=max_pos, lm_head=True, embed=emb,
                         verify=True)
    draft = ResidentModel(weights.canonical_from_fp8(wd8), 1, 1, batch=1, max_pos=max_pos, lm_head=True, embed=emb,
                          fc=weights.FP8Matrix(fq.cuda(), fs.cuda()))
    s = SpecDecoder(main, draft, drafts=K)
    yield s
    main.close()
    draft.close()


PROMPT = [17, 400, 9, 1234, 5, 77, 3000, 12, 8]


def test_spec_decode_equals_greedy(spec):
    want = spec.greedy(PROMPT, N_NEW + K + 1)
    got, stats = spec.generate(PROMPT, N_NEW)
    assert got == want[: len(PROMPT) + N_NEW]
    print("random draft layer:", stats)
    # planted drafts: right up to the first mistake at index (position % 5) (5, 4: none), so every accept length
    # 0..3 occurs
    def planted(seq, p, k):
        d = [want[q] if q < len(want) else 0 for q in range(p + 1, p + 1 + k)]
        m = p % 5
        if m < k:
            d[m] = (d[m] + 1) % VOCAB
        return d

    spec.draft_fn = planted
    try:
        got2, stats2 = spec.generate(PROMPT, N_NEW)
    finally:
        spec.draft_fn = None
    assert got2 == want[: len(PROMPT) + N_NEW]
    assert stats2["accepted_drafts"] > 0 and stats2["tokens_per_step"] > 1.5, stats2
    print("planted drafts:", stats2)


def test_block_adapter_streams_greedy(spec):
    want = spec.greedy(PROMPT, N_NEW + K + 1)
    a = Qwen36ResidentMTPForCausalLM(spec, max_seq_len=128, eos=0)
    lg = a.prefill_forward(torch.tensor([PROMPT]), None, None, torch.tensor([len(PROMPT)]))
    first = int(lg.view(-1).argmax())
    assert first == want[len(PROMPT)]
    out = [first]
    with pytest.raises(RuntimeError):  # greedy only: a first token that is not the argmax is refused
        a.decode_forward(torch.tensor([[first + 1]]), torch.tensor([len(PROMPT)]))
    while len(out) < N_NEW:
        blk = a.decode_forward(torch.tensor([[out[-1]]]), torch.tensor([len(PROMPT) + len(out) - 1]))
        assert blk.shape == (1, 4) and blk.dtype == torch.int32
        out += blk[0].tolist()
    assert out[:N_NEW] == want[len(PROMPT) : len(PROMPT) + N_NEW]
    a.release_request(0)
