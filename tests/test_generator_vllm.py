"""The vLLM adapter's call contract on the CPU (no GPU): Qwen36ResidentForCausalLM over a stand-in model that
records what the adapter asks of it, after the reference adapter (qwen36_resident/generator_vllm.py:34-160):
the prompt runs through the decode step (all but the last token host-fed, then the last for the first logits);
a decode step without sampling parameters is host-fed and returns the logits; with them the sampling words are
reloaded on request, the token state is written (fed on the device) only on reload_inputs, otherwise the step
just replays, and read_from_device returns the fed token as an int32 [1, 1]."""
from types import SimpleNamespace

import pytest
import torch

from tt_qwen_resident_b200.generator_vllm import Qwen36ResidentForCausalLM

V = 64


class StandIn:
    """the ResidentModel surface the adapter uses, recording every call"""

    batch, lm_head, vocab, embed = 1, True, V, object()

    def __init__(self):
        self.calls = []
        self.out_d = torch.tensor([[7, 0, 7, 0]], dtype=torch.int32)

    def capture_trace(self):
        self.calls.append(("capture",))

    def reset(self):
        self.calls.append(("reset",))

    def token_state(self, tokens, pos, feed=False):
        return ("tok", tokens, pos, feed)

    def step(self, tok=None):
        self.calls.append(("step", tok))
        if tok is not None:
            self.out_d[0, 1] = tok[2] + 1
        else:
            self.out_d[0, 1] += 1

    def logits(self):
        return torch.arange(V, dtype=torch.float32)

    def set_sampling(self, temperature, top_k, top_p, seed):
        self.calls.append(("sampling", temperature, top_k, top_p, seed))


def test_prefill_runs_the_prompt_through_the_decode_step():
    m = StandIn()
    a = Qwen36ResidentForCausalLM(m, max_seq_len=32)
    assert a.allocate_kv_cache((1,), torch.bfloat16, 64) == []
    assert Qwen36ResidentForCausalLM.get_max_tokens_all_users(max_model_len=32, max_num_seqs=1) == 32
    lg = a.prefill_forward(torch.tensor([[5, 6, 7, 8, 9]]), None, None, torch.tensor([5]))
    assert lg.shape == (1, 1, V)
    steps = [c for c in m.calls if c[0] == "step"]
    assert m.calls[:2] == [("capture",), ("reset",)]
    assert [s[1] for s in steps] == [("tok", t, p, False) for p, t in enumerate([5, 6, 7, 8, 9])]


def test_decode_contract():
    m = StandIn()
    a = Qwen36ResidentForCausalLM(m, max_seq_len=32)
    # host-sampled step: host-fed, logits back
    lg = a.decode_forward(torch.tensor([[11]]), torch.tensor([3]))
    assert lg.shape == (1, 1, V) and m.calls[-1] == ("step", ("tok", 11, 3, False))
    sp = SimpleNamespace(temperature=[0.7], top_k=[20], top_p=[0.9], seed=[42])
    # device-sampled: reload the words and the inputs, read the fed token
    t = a.decode_forward(torch.tensor([[12]]), torch.tensor([4]), reload_sampling_params=True, read_from_device=True,
                         sampling_params=sp)
    assert m.calls[-2] == ("sampling", 0.7, 20, 0.9, 42)
    assert m.calls[-1] == ("step", ("tok", 12, 4, True))
    assert t.dtype == torch.int32 and t.shape == (1, 1) and int(t) == 7
    # no reload: the device already wrote the token state, the step only replays
    out = a.decode_forward(torch.tensor([[0]]), torch.tensor([0]), reload_inputs=False, sampling_params=sp)
    assert m.calls[-1] == ("step", None) and out is m.out_d
    host = a.read_decode_output(out, async_read=True)
    assert isinstance(host, tuple) and int(a.process_decode_output_host(host[0])) == 7
    assert a.process_decode_output_host(lg) is lg  # the logits of a host-sampled step pass through
    with pytest.raises(AssertionError):
        a.decode_forward(torch.tensor([[0]]), torch.tensor([0]), reset_batch=True)
    with pytest.raises(AssertionError):
        a.decode_forward(torch.tensor([[0]]), torch.tensor([32]))  # past max_model_len


class StandInSpec:
    """the SpecDecoder surface the MTP block adapter uses"""

    def __init__(self):
        self.main = SimpleNamespace(vocab=V)
        self.calls = []

    def start(self, prompt):
        self.calls.append(("start", list(prompt)))
        lg = torch.zeros(V)
        lg[5] = 3.0
        return lg

    def next_block(self, n, limit):
        self.calls.append(("block", n, limit))
        return [1, 2, 3] if limit > 20 else [1]

    def stop(self):
        self.calls.append(("stop",))


def test_mtp_block_adapter_contract():
    from tt_qwen_resident_b200.generator_vllm import MTP_BLOCK, Qwen36ResidentMTPForCausalLM

    s = StandInSpec()
    a = Qwen36ResidentMTPForCausalLM(s, max_seq_len=32, eos=9)
    lg = a.prefill_forward(torch.tensor([[4, 4, 4]]), None, None, torch.tensor([3]))
    assert s.calls[0] == ("start", [4, 4, 4])
    assert lg.shape == (1, 1, V) and int(lg.view(-1).argmax()) == 5 and float(lg.view(-1)[0]) == float("-inf")
    with pytest.raises(RuntimeError):
        a.decode_forward(torch.tensor([[6]]), torch.tensor([3]))  # not the argmax the device decodes from
    out = a.decode_forward(torch.tensor([[5]]), torch.tensor([3]))
    assert out.dtype == torch.int32 and out.shape == (1, MTP_BLOCK)
    assert out[0].tolist() == [1, 2, 3] + [9] * (MTP_BLOCK - 3)  # short blocks padded with eos
    a.release_request(0)
    assert s.calls[-1] == ("stop",)
