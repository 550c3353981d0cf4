"""vLLM-facing adapter of the resident decode model on B200: the call contract of sott0n/tt-qwen-resident's
``Qwen36ResidentForCausalLM`` (qwen36_resident/generator_vllm.py:34-160) over ``ResidentModel``.

One user. The model owns its KV cache, GDN state and conv history, so the plugin's paged KV cache is not used
(``allocate_kv_cache`` returns nothing). Decode steps whose sampling the runner hands to the device (greedy, or
top-k <= 32 with temperature / top-p) run asynchronously under decode input update contract 1: every step draws
the next token on the device from the merged top-32 list and writes the next step's token state, so a step
without ``reload_inputs`` only replays the captured step, and the runner reads the (token, position) word one step
late. Any other step (``sampling_params`` None) returns the full logits for the host to sample, the host writing
the token state.

Differences by design: the prompt runs through the decode step itself, one token per step (the reference's
chunked pipeline-parallel prefill is not part of this build); weights come from the caller (``weights=``, e.g.
``weights.random_canonical`` or a converted checkpoint) since the reference's Tenstorrent checkpoint loader does
not apply.
"""
import os

import torch

from . import weights as W
from .model import TOP_K, ResidentModel


def _field(cfg, name, default=None):
    if isinstance(cfg, dict):
        return cfg.get(name, default)
    return getattr(cfg, name, default)


class Qwen36ResidentForCausalLM:
    model_capabilities = {
        "supports_prefix_caching": False,
        "supports_async_decode": True,
        # the device draws from the top TOP_K logits; anything else samples on the host from the logits
        "supports_sample_on_device": True,
        "max_device_top_k": TOP_K,
        "supports_device_penalties": False,
    }
    decode_input_update_contract = 1

    def __init__(self, model, max_seq_len, mrope=False):
        assert model.batch == 1 and model.lm_head and model.embed is not None, "one user with an lm_head and embedding"
        self.model = model
        self.vocab = model.vocab
        self.max_seq_len = max_seq_len
        self.mrope = mrope
        self._host_out = None  # pinned host copy of the output word, made at the first device read
        model.capture_trace()

    @classmethod
    def initialize_vllm_model(cls, hf_config, mesh_device, max_batch_size, max_seq_len, weights=None, embed=None,
                              mrope=False, **kwargs):
        """hf_config: num_hidden_layers, full_attention_interval, vocab_size (a dict or a config object);
        mesh_device: the torch device of this rank (one GPU per process); weights / embed: canonical FP8 weights
        and the bf16 embedding table (random-init of the named shape when None)"""
        assert max_batch_size == 1, "one decode user per model: serve with max_num_seqs=1"
        layers, interval = int(_field(hf_config, "num_hidden_layers")), int(_field(hf_config, "full_attention_interval"))
        vocab = int(_field(hf_config, "vocab_size"))
        dev = torch.device(mesh_device) if mesh_device is not None else torch.device("cuda", torch.cuda.current_device())
        if weights is None:
            weights = W.random_canonical(layers, interval, vocab, seed=0, device=dev)
        if embed is None:
            g = torch.Generator(device=dev).manual_seed(1)
            embed = torch.randn(vocab, W.HIDDEN, generator=g, device=dev).bfloat16()
        model = ResidentModel(weights, layers, interval, batch=1, max_pos=max_seq_len + 8, lm_head=True, embed=embed,
                              device=dev)
        return cls(model, max_seq_len, mrope=mrope)

    @classmethod
    def get_max_tokens_all_users(cls, max_model_len=None, max_num_seqs=None, **kwargs):
        return int(max_model_len) * int(max_num_seqs or 1)

    def allocate_kv_cache(self, kv_cache_shape, dtype, num_layers):
        return []

    def warmup_model_prefill(self, *args, **kwargs):
        pass

    def warmup_model_decode(self, *args, **kwargs):
        pass

    def _write_token(self, token, pos, feed=False):
        assert pos < self.max_seq_len, f"position {pos} is past max_model_len {self.max_seq_len}"
        return self.model.token_state(tokens=int(token), pos=int(pos), feed=feed)

    def _step(self, token, pos):
        """one host-fed step: the logits [1, 1, vocab] for the host to sample"""
        self.model.step(self._write_token(token, pos))
        return self.model.logits().view(1, 1, -1)

    def prefill_forward(self, tokens, page_table, kv_cache, prompt_lens, **kwargs):
        assert tokens.shape[0] == 1, "one user per prefill"
        T = int(prompt_lens[0]) if prompt_lens is not None else tokens.shape[1]
        ids = tokens[0, :T].tolist()
        self.model.reset()
        for p, t in enumerate(ids[:-1]):
            self.model.step(self._write_token(t, p))
        logits = self._step(ids[-1], T - 1)
        return (logits, torch.zeros(1, dtype=torch.long)) if self.mrope else logits

    def decode_forward(self, tokens, start_pos, *args, reload_inputs=True, reload_page_table=False,
                       reload_sampling_params=False, reset_sampling_state=False, read_from_device=False,
                       sampling_params=None, **kwargs):
        assert "reset_batch" not in kwargs, "contract 1 adapters take the explicit reload commands"
        token, pos = tokens.reshape(-1)[0], start_pos.reshape(-1)[0]
        # sampling_params arrive only on the steps the runner samples on device (top-k <= TOP_K or greedy)
        if sampling_params is None:
            return self._step(token, pos)
        if reload_sampling_params:
            self.model.set_sampling(float(sampling_params.temperature[0]), int(sampling_params.top_k[0]),
                                    float(sampling_params.top_p[0]), int(sampling_params.seed[0]))
        # without reload_inputs, tokens and start_pos are one step behind: the device wrote the token state
        self.model.step(self._write_token(token, pos, feed=True) if reload_inputs else None)
        if read_from_device:
            return self.process_decode_output_host(self.read_decode_output(self.model.out_d))
        return self.model.out_d

    def read_decode_output(self, out, async_read=False, **kwargs):
        """enqueue the read of the fed (token, position) word, ahead of the next replay; host tensors (the logits
        of a host-sampled step) pass through"""
        if not out.is_cuda:
            return (out, []) if async_read else out
        if self._host_out is None:
            self._host_out = torch.zeros(out.shape, dtype=torch.int32).pin_memory()
        host = self._host_out
        host.copy_(out, non_blocking=True)
        if async_read:
            ev = torch.cuda.Event()
            ev.record()
            return host, [ev]
        torch.cuda.current_stream(out.device).synchronize()
        return host

    def process_decode_output_host(self, out, is_tokens=True, **kwargs):
        if out.dtype != torch.int32:  # logits of a host-sampled step
            return out
        return out.reshape(-1)[:1].to(torch.int32).view(1, 1).clone()


MTP_BLOCK = int(os.environ.get("QWEN36_MTP_BLOCK", "4"))


class Qwen36ResidentMTPForCausalLM(Qwen36ResidentForCausalLM):
    """Greedy MTP speculative decode through the plugin's block output (generator_vllm.py:167-228): every decode
    step commits MTP_BLOCK tokens (fewer only at the position limit, padded with eos). Greedy only: the device
    decodes from its own greedy tokens, so the runner's first token (sampled from the prefill's logits) must be
    their argmax; anything else raises. One user (max_num_seqs=1)."""

    model_capabilities = {
        "supports_prefix_caching": False,
        "supports_async_decode": True,
        "supports_sample_on_device": True,
        "supports_device_penalties": False,
        "output_tokens_per_step": MTP_BLOCK,
        "tt_adaptive_block_output": True,
    }

    def __init__(self, spec, max_seq_len, eos, mrope=False):
        self.spec = spec
        self.vocab = spec.main.vocab
        self.max_seq_len = max_seq_len
        self.eos = int(eos)
        self.mrope = mrope
        self._first = None

    def prefill_forward(self, tokens, page_table, kv_cache, prompt_lens, **kwargs):
        assert tokens.shape[0] == 1, "one user per prefill"
        T = int(prompt_lens[0]) if prompt_lens is not None else tokens.shape[1]
        logits = self.spec.start(tokens[0, :T].tolist())
        self._first = int(logits.argmax())
        # only the argmax the device decodes from may be sampled (the plugin samples block models' prefill
        # logits at temperature 1)
        logits = torch.full_like(logits, float("-inf"))
        logits[self._first] = 0
        logits = logits.view(1, 1, -1)
        return (logits, torch.zeros(1, dtype=torch.long)) if self.mrope else logits

    def decode_forward(self, tokens, start_pos, *args, **kwargs):
        if self._first is not None:
            token = int(tokens.reshape(-1)[0])
            if token != self._first:
                raise RuntimeError(f"MTP serving is greedy only: the runner's first token {token} is not the argmax "
                                   f"{self._first} the device decodes from")
            self._first = None
        block = self.spec.next_block(MTP_BLOCK, self.max_seq_len)
        out = torch.full((1, MTP_BLOCK), self.eos, dtype=torch.int32)
        out[0, : len(block)] = torch.tensor(block, dtype=torch.int32)
        return out

    def release_request(self, row):
        self.spec.stop()
        self._first = None
