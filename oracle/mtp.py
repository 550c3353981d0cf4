"""MTP draft layer -- CPU restatement, TEST INFRASTRUCTURE ONLY (imported by tests/, never by the product).

The reference's draft entry (qwen36_resident/mtp.py:1-14 and :54-60, the fc on device at
kernels/streamer_compute.cpp:424-435 / streamer_common.hpp fc; the host math at tests/mtp_acceptance.py:70-81):
the draft model is one full-attention decoder layer with its own KV cache and the main model's lm_head; its
entry at position q takes x0 = fc([norm_e(e) | norm_h(h)]) for e = the embedding of the token at q + 1 and h
= the last x of the step at q (the main model's, or the previous draft's), with the pre-fc norm weights
(1 + w) folded into fc's columns (mtp.py:56-59). A chain of drafts feeds each draft's token and last x into
the next entry. Rounding points follow the device: e and h enter the fc as bf16 rows of their rmsnorm, the
fc's result (layer 0's residual) stays fp32, then the decode step of oracle.step runs the layer and the head.
Parity: pinned to nothing beyond the reference's formulas (the reference's MTP test needs the HF checkpoint,
absent here).
"""
import torch

from . import step
from .refgen import bf16


def draft_x0(e, h, fc):
    """e, h: [5120] fp32 rows; fc: [5120, 10240] fp32 (dequantised, norm weights folded) -> x0 [5120]"""
    return torch.cat([bf16(step.rmsnorm(e)), bf16(step.rmsnorm(h))]) @ fc.T


def draft_step(token, h, emb, fc, P, st, lm_head=True):
    """one draft entry at st.pos: returns (x, per-rank logits) of the draft model (one attention layer)"""
    x0 = draft_x0(emb[token].float(), h, fc)
    return step.torch_step(x0, P, st, 1, 1, lm_head=lm_head)
