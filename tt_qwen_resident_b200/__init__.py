"""B200-native resident decode step of a Qwen3.6-27B-shaped hybrid model (48 Gated DeltaNet + 16 gated
full-attention layers): hand-written sm_100a kernels in libqres.so (C ABI: include/qres.h) and the host
objects of sott0n/tt-qwen-resident's decode path (``ResidentModel``, the vLLM adapter) over them."""

from . import ops  # noqa: F401,E402  (registers torch.ops.qres.*)
