"""torch.ops.qres: PyTorch custom ops over libqres's C ABI, registered when the package is imported.

The reference dispatches its device work as ttnn ops (``ttnn.generic_op`` per chip for the step,
qwen36_resident/model.py:1499-1508); here the same entry points are PyTorch custom ops that call the sm_100a
kernels of libqres on the current CUDA stream:

  qres::decode_step(ctx, tok, x, out, replay)  one decode step of a context (replay: its captured CUDA graph);
                                               tok / x / out must be the token state, residual and output
                                               buffers bound to that context (they are what the step mutates
                                               and what a caller reads)
  qres::topk(logits, base) -> (lists, argmax)  top-32 list and argmax per row (sampling.hpp order and ties)
  qres::sample(lists, words, pos) -> tokens    the sampling draw per row (sampling.hpp:113-143)
  qres::quantize_fp8(w) -> (q, scales)         FP8-e4m3 with one fp32 scale per 128 x 128 block

There is no CPU implementation of any of them: on a tensor that is not on a CUDA device they raise.
"""
import torch

from . import _lib

_BOUND = {}  # context handle -> data pointers of its bound (tok, x, out)


def bind_context(ctx, tok, x, out):
    """record the buffers a context was bound with, so decode_step can refuse other tensors"""
    _BOUND[int(ctx.value if hasattr(ctx, "value") else ctx)] = (tok.data_ptr(), x.data_ptr(), out.data_ptr())


def unbind_context(ctx):
    _BOUND.pop(int(ctx.value if hasattr(ctx, "value") else ctx), None)


def _cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise _lib.QresError("torch.ops.qres runs on CUDA tensors only (there is no CPU implementation)")


@torch.library.custom_op("qres::decode_step", mutates_args=("tok", "x", "out"))
def decode_step(ctx: int, tok: torch.Tensor, x: torch.Tensor, out: torch.Tensor, replay: bool) -> None:
    _cuda(tok, x, out)
    if _BOUND.get(ctx) != (tok.data_ptr(), x.data_ptr(), out.data_ptr()):
        raise _lib.QresError("qres::decode_step: tok / x / out are not the buffers bound to this context")
    c, s, L = _lib.ctypes.c_void_p(ctx), _lib.stream_ptr(), _lib.lib()
    if replay:
        _lib.check(L.qres_replay(c, s), c, "replay")
    else:
        _lib.check(L.qres_decode_step(c, s), c, "decode step")


@decode_step.register_fake
def _(ctx, tok, x, out, replay):
    return None


@torch.library.custom_op("qres::topk", mutates_args=())
def topk(logits: torch.Tensor, base: int) -> tuple[torch.Tensor, torch.Tensor]:
    _cuda(logits)
    return _lib.topk(logits.contiguous(), base)


@topk.register_fake
def _(logits, base):
    rows = logits.shape[0]
    return logits.new_empty(rows, 2 * _lib.QRES_TOPK, dtype=torch.int32), logits.new_empty(rows, dtype=torch.int32)


@torch.library.custom_op("qres::sample", mutates_args=())
def sample(lists: torch.Tensor, words: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    _cuda(lists, words, pos)
    rows = lists.shape[0]
    lists, words, pos = lists.contiguous(), words.contiguous(), pos.to(torch.int32).contiguous()
    tok = torch.empty(rows, dtype=torch.int32, device=lists.device)
    _lib.check(_lib.lib().qres_sample(rows, _lib.ptr(lists), _lib.ptr(words), _lib.ptr(pos), _lib.ptr(tok),
                                      _lib.stream_ptr()), None, "sample")
    return tok


@sample.register_fake
def _(lists, words, pos):
    return lists.new_empty(lists.shape[0], dtype=torch.int32)


@torch.library.custom_op("qres::quantize_fp8", mutates_args=())
def quantize_fp8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _cuda(w)
    return _lib.quantize_fp8(w.float().contiguous())


@quantize_fp8.register_fake
def _(w):
    N, K = w.shape
    return w.new_empty(N, K, dtype=torch.uint8), w.new_empty(-(-N // 128), -(-K // 128), dtype=torch.float32)
