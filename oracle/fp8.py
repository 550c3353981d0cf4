"""FP8-e4m3 weights with one fp32 scale per 128x128 block (TEST INFRASTRUCTURE ONLY).

The weight format the build streams (BASELINE: FP8-e4m3, one fp32 scale per 128 x 128 block). The reference
quantises to Tenstorrent block-float instead (``qwen36_resident/common.py:115-116``, ``model.py:53-59``); this
is the stand-in the oracle uses for its ``quantize`` and the byte format the GPU path must reproduce bit-exactly:

    scale = amax(|block|) / 448   (1 when the block is all zero)
    q     = fp8_e4m3(w / scale)   (fp32 division, round to nearest even)
    w'    = float(q) * scale      (what the oracle multiplies with)
"""
import torch

BLOCK = 128
E4M3_MAX = 448.0


def quantize_blocks(w):
    """w [N, K] float -> (q uint8 [N, K], scales float32 [ceil(N/128), ceil(K/128)])"""
    w = w.float()
    N, K = w.shape
    nb, kb = -(-N // BLOCK), -(-K // BLOCK)
    pad = torch.zeros(nb * BLOCK, kb * BLOCK)
    pad[:N, :K] = w
    blocks = pad.view(nb, BLOCK, kb, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn)
    q = q.view(nb * BLOCK, kb * BLOCK)[:N, :K].contiguous()
    return q.view(torch.uint8), scale.contiguous()


def dequantize_blocks(q, scales):
    """inverse of quantize_blocks: float32 [N, K]"""
    N, K = q.shape
    f = q.view(torch.float8_e4m3fn).float()
    s = scales.repeat_interleave(BLOCK, 0)[:N].repeat_interleave(BLOCK, 1)[:, :K]
    return f * s


def fake_quant(w):
    """w -> dequantize(quantize(w)): the values the GPU multiplies with"""
    return dequantize_blocks(*quantize_blocks(w))
