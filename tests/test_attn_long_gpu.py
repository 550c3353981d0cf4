"""The gated-attention mixer at long context, through the C ABI, against the oracle (model.py:233-247):
BASELINE config 2's context (4096 positions, all 4 KV heads on one rank) and config 5's (131,072 positions, one KV
head: a rank of 4). K and V are N(0, 1) bf16 behind a shuffled page table of 64-position pages; the step decodes
the last position. The output must be within the bf16 rounding bound of test_kernels_gpu.bf16_close, the
appended K row likewise, the appended V row exact, and every other cache row untouched (bit-exact).
"""
import ctypes

import pytest
import torch

from oracle import step
from oracle.refgen import bf16
from tt_qwen_resident_b200 import _lib, weights
from test_kernels_gpu import bf16_close

pytestmark = pytest.mark.gpu


def rope_rows(max_pos):
    """cos / sin [max_pos, 32] exactly as step.rope_tables computes each row (fp64 angle pos * inv, to fp32)"""
    inv = 1.0 / step.ROPE_THETA ** (torch.arange(0, step.ROT, 2, dtype=torch.float64) / step.ROT)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv
    return torch.cos(ang).float(), torch.sin(ang).float()


@pytest.mark.parametrize("n,r,ctx", [(1, 0, 4096), (4, 1, 4096), (4, 2, 131072)])
def test_attn_mixer_long_context(cuda, n, r, ctx):
    s = step.Shard(r, n)
    d = weights.RankDims(r, n)
    pos = ctx - 1  # the new row is the context's last position
    max_pages = ctx // 64
    g = torch.Generator().manual_seed(ctx + r)
    y = bf16(torch.randn(1, d.attn_rows_n, generator=g))
    wq, wk = bf16(1 + 0.1 * torch.randn(256, generator=g)), bf16(1 + 0.1 * torch.randn(256, generator=g))
    K = {d.kv0 + j: bf16(torch.randn(ctx, 256, generator=g)) for j in range(d.nkv)}
    V = {d.kv0 + j: bf16(torch.randn(ctx, 256, generator=g)) for j in range(d.nkv)}
    for t in list(K.values()) + list(V.values()):
        t[pos:] = 0
    perm = torch.randperm(max_pages, generator=g).to(torch.int32)

    def pool_of(rows):  # [nkv][ctx, 256] -> [pages, nkv, 64, 256] at the page table's pages
        pl = torch.zeros(max_pages, d.nkv, 64, 256, dtype=torch.bfloat16)
        st = torch.stack([rows[d.kv0 + j] for j in range(d.nkv)]).bfloat16()  # [nkv, ctx, 256]
        pl[perm.long()] = st.view(d.nkv, max_pages, 64, 256).permute(1, 0, 2, 3)
        return pl

    kp0, vp0 = pool_of(K), pool_of(V)
    kp_d, vp_d = kp0.to(cuda), vp0.to(cuda)
    cos, sin = rope_rows(ctx)
    c_ref, s_ref = step.rope_tables(pos)
    assert torch.equal(cos[pos], c_ref) and torch.equal(sin[pos], s_ref)
    sz = ctypes.c_size_t()
    L = _lib.lib()
    _lib.check(L.qres_attn_workspace_size(n, 1, ctx, ctypes.byref(sz)), None, "ws")
    work = torch.zeros(sz.value, dtype=torch.uint8, device=cuda)
    o_d = torch.empty(1, d.gv, dtype=torch.bfloat16, device=cuda)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    y_d, pt_d, wq_d, wk_d = y.bfloat16().to(cuda), perm.view(1, -1).to(cuda), (wq / 16).to(cuda), wk.to(cuda)
    cos_d, sin_d = cos.to(cuda), sin.to(cuda)
    _lib.check(
        L.qres_attn_mixer(n, 1, _lib.ptr(y_d), d.attn_rows_n, _lib.ptr(pos_d), _lib.ptr(pt_d), max_pages, _lib.ptr(wq_d),
                          _lib.ptr(wk_d), _lib.ptr(cos_d), _lib.ptr(sin_d), _lib.ptr(kp_d), _lib.ptr(vp_d), _lib.ptr(o_d),
                          _lib.ptr(work), sz.value, _lib.ptr(err), _lib.stream_ptr()),
        None, "attn")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.set_num_threads(8)
    o_ref = step.attn_mixer(y[0], s, wq, wk, K, V, pos, c_ref, s_ref)  # writes row pos of K / V
    bf16_close(o_d[0], o_ref)
    kp, vp = kp_d.cpu(), vp_d.cpu()
    pg, row = int(perm[pos // 64]), pos % 64
    for j in range(d.nkv):
        bf16_close(kp[pg, j, row].float(), K[d.kv0 + j][pos], frac=0.05)
        assert torch.equal(vp[pg, j, row].float(), V[d.kv0 + j][pos])
    kp[pg, :, row] = kp0[pg, :, row]
    vp[pg, :, row] = vp0[pg, :, row]
    assert torch.equal(kp, kp0) and torch.equal(vp, vp0)  # every other row untouched
