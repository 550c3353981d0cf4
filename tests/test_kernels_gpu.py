"""Kernel-level parity of libqres (through its C ABI) against the CPU oracle, on seeded inputs.

Tolerances: FP8 quantisation, weight tiling, paged-KV indexing and top-k / argmax are bit-exact. bf16
outputs (projections, mixer outputs) may differ from the oracle by one bf16 rounding where fp32 summation order
moves a value across a rounding boundary: at most 2% of the elements differ, each by at most one bf16 ulp of
its magnitude plus 1e-3 of the vector's largest magnitude (values near zero carry the fp32 sum's absolute
error), and every element below magnitude 4 -- where one bf16 ulp is at most 2^-6 -- within an absolute 2e-2
(bf16 activations within atol 2e-2; above 4 a single rounding flip is 2^-5 or more, which only the ulp bound
can state). fp32 outputs (residual updates, the GDN state) match to a relative error of 1e-5.

Every device argument is held in a variable until the kernel has run: a temporary's memory returns to torch's
caching allocator at once and would be handed to the next tensor.
"""
import ctypes

import pytest
import torch

from oracle import fp8, paged, sampling, step
from oracle.refgen import bf16
from tt_qwen_resident_b200 import _lib, weights

pytestmark = pytest.mark.gpu


def ulp_mismatch(got, ref):
    """(fraction of differing bf16 values, max |diff| in ulps of the reference)"""
    g, r = got.float().cpu(), ref.float().cpu()
    diff = (g - r).abs()
    ulp = torch.clamp(r.abs(), min=1e-30)
    ulp = 2.0 ** (torch.floor(torch.log2(ulp)) - 7)
    return float((g != r).float().mean()), float((diff / ulp).max())


def bf16_close(got, ref, frac=2e-2, atol=2e-2):
    g, r = got.float().cpu().flatten(), ref.float().cpu().flatten()
    diff = (g - r).abs()
    ulp = 2.0 ** (torch.floor(torch.log2(r.abs().clamp(min=1e-30))) - 7)  # one bf16 ulp at |r|
    bound = ulp + 1e-3 * r.abs().max()
    f = float((g != r).float().mean())
    err = float(diff[r.abs() < 4].max()) if bool((r.abs() < 4).any()) else 0.0
    worst = float((diff / bound).max())
    assert f <= frac and worst <= 1.0 and err <= atol, (f, worst, err)


def test_quantize_bitexact(cuda):
    g = torch.Generator().manual_seed(0)
    for N, K in ((300, 640), (128, 5120), (517, 384)):
        w = torch.randn(N, K, generator=g) * 0.02
        w[:3, :5] = 0.0
        w[130:140, 200:260] *= 50.0  # a block with a large amax
        q_ref, s_ref = fp8.quantize_blocks(w)
        q, s = _lib.quantize_fp8(w.to(cuda))
        assert torch.equal(s.cpu(), s_ref)
        assert torch.equal(q.cpu(), q_ref)


def test_tile_layout_bitexact(cuda):
    """128-row tiles of 16 KB units; inside a unit the tensor core's 128-byte-swizzled K-major rows: byte (r, c)
    at r * 128 + ((c / 16) ^ (r % 8)) * 16 + c % 16"""
    g = torch.Generator().manual_seed(1)
    for rows, K in ((10, 640), (200, 768), (5, 2176), (257, 128)):
        q = torch.randint(0, 255, (rows, K), generator=g, dtype=torch.uint8)
        q_d = q.to(cuda)
        t = _lib.tile_weight(q_d).cpu()
        rows_pad = (rows + 127) // 128 * 128
        qp = torch.zeros(rows_pad, K, dtype=torch.uint8)
        qp[:rows] = q
        units = qp.view(rows_pad // 128, 128, K // 128, 8, 16).permute(0, 2, 1, 3, 4)  # [T, kb, r, chunk, 16]
        r = torch.arange(128).view(128, 1)
        src_chunk = torch.arange(8).view(1, 8) ^ (r % 8)  # stored chunk position c' holds chunk c' ^ (r % 8)
        ref = units[:, :, torch.arange(128).view(128, 1), src_chunk].reshape(-1)
        assert torch.equal(t, ref)


def _proj(N, K, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * scale
    q, s = fp8.quantize_blocks(w)
    return weights.FP8Matrix(q, s), fp8.dequantize_blocks(q, s)


@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("N,K", [(16480, 5120), (2060, 5120), (5120, 768), (5120, 2176), (5120, 17408), (300, 128)])
def test_gemv_parity(cuda, rows, N, K):
    m, wd = _proj(N, K, seed=N + K)
    gw = weights.shard(weights.FP8Matrix(m.q.to(cuda), m.scales.to(cuda)))
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, K, generator=g) * 3.0
    # rmsnorm prologue, bf16 out
    out = torch.empty(rows, N, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    x_d = x.to(cuda)
    _lib.gemv(gw, x_d, 0, 0, out, err)
    h = bf16(step.rmsnorm(x))
    ref = bf16(h @ wd.T)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    bf16_close(out, ref)
    # bf16 input, residual epilogue (fp32)
    hb = bf16(torch.randn(rows, K, generator=g))
    resid = torch.randn(rows, N, generator=g)
    o2 = resid.clone().to(cuda)
    hb_d = hb.to(cuda).bfloat16()
    _lib.gemv(gw, hb_d, 1, 2, o2, err)
    ref2 = hb @ wd.T + resid
    rel = float((o2.cpu() - ref2).norm() / ref2.norm())
    assert rel < 1e-5, rel
    # the step's fixed-point accumulation (epi 4; with 4 or more rows the units walk in K groups): value = out 2^-30
    acc = torch.zeros(rows, N, dtype=torch.int64, device=cuda)
    _lib.gemv(gw, hb_d, 1, 4, acc, err)
    got = acc.cpu().double() * 2.0**-30
    ref3 = hb.double() @ wd.T.double()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    rel = float((got - ref3).norm() / ref3.norm())
    assert rel < 1e-5, rel


@pytest.mark.parametrize("rows", [1, 5])
def test_gemv_swiglu_parity(cuda, rows):
    n = 8
    d = weights.RankDims(3, n)
    G, Gd = _proj(17408, 5120, seed=11, scale=1 / 70)
    U, Ud = _proj(17408, 5120, seed=12, scale=1 / 70)
    GU = weights.stack_matrices(weights.FP8Matrix(G.q.to(cuda), G.scales.to(cuda)), weights.FP8Matrix(U.q.to(cuda), U.scales.to(cuda)))
    gw = weights.shard(GU, d.gateup_rows())
    x = torch.randn(rows, 5120, generator=torch.Generator().manual_seed(3)) * 2
    out = torch.empty(rows, d.ic, dtype=torch.bfloat16, device=cuda)
    x_d = x.to(cuda)
    _lib.gemv(gw, x_d, 0, 1, out)
    h = bf16(step.rmsnorm(x))
    cols = torch.arange(3 * d.ic, 4 * d.ic)
    ref = bf16(torch.nn.functional.silu(h @ Gd[cols].T) * (h @ Ud[cols].T))
    bf16_close(out, ref)


@pytest.mark.parametrize("n,r", [(1, 0), (4, 1), (8, 7)])
@pytest.mark.parametrize("rows", [1, 2, 3, 5, 8])
def test_gdn_mixer_parity(cuda, n, r, rows):
    s = step.Shard(r, n)
    d = weights.RankDims(r, n)
    g = torch.Generator().manual_seed(10 * n + r + rows)
    ld_y = d.gdn_rows_n + 8
    y = bf16(torch.randn(rows, ld_y, generator=g))
    taps = bf16(0.5 * torch.randn(d.conv, 4, generator=g))
    wg = dict(dt=0.5 * torch.randn(48, generator=g), neg_a=-torch.exp(torch.rand(48, generator=g) * 2 - 1),
              norm_w=bf16(1 + 0.1 * torch.randn(128, generator=g)))
    S = 0.05 * torch.randn(rows, 48, 128, 128, generator=g)
    hist = bf16(torch.randn(rows, 3, d.conv, generator=g))
    pos = [5 + 3 * b for b in range(rows)]
    # device state
    S_d = S[:, s.r * s.nv : (s.r + 1) * s.nv].contiguous().to(cuda)
    H_d = torch.zeros(rows, 8, d.conv, dtype=torch.bfloat16, device=cuda)
    for b in range(rows):
        for age in range(3):
            H_d[b, (pos[b] - 3 + age) % 8] = hist[b, age].bfloat16().to(cuda)
    o_d = torch.empty(rows, d.gv, dtype=torch.bfloat16, device=cuda)
    pos_d = torch.tensor(pos, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    y_d = y.bfloat16().to(cuda)
    taps_d = taps.bfloat16().to(cuda)
    dt_d = wg["dt"][s.r * s.nv:(s.r + 1) * s.nv].contiguous().to(cuda)
    na_d = wg["neg_a"][s.r * s.nv:(s.r + 1) * s.nv].contiguous().to(cuda)
    nw_d = wg["norm_w"].to(cuda)
    L = _lib.lib()
    _lib.check(
        L.qres_gdn_mixer(n, rows, _lib.ptr(y_d), ld_y, _lib.ptr(pos_d), _lib.ptr(taps_d), _lib.ptr(dt_d), _lib.ptr(na_d),
                         _lib.ptr(nw_d), _lib.ptr(S_d), _lib.ptr(H_d), _lib.ptr(o_d), _lib.ptr(err), _lib.stream_ptr()),
        None, "gdn")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for b in range(rows):
        Sb = S[b].clone()
        o_ref, hist_new = step.gdn_mixer(y[b], s, taps, wg, hist[b], Sb)
        bf16_close(o_d[b], o_ref)
        got = S_d[b].cpu()
        ref = Sb[s.r * s.nv:(s.r + 1) * s.nv]
        assert float((got - ref).norm() / ref.norm()) < 1e-5
        # the history ring: slot of pos holds the new input, the read slots untouched
        assert torch.equal(H_d[b, pos[b] % 8].float().cpu(), hist_new[2])
        assert torch.equal(H_d[b, (pos[b] - 1) % 8].float().cpu(), hist_new[1])


def _rope(pos, max_pos):
    cos, sin = [], []
    for p in range(max_pos):
        c, s_ = step.rope_tables(p)
        cos.append(c)
        sin.append(s_)
    return torch.stack(cos), torch.stack(sin)


@pytest.mark.parametrize("n,r", [(1, 0), (2, 1), (8, 5)])
@pytest.mark.parametrize("pos", [0, 63, 64, 700])
def test_attn_mixer_parity_paged(cuda, n, r, pos):
    s = step.Shard(r, n)
    d = weights.RankDims(r, n)
    rows = 2
    max_pos = 1024
    max_pages = max_pos // 64
    g = torch.Generator().manual_seed(pos + 7 * n)
    ld_y = d.attn_rows_n
    y = bf16(torch.randn(rows, ld_y, generator=g))
    wq, wk = bf16(1 + 0.1 * torch.randn(256, generator=g)), bf16(1 + 0.1 * torch.randn(256, generator=g))
    K = [bf16(torch.randn(4, max_pos, 256, generator=g)) for _ in range(rows)]
    V = [bf16(torch.randn(4, max_pos, 256, generator=g)) for _ in range(rows)]
    # shuffled page table over a shared pool
    perm = torch.randperm(rows * max_pages, generator=g).to(torch.int32).view(rows, max_pages)
    kp = torch.zeros(rows * max_pages, d.nkv, 64, 256)
    vp = torch.zeros_like(kp)
    for b in range(rows):
        for j in range(d.nkv):
            paged.scatter(kp[:, j:j + 1], perm[b], K[b][d.kv0 + j:d.kv0 + j + 1])
            paged.scatter(vp[:, j:j + 1], perm[b], V[b][d.kv0 + j:d.kv0 + j + 1])
    kp_d, vp_d = kp.bfloat16().to(cuda), vp.bfloat16().to(cuda)
    cos, sin = _rope(pos, max_pos)
    sz = ctypes.c_size_t()
    L = _lib.lib()
    _lib.check(L.qres_attn_workspace_size(n, rows, max_pos, ctypes.byref(sz)), None, "ws")
    work = torch.zeros(sz.value, dtype=torch.uint8, device=cuda)
    o_d = torch.empty(rows, d.gv, dtype=torch.bfloat16, device=cuda)
    pos_d = torch.tensor([pos, pos + 5], dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    keep = [y.bfloat16().to(cuda), perm.to(cuda), (wq / 16).to(cuda), wk.to(cuda), cos.to(cuda), sin.to(cuda)]
    y_d, pt_d, wq_d, wk_d, cos_d, sin_d = keep
    args = (n, rows, _lib.ptr(y_d), ld_y, _lib.ptr(pos_d), _lib.ptr(pt_d), max_pages, _lib.ptr(wq_d), _lib.ptr(wk_d),
            _lib.ptr(cos_d), _lib.ptr(sin_d), _lib.ptr(kp_d), _lib.ptr(vp_d), _lib.ptr(o_d), _lib.ptr(work), sz.value,
            _lib.ptr(err), _lib.stream_ptr())
    _lib.check(L.qres_attn_mixer(*args), None, "attn")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for b in range(rows):
        p = pos + 5 * b
        c, sn = step.rope_tables(p)
        Kb, Vb = K[b].clone(), V[b].clone()
        o_ref = step.attn_mixer(y[b], s, wq, wk, Kb, Vb, p, c, sn)
        bf16_close(o_d[b], o_ref)
        # the appended row sits in its page slot; every other row of the cache is untouched (bit-exact)
        got_k = paged.gather(kp_d[:, :].float().cpu(), perm[b], p + 1)
        got_v = paged.gather(vp_d[:, :].float().cpu(), perm[b], p + 1)
        for j in range(d.nkv):
            assert torch.equal(got_k[j, :p], K[b][d.kv0 + j, :p])
            assert torch.equal(got_v[j, :p], V[b][d.kv0 + j, :p])
            assert torch.equal(got_v[j, p], Vb[d.kv0 + j, p])
            bf16_close(got_k[j, p], Kb[d.kv0 + j, p], frac=0.05)


@pytest.mark.parametrize("n", [248320, 31040, 1000, 7])
@pytest.mark.parametrize("rows", [1, 8])
def test_topk_bitexact(cuda, n, rows):
    g = torch.Generator().manual_seed(n + rows)
    lg = (torch.randn(rows, n, generator=g) * 2).bfloat16()
    for b in range(rows):
        if n > 40:
            top = int(lg[b].float().argmax())
            for j in (3, n // 2, n - 1, 17 + b):
                lg[b, j] = lg[b, top]  # ties at the maximum
            lg[b, 20:25] = lg[b].float().kthvalue(n - 31).values  # ties at the 32nd place
    lg_d = lg.to(cuda)
    lists, am = _lib.topk(lg_d, base=123)
    lists = lists.cpu().to(torch.int64) & 0xFFFFFFFF
    for b in range(rows):
        ks, ix = sampling.topk_list(lg[b].float(), base=123)
        assert lists[b, :32].tolist() == ks
        assert lists[b, 32:].tolist() == ix
        assert int(am[b]) == 123 + sampling.argmax_rule(lg[b].float())
