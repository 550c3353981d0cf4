"""Kernel microbenchmarks of libqres (one kernel at a time, CUDA events, L2 flushed between launches).

  python -m tt_qwen_resident_b200.microbench gemv [--rows 1] [--n 34816] [--k 5120] [--pro 0] [--epi 1]  (epi 4: fixed-point accumulators)
  python -m tt_qwen_resident_b200.microbench gdn [--rows 1] [--tp 1]
  python -m tt_qwen_resident_b200.microbench attn [--rows 1] [--tp 1] [--ctx 4096]

Each prints one JSON line: time per launch, algorithmic bytes per launch and the achieved bandwidth against
MEASURED_PEAKS.json (the repository root) when present. Inputs are random; the kernels are the ones the decode
step runs.
"""
import argparse
import ctypes
import json
import os
import statistics

import torch

from . import _lib, weights

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def timed(fn, reps, warm=3, flush_mb=256):
    dev = torch.device("cuda")
    flush = torch.empty(flush_mb << 20, dtype=torch.uint8, device=dev)
    for _ in range(warm):
        fn()
    ev = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    ts = [a.elapsed_time(b) for a, b in ev]
    return statistics.median(ts), min(ts)


def bench_gemv(a):
    dev = torch.device("cuda")
    N, K = a.n, a.k
    g = torch.Generator(device=dev).manual_seed(0)
    w32 = torch.randn(N, K, generator=g, device=dev) * 0.02
    m = weights.quantize(w32)
    del w32
    gw = weights.shard(m)
    x = torch.randn(a.rows, K, device=dev)
    if a.pro == 1:
        x = x.bfloat16()
    if a.epi == 1:
        out = torch.empty(a.rows, N // 2, dtype=torch.bfloat16, device=dev)
    elif a.epi == 0:
        out = torch.empty(a.rows, N, dtype=torch.bfloat16, device=dev)
    elif a.epi == 4:  # the step's fixed-point accumulators (int64; the sums grow over the repetitions)
        out = torch.zeros(a.rows, N, dtype=torch.int64, device=dev)
    else:
        out = torch.zeros(a.rows, N, device=dev)
    work = _lib.gemv_work(dev, gw.rows_pad, a.grid)
    fn = lambda: _lib.gemv(gw, x, a.pro, a.epi, out, grid=a.grid, work=work)
    med, best = timed(fn, a.reps)
    pk, kind = peak()
    gbs = gw.nbytes / (med * 1e-3) / 1e9
    return dict(kernel="gemv_fp8", rows=a.rows, N=N, K=K, pro=a.pro, epi=a.epi, ms=med, ms_best=best,
                bytes=gw.nbytes, GBps=gbs, frac=gbs / pk, peak=pk, peak_kind=kind)


def bench_gdn(a):
    dev = torch.device("cuda")
    n, R = a.tp, a.rows
    d = weights.RankDims(0, n)
    ld_y = d.gdn_rows_n
    y = torch.randn(R, ld_y, device=dev).bfloat16()
    taps = (0.5 * torch.randn(d.conv, 4, device=dev)).bfloat16()
    dt = torch.randn(d.nv, device=dev) * 0.5
    na = -torch.rand(d.nv, device=dev) - 0.5
    nw = torch.ones(128, device=dev)
    S = torch.randn(R, d.nv, 128, 128, device=dev) * 0.05
    H = torch.randn(R, 8, d.conv, device=dev).bfloat16()
    o = torch.empty(R, d.gv, dtype=torch.bfloat16, device=dev)
    pos = torch.full((R,), 100, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    args = [n, R, _lib.ptr(y), ld_y, _lib.ptr(pos), _lib.ptr(taps), _lib.ptr(dt), _lib.ptr(na), _lib.ptr(nw),
            _lib.ptr(S), _lib.ptr(H), _lib.ptr(o), _lib.ptr(err)]
    fn = lambda: _lib.check(L.qres_gdn_mixer(*args, _lib.stream_ptr()), None, "gdn")
    med, best = timed(fn, a.reps)
    nbytes = R * d.nv * 128 * 128 * 4 * 2 + R * 4 * d.conv * 2 + R * ld_y * 2
    pk, kind = peak()
    gbs = nbytes / (med * 1e-3) / 1e9
    return dict(kernel="gdn_decode", rows=R, tp=n, ms=med, ms_best=best, bytes=nbytes, GBps=gbs, frac=gbs / pk,
                peak=pk, peak_kind=kind)


def bench_attn(a):
    dev = torch.device("cuda")
    n, R, ctx = a.tp, a.rows, a.ctx
    d = weights.RankDims(0, n)
    max_pos = ctx + 64
    max_pages = -(-max_pos // 64)
    ld_y = d.attn_rows_n
    y = torch.randn(R, ld_y, device=dev).bfloat16()
    wq = torch.ones(256, device=dev) / 16
    wk = torch.ones(256, device=dev)
    ang = torch.arange(max_pos, dtype=torch.float64, device=dev)[:, None] * (
        1.0 / 1e7 ** (torch.arange(0, 64, 2, dtype=torch.float64, device=dev) / 64))
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    kp = torch.randn(R * max_pages, d.nkv, 64, 256, device=dev).bfloat16()
    vp = torch.randn(R * max_pages, d.nkv, 64, 256, device=dev).bfloat16()
    pt = torch.arange(R * max_pages, dtype=torch.int32, device=dev).view(R, max_pages)
    o = torch.empty(R, d.gv, dtype=torch.bfloat16, device=dev)
    pos = torch.full((R,), ctx, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    sz = ctypes.c_size_t()
    L = _lib.lib()
    _lib.check(L.qres_attn_workspace_size(n, R, max_pos, ctypes.byref(sz)), None, "ws")
    work = torch.zeros(sz.value, dtype=torch.uint8, device=dev)
    args = [n, R, _lib.ptr(y), ld_y, _lib.ptr(pos), _lib.ptr(pt), max_pages, _lib.ptr(wq), _lib.ptr(wk), _lib.ptr(cos),
            _lib.ptr(sin), _lib.ptr(kp), _lib.ptr(vp), _lib.ptr(o), _lib.ptr(work), sz.value, _lib.ptr(err)]
    fn = lambda: _lib.check(L.qres_attn_mixer(*args, _lib.stream_ptr()), None, "attn")
    med, best = timed(fn, a.reps)
    nbytes = R * (ctx + 1) * d.nkv * 256 * 2 * 2
    pk, kind = peak()
    gbs = nbytes / (med * 1e-3) / 1e9
    return dict(kernel="attn_decode", rows=R, tp=n, ctx=ctx, ms=med, ms_best=best, bytes=nbytes, GBps=gbs,
                frac=gbs / pk, peak=pk, peak_kind=kind)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemv", "gdn", "attn"])
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--n", type=int, default=34816)
    ap.add_argument("--k", type=int, default=5120)
    ap.add_argument("--pro", type=int, default=0)
    ap.add_argument("--epi", type=int, default=1)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--grid", type=int, default=0)
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    r = {"gemv": bench_gemv, "gdn": bench_gdn, "attn": bench_attn}[a.what](a)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
