"""Benchmark of the resident decode step (BASELINE.json metric: decode tok/s/user at batch 1, total tok/s at
batch 8, on 1/2/4/8 B200; % of the HBM roofline).

Default workload (N GPUs, one process each): BASELINE config 3 -- the full 64-layer Qwen3.6-27B-shaped model (48
GDN + 16 attention layers, every 4th attention), vocab 248,320, FP8 block-scaled random-init weights, batch 1; a
2,048-token uniform-random prompt is run through the decode step itself (prefill is out of scope), then greedy
decode steps are timed. The same run adds a `batch8` record (config 4: 8 users, 128-token prompts each, on the
same device weights) and, at N > 1, a `tp_check` of the tensor-parallel exchange. `--batch 8` makes config 4 the
headline; `--ctx 131072` gives config 5 (the attention KV random-filled to that context, decode from there).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--ctx C] [--impl ours|reference]

Arms:
  ours       timed region: K device-fed greedy steps (one CUDA-graph replay each), inputs resident in HBM (25.6 GB
             of weights per step, larger than L2), CUDA events on the launching stream, barrier + synchronize on
             both sides, max over ranks. e2e: the same metric through the public step call with host buffers:
             each step copies the token state from pinned host memory, replays the step and reads the picked
             token back.
  reference  the reference's decode math (its torch_step, restated in oracle/) on the host cores: every step one
             full 64-layer step with the reference's own weight-copies mechanism (2 distinct weight sets per
             layer kind, tests/bench_resident_batch.py) and the full lm_head, fp32; at batch 8 one user's step
             per sample (the oracle runs users one after another). Rank 0 only.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, INTERVAL, VOCAB = 64, 4, 248320


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=None, help="prompt tokens (default 2048 at batch 1, 128 at batch 8)")
    ap.add_argument("--ctx", type=int, default=0,
                    help="long context (config 5): random-fill the KV to this many positions instead of a prompt")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch8", action="store_true", help="skip the batch-8 record of a batch-1 run")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--tile-finish", action="store_true",
                    help="finish split projection tiles by ticket instead of the fixed-point accumulators (1 rank)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel exchange: the fused NVLink peer exchange (default) or NCCL (baseline)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def metric_name(batch):
    return "decode_tok_s_per_user" if batch == 1 else "decode_total_tok_s"


def prompt_of(args):
    return 0 if args.ctx else (args.prompt or (2048 if args.batch == 1 else 128))


def config_of(args, world):
    """the workload, identical in both arms"""
    batch, prompt = args.batch, prompt_of(args)
    cfg = 5 if args.ctx else (3 if batch == 1 else 4)
    start = f"KV random-filled to {args.ctx}" if args.ctx else f"{prompt}-token prompt"
    return {
        "workload": f"config{cfg}: 64-layer Qwen3.6-27B-shaped hybrid, vocab 248320, FP8 weights, batch {batch}, {start}",
        "batch": batch,
        "prompt": prompt,
        "ctx": args.ctx or None,
        "layers": args.layers,
        "parallelism": f"tp{world}",
        "l2": "inputs larger than L2 (25.6 GB of weights streamed per step)",
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region"""

    Q = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p is None:
            return
        time.sleep(0.25)
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out = ""
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) >= 9:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(self.rows),
        }


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ============================================================================================== CPU (reference)
class CpuStep:
    """the oracle (the reference's torch_step, restated) over a full 64-layer schedule in fp32 on the host cores,
    with the reference's weight-copies mechanism: 2 distinct weight sets per layer kind (layer l of a kind uses copy
    k % 2), every layer its own decode state, the full lm_head"""

    def __init__(self, ctx, threads):
        from oracle import refgen, step

        torch.set_num_threads(threads)
        self.threads = threads
        g = torch.Generator().manual_seed(0)
        rn = lambda *s: torch.randn(*s, generator=g) * 0.02
        w = refgen.Canon()
        w.gdn = [dict(Win=rn(refgen.GDN_ROWS, 5120), taps=refgen.bf16(rn(refgen.CONV_CH, 4)), dt=rn(48),
                      neg_a=-torch.rand(48, generator=g) - 0.5, norm_w=torch.ones(128)) for _ in range(2)]
        w.attn = [dict(Win=rn(refgen.ATTN_ROWS, 5120), wq=torch.ones(256), wk=torch.ones(256)) for _ in range(2)]
        w.out = [rn(5120, 6144) for _ in range(2)]
        w.mlp = [dict(G=rn(17408, 5120), U=rn(17408, 5120), D=rn(5120, 17408)) for _ in range(2)]
        w.head = rn(VOCAB, 5120)
        self.P = step.Prepared(w, 1)
        # the step multiplies with the transposed per-rank copies Prepared made; drop the canonical matrices
        for g_ in w.gdn:
            g_["Win"] = None
        for a_ in w.attn:
            a_["Win"] = None
        w.out = [None] * len(w.out)
        w.mlp = [None] * len(w.mlp)
        w.head = None
        n_attn = LAYERS // INTERVAL
        self.st = refgen.random_state(LAYERS - n_attn, n_attn, ctx, ctx + 64, seed=1)
        self.x0 = refgen.bf16(torch.randn(5120, generator=g))
        self.step = step

    def time_one(self):
        t0 = time.perf_counter()
        self.step.torch_step(self.x0, self.P, self.st, LAYERS, INTERVAL, lm_head=True)
        return time.perf_counter() - t0


def cpu_sample(batch, ctx, nsteps):
    """the CPU baseline: nsteps full 64-layer oracle steps of one user (median); tok/s/user, or tok/s at batch 8
    (users one after another)"""
    threads = os.cpu_count() or 1
    c = CpuStep(ctx, threads)
    c.time_one()  # first touch of the weights
    per_user = statistics.median(c.time_one() for _ in range(nsteps))
    return {
        "value": (1.0 / per_user) if batch == 1 else 1.0 / per_user,
        "unit": "tok/s/user" if batch == 1 else "tok/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{nsteps} full 64-layer oracle steps (ctx {ctx}, 2 weight copies per kind, full lm_head) of one user, "
        f"median {per_user:.2f} s, fp32 torch on {threads} host threads" + (", users sequential" if batch > 1 else ""),
    }


def run_reference(args, rank, world):
    if rank != 0:
        return
    batch = args.batch
    ctx = args.ctx or prompt_of(args)
    threads = os.cpu_count() or 1
    c = CpuStep(ctx, threads)
    for _ in range(args.warmup):
        c.time_one()
    ts = [c.time_one() for _ in range(args.steps)]
    per_user = statistics.median(ts)
    v = 1.0 / per_user  # batch 8: tok/s with users one after another = 1 / (per-user step time)
    unit = "tok/s/user" if batch == 1 else "tok/s"
    line = {
        "impl": "reference",
        "metric": metric_name(batch),
        "value": v,
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_user * 1e3 * batch,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (random-init weights of the named shape, uniform-random prompt tokens)",
        "config": config_of(args, world),
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"each step one full 64-layer oracle step of one user (ctx {ctx}, 2 weight copies "
                         f"per kind, full lm_head), fp32 torch on {threads} host threads"},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ============================================================================================== GPU (ours)
def max_over_ranks(v, world, dev):
    if world == 1:
        return v
    t = torch.tensor([v], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t)


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def nccl_id_bcast(rank):
    from tt_qwen_resident_b200.model import nccl_unique_id

    obj = [nccl_unique_id() if rank == 0 else None]
    torch.distributed.broadcast_object_list(obj, src=0)
    return obj[0]


def tp_check(rank, world, dev, exchange):
    """The tensor-parallel path checked on the ranks themselves (N > 1), before the timed run: a 4-layer G G G A
    model with the full lm_head from the same seeded weights and decode state on every rank. Its first step, eager
    and as a graph replay, must leave x bit-identical on every rank and between the two; x must agree with NCCL's
    (the baseline exchange) within 1e-2 and with one rank running the whole model (rank 0 only) within 2e-2."""
    import torch.distributed as dist

    from oracle import refgen
    from tt_qwen_resident_b200 import weights
    from tt_qwen_resident_b200.model import ResidentModel

    layers, pos = 4, 70
    w = weights.random_canonical(layers, INTERVAL, VOCAB, seed=5, device=dev)
    st = refgen.random_state(3, 1, pos, pos + 16, seed=1)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(3)).bfloat16().float()

    def first_step(model):
        model.load_state(st)
        model.step(model.token_state(x0, pos))
        model.check()
        return model.x().clone(), model.argmax()

    m = ResidentModel(w, layers, INTERVAL, max_pos=pos + 16, lm_head=True, rank=rank, nranks=world, device=dev,
                      p2p=exchange == "p2p", nccl_id=nccl_id_bcast(rank) if exchange == "nccl" else None)
    mode = m.exchange
    x_eager, am = first_step(m)
    m.capture_trace()
    x_graph, am_g = first_step(m)
    m.release_trace()
    m.close()
    barrier(world)
    nid = nccl_id_bcast(rank)
    mn = ResidentModel(w, layers, INTERVAL, max_pos=pos + 16, lm_head=True, rank=rank, nranks=world, device=dev, nccl_id=nid)
    x_nccl, am_n = first_step(mn)
    mn.close()
    barrier(world)
    xs = [torch.empty_like(x_eager) for _ in range(world)]
    dist.all_gather_object(xs, x_eager)
    identical = all(torch.equal(x, xs[0]) for x in xs) and torch.equal(x_eager, x_graph) and am == am_g
    rel = lambda a, b: float((a - b).norm() / b.norm())
    res = {"exchange": mode, "ranks_identical": bool(identical), "rel_err_vs_nccl": rel(x_eager, x_nccl),
           "argmax_equal_nccl": am == am_n}
    if rank == 0:
        one = ResidentModel(w, layers, INTERVAL, max_pos=pos + 16, lm_head=True, device=dev)
        x1, am1 = first_step(one)
        one.close()
        res["rel_err_vs_1rank"] = rel(x_eager, x1)
        res["argmax_1rank"] = (am, am1)
    del w
    torch.cuda.empty_cache()
    ok = [res["ranks_identical"] and res["rel_err_vs_nccl"] < 1e-2 and res.get("rel_err_vs_1rank", 0.0) < 2e-2]
    dist.broadcast_object_list(ok, src=0)
    res["ok"] = bool(ok[0])
    barrier(world)
    return res


def random_long_state(model, ctx, seed=4):
    """config 5: every attention layer's K / V random-filled N(0, 1) for positions 0 .. ctx-1 (on the device, the
    pool of the default contiguous page table), GDN states and conv histories random"""
    g = torch.Generator(device=model.device).manual_seed(seed)
    for t in model.k_pool + model.v_pool:
        t.normal_(generator=g)
    for t in model.gdn_state:
        t.normal_(generator=g).mul_(0.05)
    for t in model.conv_hist:
        t.normal_(generator=g)


def decode_run(model, args, batch, prompt, stream, world, dev, local, pos0=0):
    """prompt through the decode step (host-fed uniform-random tokens), then device-fed greedy decode: W warmup
    replays, K timed replays (max over ranks). Returns (ms per step, clocks, position after the run)."""
    gen = torch.Generator().manual_seed(2)
    with torch.cuda.stream(stream):
        for p in range(pos0, pos0 + prompt):
            toks = torch.randint(0, VOCAB, (batch,), generator=gen).tolist()
            model.step(model.token_state(tokens=toks, pos=[p] * batch), stream=stream)
        first = model.argmax() if prompt else [0] * batch
        first = first if isinstance(first, list) else [first]
        model.step(model.token_state(tokens=first, pos=[pos0 + prompt] * batch, feed=True), stream=stream)
        for _ in range(args.warmup):
            model.step(None, stream=stream)
    model.check(stream)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            model.step(None, stream=stream)
        e1.record(stream)
        e1.synchronize()
        barrier(world)
    model.check(stream)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
    return ms, clk.summary(), model.fed_token()[1]


def e2e_run(model, args, batch, stream, world, dev):
    """the public step call with host buffers: token state from pinned host memory in, the picked token out"""
    from tt_qwen_resident_b200 import _lib

    pos0 = model.fed_token()[1]
    words = torch.zeros(_lib.TOK_WORDS, dtype=torch.int32).pin_memory()
    out_h = torch.zeros(batch, 4, dtype=torch.int32).pin_memory()
    tok = model.argmax()
    tok = tok if isinstance(tok, list) else [tok]
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        words.copy_(model.token_state(tokens=tok, pos=[pos0 + i] * batch)[0])
        with torch.cuda.stream(stream):
            model.tok_d.copy_(words, non_blocking=True)
            model.step(None, stream=stream)
            out_h.copy_(model.out_d, non_blocking=True)
        stream.synchronize()
        tok = out_h[:, 0].tolist()
    ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps, world, dev)
    model.check(stream)
    return ms, _lib.TOK_WORDS * 4, batch * 16


def gateup_alone(model, rows, stream, dev, epi=1):
    """the dominant kernel, the gate|up GEMV (rmsnorm prologue; epi 1: SwiGLU epilogue, 4: the step's fixed-point
    accumulators), timed alone with CUDA events on its stream: layers 0 and 1 alternate, so every launch streams
    weights that are not in L2 (2 x 178 MB > 126 MB). Returns (ms per launch, algorithmic bytes per launch)."""
    from tt_qwen_resident_b200 import _lib

    gws = model.w_gu[:2] if len(model.w_gu) > 1 else model.w_gu[:1]
    xin = torch.randn(rows, 5120, device=dev)
    if epi == 4:
        aout = torch.zeros(rows, 2 * model.d.ic, dtype=torch.int64, device=dev)
    else:
        aout = torch.empty(rows, model.d.ic, dtype=torch.bfloat16, device=dev)
    flush = None if len(gws) > 1 else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        for k in range(4):
            _lib.gemv(gws[k % len(gws)], xin, 0, epi, aout, stream=stream)
        ts = []
        for k in range(20):
            if flush is not None:
                flush.zero_()  # one layer only: evict L2 between launches
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            _lib.gemv(gws[k % len(gws)], xin, 0, epi, aout, stream=stream)
            b.record(stream)
            ts.append((a, b))
    stream.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in ts), gws[0].nbytes


# dram__bytes_read.sum + dram__bytes_write.sum of the gate|up GEMV at one rank, from the committed ncu captures
# (profiles/gemv_fp8_gateup_34816x5120_b1.md; profiles/gemv_fp8_gateup_34816x5120_b8.md: 8 rows, with the tensor
# pipe's share of the active cycles)
NCU_GATEUP = {1: dict(traffic=181963264, src="profiles/gemv_fp8_gateup_34816x5120_b1.md"),
              8: dict(traffic=184298752, tensor_pipe=0.0252, src="profiles/gemv_fp8_gateup_34816x5120_b8.md")}


def run_ours(args, rank, world, local):
    from tt_qwen_resident_b200 import weights
    from tt_qwen_resident_b200.model import ResidentModel

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    tpc = tp_check(rank, world, dev, args.exchange) if world > 1 else None
    batch, prompt = args.batch, prompt_of(args)
    layers = args.layers
    start = args.ctx or prompt
    max_pos = start + args.warmup + 2 * args.steps + 16
    t_build = time.perf_counter()
    w = weights.random_canonical(layers, INTERVAL, VOCAB, seed=0, device=dev)
    emb = torch.randn(VOCAB, 5120, generator=torch.Generator(device=dev).manual_seed(1), device=dev).bfloat16()
    nid = nccl_id_bcast(rank) if world > 1 and args.exchange == "nccl" else None
    model = ResidentModel(w, layers, INTERVAL, batch=batch, max_pos=max_pos, lm_head=True, embed=emb, rank=rank,
                          nranks=world, nccl_id=nid, p2p=world > 1 and args.exchange == "p2p", device=dev,
                          tile_finish=args.tile_finish)
    del w
    torch.cuda.empty_cache()
    build_s = time.perf_counter() - t_build
    if args.ctx:
        random_long_state(model, args.ctx)
    stream = torch.cuda.Stream(device=dev)
    model.capture_trace(stream)
    ms, clocks, end_pos = decode_run(model, args, batch, prompt, stream, world, dev, local, pos0=args.ctx)
    launches_per_step = model.launches
    e2e_ms, h2d, d2h = e2e_run(model, args, batch, stream, world, dev)
    # at 4 or more rows the step's accumulating form walks K groups: time that form
    gemv_ms, gemv_bytes = gateup_alone(model, batch, stream, dev,
                                       epi=4 if batch >= 4 and model.exchange in ("none", "counted") else 1)
    peak, peak_kind = peaks()
    gemv_gbs = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    step_bytes = model.weight_bytes + model.state_bytes_per_step(ctx=end_pos - args.steps // 2)
    step_gbs = step_bytes / (ms * 1e-3) / 1e9
    exchange = model.exchange
    # config 4 beside config 3: 8 users on the same device weights, 128-token prompts
    b8 = None
    if batch == 1 and not args.no_batch8 and not args.ctx:
        m8 = ResidentModel(None, layers, INTERVAL, batch=8, max_pos=128 + args.warmup + args.steps + 16, lm_head=True,
                           embed=emb, rank=rank, nranks=world, nccl_id=nccl_id_bcast(rank) if nid else None,
                           p2p=world > 1 and args.exchange == "p2p", device=dev, share=model)
        m8.capture_trace(stream)
        ms8, clocks8, end8 = decode_run(m8, args, 8, 128, stream, world, dev, local)
        g8_ms, g8_bytes = gateup_alone(m8, 8, stream, dev, epi=4 if m8.exchange in ("none", "counted") else 1)
        sb8 = m8.weight_bytes + m8.state_bytes_per_step(ctx=end8 - args.steps // 2)
        b8 = {
            "metric": metric_name(8), "value": 8e3 / ms8, "unit": "tok/s", "ms_per_step": ms8,
            "workload": "config4: 8 users, 128-token uniform-random prompts each, greedy decode",
            "exchange": m8.exchange, "launches_per_step": m8.launches, "clocks": clocks8,
            "split_tiles": "fixed-point accumulators" if m8.exchange in ("none", "counted") else "finished by ticket",
            "step_roofline": {"bytes_per_step_per_gpu": sb8, "achieved_GBps": sb8 / (ms8 * 1e-3) / 1e9,
                              "frac": sb8 / (ms8 * 1e-3) / 1e9 / peak},
            "gateup_8rows": {"ms_per_launch": g8_ms, "achieved_GBps": g8_bytes / (g8_ms * 1e-3) / 1e9,
                             "frac": g8_bytes / (g8_ms * 1e-3) / 1e9 / peak,
                             "traffic": NCU_GATEUP[8]["traffic"], "bytes_per_launch": g8_bytes,
                             "tensor_pipe_active": NCU_GATEUP[8]["tensor_pipe"], "ncu": NCU_GATEUP[8]["src"]},
        }
        m8.close()
    if rank == 0:
        value = batch * 1e3 / ms if batch > 1 else 1e3 / ms
        e2e_v = batch * 1e3 / e2e_ms if batch > 1 else 1e3 / e2e_ms
        cfg = config_of(args, world)
        cfg.update({
            "split_tiles": "fixed-point accumulators" if exchange in ("none", "counted") and not args.tile_finish
            else "finished by ticket",
            "exchange": {"none": None, "counted": "counted fixed-point words over NVLink (GEMV epilogue)",
                         "tagged": "tagged words over NVLink (GEMV epilogue)", "nccl": "NCCL"}[exchange],
        })
        ncu = NCU_GATEUP.get(batch, {}) if world == 1 else {}
        line = {
            "metric": metric_name(batch),
            "value": value,
            "unit": "tok/s/user" if batch == 1 else "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong",
            "vs_baseline": None,
            "dtype": "fp8-e4m3 weights x bf16 activations, fp32 accumulate / state",
            "data": "synthetic (random-init weights of the named shape, uniform-random prompt tokens)",
            "config": cfg,
            "e2e": {"value": e2e_v, "unit": "tok/s/user" if batch == 1 else "tok/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {
                "bound": "hbm",
                "kernel": "gemv_fp8 gate|up (rmsnorm prologue + SwiGLU epilogue) timed alone, layers 0 / 1 alternating",
                "achieved": gemv_gbs,
                "peak": peak,
                "unit": "GB/s",
                "frac": gemv_gbs / peak,
                "peak_kind": peak_kind,
                "traffic": ncu.get("traffic"),
                "traffic_source": ncu.get("src"),
                "bytes_per_launch": gemv_bytes,
                "ms_per_launch": gemv_ms,
            },
            "step_roofline": {"bytes_per_step_per_gpu": step_bytes, "achieved_GBps": step_gbs, "frac": step_gbs / peak},
            "gpu_launches": launches_per_step * (2 * args.steps),
            "launches_per_step": launches_per_step,
            "clocks": clocks,
            "build_s": build_s,
        }
        if b8 is not None:
            line["batch8"] = b8
        if tpc is not None:
            line["tp_check"] = tpc
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_sample(batch, args.ctx or prompt, 3)
        print(json.dumps(line), flush=True)
    model.close()
    ok = tpc is None or tpc["ok"]
    if world > 1:
        torch.distributed.destroy_process_group()
    if not ok:
        sys.exit(f"tp_check failed: {tpc}")


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
