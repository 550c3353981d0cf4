"""Benchmark of the resident decode step (BASELINE.json metric: decode tok/s/user at batch 1, total tok/s at
batch 8, on 1/2/4/8 B200; % of the HBM roofline).

Default workload (N=1): BASELINE config 3 -- the full 64-layer Qwen3.6-27B-shaped model (48 GDN + 16
attention layers, every 4th attention), vocab 248,320, FP8 block-scaled random-init weights, batch 1; a
2,048-token uniform-random prompt is run through the decode step itself (prefill is out of scope), then greedy
decode steps are timed. `--batch 8` gives config 4 (8 users, 128-token prompts).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Arms:
  ours       timed region: K device-fed greedy steps (one CUDA-graph replay each), inputs resident in HBM,
             CUDA events on the launching stream, barrier + synchronize on both sides, max over ranks.
             e2e: the same metric through the public step call with host buffers: each step copies the token
             state from pinned host memory, replays the step and reads the picked token back to the host.
  reference  the reference's own decode math (its torch_step, restated in oracle/) on the host cores, every
             step a bounded sample (4 layers G G G A + the lm_head, extrapolated to 64 layers); rank 0 only.
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
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--tile-finish", action="store_true",
                    help="finish split projection tiles by ticket instead of the fixed-point accumulators (1 rank)")
    ap.add_argument("--chain", action="store_true",
                    help="the chained projections between two mixers (one persistent launch) instead of one launch each")
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


def workload_name(batch, prompt):
    return (
        f"config{3 if batch == 1 else 4}: 64-layer Qwen3.6-27B-shaped hybrid (48 GDN + 16 attn), vocab 248320, FP8 "
        f"block-scaled random weights, batch {batch}, {prompt}-token prompt then greedy decode"
    )


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


def cpu_baseline(batch, seconds_budget=30.0):
    """the oracle (the reference's torch_step, restated) on the host cores: one step of 4 layers (G G G A) plus
    the lm_head on random fp32 weights of the real shapes, extrapolated to 64 layers; tok/s/user"""
    from oracle import refgen, step

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    rn = lambda *s: torch.randn(*s, generator=g) * 0.02
    w = refgen.Canon()
    w.gdn = [
        dict(Win=rn(refgen.GDN_ROWS, 5120), taps=refgen.bf16(rn(refgen.CONV_CH, 4)), dt=rn(48), neg_a=-torch.rand(48) - 0.5,
             norm_w=torch.ones(128))
    ]
    w.attn = [dict(Win=rn(refgen.ATTN_ROWS, 5120), wq=torch.ones(256), wk=torch.ones(256))]
    w.out = [rn(5120, 6144)]
    w.mlp = [dict(G=rn(17408, 5120), U=rn(17408, 5120), D=rn(5120, 17408))]
    P = step.Prepared(w, 1)
    ctx = 2048 if batch == 1 else 128
    st = refgen.random_state(1, 1, ctx, ctx + 8, seed=1)
    x0 = refgen.bf16(torch.randn(5120, generator=g))
    t0 = time.perf_counter()
    step.torch_step(x0, P, st, 4, 4)
    t4 = time.perf_counter() - t0
    head = rn(VOCAB // 8, 5120).T.contiguous()  # an eighth of the lm_head, timed and scaled by 8
    h = refgen.bf16(step.rmsnorm(x0))
    t0 = time.perf_counter()
    _ = h @ head
    th = (time.perf_counter() - t0) * 8
    per_step = t4 * (LAYERS / 4) + th
    per_user = per_step * batch  # the oracle runs users one after another
    return {
        "value": (1.0 / per_user) if batch == 1 else batch / per_user,
        "unit": "tok/s/user" if batch == 1 else "tok/s",
        "cores": threads,
        "kind": "port",
        "sample": f"1 oracle step of 4 layers (G G G A, ctx {ctx}) = {t4:.2f} s x 16 + lm_head ({th:.2f} s from 1/8 of "
        f"it) per user, fp32 torch on {threads} host threads",
    }


def run_reference(args, rank, world):
    if rank != 0:
        return
    batch = args.batch
    prompt = args.prompt or (2048 if batch == 1 else 128)
    vals = []
    cb = None
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(batch)
        if i >= args.warmup:
            vals.append(cb["value"])
    v = statistics.median(vals) if vals else cb["value"]
    line = {
        "impl": "reference",
        "metric": metric_name(batch),
        "value": v,
        "unit": cb["unit"],
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 / v * (1 if batch == 1 else batch),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (random weights of the named shape, uniform-random prompt)",
        "config": {"workload": workload_name(batch, prompt), "batch": batch, "prompt": prompt},
        "cpu_baseline": {k: cb[k] for k in ("cores", "kind", "sample")} | {"value": v, "unit": cb["unit"]},
        "e2e": {"value": v, "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local):
    from tt_qwen_resident_b200 import _lib, weights
    from tt_qwen_resident_b200.model import ResidentModel, nccl_unique_id

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    batch = args.batch
    prompt = args.prompt or (2048 if batch == 1 else 128)
    layers = args.layers
    total_steps = prompt + args.warmup + args.steps + 2 * args.steps + 8
    max_pos = total_steps + 64
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        if args.exchange == "nccl":
            obj = [nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            nid = obj[0]
        else:
            nid = None
    else:
        nid = None

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    t_build = time.perf_counter()
    w = weights.random_canonical(layers, INTERVAL, VOCAB, seed=0, device=dev)
    emb = torch.randn(VOCAB, 5120, generator=torch.Generator(device=dev).manual_seed(1), device=dev).bfloat16()
    model = ResidentModel(w, layers, INTERVAL, batch=batch, max_pos=max_pos, lm_head=True, embed=emb, rank=rank,
                          nranks=world, nccl_id=nid, p2p=world > 1 and args.exchange == "p2p", device=dev,
                          chain=args.chain, tile_finish=args.tile_finish)
    del w
    torch.cuda.empty_cache()
    build_s = time.perf_counter() - t_build
    stream = torch.cuda.Stream(device=dev)
    model.capture_trace(stream)
    gen = torch.Generator().manual_seed(2)
    # prompt through the decode step (host-fed tokens), then device-fed greedy decode
    with torch.cuda.stream(stream):
        for p in range(prompt):
            toks = torch.randint(0, VOCAB, (batch,), generator=gen).tolist()
            model.step(model.token_state(tokens=toks, pos=[p] * batch), stream=stream)
        model.step(model.token_state(tokens=model.argmax() if batch == 1 else [0] * batch, pos=[prompt] * batch, feed=True),
                   stream=stream)
        for _ in range(args.warmup):
            model.step(None, stream=stream)
    model.check(stream)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            model.step(None, stream=stream)
        e1.record(stream)
        e1.synchronize()
        barrier()
    model.check(stream)
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t)
    launches_per_step = model.launches
    # e2e: host buffers, one token per step through the public step call
    pos0 = model.fed_token()[1]
    words = torch.zeros(_lib.TOK_WORDS, dtype=torch.int32).pin_memory()
    out_h = torch.zeros(batch, 4, dtype=torch.int32).pin_memory()
    tok = model.argmax()
    tok = tok if isinstance(tok, list) else [tok]
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        w_ = model.token_state(tokens=tok, pos=[pos0 + i] * batch)[0]
        words.copy_(w_)
        with torch.cuda.stream(stream):
            model.tok_d.copy_(words, non_blocking=True)
            model.step(None, stream=stream)
            out_h.copy_(model.out_d, non_blocking=True)
        stream.synchronize()
        tok = out_h[:, 0].tolist()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t)
    model.check(stream)
    # dominant kernel: the gate|up GEMV (the largest per-layer weight stream), timed alone: layers 0 and 1
    # alternate, so each launch streams weights that are not in L2 (2 x 178 MB > 126 MB)
    gws = model.w_gu[:2] if len(model.w_gu) > 1 else model.w_gu[:1]
    gw = gws[0]
    xin = torch.randn(batch, 5120, device=dev)
    aout = torch.empty(batch, model.d.ic, dtype=torch.bfloat16, device=dev)
    flush = None if len(gws) > 1 else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        for k in range(4):
            _lib.gemv(gws[k % len(gws)], xin, 0, 1, aout, stream=stream)
        ts = []
        for k in range(20):
            if flush is not None:
                flush.zero_()  # one layer only: evict L2 between launches
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            _lib.gemv(gws[k % len(gws)], xin, 0, 1, aout, stream=stream)
            b.record(stream)
            ts.append((a, b))
    stream.synchronize()
    gemv_ms = statistics.mean(a.elapsed_time(b) for a, b in ts)
    peak, peak_kind = peaks()
    gemv_gbs = gw.nbytes / (gemv_ms * 1e-3) / 1e9
    step_bytes = model.weight_bytes + model.state_bytes_per_step(ctx=prompt + args.warmup + args.steps)
    step_gbs = step_bytes / (ms * 1e-3) / 1e9
    if rank == 0:
        value = batch * 1e3 / ms if batch > 1 else 1e3 / ms
        e2e_v = batch * 1e3 / e2e_ms if batch > 1 else 1e3 / e2e_ms
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
            "config": {
                "workload": workload_name(batch, prompt),
                "batch": batch,
                "prompt": prompt,
                "layers": layers,
                "parallelism": f"tp{world}",
                "projections": "chained between mixers (gemv_chain)" if args.chain else "per-projection launches",
                "split_tiles": ("fixed-point accumulators" + (" (counted exchange over NVLink)" if world > 1 else "")
                                if batch <= 2 and not args.chain and not args.tile_finish
                                and (world == 1 or args.exchange == "p2p") else "finished by ticket"),
                "exchange": ("fused NVLink peer exchange in the GEMV epilogue" if args.exchange == "p2p" else "NCCL")
                if world > 1 else None,
                "l2": "inputs larger than L2 (25.6 GB of weights streamed per step)",
            },
            "e2e": {
                "value": e2e_v,
                "unit": "tok/s/user" if batch == 1 else "tok/s",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": _lib.TOK_WORDS * 4,
                "d2h_bytes_per_step": batch * 16,
            },
            "roofline": {
                "bound": "hbm",
                "kernel": "gemv_fp8 (gate|up, rmsnorm prologue + SwiGLU epilogue), timed alone; layers 0 and 1 alternate "
                          "(2 x 178 MB, larger than L2)",
                "achieved": gemv_gbs,
                "peak": peak,
                "unit": "GB/s",
                "frac": gemv_gbs / peak,
                "peak_kind": peak_kind,
                # dram__bytes_read.sum + dram__bytes_write.sum of this kernel at this shape, from the committed
                # ncu capture (profiles/gemv_fp8_gateup_34816x5120_b1.md): 178.76 MB + 3.97 MB
                "traffic": 182731008 if (batch == 1 and world == 1) else None,
                "traffic_source": "ncu --set full, profiles/gemv_fp8_gateup_34816x5120_b1.md" if (batch == 1 and world == 1) else None,
                "bytes_per_launch": gw.nbytes,
                "ms_per_launch": gemv_ms,
            },
            "step_roofline": {
                "bytes_per_step_per_gpu": step_bytes,
                "achieved_GBps": step_gbs,
                "frac": step_gbs / peak,
            },
            "gpu_launches": launches_per_step * (2 * args.steps),
            "launches_per_step": launches_per_step,
            "clocks": clk.summary(),
            "build_s": build_s,
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(batch)
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
