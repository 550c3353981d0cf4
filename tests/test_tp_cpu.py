"""Tensor-parallel host logic on the CPU (no GPU): the rank partition and the row-parallel all-reduce.

The reference splits heads, MLP columns and vocab over its chips and all-reduces the out- and down-projection
partials (qwen36_resident/weights.py:1-7, model.py:279-287, kernels/mlp_hub.cpp:309-364). Here:
- every rank's slices (weights.RankDims, the ones the GPU shards use) cover each canonical row exactly once
  (KV heads: twice at n = 8, replicated on rank pairs);
- two gloo ranks, each running the oracle for its own shard, all-reduce their partials and reproduce the
  single-rank step -- the decomposition the GPU path computes with NCCL.
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import refgen, step
from tt_qwen_resident_b200 import weights

GDN_ROWS, ATTN_ROWS = weights.GDN_ROWS, weights.ATTN_ROWS


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_rank_partition_covers_rows(n):
    gdn = torch.cat([weights.RankDims(r, n).gdn_rows() for r in range(n)])
    assert torch.equal(gdn.sort().values, torch.arange(GDN_ROWS))
    gu = torch.cat([weights.RankDims(r, n).gateup_rows() for r in range(n)])
    assert torch.equal(gu.sort().values, torch.arange(2 * weights.INTER))
    voc = torch.cat([weights.RankDims(r, n, vocab=248320).vocab_rows() for r in range(n)])
    assert torch.equal(voc, torch.arange(248320))
    att = torch.cat([weights.RankDims(r, n).attn_rows() for r in range(n)])
    q_gate = att[att < 2 * weights.NQ * weights.HD]
    assert torch.equal(q_gate.sort().values, torch.arange(2 * weights.NQ * weights.HD))
    kv = att[att >= 2 * weights.NQ * weights.HD]
    reps = 2 if n == 8 else 1  # KV heads replicated on rank pairs at n = 8
    assert kv.numel() == reps * 2 * weights.NKV * weights.HD
    # the oracle's shard (an independent restatement) agrees with the product's
    for r in range(n):
        s, d = step.Shard(r, n), weights.RankDims(r, n)
        assert torch.equal(s.gdn_rows(), d.gdn_rows()) and torch.equal(s.attn_rows(), d.attn_rows())
        assert torch.equal(s.conv_channels(), d.conv_channels())
        assert s.kv0 == d.kv0 and s.nkv == d.nkv


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(2)
    w = refgen.random_weights(2, 1, 1, vocab=0, seed=0)
    P = step.Prepared(w, world)
    s = P.sh[rank]
    x = refgen.bf16(torch.randn(5120, generator=torch.Generator().manual_seed(4)))
    h = refgen.bf16(step.rmsnorm(x))
    # one MLP half-layer: rank-local SwiGLU + row-parallel down projection, all-reduced
    cm = P.mlp[0][rank]
    part = refgen.bf16(torch.nn.functional.silu(h @ cm["G"]) * (h @ cm["U"])) @ cm["D"]
    dist.all_reduce(part)
    out[rank] = (x + part).clone()
    dist.destroy_process_group()


def test_row_parallel_all_reduce_two_gloo_ranks():
    world = 2
    port = 29500 + (os.getpid() % 1000)
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    w = refgen.random_weights(2, 1, 1, vocab=0, seed=0)
    P1 = step.Prepared(w, 1)
    x = refgen.bf16(torch.randn(5120, generator=torch.Generator().manual_seed(4)))
    h = refgen.bf16(step.rmsnorm(x))
    cm = P1.mlp[0][0]
    ref = x + refgen.bf16(torch.nn.functional.silu(h @ cm["G"]) * (h @ cm["U"])) @ cm["D"]
    for r in range(world):
        got = out[r]
        assert (got - ref).norm() / ref.norm() < 1e-4  # the same math up to fp32 summation order
    assert torch.equal(out[0], out[1])  # every rank holds the same x after the all-reduce
