"""Tensor parallelism on 2 GPUs: each rank runs ResidentModel on its shard (heads, MLP columns, vocab), the
out- and down-projection partials are all-reduced over NCCL, the lm_head's per-rank top-32 lists are gathered
and merged. The result must match the oracle run at n = 2 from the same state (x and each rank's logits within
2e-2 relative, the greedy pick by the argmax rule over the gathered logits), and both ranks must hold the same x
bit for bit. Skipped with fewer than 2 GPUs."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, w8, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import refgen
    from tt_qwen_resident_b200 import weights
    from tt_qwen_resident_b200.model import ResidentModel, nccl_unique_id

    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    dev = torch.device("cuda", rank)
    st = refgen.random_state(3, 1, 70, 134, seed=1)
    model = ResidentModel(weights.canonical_from_fp8(w8, device=dev), 4, 4, batch=1, max_pos=134, lm_head=True,
                          rank=rank, nranks=world, nccl_id=obj[0], device=dev)
    model.load_state(st)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(3)).bfloat16().float()
    for trace in (False, True):
        if trace:
            model.load_state(st)
            model.capture_trace()
        model.step(model.token_state(x0, st.pos))
        model.check()
        out[(rank, trace)] = (model.x().clone(), model.logits().clone(), model.argmax())
    model.close()
    dist.barrier()
    dist.destroy_process_group()


def test_tp2_decode_step_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle import fp8, refgen, sampling, step
    from test_model_gpu import dequantized, quantized

    torch.set_num_threads(8)
    w32 = refgen.random_weights(2, 1, 2, vocab=16384, seed=0)
    w8 = quantized(w32)
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(world, 29600 + os.getpid() % 300, w8, out), nprocs=world, join=True)
    P = step.Prepared(dequantized(w8, w32), world)
    st = refgen.random_state(3, 1, 70, 134, seed=1)
    x0 = torch.randn(5120, generator=torch.Generator().manual_seed(3)).bfloat16().float()
    x_ref, lg = step.torch_step(x0, P, st, 4, 4, lm_head=True)
    rel = lambda a, b: float((a - b).norm() / b.norm())
    for trace in (False, True):
        x0_, l0, a0 = out[(0, trace)]
        x1_, l1, a1 = out[(1, trace)]
        assert torch.equal(x0_, x1_)
        assert rel(x0_, x_ref) < 2e-2
        assert rel(l0, step.logits_bf16([lg[0]])) < 2e-2 and rel(l1, step.logits_bf16([lg[1]])) < 2e-2
        got = torch.cat([l0, l1])
        assert a0 == a1 == sampling.argmax_rule(got)
    assert torch.equal(out[(0, False)][0], out[(0, True)][0])  # graph replay == eager
