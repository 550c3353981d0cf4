"""Host-side failure detection between steps, on the CPU with gloo ranks (no GPU): two ranks step together; one
rank leaves between steps (it returns without reaching the next step barrier); the survivor's RankWatch.check
(a monitored barrier with a 2 s timeout, tt_qwen_resident_b200/ranks.py) raises PeerLost within the timeout
instead of launching a step whose exchange would wait for the lost rank."""
import os
import time

import torch.distributed as dist
import torch.multiprocessing as mp


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tt_qwen_resident_b200.ranks import PeerLost, RankWatch

    watch = RankWatch(timeout_s=2.0)
    watch.check()  # step 1: both ranks present
    out[(rank, "step1")] = True
    if rank == 1:
        return  # rank 1 leaves between steps
    t0 = time.time()
    try:
        watch.check()  # step 2
        out[(rank, "step2")] = "passed"
    except PeerLost as e:
        out[(rank, "step2")] = ("lost", time.time() - t0, str(e))


def test_survivor_detects_lost_rank():
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(2, 29700 + os.getpid() % 200, out), nprocs=2, join=True)
    assert out[(0, "step1")] and out[(1, "step1")]
    res = out[(0, "step2")]
    assert res[0] == "lost", res
    assert res[1] < 30, res  # detected by the timeout, not hung
