"""Host-side liveness of the tensor-parallel ranks between decode steps.

The reference's chips wait for each other inside the device program with no limit, and a lost chip is recovered
by a card reset (README.md:84). Here every wait inside the kernels is bounded (a timeout sets the context's error
word, reported by qres_check), and between steps the host can check that every rank is still there before it
launches the next step, whose exchange would otherwise wait on a rank that left: ``RankWatch.check`` is a
monitored barrier over a gloo group with a short timeout that raises ``PeerLost`` naming the ranks that did not
arrive.
"""
import datetime

import torch.distributed as dist


class PeerLost(RuntimeError):
    pass


class RankWatch:
    def __init__(self, timeout_s=2.0, group=None):
        """a gloo group over the default group's ranks (monitored barriers need gloo), made collectively"""
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.group = group if group is not None else dist.new_group(backend="gloo")

    def check(self):
        """return once every rank has called check(); raise PeerLost if one has not within the timeout"""
        try:
            dist.monitored_barrier(group=self.group, timeout=self.timeout, wait_all_ranks=True)
        except RuntimeError as e:
            raise PeerLost(f"rank {dist.get_rank()}: a peer did not reach the step barrier: {e}") from e
