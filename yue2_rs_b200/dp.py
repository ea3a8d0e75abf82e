"""Data parallelism over songs (one process per GPU, no data-path collective).

The decode path shards by song: each request's cond and uncond rows must share one weight
pass (the CFG mix needs both), so a song never splits across GPUs, and songs are
independent. Song i runs on rank i % world. The only cross-rank traffic is the timing
reduction (max over ranks) and the barriers around the timed region; with NCCL on GPUs,
with gloo in the CPU tests.
"""
import os


class DataParallel:
    """Rank/world from the torchrun environment, plus the three reductions bench.py needs."""

    def __init__(self, backend=None):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self._dist = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            kw = {}
            if backend == "nccl":
                kw["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
            self._dist = dist

    def songs(self, n_total):
        """Indices of the songs this rank runs out of n_total (song i on rank i % world)."""
        return list(range(self.rank, n_total, self.world))

    def _device(self):
        import torch
        return torch.device("cuda", self.local) if self.backend == "nccl" else torch.device("cpu")

    def barrier(self):
        if self._dist is not None:
            self._dist.barrier()

    def max(self, x):
        """Max over ranks (every rank gets it): the timed region ends when the slowest rank does."""
        if self._dist is None:
            return float(x)
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self._device())
        self._dist.all_reduce(t, op=self._dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        """Sum over ranks (every rank gets it), e.g. tokens produced by all ranks."""
        if self._dist is None:
            return float(x)
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self._device())
        self._dist.all_reduce(t, op=self._dist.ReduceOp.SUM)
        return float(t.item())

    def throughput(self, tokens_this_rank, seconds_this_rank):
        """Whole-job tokens/s: tokens of every rank over the slowest rank's time."""
        return self.sum(tokens_this_rank) / self.max(seconds_this_rank)

    def close(self):
        if self._dist is not None:
            self._dist.destroy_process_group()
            self._dist = None
