"""Data-parallel plumbing over independent sequences: one process per GPU.

The denoising path shards only across independent sequences (a sequence's steps depend
on each other; different sequences share nothing but the read-only weights), so every
rank holds a full weight replica and generates its own contiguous share of the
sequences.  Nothing crosses ranks on the data path.  torch.distributed carries only the
host-side steps: barriers around timed regions, the max-over-ranks of device times, and
gathering generated tokens to rank 0 (the reference's single-process loop,
src/diffuse-sampler.cpp:60-370, run once per sequence, is what each rank executes).

Backend: "nccl" when CUDA is available (tensors on the rank's device), else "gloo"
(CPU tests).  Every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import numpy as np


def shard(n_items: int, rank: int, world: int) -> range:
    """Contiguous, balanced share of n_items for `rank` of `world` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    lo = n_items * rank // world
    hi = n_items * (rank + 1) // world
    return range(lo, hi)


@dataclass
class DataParallel:
    rank: int = 0
    world: int = 1
    local: int = 0
    backend: str | None = None
    _dist: object = None

    @classmethod
    def from_env(cls, timeout_s: float = 300.0, backend: str | None = None) -> "DataParallel":
        """Joins the process group torchrun describes (RANK / WORLD_SIZE / LOCAL_RANK /
        MASTER_ADDR / MASTER_PORT); a single process without them is world 1."""
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        dp = cls(rank=rank, world=world, local=local)
        if world > 1:
            import torch
            import torch.distributed as dist
            if backend is None:
                backend = "nccl" if torch.cuda.is_available() else "gloo"
            if backend == "nccl":
                torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
            dp.backend, dp._dist = backend, dist
        return dp

    def _device(self):
        import torch
        return torch.device(f"cuda:{self.local}") if self.backend == "nccl" else torch.device("cpu")

    def barrier(self):
        if self._dist is None:
            return
        if self.backend == "nccl":
            import torch
            self._dist.barrier(device_ids=[self.local])
            torch.cuda.synchronize()
        else:
            self._dist.barrier()

    def _reduce(self, x: float, op) -> float:
        import torch
        t = torch.tensor([float(x)], dtype=torch.float64, device=self._device())
        self._dist.all_reduce(t, op=op)
        return float(t.item())

    def max_over_ranks(self, x: float) -> float:
        """The slowest rank's value (device times of a timed region)."""
        if self._dist is None:
            return float(x)
        return self._reduce(x, self._dist.ReduceOp.MAX)

    def sum_over_ranks(self, x: float) -> float:
        if self._dist is None:
            return float(x)
        return self._reduce(x, self._dist.ReduceOp.SUM)

    def broadcast_bytes(self, data: bytes) -> bytes:
        """Rank 0's bytes on every rank (e.g. the NCCL unique id of tensor parallelism)."""
        if self._dist is None:
            return bytes(data)
        import torch
        n = torch.tensor([len(data)], dtype=torch.int64, device=self._device())
        self._dist.broadcast(n, src=0)
        buf = np.zeros(int(n.item()), np.uint8)
        if self.rank == 0:
            buf[:] = np.frombuffer(data, np.uint8)
        t = torch.from_numpy(buf).to(self._device())
        self._dist.broadcast(t, src=0)
        return t.cpu().numpy().tobytes()

    def gather_rows(self, rows: np.ndarray, n_total: int) -> np.ndarray | None:
        """Concatenates every rank's int32 [n_local, L] block in rank order on rank 0
        (the blocks of shard(n_total, r, world)); other ranks get None."""
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        if self._dist is None:
            return rows
        import torch
        L = rows.shape[1] if rows.ndim == 2 else 0
        cap = -(-n_total // self.world)  # largest shard
        buf = np.zeros((cap, L), np.int32)
        buf[: rows.shape[0]] = rows
        t = torch.from_numpy(buf).to(self._device())
        outs = [torch.zeros_like(t) for _ in range(self.world)] if self.rank == 0 else None
        self._dist.gather(t, gather_list=outs, dst=0)
        if self.rank != 0:
            return None
        parts = [o.cpu().numpy()[: len(shard(n_total, r, self.world))] for r, o in enumerate(outs)]
        return np.concatenate(parts, axis=0)

    def close(self):
        if self._dist is not None:
            self.barrier()
            self._dist.destroy_process_group()
            self._dist = None
