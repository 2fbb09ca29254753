"""Tensor-parallel communication: process setup and the NCCL baseline.

One process per GPU, ``torch.distributed`` with the NCCL backend over
NVLink 5 / NVSwitch. The reference had no communication code of its own (its
all-reduces were vLLM's oneCCL calls, tuned by env vars in
``k8v4_v030/launch.sh:101-110``); this module is the plain-NCCL baseline the
fused compute+collective kernels are measured against.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init_from_env(timeout_s: float = 300.0, backend: str | None = None) -> tuple[int, int, int]:
    """Initialize the default process group from RANK/WORLD_SIZE/LOCAL_RANK.

    Returns (rank, world_size, local_rank). A single process without the env
    vars is rank 0 of 1 and creates no group.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


class TPComm:
    """Collectives of one TP group (NCCL baseline)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor, dim: int = 0) -> torch.Tensor:
        if self.world == 1:
            return t
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        if dim == 0:
            return out
        return torch.cat(list(out.chunk(self.world, 0)), dim=dim)

    def reduce_scatter(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        out = torch.empty((t.shape[0] // self.world,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t.contiguous(), group=self.group)
        return out

    def argmax_reduce(self, val: torch.Tensor, idx: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Per-row (value, global index) of the best vocab shard (lowest index on ties)."""
        if self.world == 1:
            return val, idx
        packed = torch.stack([val.float(), idx.float()], 0)  # exact: vocab indices < 2^24
        allp = self.all_gather(packed.unsqueeze(0)).view(self.world, 2, -1)  # [world, (val, idx), rows]
        vals, idxs = allp[:, 0], allp[:, 1]
        best = vals.max(dim=0).values
        cand = torch.where(vals == best.unsqueeze(0), idxs, torch.full_like(idxs, float("inf")))
        return best, cand.min(dim=0).values.to(torch.int64)

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    def max_scalar(self, x: float) -> float:
        """Max of a host scalar over ranks (timing: the slowest rank counts)."""
        if self.world == 1:
            return x
        dev = "cuda" if dist.get_backend(self.group) == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())
