"""Process groups of a TP x CP job (one process per GPU).

Rank ``r`` of a ``tp * cp`` world is TP rank ``r % tp`` of CP rank
``r // tp``: the ranks of one TP group are adjacent (one model replica's
shards), and a CP group holds the ranks with the same TP rank, one per CP
rank (the same KV heads, page-sharded by sequence position). With both
degrees above one, every rank creates every group, in the same order, as
``torch.distributed.new_group`` requires; with one of them, the other's group
is the whole world. A degree of one has no group (``None``). The reference
gets TP from vLLM (``k8v4_v030/launch.sh:184``) and has no CP, so there is no
counterpart for the CP x TP layout.
"""
from __future__ import annotations

import dataclasses

import torch.distributed as dist


def tp_members(tp: int, cp: int) -> list[list[int]]:
    return [[c * tp + t for t in range(tp)] for c in range(cp)]


def cp_members(tp: int, cp: int) -> list[list[int]]:
    return [[c * tp + t for c in range(cp)] for t in range(tp)]


def coords(rank: int, tp: int) -> tuple[int, int]:
    """(tp rank, cp rank) of a global rank."""
    return rank % tp, rank // tp


@dataclasses.dataclass
class ParallelGroups:
    tp: int
    cp: int
    tp_rank: int
    cp_rank: int
    tp_group: object | None
    cp_group: object | None


def build(tp: int, cp: int, backend: str | None = None) -> ParallelGroups:
    """Create the TP and CP groups of this job (world must be tp * cp)."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    if tp < 1 or cp < 1 or tp * cp != world:
        raise ValueError("tp %d x cp %d does not match the world of %d ranks" % (tp, cp, world))
    rank = dist.get_rank() if dist.is_initialized() else 0
    t, c = coords(rank, tp)
    tp_group = cp_group = None
    if tp > 1 and cp > 1:
        for members in tp_members(tp, cp):
            g = dist.new_group(members, backend=backend)
            if rank in members:
                tp_group = g
        for members in cp_members(tp, cp):
            g = dist.new_group(members, backend=backend)
            if rank in members:
                cp_group = g
    elif tp > 1:
        tp_group = dist.group.WORLD
    elif cp > 1:
        cp_group = dist.group.WORLD
    return ParallelGroups(tp, cp, t, c, tp_group, cp_group)
