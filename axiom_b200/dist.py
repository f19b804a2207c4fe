"""Multi-GPU partitioning of the KDA core (one process per GPU).

(batch, head) units are independent in the forward, the backward and decode,
so the work is split across ranks with no collective inside the kernels: each
rank runs the library on its slice, and the collective is only the final
gather of the outputs (NCCL all-gather over NVLink on GPUs).  The split is by
batch when the batch divides evenly across the ranks, else by head; anything
else is refused (fail-closed) rather than silently imbalanced.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def partition(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, even split of ``n`` items: rank's ``[start, stop)``."""
    if n % world:
        raise ValueError(f"{n} items do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_axis(B: int, H: int, world: int) -> int:
    """Axis to shard ``[B, T, H, D]`` tensors on: 0 (batch) or 2 (heads)."""
    if B % world == 0:
        return 0
    if H % world == 0:
        return 2
    raise ValueError(f"neither B={B} nor H={H} divides over {world} ranks")


def _slice(x: Optional[torch.Tensor], axis: int, start: int, stop: int) -> Optional[torch.Tensor]:
    if x is None:
        return None
    return x.narrow(axis, start, stop - start).contiguous()


def _gather(x: torch.Tensor, axis: int, group=None) -> torch.Tensor:
    world = dist.get_world_size(group)
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=axis)


def sharded_forward(q, k, v, g, beta, S0=None, *, chunk: int = 64, group=None,
                    compute: Optional[Callable] = None):
    """Forward over all ranks' share of the (batch, head) units; returns the
    full ``(o, S_T)`` on every rank (gathered).  Inputs are the full tensors
    (every rank holds them, as in data-parallel training); ``compute`` is the
    per-rank operator, by default :func:`axiom_b200.kda.kda_fwd`."""
    if compute is None:
        from .kda import kda_fwd

        def compute(q_, k_, v_, g_, b_, s_):
            o_, s_t, _ = kda_fwd(q_, k_, v_, g_, b_, s_, chunk=chunk)
            return o_, s_t

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, T, H, _ = q.shape
    axis = shard_axis(B, H, world)
    n = B if axis == 0 else H
    lo, hi = partition(n, world, rank)
    xs = [_slice(t, axis, lo, hi) for t in (q, k, v, g)]
    b_loc = _slice(beta, axis, lo, hi)
    s_axis = 0 if axis == 0 else 1  # S is [B, H, dk, dv]
    s_loc = _slice(S0, s_axis, lo, hi)
    o_loc, st_loc = compute(*xs, b_loc, s_loc)
    return _gather(o_loc, axis, group), _gather(st_loc, s_axis, group)
