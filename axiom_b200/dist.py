"""Multi-GPU partitioning of the KDA core and of the mixer layer (one process per GPU).

The KDA core.  (batch, head) units are independent in the forward, the
backward and decode, so the work is split across ranks with no collective
inside the kernels: each rank runs the library on its slice, and the only
collective is the gather of the results (NCCL all-gather over NVLink on GPUs).
The split is by batch when the batch divides evenly across the ranks, else by
head; anything else is refused (fail-closed) rather than silently imbalanced.

* :func:`sharded_forward` / :func:`sharded_backward` -- chunked forward and
  fused backward on the rank's slice, results all-gathered;
* :func:`sharded_decode_step` -- every rank keeps the recurrent states of its
  slice of (sequence, head) pairs resident and updates them in place; the
  per-token outputs are all-gathered.

The mixer layer (packed sequences, sharded by sequence x
head).  Ranks form a ``n_seq_groups x n_head_groups`` mesh (:func:`layer_mesh`):

* whole packed sequences are assigned to sequence groups, longest first onto
  the group with the fewest tokens (:func:`assign_sequences`);
* within a sequence group the heads are split: the q/k/v/gate/beta/decay
  projections and the conv taps by output column, ``W_o`` by input row
  (:func:`shard_layer_params`); the group's partial ``W_o`` products are
  summed by an all-reduce in the forward, and the input's cotangent by an
  all-reduce in the backward (:func:`kda_layer_sharded`);
* the replicated low-rank ``W_a_down``'s gradient is summed over the head
  group, then every gradient over the ranks holding the same head shard
  (data parallel over sequences), in one flat bucket per dtype
  (:func:`allreduce_layer_grads`).

The reference has no multi-GPU code for this path (data parallelism is only
designed there, ``model/ADR-034-multi-gpu-dp.md``), so these collectives follow
the partitioning the operator admits rather than a reference implementation.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist


# ---------------------------------------------------------------------------
# the KDA core: (batch, head) sharding
# ---------------------------------------------------------------------------


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


def _world_rank(group=None) -> tuple[int, int]:
    """``(world size, rank)`` of ``group``; a process without a process group is
    a world of one."""
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _gather(x: torch.Tensor, axis: int, group=None, async_op: bool = False):
    """All-gather rank slices and concatenate them along ``axis``.  Slices of
    the leading axis land in place (``all_gather_into_tensor``); other axes go
    through a stacked buffer and one reordering copy.  With ``async_op`` the
    result is ``(finish, work)``: ``finish()`` waits for the collective (on the
    current stream) and returns the gathered tensor."""
    world, _ = _world_rank(group)
    x = x.contiguous()
    if async_op:
        if world == 1:
            return (lambda: x), None
        out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        work = dist.all_gather_into_tensor(out, x, group=group, async_op=True)

        def finish():
            work.wait()
            return out if axis == 0 else _interleave(out, x.shape, axis, world)

        return finish, work
    if world == 1:
        return x
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out if axis == 0 else _interleave(out, x.shape, axis, world)


def _interleave(out, shape, axis, world):
    """``[world * s0, ...]`` rank-major gather -> the slices concatenated on ``axis``."""
    stacked = out.view((world,) + tuple(shape))
    perm = list(range(1, axis + 1)) + [0] + list(range(axis + 1, len(shape) + 1))
    full = list(shape)
    full[axis] *= world
    return stacked.permute(*perm).reshape(full)


@dataclass
class CoreShard:
    """Which slice of the ``[B, T, H, D]`` units a rank owns: ``axis`` 0 (batch)
    or 2 (heads), ``[lo, hi)`` along it; states ``[B, H, dk, dv]`` are sliced
    on ``s_axis`` (0 or 1)."""

    axis: int
    lo: int
    hi: int

    @property
    def s_axis(self) -> int:
        return 0 if self.axis == 0 else 1

    def take(self, x):
        return _slice(x, self.axis, self.lo, self.hi)

    def take_state(self, s):
        return _slice(s, self.s_axis, self.lo, self.hi)


def core_shard(B: int, H: int, group=None) -> CoreShard:
    """This rank's share of a ``B x H`` problem (batch split if it divides, else heads)."""
    world, rank = _world_rank(group)
    axis = shard_axis(B, H, world)
    lo, hi = partition(B if axis == 0 else H, world, rank)
    return CoreShard(axis, lo, hi)


def sharded_forward(q, k, v, g, beta, S0=None, *, chunk: int = 64, group=None,
                    compute: Optional[Callable] = None, need_ckpt: bool = False):
    """Forward over all ranks' share of the (batch, head) units; returns the
    full ``(o, S_T)`` on every rank (gathered), plus this rank's checkpoint for
    :func:`sharded_backward` when ``need_ckpt``.  Inputs are the full tensors
    (every rank holds them, as in data-parallel training); ``compute(q, k, v,
    g, beta, S0) -> (o, S_T[, ckpt])`` is the per-rank operator, by default
    :func:`axiom_b200.kda.kda_fwd`."""
    if compute is None:
        from .kda import kda_fwd

        def compute(q_, k_, v_, g_, b_, s_):
            o_, s_t, ck = kda_fwd(q_, k_, v_, g_, b_, s_, chunk=chunk, need_ckpt=need_ckpt)
            return (o_, s_t, ck) if need_ckpt else (o_, s_t)

    B, _, H, _ = q.shape
    sh = core_shard(B, H, group)
    res = compute(*(sh.take(t) for t in (q, k, v, g, beta)), sh.take_state(S0))
    o = _gather(res[0], sh.axis, group)
    s_t = _gather(res[1], sh.s_axis, group)
    return (o, s_t, res[2]) if need_ckpt else (o, s_t)


def sharded_backward(q, k, v, g, beta, ckpt_local, do, dST=None, *, chunk: int = 64, group=None,
                     compute: Optional[Callable] = None, need_ds0: bool = True):
    """Backward of :func:`sharded_forward` from this rank's checkpoint: every
    rank differentiates its slice with the fused backward and the gradients
    ``(dq, dk, dv, dg, dbeta, dS0)`` are all-gathered (``dS0`` None unless
    ``need_ds0``).  ``compute(q, k, v, g, beta, ckpt, do, dST)`` defaults to
    :func:`axiom_b200.kda.kda_bwd`."""
    if compute is None:
        from .kda import kda_bwd

        def compute(q_, k_, v_, g_, b_, ck, do_, ds_):
            return kda_bwd(q_, k_, v_, g_, b_, ck, do_, ds_, chunk=chunk, need_ds0=need_ds0)

    B, _, H, _ = q.shape
    sh = core_shard(B, H, group)
    grads = compute(*(sh.take(t) for t in (q, k, v, g, beta)), ckpt_local, sh.take(do),
                    sh.take_state(dST))
    out = [_gather(x, sh.axis, group) for x in grads[:5]]
    out.append(None if grads[5] is None else _gather(grads[5], sh.s_axis, group))
    return tuple(out)


def decode_shard(n_states: int, group=None) -> tuple[int, int]:
    """This rank's contiguous range of the ``n_states`` (sequence, head) states."""
    world, rank = _world_rank(group)
    return partition(n_states, world, rank)


def sharded_decode_step(S_local, q, k, v, g, beta, *, group=None, compute: Optional[Callable] = None):
    """One token for all ``N`` states, the states sharded over the ranks: this
    rank's ``S_local [N / world, dk, dv]`` (its :func:`decode_shard` range,
    resident on the device) is updated in place from the full per-token inputs
    ``q, k, g [N, dk]``, ``v [N, dv]``, ``beta [N]``; returns the full ``o
    [N, dv]`` (all-gathered).  ``compute(S, q, k, v, g, beta) -> o`` defaults to
    :func:`axiom_b200.kda.decode_step`."""
    if compute is None:
        from .kda import decode_step as compute
    lo, hi = decode_shard(q.shape[0], group)
    if S_local.shape[0] != hi - lo:
        raise ValueError(f"S_local holds {S_local.shape[0]} states, this rank owns {hi - lo}")
    o = compute(S_local, *(_slice(t, 0, lo, hi) for t in (q, k, v, g, beta)))
    return _gather(o, 0, group)


# ---------------------------------------------------------------------------
# the mixer layer: sequence x head sharding
# ---------------------------------------------------------------------------


def assign_sequences(lengths: Sequence[int], n_groups: int) -> list[list[int]]:
    """Whole sequences onto ``n_groups`` groups, balancing tokens: longest first
    (ties by index) onto the group with the fewest tokens so far (ties: lowest
    group).  Each group's sequence indices are returned in ascending order."""
    if n_groups < 1:
        raise ValueError("n_groups must be >= 1")
    load = [0] * n_groups
    groups: list[list[int]] = [[] for _ in range(n_groups)]
    for i in sorted(range(len(lengths)), key=lambda j: (-int(lengths[j]), j)):
        tgt = min(range(n_groups), key=lambda r: (load[r], r))
        groups[tgt].append(i)
        load[tgt] += int(lengths[i])
    return [sorted(gr) for gr in groups]


def local_packing(cu_seqlens: Sequence[int], seq_ids: Sequence[int]) -> tuple[list[int], list[int]]:
    """Token rows of the sequences ``seq_ids`` of a packed batch, in that order,
    and their own ``cu_seqlens``: ``(rows, cu_local)``."""
    cu = [int(c) for c in cu_seqlens]
    rows: list[int] = []
    cu_local = [0]
    for i in seq_ids:
        rows.extend(range(cu[i], cu[i + 1]))
        cu_local.append(cu_local[-1] + cu[i + 1] - cu[i])
    return rows, cu_local


@dataclass
class LayerMesh:
    """A ``n_seq_groups x n_head_groups`` mesh of ranks; rank r sits at
    ``(seq_index, head_index) = divmod(r, n_head_groups)``.  ``head_group``: the
    ranks sharing this rank's sequences (they split the heads); ``dp_group``:
    the ranks holding this rank's head shard (they split the sequences)."""

    n_seq_groups: int
    n_head_groups: int
    seq_index: int
    head_index: int
    head_group: object
    dp_group: object

    @staticmethod
    def single() -> "LayerMesh":
        """The mesh of a lone process (no process group needed)."""
        return LayerMesh(1, 1, 0, 0, None, None)


def layer_mesh(n_head_groups: int = 1, group=None) -> LayerMesh:
    """Build the mesh's process groups.  Every rank of ``group`` must call this
    with the same ``n_head_groups`` (each ``new_group`` is collective)."""
    world, rank = _world_rank(group)
    if world == 1 and n_head_groups == 1:
        return LayerMesh.single()
    if n_head_groups < 1 or world % n_head_groups:
        raise ValueError(f"{n_head_groups} head groups do not divide {world} ranks")
    n_seq = world // n_head_groups
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    head_groups = [dist.new_group([ranks[s * n_head_groups + j] for j in range(n_head_groups)])
                   for s in range(n_seq)]
    dp_groups = [dist.new_group([ranks[s * n_head_groups + j] for s in range(n_seq)])
                 for j in range(n_head_groups)]
    s_idx, h_idx = divmod(rank, n_head_groups)
    return LayerMesh(n_seq, n_head_groups, s_idx, h_idx, head_groups[s_idx], dp_groups[h_idx])


def choose_head_groups(lengths: Sequence[int], world: int, H: int, slack: float = 0.10) -> int:
    """Head-group count for a ``world``-rank mesh.  The busiest rank's work is
    (tokens of its sequence group) x (heads per rank); splitting heads balances
    it perfectly but all-reduces a ``[tokens, d_model]`` activation twice per
    step, while splitting sequences only all-reduces the weight gradients.  So
    the fewest head groups (over the divisors of ``world`` that also divide
    ``H``) whose busiest rank is within ``slack`` of the best balance wins."""
    costs = {}
    for hg in range(1, world + 1):
        if world % hg or H % hg:
            continue
        groups = assign_sequences(lengths, world // hg)
        costs[hg] = max(sum(int(lengths[i]) for i in gr) for gr in groups) * (H // hg)
    best = min(costs.values())
    return min(hg for hg, c in costs.items() if c <= (1.0 + slack) * best)


class _CopyToHeadGroup(torch.autograd.Function):
    """Identity forward; the backward all-reduces the cotangent over the head
    group (each rank's projections contribute a partial input cotangent)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, dx):
        dx = dx.contiguous()
        dist.all_reduce(dx, group=ctx.group)
        return dx, None


class _ReduceFromHeadGroup(torch.autograd.Function):
    """All-reduce (sum) forward of the ranks' partial ``W_o`` products; identity backward."""

    @staticmethod
    def forward(ctx, y, group):
        y = y.contiguous().clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, dy):
        return dy, None


_COL_SHARDED = ("W_q", "W_k", "W_v", "W_g", "W_a_up", "conv_q", "conv_k", "conv_v")


def shard_layer_params(p, H: int, mesh: LayerMesh):
    """This rank's head shard of full layer weights (``axiom_b200.layer.KDALayerParams``)
    as new leaf tensors: heads ``[h0, h1)`` of the projections' and conv taps'
    output columns, of ``W_beta``, ``b_gate`` and ``A``, and of ``W_o``'s input
    rows; ``W_a_down`` is replicated.  Returns ``(params, H_local)``."""
    if H % mesh.n_head_groups:
        raise ValueError(f"H={H} does not split over {mesh.n_head_groups} head groups")
    Hl = H // mesh.n_head_groups
    h0 = mesh.head_index * Hl
    dk = p.W_q.shape[1] // H
    dv = p.W_v.shape[1] // H
    out = {}
    for f in fields(p):
        t = getattr(p, f.name).detach()
        if f.name in _COL_SHARDED:
            w = dv if f.name in ("W_v", "W_g", "conv_v") else dk
            t = t[:, h0 * w:(h0 + Hl) * w]
        elif f.name == "W_beta":
            t = t[:, h0:h0 + Hl]
        elif f.name == "b_gate":
            t = t[h0 * dk:(h0 + Hl) * dk]
        elif f.name == "A":
            t = t[h0:h0 + Hl]
        elif f.name == "W_o":
            t = t[h0 * dv:(h0 + Hl) * dv, :]
        out[f.name] = t.contiguous().clone().requires_grad_(True)
    return type(p)(**out), Hl


def kda_layer_sharded(p_local, x_local, mesh: LayerMesh, *, H_local: int, cu_seqlens=None, **kw):
    """The layer over this rank's sequences (``x_local`` packed by
    ``cu_seqlens``) and head shard: the rank's partial output is summed over
    the head group, so every rank of it returns the full ``[T_local, d_model]``
    output of its sequences.  Differentiable; call :func:`allreduce_layer_grads`
    after the backward."""
    from .layer import kda_layer

    if mesh.n_head_groups > 1:
        x_local = _CopyToHeadGroup.apply(x_local, mesh.head_group)
    y = kda_layer(p_local, x_local, H=H_local, cu_seqlens=cu_seqlens, **kw)
    if mesh.n_head_groups > 1:
        y = _ReduceFromHeadGroup.apply(y, mesh.head_group)
    return y


def allreduce_layer_grads(p_local, mesh: LayerMesh) -> None:
    """Finish the gradients of a sharded layer step in place: ``W_a_down``'s
    (replicated in the head group, each rank holding the part from its heads)
    summed over the head group, then every gradient summed over the
    data-parallel (sequence) group, one flat bucket per dtype."""
    from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors

    if mesh.n_head_groups > 1 and p_local.W_a_down.grad is not None:
        dist.all_reduce(p_local.W_a_down.grad, group=mesh.head_group)
    if mesh.n_seq_groups == 1:
        return
    grads = [t.grad for t in p_local.tensors() if t.grad is not None]
    for dt in sorted({g_.dtype for g_ in grads}, key=str):
        part = [g_ for g_ in grads if g_.dtype == dt]
        flat = _flatten_dense_tensors(part)
        dist.all_reduce(flat, group=mesh.dp_group)
        for g_, s in zip(part, _unflatten_dense_tensors(flat, part)):
            g_.copy_(s)
