"""World-size-2 CPU (gloo) tests of the multi-rank partitioning and collectives.

The per-rank operators are replaced by the CPU oracle (the kernels need a
GPU); what is tested here is the host-side logic: the batch/head split, the
slices each rank computes, the reassembly of O, S_T, the gradients and the
decode outputs by the all-gather, the sequence assignment of the mixer layer,
the head-group all-reduces of its forward and backward, and the gradient
bucket all-reduce.  The same paths with the CUDA kernels and NCCL are in
``tests/test_gpu_dist.py``.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from axiom_b200 import dist as D
from oracle import kda_oracle as K


def _oracle_fwd(q, k, v, g, beta, S0):
    o, s = K.chunk_fwd(q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta.numpy(),
                       None if S0 is None else S0.numpy(), chunk=16)
    # the oracle needs no checkpoint beyond S0: the rank's own S0 slice stands in for it
    return torch.from_numpy(o), torch.from_numpy(s), S0


def _oracle_bwd(q, k, v, g, beta, S0_local, do, dST):
    r = K.chunk_bwd(q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta.numpy(), S0_local.numpy(),
                    do.numpy(), dST.numpy(), chunk=16)
    return tuple(torch.from_numpy(np.ascontiguousarray(a)) for a in r)


def _oracle_decode(S, q, k, v, g, beta):
    o, s_new = K.decode_step(S.numpy(), q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta.numpy())
    S.copy_(torch.from_numpy(s_new))
    return torch.from_numpy(o)


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _core_worker(rank, world, port, B, H, out_path):
    _init(rank, world, port)
    try:
        x = K.make_inputs(B, 40, H, 8, 8, seed=3, s0_std=0.1)
        t = {n: torch.from_numpy(a).double() for n, a in x.items()}
        rng = np.random.default_rng(4)
        do = torch.from_numpy(rng.standard_normal((B, 40, H, 8)))
        dST = torch.from_numpy(rng.standard_normal((B, H, 8, 8)))
        o, s, ck = D.sharded_forward(t["q"], t["k"], t["v"], t["g"], t["beta"], t["S0"],
                                     compute=_oracle_fwd, need_ckpt=True)
        grads = D.sharded_backward(t["q"], t["k"], t["v"], t["g"], t["beta"], ck, do, dST,
                                   compute=_oracle_bwd)
        # decode: N = B * H states sharded over the ranks, one token
        N = B * H
        lo, hi = D.decode_shard(N)
        S_all = t["S0"].reshape(N, 8, 8)
        S_loc = S_all[lo:hi].clone()
        tok = {n: t[n][:, 0].reshape((N,) + tuple(t[n].shape[3:])) for n in ("q", "k", "v", "g", "beta")}
        od = D.sharded_decode_step(S_loc, tok["q"], tok["k"], tok["v"], tok["g"], tok["beta"],
                                   compute=_oracle_decode)
        S_parts = [torch.empty_like(S_loc) for _ in range(world)]
        dist.all_gather(S_parts, S_loc)
        if rank == 0:
            np.savez(out_path, o=o.numpy(), s=s.numpy(), od=od.numpy(), sd=torch.cat(S_parts).numpy(),
                     **{f"g{i}": gr.numpy() for i, gr in enumerate(grads)})
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        return sck.getsockname()[1]


def _spawn(fn, *args):
    mp.start_processes(fn, args=(2, _free_port(), *args), nprocs=2, join=True, start_method="spawn")


@pytest.mark.parametrize("B,H", [(4, 3), (3, 4)])  # batch split, then head split
def test_two_rank_sharded_forward_backward_decode_equal_single_process(tmp_path, B, H):
    out = str(tmp_path / "res.npz")
    _spawn(_core_worker, B, H, out)
    got = np.load(out)
    x = K.make_inputs(B, 40, H, 8, 8, seed=3, s0_std=0.1)
    rng = np.random.default_rng(4)
    do = rng.standard_normal((B, 40, H, 8))
    dST = rng.standard_normal((B, H, 8, 8))
    o_ref, s_ref = K.chunk_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk=16)
    assert np.allclose(got["o"], o_ref, atol=1e-10)
    assert np.allclose(got["s"], s_ref, atol=1e-10)
    ref = K.chunk_bwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], do, dST, chunk=16)
    for i, r in enumerate(ref):
        assert np.allclose(got[f"g{i}"], r, atol=1e-10), i
    N = B * H
    od, sd = K.decode_step(x["S0"].reshape(N, 8, 8), *(x[n][:, 0].reshape((N,) + x[n].shape[3:])
                                                        for n in ("q", "k", "v", "g", "beta")))
    assert np.allclose(got["od"], od, atol=1e-10)
    assert np.allclose(got["sd"], sd, atol=1e-10)


def test_partition_and_axis_rules():
    assert D.partition(8, 4, 1) == (2, 4)
    assert D.shard_axis(4, 3, 2) == 0
    assert D.shard_axis(3, 4, 2) == 2
    with pytest.raises(ValueError):
        D.shard_axis(3, 5, 2)
    with pytest.raises(ValueError):
        D.partition(5, 2, 0)


def test_sequence_assignment_balances_whole_sequences():
    lengths = [100, 900, 400, 400, 300, 0, 50]
    groups = D.assign_sequences(lengths, 3)
    assert sorted(i for gr in groups for i in gr) == list(range(len(lengths)))
    # longest first onto the lightest group: 900 | 400 + 300 | 400 + 100 + 50 + 0
    assert groups == [[1], [2, 4], [0, 3, 5, 6]]
    rows, cu_local = D.local_packing([0, 2, 5, 5, 9], [2, 0, 3])
    assert rows == [0, 1, 5, 6, 7, 8] and cu_local == [0, 0, 2, 6]  # sequence 2 is empty
    # cfg5-like lengths: head groups are chosen when whole sequences cannot balance 8 ranks
    rng = np.random.default_rng(5)
    L = rng.uniform(512, 8192, 16)
    L = np.floor(L / L.sum() * 65536).astype(int)
    L[-1] += 65536 - int(L.sum())
    def cost(w, h2):
        return max(sum(L[i] for i in gr) for gr in D.assign_sequences(L.tolist(), w // h2)) * (16 // h2)

    for world in (2, 4, 8):
        hg = D.choose_head_groups(L.tolist(), world, 16)
        best = min(cost(world, h2) for h2 in (1, 2, 4, 8) if world % h2 == 0)
        # the fewest head groups within 10 % of the best-balanced mesh
        assert cost(world, hg) <= 1.1 * best
        assert all(cost(world, h2) > 1.1 * best for h2 in (1, 2, 4) if h2 < hg)
    assert D.choose_head_groups(L.tolist(), 2, 16) == 1      # sequences balance two ranks
    assert D.choose_head_groups(L.tolist(), 8, 16) == 2      # ... but not eight


def _mesh_worker(rank, world, port, n_head_groups, out_path):
    """A toy two-projection 'layer' y = (x W1) W2 with W1 column-sharded and W2
    row-sharded over the head group, plus a replicated weight R whose gradient is
    partial per head shard: checks the head-group all-reduces of the forward and
    the backward and allreduce_layer_grads against the unsharded computation."""
    _init(rank, world, port)
    try:
        from axiom_b200.layer import KDALayerParams

        mesh = D.layer_mesh(n_head_groups)
        g = torch.Generator().manual_seed(0)
        d, H, dh, T = 6, 4, 2, 5
        full = {n: torch.randn(*s, generator=g, dtype=torch.float64) for n, s in (
            ("W_q", (d, H * dh)), ("W_k", (d, H * dh)), ("W_v", (d, H * dh)), ("W_g", (d, H * dh)),
            ("W_beta", (d, H)), ("W_a_down", (d, 3)), ("W_a_up", (3, H * dh)), ("b_gate", (H * dh,)),
            ("A", (H,)), ("conv_q", (2, H * dh)), ("conv_k", (2, H * dh)), ("conv_v", (2, H * dh)),
            ("W_o", (H * dh, d)))}
        x_all = torch.randn(2 * T, d, generator=g, dtype=torch.float64)
        p = KDALayerParams(**{n: t.clone() for n, t in full.items()})
        pl, Hl = D.shard_layer_params(p, H, mesh)
        # this rank's sequences: sequence group s takes rows [s T, (s + 1) T) (two groups at most)
        x = x_all[mesh.seq_index * T * (2 // mesh.n_seq_groups):][: T * (2 // mesh.n_seq_groups)]
        x = x.clone().requires_grad_(True)
        xin = D._CopyToHeadGroup.apply(x, mesh.head_group) if n_head_groups > 1 else x
        # toy layer on the local heads: y = ((x W_q) * (x W_a_down W_a_up)) W_o
        z = (xin @ pl.W_a_down) @ pl.W_a_up
        y = ((xin @ pl.W_q) * z) @ pl.W_o
        if n_head_groups > 1:
            y = D._ReduceFromHeadGroup.apply(y, mesh.head_group)
        y.backward(torch.ones_like(y))
        for t in pl.tensors():
            if t.grad is None:
                t.grad = torch.zeros_like(t)
        D.allreduce_layer_grads(pl, mesh)
        res = {"y": y.detach().numpy(), "dx": x.grad.numpy()}
        for n in ("W_q", "W_a_down", "W_a_up", "W_o"):
            res[n] = getattr(pl, n).grad.numpy()
        np.savez(out_path.replace(".npz", f"_{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_head_groups", [(2, 1), (2, 2), (4, 2)])  # 2 x 1, 1 x 2, 2 x 2 meshes
def test_layer_mesh_collectives_equal_unsharded(tmp_path, world, n_head_groups):
    out = str(tmp_path / "mesh.npz")
    mp.start_processes(_mesh_worker, args=(world, _free_port(), n_head_groups, out), nprocs=world, join=True,
                       start_method="spawn")
    g = torch.Generator().manual_seed(0)
    d, H, dh, T = 6, 4, 2, 5
    shapes = (("W_q", (d, H * dh)), ("W_k", (d, H * dh)), ("W_v", (d, H * dh)), ("W_g", (d, H * dh)),
              ("W_beta", (d, H)), ("W_a_down", (d, 3)), ("W_a_up", (3, H * dh)), ("b_gate", (H * dh,)),
              ("A", (H,)), ("conv_q", (2, H * dh)), ("conv_k", (2, H * dh)), ("conv_v", (2, H * dh)),
              ("W_o", (H * dh, d)))
    full = {n: torch.randn(*s, generator=g, dtype=torch.float64).requires_grad_(True) for n, s in shapes}
    x = torch.randn(2 * T, d, generator=g, dtype=torch.float64).requires_grad_(True)
    y = ((x @ full["W_q"]) * ((x @ full["W_a_down"]) @ full["W_a_up"])) @ full["W_o"]
    y.backward(torch.ones_like(y))
    n_seq = world // n_head_groups
    width = H * dh // n_head_groups  # columns of one head shard
    for r in range(world):
        got = np.load(out.replace(".npz", f"_{r}.npz"))
        s_idx, j = divmod(r, n_head_groups)
        rows = slice(0, 2 * T) if n_seq == 1 else slice(s_idx * T, (s_idx + 1) * T)
        cols = slice(j * width, (j + 1) * width)
        assert np.allclose(got["y"], y.detach().numpy()[rows]), r
        assert np.allclose(got["dx"], x.grad.numpy()[rows]), r
        # every gradient is the whole batch's: summed over the sequence groups, and
        # W_a_down's also over the head group
        assert np.allclose(got["W_a_down"], full["W_a_down"].grad.numpy()), r
        assert np.allclose(got["W_q"], full["W_q"].grad.numpy()[:, cols]), r
        assert np.allclose(got["W_a_up"], full["W_a_up"].grad.numpy()[:, cols]), r
        assert np.allclose(got["W_o"], full["W_o"].grad.numpy()[cols, :]), r
