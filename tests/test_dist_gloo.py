"""World-size-2 CPU (gloo) test of the multi-rank partitioning and gather.

The per-rank operator is replaced by the CPU oracle (the kernels need a GPU);
what is tested here is the host-side logic: the batch/head split, the slices
each rank computes, and the reassembly of O and S_T by the all-gather.
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


def _oracle_compute(q, k, v, g, beta, S0):
    o, s = K.chunk_fwd(q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta.numpy(),
                       None if S0 is None else S0.numpy(), chunk=16)
    return torch.from_numpy(o), torch.from_numpy(s)


def _worker(rank, world, port, B, H, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = K.make_inputs(B, 40, H, 8, 8, seed=3, s0_std=0.1)
        t = {n: torch.from_numpy(a).double() for n, a in x.items()}
        o, s = D.sharded_forward(t["q"], t["k"], t["v"], t["g"], t["beta"], t["S0"],
                                 compute=_oracle_compute)
        if rank == 0:
            np.savez(out_path, o=o.numpy(), s=s.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        return sck.getsockname()[1]


@pytest.mark.parametrize("B,H", [(4, 3), (3, 4)])  # batch split, then head split
def test_two_rank_sharded_forward_equals_single_process(tmp_path, B, H):
    out = str(tmp_path / "res.npz")
    mp.start_processes(_worker, args=(2, _free_port(), B, H, out), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    x = K.make_inputs(B, 40, H, 8, 8, seed=3, s0_std=0.1)
    o_ref, s_ref = K.chunk_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk=16)
    assert np.allclose(got["o"], o_ref, atol=1e-10)
    assert np.allclose(got["s"], s_ref, atol=1e-10)


def test_partition_and_axis_rules():
    assert D.partition(8, 4, 1) == (2, 4)
    assert D.shard_axis(4, 3, 2) == 0
    assert D.shard_axis(3, 4, 2) == 2
    with pytest.raises(ValueError):
        D.shard_axis(3, 5, 2)
    with pytest.raises(ValueError):
        D.partition(5, 2, 0)
