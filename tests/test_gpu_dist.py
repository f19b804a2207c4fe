"""Two GPUs, NCCL: the sharded KDA core and the sharded mixer layer against one GPU.

Two ranks (one process per GPU, NCCL over NVLink) each run the sharded path
and, on the same inputs, the unsharded one on their own GPU:

* the core's forward, backward and decode split by batch (B = 2) and by head
  (B = 1): the gathered outputs, gradients and states equal the single-GPU
  ones bit for bit (every (batch, head) unit is computed by the same kernels
  with the same arithmetic whichever rank runs it);
* the mixer layer on a 2 x 1 mesh (whole sequences per rank) and a 1 x 2 mesh
  (heads split, the W_o products and the input cotangent all-reduced): output,
  input gradient and every weight gradient within 2e-2 scale-relative of the
  single-GPU layer (the gradient sums run in a different order, over bf16).

Skipped on hosts with fewer than two GPUs.  The CPU (gloo) versions of the
same host logic are in ``tests/test_dist_gloo.py``.
"""

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        return sck.getsockname()[1]


def _core_worker(rank, world, port, B, out_path):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from axiom_b200 import decode_step, kda_bwd, kda_fwd
    from axiom_b200 import dist as D

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        H, T = 4, 200
        gen = torch.Generator(device=dev).manual_seed(7)
        bf = torch.bfloat16

        def rn(*s):
            return torch.randn(*s, generator=gen, device=dev)

        q = torch.nn.functional.normalize(rn(B, T, H, 128), dim=-1).to(bf)
        k = torch.nn.functional.normalize(rn(B, T, H, 128), dim=-1).to(bf)
        v = rn(B, T, H, 128).to(bf)
        g = torch.nn.functional.logsigmoid(rn(B, T, H, 128) + 3.0).to(bf)
        beta = torch.sigmoid(rn(B, T, H)).to(bf)
        S0 = rn(B, H, 128, 128) * 0.05
        do = rn(B, T, H, 128).to(bf)
        dST = rn(B, H, 128, 128)
        o, s_t, ck = D.sharded_forward(q, k, v, g, beta, S0, need_ckpt=True)
        grads = D.sharded_backward(q, k, v, g, beta, ck, do, dST)
        o1, s1, ck1 = kda_fwd(q, k, v, g, beta, S0, need_ckpt=True)
        grads1 = kda_bwd(q, k, v, g, beta, ck1, do, dST)
        same = [bool(torch.equal(a, b)) for a, b in zip((o, s_t) + tuple(grads), (o1, s1) + tuple(grads1))]
        # decode: the B * H states split over the ranks, three tokens
        N = B * H
        lo, hi = D.decode_shard(N)
        S_all = S0.reshape(N, 128, 128).clone()
        S_loc = S_all[lo:hi].clone()
        for t in range(3):
            tok = [x[:, t].reshape(N, -1).contiguous() for x in (q, k, v, g)]
            bt = beta[:, t].reshape(N).contiguous()
            od = D.sharded_decode_step(S_loc, *tok, bt)
            od1 = decode_step(S_all, *tok, bt)
            same.append(bool(torch.equal(od, od1)))
        same.append(bool(torch.equal(S_loc, S_all[lo:hi])))
        torch.cuda.synchronize()
        if rank == 0:
            np.save(out_path, np.array(same))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [2, 1])  # batch split, then head split
def test_two_gpu_sharded_core_equals_one_gpu_bitwise(tmp_path, B):
    import torch.multiprocessing as mp

    out = str(tmp_path / "same.npy")
    mp.start_processes(_core_worker, args=(2, _free_port(), B, out), nprocs=2, join=True,
                       start_method="spawn")
    same = np.load(out)
    assert same.all(), same.tolist()


def _layer_worker(rank, world, port, n_head_groups, out_path):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from axiom_b200 import dist as D
    from axiom_b200 import layer
    from oracle.kda_oracle import scale_rel_err

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        d_model, H, dk = 256, 4, 128
        cu = [0, 150, 230, 400, 471]
        T = cu[-1]
        p = layer.init_params(d_model, H, dk, dk, rank=32, K=4, gate_kind="softplus", dtype=torch.bfloat16,
                              device=dev, seed=9)
        gen = torch.Generator(device="cpu").manual_seed(10)
        x = torch.randn(T, d_model, generator=gen).to(dev, torch.bfloat16)
        dout = torch.randn(T, d_model, generator=gen).to(dev, torch.bfloat16)
        # one GPU: the whole layer
        x1 = x.clone().requires_grad_(True)
        layer.kda_layer(p, x1, H=H, cu_seqlens=cu, gate_kind="softplus").backward(dout)
        # the mesh
        mesh = D.layer_mesh(n_head_groups)
        pl, Hl = D.shard_layer_params(p, H, mesh)
        ids = D.assign_sequences([b - a for a, b in zip(cu[:-1], cu[1:])], mesh.n_seq_groups)[mesh.seq_index]
        rows, cu_loc = D.local_packing(cu, ids)
        ridx = torch.tensor(rows, device=dev, dtype=torch.long)
        xl = x[ridx].clone().requires_grad_(True)
        y = D.kda_layer_sharded(pl, xl, mesh, H_local=Hl, cu_seqlens=cu_loc, gate_kind="softplus")
        y.backward(dout[ridx])
        D.allreduce_layer_grads(pl, mesh)
        with torch.no_grad():
            y_ref = layer.kda_layer(p, x, H=H, cu_seqlens=cu, gate_kind="softplus")[ridx]
        errs = {"y": scale_rel_err(y.detach().double().cpu().numpy(), y_ref.double().cpu().numpy()),
                "x": scale_rel_err(xl.grad.double().cpu().numpy(), x1.grad[ridx].double().cpu().numpy())}
        h0 = mesh.head_index * Hl
        for name in ("W_q", "W_k", "W_v", "W_g", "W_beta", "W_a_down", "W_a_up", "b_gate", "A", "conv_q",
                     "conv_k", "conv_v", "W_o"):
            full = getattr(p, name).grad
            if name in ("W_beta",):
                full = full[:, h0:h0 + Hl]
            elif name == "A":
                full = full[h0:h0 + Hl]
            elif name == "b_gate":
                full = full[h0 * dk:(h0 + Hl) * dk]
            elif name == "W_o":
                full = full[h0 * dk:(h0 + Hl) * dk]
            elif name != "W_a_down":
                full = full[:, h0 * dk:(h0 + Hl) * dk]
            errs[name] = scale_rel_err(getattr(pl, name).grad.double().cpu().numpy(), full.double().cpu().numpy())
        torch.cuda.synchronize()
        np.save(out_path.replace(".npy", f"_{rank}.npy"), np.array([errs[k_] for k_ in sorted(errs)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_head_groups", [1, 2])  # 2 x 1 (sequences), 1 x 2 (heads)
def test_two_gpu_sharded_layer_matches_one_gpu(tmp_path, n_head_groups):
    import torch.multiprocessing as mp

    out = str(tmp_path / "errs.npy")
    mp.start_processes(_layer_worker, args=(2, _free_port(), n_head_groups, out), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        errs = np.load(out.replace(".npy", f"_{r}.npy"))
        assert (errs <= 2e-2).all(), errs.tolist()
