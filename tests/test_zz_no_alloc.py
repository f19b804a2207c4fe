"""kda_bwd_noalloc: the backward for callers that cannot allocate device memory.

A framework's custom-call handler, or a serving loop on a fixed memory budget,
cannot hand kda_bwd a workspace: allocating one would take device memory the
framework has already reserved for itself and would synchronise the device.
kda_bwd_noalloc runs the same backward on a fixed scratch array built into the
library.  These tests call it through the C ABI and check it against kda_bwd
(the entry point that takes a caller workspace) on two calls in a row, on the
tensor-core path and on the exact fp32 path, and check that an oversized
problem is refused before anything runs.  This file is collected last so that a
failure here cannot hide the result of any other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from axiom_b200 import _lib
from oracle import kda_oracle as K

KDA_ERR_SCRATCH_LIMIT = -8


def _ptr(x):
    return None if x is None else ctypes.c_void_p(x.data_ptr())


def _noalloc(q, k, v, g, beta, ckpt, do, dST, chunk):
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    outs = [torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(g),
            torch.empty_like(beta), torch.empty((B, H, dk, dv), dtype=torch.float32, device=q.device)]
    dt = {torch.float32: 0, torch.bfloat16: 1}
    rc = _lib.lib().kda_bwd_noalloc(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(ckpt), _ptr(do), _ptr(dST),
        *(_ptr(o) for o in outs), B, T, H, dk, dv, chunk, dt[q.dtype], dt[do.dtype],
        dt[ckpt.dtype], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check("kda_bwd_noalloc", rc)
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol,dims", [
    (torch.bfloat16, 1e-2, (1, 256, 2, 128, 128, 64)),   # tensor-core path
    (torch.float32, 1e-4, (1, 100, 2, 32, 32, 32)),      # exact fp32 path
])
def test_noalloc_matches_workspace_backward_twice(dtype, tol, dims):
    from axiom_b200 import kda_bwd, kda_fwd

    B, T, H, dk, dv, C = dims
    x = K.make_inputs(B, T, H, dk, dv, seed=31, s0_std=0.05)
    d = {n: torch.as_tensor(a).cuda().to(dtype if n != "S0" else torch.float32).contiguous()
         for n, a in x.items()}
    rng = np.random.default_rng(32)
    do = torch.as_tensor(rng.standard_normal((B, T, H, dv)), dtype=torch.float32).cuda().to(dtype)
    dST = torch.as_tensor(rng.standard_normal((B, H, dk, dv)), dtype=torch.float32).cuda()
    _, _, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], chunk=C, need_ckpt=True)
    ref = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, do, dST, chunk=C)
    for _ in range(2):
        got = _noalloc(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, do, dST, C)
        torch.cuda.synchronize()
        for name, a, b in zip(["dq", "dk", "dv", "dg", "dbeta", "dS0"], got, ref):
            err = K.scale_rel_err(a.float().cpu().numpy(), b.float().cpu().numpy())
            assert err <= tol, f"{name}: {err}"


def test_noalloc_refuses_problems_larger_than_its_scratch():
    lib = _lib.lib()
    need = lib.kda_bwd_workspace_bytes(4, 8192, 32, 128, 128, 64, 1)
    assert need > (32 << 20)
    rc = lib.kda_bwd_noalloc(*([None] * 14), 4, 8192, 32, 128, 128, 64, 1, 1, 1, None)
    assert rc == KDA_ERR_SCRATCH_LIMIT
    assert b"kda_bwd_noalloc" in lib.kda_strerror(rc)
