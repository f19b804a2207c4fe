"""Host-side checks of the C ABI and the Python mirror (no GPU needed).

* the library loads and exports every function ``include/*.h`` declares;
* argument validation fails closed before any launch (typed error codes);
* the implementation switch fails closed on unknown values
  (``net/kda.py:708-729``) and the operators refuse a GPU-less host with a
  typed error instead of falling back (``net/kda.py:759-763``).
"""

import ctypes
import glob
import os
import re

import pytest
import torch

from axiom_b200 import _lib
from axiom_b200 import kda as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def _declared_functions(header):
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(kda_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    assert len(HEADERS) >= 2
    for header in HEADERS:
        names = _declared_functions(header)
        assert names, f"no declarations parsed from {header}"
        for name in names:
            assert hasattr(lib, name), f"{name} declared in {os.path.basename(header)} but not exported"
            assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.kda_version() >= 100
    assert lib.kda_strerror(0) == b"ok"
    assert b"dimensions" in lib.kda_strerror(-1)


def test_ckpt_bytes():
    lib = _lib.lib()
    units = 4 * 32 * 128
    # tensor-core path: states, then per chunk-head T, Aqk, Akk (3 x 64 x 64 bf16),
    # W, Q Gam, K Gam, K Gam^-1, lam K, v~, U (7 x 64 x 128 bf16), Gam_C (128 fp32)
    # and the flags (padded to 16 bytes), then the state-chain operands of the
    # split forward: NP (128 x 128 bf16), Q~ and Aqk U (2 x 64 x 128 bf16)
    factors = 3 * 64 * 64 * 2 + 7 * 64 * 128 * 2 + 128 * 4 + 512 + 128 * 128 * 2 + 2 * 64 * 128 * 2
    assert factors == 205824
    assert lib.kda_ckpt_bytes(4, 8192, 32, 128, 128, 64, 1, 1) == units * (128 * 128 * 2 + factors)
    assert lib.kda_ckpt_bytes(4, 8192, 32, 128, 128, 64, 1, 0) == units * (128 * 128 * 4 + factors)
    # exact path: states only
    assert lib.kda_ckpt_bytes(1, 100, 2, 16, 8, 64, 0, 0) == 1 * 2 * 2 * 16 * 8 * 4
    assert lib.kda_ckpt_bytes(1, 64, 1, 64, 64, 48, 1, 1) == 0  # unsupported chunk


def test_ckpt_states_undoes_the_operand_image():
    # byte offset of element (r, c) in a CM tile with `cols` columns, as in the kernels:
    # 8 x 8 core matrices of 128 bytes, core (r/8, c/8) at ((r/8)*(cols/8) + c/8)*128
    def cm_off(r, c, cols):
        return ((r // 8) * (cols // 8) + c // 8) * 128 + (r % 8) * 16 + (c % 8) * 2

    B, T, H, n = 1, 130, 2, 3
    states = torch.randn(B, H, n, 128, 128).to(torch.bfloat16)
    image = torch.empty(B * H * n * 128 * 128, dtype=torch.bfloat16)
    r = torch.arange(128).view(128, 1).expand(128, 128)
    c = torch.arange(128).view(1, 128).expand(128, 128)
    elem = torch.tensor([[cm_off(i, j, 128) // 2 for j in range(128)] for i in range(128)])
    assert torch.equal(elem, ((r // 8) * 16 + c // 8) * 64 + (r % 8) * 8 + c % 8)
    for u in range(B * H * n):
        image[u * 16384 + elem.reshape(-1)] = states.reshape(-1, 128, 128)[u].reshape(-1)
    ckpt = torch.cat([image, torch.zeros(B * H * n * 3 * 64 * 64, dtype=torch.bfloat16)])
    assert torch.equal(K.ckpt_states(ckpt, B, T, H, 128, 128), states)
    # other layouts are row-major
    flat = torch.randn(B * H * n * 64 * 64)
    assert torch.equal(K.ckpt_states(flat, B, T, H, 64, 64, in_dtype=torch.float32),
                       flat.reshape(B, H, n, 64, 64))


@pytest.mark.parametrize("dims", [
    (1, 64, 1, 7, 64, 64),     # dk not a multiple of 8
    (1, 64, 1, 64, 136, 64),   # dv too large
    (1, 64, 1, 64, 64, 48),    # unsupported chunk
    (-1, 64, 1, 64, 64, 64),   # negative batch
])
def test_fwd_rejects_bad_shapes_before_launch(dims):
    lib = _lib.lib()
    B, T, H, dk, dv, C = dims
    rc = lib.kda_fwd(None, None, None, None, None, None, None, None, None,
                     B, T, H, dk, dv, C, 1, 1, 1, None)
    assert rc == -1


def test_fwd_rejects_bad_dtype_and_null_pointers():
    lib = _lib.lib()
    assert lib.kda_fwd(*([None] * 9), 1, 64, 1, 64, 64, 64, 7, 1, 1, None) == -2
    assert lib.kda_fwd(*([None] * 9), 1, 64, 1, 64, 64, 64, 1, 1, 1, None) == -4


def test_bwd_validation():
    lib = _lib.lib()
    args = [None] * 14 + [None, 0]
    assert lib.kda_bwd(*args, 1, 64, 1, 64, 64, 63, 1, 1, 1, None) == -1
    assert lib.kda_bwd(*args, 1, 64, 1, 64, 64, 64, 1, 1, 1, None) == -4
    fake = ctypes.c_void_p(16)
    full = [fake] * 14 + [None, 0]
    assert lib.kda_bwd(*full, 1, 64, 1, 64, 64, 64, 1, 1, 1, None) == -6  # workspace missing
    assert lib.kda_bwd_workspace_bytes(1, 64, 1, 64, 64, 64, 1) > 0


def test_decode_validation():
    lib = _lib.lib()
    assert lib.kda_decode(*([None] * 7), 4, 96, 128, 1, 1, None) == -1
    assert lib.kda_decode(*([None] * 7), 4, 128, 128, 1, 1, None) == -4
    assert lib.kda_decode(*([None] * 7), 0, 128, 128, 1, 1, None) == 0
    odd = ctypes.c_void_p(8)
    assert lib.kda_decode(odd, *([ctypes.c_void_p(16)] * 6), 4, 128, 128, 1, 1, None) == -3


def test_prologue_validation():
    lib = _lib.lib()
    w = [None] * 10
    outs = [None] * 5

    def fwd(*, kind=0, st=(None, None), cu=None, n_seqs=0, rows=None, dims=(1, 64, 2, 128, 128, 4), dt=(1, 1),
            ptrs=None, o=None):
        return lib.kda_prologue_fwd(*(ptrs or w), -5.0, kind, st[0], st[1], cu, n_seqs, rows, *(o or outs), *dims,
                                    *dt, None)

    assert fwd(dims=(1, 64, 2, 96, 128, 4)) == -1       # dk not 64/128
    assert fwd(dims=(1, 64, 2, 128, 128, 5)) == -1      # K > 4
    assert fwd(dims=(1, 64, 2, 128, 128, 0)) == -1      # K < 1
    assert fwd(kind=7) == -1                              # unknown gate form
    assert fwd(dt=(1, 9)) == -2
    assert fwd(dims=(0, 64, 2, 128, 128, 4)) == 0        # nothing to do
    assert fwd() == -4                                    # null inputs
    fake, odd = ctypes.c_void_p(16), ctypes.c_void_p(8)
    # packed sequences need B = 1 and no conv state
    assert fwd(cu=fake, n_seqs=2, dims=(2, 64, 2, 128, 128, 4)) == -1
    assert fwd(cu=fake, n_seqs=2, st=(fake, None)) == -1
    assert fwd(ptrs=[odd] + [fake] * 9, o=[fake] * 5) == -3
    assert fwd(rows=fake, ptrs=[fake] * 10, o=[fake] * 5) == -1  # out_rows without cu_seqlens
    assert lib.kda_prologue_bwd_workspace_bytes(1, 64, 2, 128, 128, 4) > 0
    assert lib.kda_prologue_bwd_workspace_bytes(1, 64, 2, 100, 128, 4) == 0
    bw = lib.kda_prologue_bwd(*([fake] * 10), -5.0, 0, None, None, 0, None, *([fake] * 10), *([fake] * 5), None,
                              None, 0, 1, 64, 2, 128, 128, 4, 1, 1, None)
    assert bw == -6                                       # workspace missing


def test_gated_rmsnorm_and_fused_decode_validation():
    lib = _lib.lib()
    nomap = (None, None, 0)
    assert lib.kda_gated_rmsnorm_fwd(None, None, None, *nomap, 4, 2, 96, 1e-6, 1, 1, 1, None) == -1
    assert lib.kda_gated_rmsnorm_fwd(None, None, None, *nomap, 0, 2, 128, 1e-6, 1, 1, 1, None) == 0
    assert lib.kda_gated_rmsnorm_fwd(None, None, None, *nomap, 4, 2, 128, 1e-6, 1, 1, 1, None) == -4
    assert lib.kda_gated_rmsnorm_bwd(*([None] * 5), *nomap, 4, 2, 128, 1e-6, 3, 1, 1, None) == -2
    fake = ctypes.c_void_p(16)
    # a row map needs the sequence offsets
    assert lib.kda_gated_rmsnorm_fwd(fake, fake, fake, None, fake, 2, 4, 2, 128, 1e-6, 1, 1, 1, None) == -1
    args = [fake, fake] + [fake] * 11
    assert lib.kda_decode_fused(*args, -5.0, 0, 1e-6, fake, 4, 2, 96, 128, 4, 1, 1, None) == -1
    assert lib.kda_decode_fused(*args, -5.0, 2, 1e-6, fake, 4, 2, 128, 128, 4, 1, 1, None) == -1
    no_buf = [fake, None] + [fake] * 11
    assert lib.kda_decode_fused(*no_buf, -5.0, 0, 1e-6, fake, 4, 2, 128, 128, 4, 1, 1, None) == -4
    assert lib.kda_decode_fused(*args, -5.0, 0, 1e-6, fake, 0, 2, 128, 128, 4, 1, 1, None) == 0


def test_varlen_core_validation():
    lib = _lib.lib()
    fake = ctypes.c_void_p(16)
    # T must be a multiple of the chunk; the chunk offsets are required
    assert lib.kda_fwd_varlen(*([fake] * 9), fake, 2, 100, 2, 128, 128, 64, 1, 1, 1, None) == -1
    assert lib.kda_fwd_varlen(*([fake] * 9), None, 2, 128, 2, 128, 128, 64, 1, 1, 1, None) == -4
    assert lib.kda_fwd_varlen(*([fake] * 9), fake, -1, 128, 2, 128, 128, 64, 1, 1, 1, None) == -1
    assert lib.kda_fwd_varlen(*([None] * 10), 0, 128, 2, 128, 128, 64, 1, 1, 1, None) == 0
    args = [fake] * 14 + [None, 0]
    assert lib.kda_bwd_varlen(*args, fake, 2, 128, 2, 128, 128, 64, 1, 1, 1, None) == -6  # workspace missing
    assert lib.kda_bwd_varlen_workspace_bytes(2, 128, 2, 128, 128, 64, 1) >= \
        lib.kda_bwd_workspace_bytes(1, 128, 2, 128, 128, 64, 1)
    # the CUDA-core path's scratch is per sequence
    assert lib.kda_bwd_varlen_workspace_bytes(3, 96, 2, 32, 32, 32, 0) == \
        lib.kda_bwd_workspace_bytes(3, 96, 2, 32, 32, 32, 0)


def test_impl_switch_fails_closed(monkeypatch):
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "b200")
    assert K.kda_cc_impl() == "b200"
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "jax")
    assert K.kda_cc_impl() == "jax"
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "triton")
    with pytest.raises(ValueError):
        K.kda_cc_impl()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the GPU-less refusal")
def test_operators_refuse_a_gpu_less_host():
    x = torch.zeros(1, 64, 1, 64)
    with pytest.raises(RuntimeError, match="no CPU"):
        K.kda_fwd(x, x, x, x, torch.zeros(1, 64, 1))
    with pytest.raises(RuntimeError, match="no CPU"):
        K.decode_step(torch.zeros(2, 64, 64), *([torch.zeros(2, 64)] * 4), torch.zeros(2))


def test_missing_library_raises(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", os.path.join(ROOT, "does_not_exist.so"))
    with pytest.raises(RuntimeError, match="not built"):
        _lib.lib()


def test_device_status_entry_points_validate_before_any_cuda_call():
    lib = _lib.lib()
    assert lib.kda_device_status(None, 0, None) == -4  # KDA_ERR_NULL
    assert lib.kda_selftest_wait_timeout(0, None) == -1  # KDA_ERR_SHAPE: zero polls
    assert b"bounded wait" in lib.kda_strerror(-9)
