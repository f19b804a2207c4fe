"""JAX registration of the B200 KDA kernels (jax.ffi custom calls + custom_vjp).

The reference binds its KDA core interval as ``cc_scan`` (a ``jax.custom_vjp``
over the persistent Mosaic kernels, ``net/kernels/kda_cc_fused_persist.py:874-932``)
and selects it through ``AXIOM_KDA_CC_IMPL`` (``net/kda.py:708-729, 888-926``).
This module is the same boundary over ``libkda_b200.so``: ``cc_scan_b200`` is a
custom_vjp whose forward rule is the ``kda_fwd`` custom call (keeping the
forward's checkpoint as the residual) and whose backward rule is ``kda_bwd``;
``decode_step_b200`` is ``_delta_step`` + ``o = S^T q`` (``net/kda.py:298-310``).

It needs JAX and the handler library built from ``kda_ffi.cc`` (beside this
file); neither is available in the environment this package is built and
tested in, so nothing imports this module by default.  With them installed::

    from axiom_b200.jax_ffi.cc_scan_b200 import register, cc_scan_b200
    register("/path/to/libkda_ffi.so")
    o, S_T = cc_scan_b200(q, k, v, g, beta, S0)        # [B, T, H, D], g = log alpha

The reference calls its scan per batch element under ``vmap``
(``net/model.py:341-347``); these calls take the batch dimension directly, so
the caller drops the ``vmap`` around the core interval and makes one launch for
the batch.  Under a ``vmap`` that stays, each call declares
``vmap_method="sequential"``: one call per mapped element.
"""

from __future__ import annotations

import ctypes
import os
from functools import partial

import jax
import jax.numpy as jnp

_KDA_F32, _KDA_BF16 = 0, 1
_core = None


def _kda_dtype(dt) -> int:
    if dt == jnp.float32:
        return _KDA_F32
    if dt == jnp.bfloat16:
        return _KDA_BF16
    raise TypeError(f"KDA custom calls take float32 or bfloat16, got {dt}")


def register(ffi_lib_path: str, core_lib_path: str | None = None) -> None:
    """Load the handler library and register the three targets for CUDA."""
    global _core
    core_lib_path = core_lib_path or os.path.join(os.path.dirname(os.path.dirname(__file__)),
                                                  "libkda_b200.so")
    _core = ctypes.CDLL(core_lib_path)
    _core.kda_ckpt_bytes.restype = ctypes.c_size_t
    _core.kda_ckpt_bytes.argtypes = [ctypes.c_int] * 8
    handlers = ctypes.CDLL(ffi_lib_path)
    for name in ("kda_fwd", "kda_bwd", "kda_decode"):
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(handlers, name + "_handler")),
                                    platform="CUDA")


def _ckpt_bytes(B, T, H, dk, dv, chunk, dt) -> int:
    if _core is None:
        raise RuntimeError("call register() first: the KDA library is not loaded")
    code = _kda_dtype(dt)
    return int(_core.kda_ckpt_bytes(B, T, H, dk, dv, chunk, code, code))


def _fwd_call(q, k, v, g, beta, S0, chunk):
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    nbytes = _ckpt_bytes(B, T, H, dk, dv, chunk, q.dtype)
    return jax.ffi.ffi_call("kda_fwd", (
        jax.ShapeDtypeStruct((B, T, H, dv), q.dtype),
        jax.ShapeDtypeStruct((B, H, dk, dv), jnp.float32),
        jax.ShapeDtypeStruct((nbytes,), jnp.uint8),
    ), vmap_method="sequential")(q, k, v, g, beta, S0.astype(jnp.float32), chunk=chunk)


@partial(jax.custom_vjp, nondiff_argnums=(6,))
def cc_scan_b200(q, k, v, g, beta, S0, chunk=64):
    """Chunked KDA core: ``(o, S_T)`` from ``q, k, g [B, T, H, dk]``, ``v [B, T, H, dv]``,
    ``beta [B, T, H]`` and ``S0 [B, H, dk, dv]`` (fp32)."""
    o, s_t, _ = _fwd_call(q, k, v, g, beta, S0, chunk)
    return o, s_t


def _cc_fwd(q, k, v, g, beta, S0, chunk):
    o, s_t, ckpt = _fwd_call(q, k, v, g, beta, S0, chunk)
    return (o, s_t), (q, k, v, g, beta, ckpt, S0)


def _cc_bwd(chunk, res, cot):
    q, k, v, g, beta, ckpt, S0 = res
    do, dsT = cot
    dq, dk_, dv_, dg, dbeta, ds0 = jax.ffi.ffi_call("kda_bwd", (
        jax.ShapeDtypeStruct(q.shape, q.dtype), jax.ShapeDtypeStruct(k.shape, k.dtype),
        jax.ShapeDtypeStruct(v.shape, v.dtype), jax.ShapeDtypeStruct(g.shape, g.dtype),
        jax.ShapeDtypeStruct(beta.shape, beta.dtype), jax.ShapeDtypeStruct(S0.shape, jnp.float32),
    ), vmap_method="sequential")(q, k, v, g, beta, ckpt, do.astype(q.dtype), dsT.astype(jnp.float32), chunk=chunk)
    # cotangents in the primal dtypes (kda_cc_fused_persist.py:1716-1719)
    return dq, dk_, dv_, dg, dbeta, ds0.astype(S0.dtype)


cc_scan_b200.defvjp(_cc_fwd, _cc_bwd)


def decode_step_b200(S, q, k, v, g, beta):
    """One token for every (sequence, head): returns ``(o, S_new)``; ``S`` is donated
    to the result (updated in place on the device)."""
    o_shape = q.shape[:-1] + (S.shape[-1],)
    return jax.ffi.ffi_call("kda_decode", (
        jax.ShapeDtypeStruct(o_shape, q.dtype), jax.ShapeDtypeStruct(S.shape, jnp.float32),
    ), input_output_aliases={0: 1}, vmap_method="sequential")(S, q, k, v, g, beta)
