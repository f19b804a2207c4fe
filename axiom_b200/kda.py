"""Host-side operator interface of the B200 KDA core.

Mirrors the reference's operator API for the KDA core interval so that a
caller of the reference finds the same names, argument meanings and error
behaviour (AXIOM, ``net/kernels/kda_cc_fused_persist.py`` and ``net/kda.py``):

* :func:`kernel` / :func:`kernel_bwd` / :func:`cc_scan` -- the operand form
  ``(q, k, v, alpha, beta32, S)`` of ``kda_cc_fused_persist.kernel`` (:718),
  ``kernel_bwd`` (:1707) and the differentiable ``cc_scan`` (:920);
* :func:`chunk_kda` -- the same operator in the BASELINE form
  ``(q, k, v, g, beta, S0)`` over ``[B, T, H, D]``, differentiable;
* :func:`kda_fwd` / :func:`kda_bwd` -- the raw launches;
* :func:`decode_step` -- the recurrent single-token update
  (``_delta_step`` + ``o = S^T q``, ``net/kda.py:298-310, :293``);
* :func:`kda_cc_impl` -- the fail-closed implementation switch
  (``net/kda.py:708-729``) with the added value ``b200``.

PyTorch provides device memory, streams and autograd plumbing only; every
computation runs in ``libkda_b200.so`` and there is no eager or CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

import torch

from ._lib import KDA_BF16, KDA_F32, KDAError, check, lib

#: Chunk width of the tensor-core path (the reference's persistent kernel uses 32
#: because of the GB10 SMEM budget, ``kda_cc_fused_persist.py:228``; B200 runs 64).
CHUNK = 64
#: Decay-factor tile width of the reference (``net/kda.py:561``); kept for
#: signature compatibility, the kernels' tiling is fixed by their design.
TILE = 16

#: Accepted values of ``AXIOM_KDA_CC_IMPL`` (the reference's three plus ``b200``).
KDA_CC_IMPLS = ("jax", "mosaic", "persistent", "b200")

_DT = {torch.float32: KDA_F32, torch.bfloat16: KDA_BF16}


def kda_cc_impl() -> str:
    """Read ``AXIOM_KDA_CC_IMPL`` on every call; unknown values raise (fail-closed)."""
    value = (os.environ.get("AXIOM_KDA_CC_IMPL") or "b200").strip().lower()
    if value not in KDA_CC_IMPLS:
        raise ValueError(f"AXIOM_KDA_CC_IMPL={value!r}: expected one of {KDA_CC_IMPLS}")
    return value


def device_available() -> bool:
    """True when a CUDA device is present (the library itself checks sm_100)."""
    return torch.cuda.is_available()


def _require_device(what: str) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(
            f"{what}: the B200 KDA kernels run only on a CUDA device; there is no CPU "
            "fallback -- select another implementation explicitly.")


def _dt(x: torch.Tensor, name: str) -> int:
    try:
        return _DT[x.dtype]
    except KeyError:
        raise TypeError(f"{name}: dtype {x.dtype} is not supported (float32 or bfloat16)") from None


def _ptr(x):
    return None if x is None else x.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


STATUS_BITS = {"fwd": 1, "bwd": 2, "decode_fused": 4, "selftest": 8}  # KDA_STATUS_* (kda_b200.h)


def device_status(clear=False) -> dict:
    """Which kernel families had a bounded wait give up since the last clear
    (``kda_device_status``; synchronises the current stream).  A kernel that
    gives up skips its remaining work, so its outputs are not valid."""
    _require_device("device_status")
    flags = ctypes.c_int(0)
    check("kda_device_status", lib().kda_device_status(ctypes.byref(flags), int(bool(clear)), _stream()))
    return {name: bool(flags.value & bit) for name, bit in STATUS_BITS.items()}


def check_device(clear=True) -> None:
    """Raise ``KDAError`` (``KDA_ERR_TIMEOUT``) if any kernel's wait gave up."""
    st = device_status(clear=clear)
    bad = [name for name, hit in st.items() if hit]
    if bad:
        raise KDAError("check_device", -9, "bounded wait gave up in: " + ", ".join(bad))


def selftest_wait_timeout(polls=4096) -> None:
    """Run the bounded-wait failure path once (``kda_selftest_wait_timeout``):
    a wait that nothing completes gives up and sets the ``selftest`` bit."""
    _require_device("selftest_wait_timeout")
    check("kda_selftest_wait_timeout", lib().kda_selftest_wait_timeout(int(polls), _stream()))


def _check_tensor(x: torch.Tensor, name: str, shape, dtype=None):
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if tuple(x.shape) != tuple(shape):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(x.shape)}")
    if dtype is not None and x.dtype != dtype:
        raise TypeError(f"{name}: expected dtype {dtype}, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ---------------------------------------------------------------------------
# raw launches (BASELINE form)
# ---------------------------------------------------------------------------


def kda_fwd(q, k, v, g, beta, S0=None, *, chunk=CHUNK, o_dtype=None, need_ckpt=False,
            ckpt_dtype=None):
    """Chunked forward; returns ``(o, S_T, ckpt)`` (``ckpt`` is None unless requested).

    ``ckpt`` (1-D, ``kda_ckpt_bytes`` bytes) is opaque: it starts with the
    chunk-boundary states (``ckpt_states`` gives them as ``[B, H, n, dk, dv]``)
    and, on the tensor-core path, per-chunk factors for the backward follow.

    ``q, k, g``: ``[B, T, H, dk]``; ``v``: ``[B, T, H, dv]``; ``beta``: ``[B, T, H]``,
    all of one dtype (bf16 or fp32); ``S0``: ``[B, H, dk, dv]`` fp32 or None.
    """
    _require_device("kda_fwd")
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    dt = q.dtype
    for x, n, s in ((q, "q", (B, T, H, dk)), (k, "k", (B, T, H, dk)), (v, "v", (B, T, H, dv)),
                    (g, "g", (B, T, H, dk)), (beta, "beta", (B, T, H))):
        _check_tensor(x, n, s, dt)
    if S0 is not None:
        _check_tensor(S0, "S0", (B, H, dk, dv), torch.float32)
    o_dtype = dt if o_dtype is None else o_dtype
    ckpt_dtype = (torch.float32 if dt == torch.float32 else torch.bfloat16) if ckpt_dtype is None else ckpt_dtype
    o = torch.empty((B, T, H, dv), dtype=o_dtype, device=q.device)
    s_out = torch.empty((B, H, dk, dv), dtype=torch.float32, device=q.device)
    ckpt = None
    if need_ckpt:
        nbytes = lib().kda_ckpt_bytes(B, T, H, dk, dv, chunk, _dt(q, "q"), _DT[ckpt_dtype])
        esz = 4 if ckpt_dtype == torch.float32 else 2
        ckpt = torch.empty(-(-nbytes // esz), dtype=ckpt_dtype, device=q.device)
    rc = lib().kda_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(S0), _ptr(o),
                       _ptr(s_out), _ptr(ckpt), B, T, H, dk, dv, int(chunk), _dt(q, "q"),
                       _DT[o_dtype], _DT[ckpt_dtype], _stream())
    check("kda_fwd", rc)
    return o, s_out, ckpt


def ckpt_states(ckpt, B, T, H, dk, dv, *, chunk=CHUNK, in_dtype=torch.bfloat16):
    """The chunk-boundary states held in a forward checkpoint, ``[B, H, n, dk, dv]``
    (entry ``c`` is the state entering chunk ``c``), in the checkpoint's dtype.

    A bf16 checkpoint written by the tensor-core forward stores each state as
    its 8 x 8 core-matrix operand image (core ``(i, j)`` holds rows ``8i..8i+7``
    and columns ``8j..8j+7`` row-major); this undoes that arrangement.
    """
    n = -(-T // chunk)
    flat = ckpt[: B * H * n * dk * dv]
    tc = (in_dtype == torch.bfloat16 and dk == 128 and dv == 128 and chunk == 64
          and ckpt.dtype == torch.bfloat16)
    if not tc:
        return flat.reshape(B, H, n, dk, dv)
    cores = flat.reshape(B, H, n, dk // 8, dv // 8, 8, 8)
    return cores.permute(0, 1, 2, 3, 5, 4, 6).reshape(B, H, n, dk, dv)


def kda_bwd(q, k, v, g, beta, ckpt, do, dST=None, *, chunk=CHUNK, need_ds0=True):
    """Fused backward from the forward's checkpoint; returns ``(dq, dk, dv, dg, dbeta, dS0)``."""
    _require_device("kda_bwd")
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    dt = q.dtype
    for x, n, s in ((q, "q", (B, T, H, dk)), (k, "k", (B, T, H, dk)), (v, "v", (B, T, H, dv)),
                    (g, "g", (B, T, H, dk)), (beta, "beta", (B, T, H))):
        _check_tensor(x, n, s, dt)
    _check_tensor(do, "do", (B, T, H, dv))
    if dST is not None:
        _check_tensor(dST, "dST", (B, H, dk, dv), torch.float32)
    if ckpt is None or ckpt.dtype not in _DT or not ckpt.is_contiguous():
        raise ValueError("kda_bwd: ckpt must be the forward's checkpoint")
    nbytes = lib().kda_ckpt_bytes(B, T, H, dk, dv, chunk, _dt(q, "q"), _DT[ckpt.dtype])
    if ckpt.numel() * ckpt.element_size() < nbytes:
        raise ValueError("kda_bwd: ckpt is smaller than the forward's checkpoint for these shapes")
    dq = torch.empty_like(q)
    dk_ = torch.empty_like(k)
    dv_ = torch.empty_like(v)
    dg = torch.empty_like(g)
    dbeta = torch.empty_like(beta)
    ds0 = torch.empty((B, H, dk, dv), dtype=torch.float32, device=q.device) if need_ds0 else None
    wbytes = lib().kda_bwd_workspace_bytes(B, T, H, dk, dv, int(chunk), _dt(q, "q"))
    work = torch.empty(max(wbytes, 1), dtype=torch.uint8, device=q.device)
    rc = lib().kda_bwd(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(ckpt), _ptr(do),
                       _ptr(dST), _ptr(dq), _ptr(dk_), _ptr(dv_), _ptr(dg), _ptr(dbeta),
                       _ptr(ds0), _ptr(work), wbytes, B, T, H, dk, dv, int(chunk),
                       _dt(q, "q"), _dt(do, "do"), _dt(ckpt, "ckpt"), _stream())
    check("kda_bwd", rc)
    return dq, dk_, dv_, dg, dbeta, ds0


# ---------------------------------------------------------------------------
# packed (variable-length) sequences
# ---------------------------------------------------------------------------


def packing(cu_seqlens, chunk=CHUNK):
    """Chunk-aligned packing of the sequences ``cu_seqlens`` delimits (host
    integers, or a tensor read back once): ``(chunk_offsets, out_rows, T_pad)``
    with ``chunk_offsets[s]`` the first chunk of sequence ``s`` (last entry: the
    total), ``out_rows = chunk * chunk_offsets`` (the rows
    :func:`axiom_b200.mixer.prologue_fwd` writes each sequence from) and
    ``T_pad`` the packed length.  Each sequence is padded to its next chunk
    boundary (at most ``chunk - 1`` rows)."""
    cu = [int(x) for x in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
    if not cu or cu[0] != 0 or any(b < a for a, b in zip(cu[:-1], cu[1:])):
        raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
    offs = [0]
    for a, b in zip(cu[:-1], cu[1:]):
        offs.append(offs[-1] + -(-(b - a) // chunk))
    return offs, [chunk * o for o in offs], chunk * offs[-1]


def _offsets_tensor(chunk_offsets, device):
    if isinstance(chunk_offsets, torch.Tensor):
        return chunk_offsets.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(chunk_offsets), dtype=torch.int32, device=device)


def kda_fwd_varlen(q, k, v, g, beta, chunk_offsets, S0=None, *, chunk=CHUNK, o_dtype=None,
                   need_ckpt=False, ckpt_dtype=None):
    """Chunked forward over packed sequences; returns ``(o, S_T, ckpt)``.

    ``q, k, g``: ``[1, T, H, dk]``, ``v``: ``[1, T, H, dv]``, ``beta``: ``[1, T, H]``
    in the chunk-aligned packed layout (see :func:`packing`); ``chunk_offsets``:
    ``[n + 1]`` (device int32 tensor or host integers); ``S0`` and ``S_T``:
    ``[n, H, dk, dv]`` fp32, one state per sequence.
    """
    _require_device("kda_fwd_varlen")
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    dt = q.dtype
    if B != 1:
        raise ValueError("kda_fwd_varlen: packed sequences share one batch row (B = 1)")
    for x, n, s in ((q, "q", (1, T, H, dk)), (k, "k", (1, T, H, dk)), (v, "v", (1, T, H, dv)),
                    (g, "g", (1, T, H, dk)), (beta, "beta", (1, T, H))):
        _check_tensor(x, n, s, dt)
    cs = _offsets_tensor(chunk_offsets, q.device)
    n_seqs = cs.numel() - 1
    if S0 is not None:
        _check_tensor(S0, "S0", (n_seqs, H, dk, dv), torch.float32)
    o_dtype = dt if o_dtype is None else o_dtype
    ckpt_dtype = (torch.float32 if dt == torch.float32 else torch.bfloat16) if ckpt_dtype is None else ckpt_dtype
    o = torch.empty((1, T, H, dv), dtype=o_dtype, device=q.device)
    s_out = torch.empty((n_seqs, H, dk, dv), dtype=torch.float32, device=q.device)
    ckpt = None
    if need_ckpt:
        nbytes = lib().kda_ckpt_bytes(1, T, H, dk, dv, chunk, _dt(q, "q"), _DT[ckpt_dtype])
        esz = 4 if ckpt_dtype == torch.float32 else 2
        ckpt = torch.empty(max(-(-nbytes // esz), 1), dtype=ckpt_dtype, device=q.device)
    rc = lib().kda_fwd_varlen(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(S0), _ptr(o),
                              _ptr(s_out), _ptr(ckpt), _ptr(cs), n_seqs, T, H, dk, dv, int(chunk),
                              _dt(q, "q"), _DT[o_dtype], _DT[ckpt_dtype], _stream())
    check("kda_fwd_varlen", rc)
    return o, s_out, ckpt


def kda_bwd_varlen(q, k, v, g, beta, ckpt, do, chunk_offsets, dST=None, *, chunk=CHUNK, need_ds0=True):
    """Fused backward over packed sequences; returns ``(dq, dk, dv, dg, dbeta, dS0)``
    (``dS0``: ``[n, H, dk, dv]``).  ``do``'s pad rows must be zero."""
    _require_device("kda_bwd_varlen")
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    dt = q.dtype
    for x, n, s in ((q, "q", (1, T, H, dk)), (k, "k", (1, T, H, dk)), (v, "v", (1, T, H, dv)),
                    (g, "g", (1, T, H, dk)), (beta, "beta", (1, T, H))):
        _check_tensor(x, n, s, dt)
    _check_tensor(do, "do", (1, T, H, dv))
    cs = _offsets_tensor(chunk_offsets, q.device)
    n_seqs = cs.numel() - 1
    if dST is not None:
        _check_tensor(dST, "dST", (n_seqs, H, dk, dv), torch.float32)
    if ckpt is None or ckpt.dtype not in _DT or not ckpt.is_contiguous():
        raise ValueError("kda_bwd_varlen: ckpt must be the forward's checkpoint")
    dq, dk_, dv_, dg, dbeta = (torch.empty_like(x) for x in (q, k, v, g, beta))
    ds0 = torch.empty((n_seqs, H, dk, dv), dtype=torch.float32, device=q.device) if need_ds0 else None
    wbytes = lib().kda_bwd_varlen_workspace_bytes(n_seqs, T, H, dk, dv, int(chunk), _dt(q, "q"))
    work = torch.empty(max(wbytes, 1), dtype=torch.uint8, device=q.device)
    rc = lib().kda_bwd_varlen(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(ckpt), _ptr(do),
                              _ptr(dST), _ptr(dq), _ptr(dk_), _ptr(dv_), _ptr(dg), _ptr(dbeta),
                              _ptr(ds0), _ptr(work), wbytes, _ptr(cs), n_seqs, T, H, dk, dv, int(chunk),
                              _dt(q, "q"), _dt(do, "do"), _dt(ckpt, "ckpt"), _stream())
    check("kda_bwd_varlen", rc)
    return dq, dk_, dv_, dg, dbeta, ds0


def decode_step(S, q, k, v, g, beta, *, o_dtype=None):
    """One recurrent token for ``N`` states; updates ``S`` in place, returns ``o``.

    ``S``: ``[..., dk, dv]`` fp32; ``q, k, g``: ``[..., dk]``; ``v``: ``[..., dv]``;
    ``beta``: ``[...]`` (leading dims flattened to N).
    """
    _require_device("decode_step")
    dk, dv = S.shape[-2], S.shape[-1]
    lead = tuple(S.shape[:-2])
    N = 1
    for s_ in lead:
        N *= s_
    dt = q.dtype
    _check_tensor(S, "S", lead + (dk, dv), torch.float32)
    for x, n, s in ((q, "q", lead + (dk,)), (k, "k", lead + (dk,)), (v, "v", lead + (dv,)),
                    (g, "g", lead + (dk,)), (beta, "beta", lead)):
        _check_tensor(x, n, s, dt)
    o_dtype = dt if o_dtype is None else o_dtype
    o = torch.empty(lead + (dv,), dtype=o_dtype, device=S.device)
    rc = lib().kda_decode(_ptr(S), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(o),
                          N, dk, dv, _dt(q, "q"), _DT[o_dtype], _stream())
    check("kda_decode", rc)
    return o


# ---------------------------------------------------------------------------
# differentiable operator (BASELINE form) -- the custom_vjp wiring
# ---------------------------------------------------------------------------


class _ChunkKDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, S0, chunk):
        o, s_t, ckpt = kda_fwd(q, k, v, g, beta, S0, chunk=chunk, need_ckpt=True)
        ctx.save_for_backward(q, k, v, g, beta, ckpt)
        ctx.chunk = chunk
        ctx.has_s0 = S0 is not None
        return o, s_t

    @staticmethod
    def backward(ctx, do, dst):
        q, k, v, g, beta, ckpt = ctx.saved_tensors
        if do is None:
            do = torch.zeros(q.shape[:-1] + (v.shape[-1],), dtype=q.dtype, device=q.device)
        do = do.to(q.dtype).contiguous()
        dst = None if dst is None else dst.to(torch.float32).contiguous()
        dq, dk, dv, dg, dbeta, ds0 = kda_bwd(q, k, v, g, beta, ckpt, do, dst, chunk=ctx.chunk,
                                             need_ds0=ctx.has_s0)
        return dq, dk, dv, dg, dbeta, (ds0 if ctx.has_s0 else None), None


def chunk_kda(q, k, v, g, beta, S0=None, chunk=CHUNK):
    """Differentiable chunked KDA core: ``(o, S_T)``; gradients via the fused backward."""
    return _ChunkKDA.apply(q, k, v, g, beta, S0, int(chunk))


class _ChunkKDAVarlen(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, cs, S0, chunk):
        o, s_t, ckpt = kda_fwd_varlen(q, k, v, g, beta, cs, S0, chunk=chunk, need_ckpt=True)
        ctx.save_for_backward(q, k, v, g, beta, ckpt, cs)
        ctx.chunk = chunk
        ctx.has_s0 = S0 is not None
        return o, s_t

    @staticmethod
    def backward(ctx, do, dst):
        q, k, v, g, beta, ckpt, cs = ctx.saved_tensors
        if do is None:
            do = torch.zeros(q.shape[:-1] + (v.shape[-1],), dtype=q.dtype, device=q.device)
        do = do.to(q.dtype).contiguous()
        dst = None if dst is None else dst.to(torch.float32).contiguous()
        dq, dk, dv, dg, dbeta, ds0 = kda_bwd_varlen(q, k, v, g, beta, ckpt, do, cs, dst, chunk=ctx.chunk,
                                                    need_ds0=ctx.has_s0)
        return dq, dk, dv, dg, dbeta, None, (ds0 if ctx.has_s0 else None), None


def chunk_kda_varlen(q, k, v, g, beta, chunk_offsets, S0=None, chunk=CHUNK):
    """Differentiable chunked KDA core over packed sequences (``[1, T, H, *]`` in
    the chunk-aligned layout of :func:`packing`): ``(o, S_T)``, one state per
    sequence.  The pad rows of ``o``'s cotangent must be zero (the output gate's
    backward writes them so)."""
    cs = _offsets_tensor(chunk_offsets, q.device)
    return _ChunkKDAVarlen.apply(q, k, v, g, beta, cs, S0, int(chunk))


# ---------------------------------------------------------------------------
# the reference's operand form: (q, k, v, alpha, beta32, S) over (T, H*D)
# ---------------------------------------------------------------------------


def _operand_to_native(q, k, v, alpha, beta32, S):
    T = q.shape[0]
    H, dk, dv = S.shape
    if q.shape != (T, H * dk) or k.shape != (T, H * dk) or v.shape != (T, H * dv):
        raise ValueError("q/k must be (T, H*dk) and v (T, H*dv) for S of shape (H, dk, dv)")
    if alpha.shape != (T, H * dk) or beta32.shape != (T, H * 32):
        raise ValueError("alpha must be (T, H*dk) and beta32 (T, H*32)")
    dt = q.dtype
    g = torch.log(alpha.to(torch.float32)).to(dt).reshape(1, T, H, dk).contiguous()
    beta = beta32.to(torch.float32).reshape(T, H, 32).mean(-1).to(dt).reshape(1, T, H).contiguous()
    return (q.reshape(1, T, H, dk).contiguous(), k.reshape(1, T, H, dk).contiguous(),
            v.reshape(1, T, H, dv).contiguous(), g, beta, S.to(torch.float32).reshape(1, H, dk, dv).contiguous())


def _check_operand(q, v, T, chunk):
    dt = q.dtype
    if v.dtype != dt or dt not in (torch.bfloat16, torch.float32):
        raise ValueError(f"kernel consumes bf16 or fp32 q/k/v of one dtype; got q.dtype={dt}, v.dtype={v.dtype}")
    if T % int(chunk):
        raise ValueError(f"T={T} must be a multiple of the chunk width C={int(chunk)}")


def kernel(q, k, v, alpha, beta32, S, *, tile=TILE, chunk=CHUNK):
    """``(q, k, v, alpha, beta32, S) -> (o, S_new)``: one launch over the whole sequence.

    Same contract as ``kda_cc_fused_persist.kernel`` (:718-759): ``q``/``k``
    ``(T, H*dk)``, ``v`` ``(T, H*dv)``, ``alpha`` ``(T, H*dk)`` fp32 decay,
    ``beta32`` ``(T, H*32)`` fp32, ``S`` ``(H, dk, dv)`` fp32; ``T`` must be a
    multiple of ``chunk``.  Returns ``o`` ``(T, H*dv)`` fp32 and the final state.
    """
    T = q.shape[0]
    _check_operand(q, v, T, chunk)
    qn, kn, vn, g, beta, S0 = _operand_to_native(q, k, v, alpha, beta32, S)
    o, s_t, _ = kda_fwd(qn, kn, vn, g, beta, S0, chunk=chunk, o_dtype=torch.float32)
    return o.reshape(T, -1), s_t[0]


def kernel_bwd(q, k, v, alpha, beta32, S, do, dS, *, tile=TILE, chunk=CHUNK, debug_outputs=False):
    """Backward of :func:`kernel`: ``(dq, dk, dv, dalpha, dbeta32, dS_in)`` in primal dtypes.

    Same contract as ``kda_cc_fused_persist.kernel_bwd`` (:1707-1763); the
    forward is re-run once to produce the chunk-boundary states.
    """
    T = q.shape[0]
    _check_operand(q, v, T, chunk)
    H, dk, dv = S.shape
    qn, kn, vn, g, beta, S0 = _operand_to_native(q, k, v, alpha, beta32, S)
    _, _, ckpt = kda_fwd(qn, kn, vn, g, beta, S0, chunk=chunk, need_ckpt=True)
    don = do.to(q.dtype).reshape(1, T, H, dv).contiguous()
    dq, dk_, dv_, dg, dbeta, ds0 = kda_bwd(qn, kn, vn, g, beta, ckpt, don,
                                           dS.to(torch.float32).reshape(1, H, dk, dv).contiguous(),
                                           chunk=chunk)
    dalpha = (dg.to(torch.float32) / alpha.to(torch.float32).reshape(1, T, H, dk)).reshape(T, H * dk)
    dbeta32 = (dbeta.to(torch.float32)[..., None] / 32.0).expand(1, T, H, 32).reshape(T, H * 32)
    return (dq.reshape(T, -1).to(q.dtype), dk_.reshape(T, -1).to(k.dtype),
            dv_.reshape(T, -1).to(v.dtype), dalpha.to(alpha.dtype), dbeta32.to(beta32.dtype),
            ds0[0])


class _CCScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, alpha, beta32, S, tile, chunk):
        ctx.save_for_backward(q, k, v, alpha, beta32, S)
        ctx.tile, ctx.chunk = tile, chunk
        return kernel(q, k, v, alpha, beta32, S, tile=tile, chunk=chunk)

    @staticmethod
    def backward(ctx, do, dS):
        q, k, v, alpha, beta32, S = ctx.saved_tensors
        if do is None:
            do = torch.zeros(q.shape[0], v.shape[1], dtype=torch.float32, device=q.device)
        if dS is None:
            dS = torch.zeros_like(S, dtype=torch.float32)
        grads = kernel_bwd(q, k, v, alpha, beta32, S, do, dS, tile=ctx.tile, chunk=ctx.chunk)
        return (*grads, None, None)


def cc_scan(q, k, v, alpha, beta32, S, tile=TILE, chunk=CHUNK):
    """Differentiable whole-sequence entry point (``kda_cc_fused_persist.cc_scan`` :920-932)."""
    return _CCScan.apply(q, k, v, alpha, beta32, S, int(tile), int(chunk))
