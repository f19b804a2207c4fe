"""Host-side interface of the per-token work around the KDA core.

Mirrors the reference's layer functions (AXIOM, ``net/kda.py``,
``net/shortconv.py``, ``net/norm.py``) over the C ABI of
``include/kda_mixer.h``:

* :func:`prologue_fwd` / :func:`prologue_bwd` / :func:`kda_prologue` --
  ShortConv -> Swish -> L2 norm of q, k, ShortConv -> Swish of v, the sigmoid
  write gate and the decay gate (``_postprocess`` ``net/kda.py:194-203``,
  ``short_conv`` ``net/shortconv.py:14-30``, ``_project``'s activations
  ``net/kda.py:169-180``), differentiable;
* :func:`gated_rmsnorm` -- ``sigmoid(gate) * headwise_rms_norm(o)``, the output
  gate before ``W_o`` (``_output_gate`` ``net/kda.py:206-214``), differentiable;
* :func:`decode_fused` -- one streaming token (``recurrent_step``
  ``net/kda.py:277-295`` without the projection GEMMs).

Every computation runs in ``libkda_b200.so``; PyTorch provides memory, streams
and autograd plumbing, and there is no eager or CPU fallback.
"""

from __future__ import annotations

import torch

from ._lib import check, lib
from .kda import _check_tensor, _dt, _ptr, _require_device, _stream

#: ``l2_norm``'s eps (``net/norm.py:51``); ``headwise_rms_norm``'s (``net/norm.py:70``)
L2_EPS = 1e-12
RMS_EPS = 1e-6
#: the reference's lower bound of the log-decay (``net/config.py:131``)
G_MIN = -5.0
#: decay-gate forms: the reference's ``g_min * sigmoid(exp(A) * z)`` and
#: ``-exp(A_log) * softplus(z + b)``
GATE_KINDS = {"sigmoid_min": 0, "softplus": 1}


def _gate_kind(kind) -> int:
    if kind not in GATE_KINDS:
        raise ValueError(f"gate_kind={kind!r}: expected one of {tuple(GATE_KINDS)}")
    return GATE_KINDS[kind]


def _cu(cu_seqlens, B, device):
    if cu_seqlens is None:
        return None, 0
    if B != 1:
        raise ValueError("cu_seqlens packs sequences along T: B must be 1")
    cu = cu_seqlens.to(device=device, dtype=torch.int32).contiguous()
    return cu, cu.numel() - 1


def _rows(out_rows, cu, n_seqs, T, device):
    """``(device int32 rows or None, output length)``."""
    if out_rows is None:
        return None, T
    if cu is None:
        raise ValueError("out_rows places packed sequences: cu_seqlens is required")
    host = [int(x) for x in (out_rows.tolist() if isinstance(out_rows, torch.Tensor) else out_rows)]
    if len(host) != n_seqs + 1:
        raise ValueError("out_rows needs one entry per sequence plus the total")
    return torch.tensor(host, dtype=torch.int32, device=device), host[-1]


def _state_width(H, dk, dv):
    return H * (2 * dk + dv)


def prologue_fwd(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, *, H, b_gate=None, g_min=G_MIN,
                 gate_kind="sigmoid_min", conv_state=None, return_state=False, cu_seqlens=None,
                 out_rows=None, out_dtype=None):
    """The KDA core's inputs from the layer's projections.

    ``qp, kp, z``: ``[B, T, H*dk]``; ``vp``: ``[B, T, H*dv]``; ``beta_logit``:
    ``[B, T, H]`` (one dtype, bf16 or fp32); ``conv_q, conv_k``: ``[K, H*dk]``,
    ``conv_v``: ``[K, H*dv]``, ``b_gate``: ``[H*dk]``, ``A``: ``[H]`` (fp32).
    ``conv_state``: ``[B, K-1, H*(2dk+dv)]`` fp32 (the q, k, v buffers of
    ``KDAState``) or None.  ``cu_seqlens`` (``[n + 1]``) packs sequences along T
    (B = 1; each restarts the convolution); ``out_rows`` (``[n + 1]``, e.g.
    :func:`axiom_b200.kda.packing`'s) then places sequence ``s`` from output row
    ``out_rows[s]`` with zero rows up to the next.  Returns ``q, k, v, g, beta``
    in the core's layout (``[B, T', H, d]``, ``[B, T', H]``, ``T' = T`` or
    ``out_rows[-1]``), plus the next conv state when ``return_state``.
    """
    _require_device("prologue_fwd")
    B, T, HK = qp.shape
    dk, dv, K = HK // H, vp.shape[-1] // H, conv_q.shape[0]
    dt = qp.dtype
    for x, n, s in ((qp, "qp", (B, T, H * dk)), (kp, "kp", (B, T, H * dk)), (vp, "vp", (B, T, H * dv)),
                    (z, "z", (B, T, H * dk)), (beta_logit, "beta_logit", (B, T, H))):
        _check_tensor(x, n, s, dt)
    for x, n, s in ((conv_q, "conv_q", (K, H * dk)), (conv_k, "conv_k", (K, H * dk)),
                    (conv_v, "conv_v", (K, H * dv)), (A, "A", (H,))):
        _check_tensor(x, n, s, torch.float32)
    if b_gate is not None:
        _check_tensor(b_gate, "b_gate", (H * dk,), torch.float32)
    if conv_state is not None:
        _check_tensor(conv_state, "conv_state", (B, K - 1, _state_width(H, dk, dv)), torch.float32)
    out_dtype = dt if out_dtype is None else out_dtype
    dev = qp.device
    cu, n_seqs = _cu(cu_seqlens, B, dev)
    rows, To = _rows(out_rows, cu, n_seqs, T, dev)
    q = torch.empty((B, To, H, dk), dtype=out_dtype, device=dev)
    k = torch.empty_like(q)
    g = torch.empty_like(q)
    v = torch.empty((B, To, H, dv), dtype=out_dtype, device=dev)
    beta = torch.empty((B, To, H), dtype=out_dtype, device=dev)
    st_out = None
    if return_state and K > 1:
        st_out = torch.empty((B, K - 1, _state_width(H, dk, dv)), dtype=torch.float32, device=dev)
    rc = lib().kda_prologue_fwd(
        _ptr(qp), _ptr(kp), _ptr(vp), _ptr(z), _ptr(beta_logit), _ptr(conv_q), _ptr(conv_k), _ptr(conv_v),
        _ptr(b_gate), _ptr(A), float(g_min), _gate_kind(gate_kind), _ptr(conv_state), _ptr(st_out), _ptr(cu),
        n_seqs, _ptr(rows), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), B, T, H, dk, dv, K, _dt(qp, "qp"),
        _dt(q, "out"), _stream())
    check("kda_prologue_fwd", rc)
    if return_state:
        return q, k, v, g, beta, st_out
    return q, k, v, g, beta


def prologue_bwd(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, dq, dk, dv, dg, dbeta, *, H,
                 b_gate=None, g_min=G_MIN, gate_kind="sigmoid_min", conv_state=None, cu_seqlens=None,
                 out_rows=None):
    """Cotangents of :func:`prologue_fwd`'s inputs; returns a dict with
    ``dqp, dkp, dvp, dz, dbeta_logit`` (input dtype), ``dconv_q, dconv_k,
    dconv_v, db_gate, dA`` (fp32) and ``dconv_state`` (fp32, or None)."""
    _require_device("prologue_bwd")
    B, T, HK = qp.shape
    dk_, dv_, K = HK // H, vp.shape[-1] // H, conv_q.shape[0]
    odt = dq.dtype
    dev = qp.device
    cu, n_seqs = _cu(cu_seqlens, B, dev)
    rows, To = _rows(out_rows, cu, n_seqs, T, dev)
    for x, n, s in ((dq, "dq", (B, To, H, dk_)), (dk, "dk", (B, To, H, dk_)), (dv, "dv", (B, To, H, dv_)),
                    (dg, "dg", (B, To, H, dk_)), (dbeta, "dbeta", (B, To, H))):
        _check_tensor(x, n, s, odt)
    out = {
        "dqp": torch.empty_like(qp), "dkp": torch.empty_like(kp), "dvp": torch.empty_like(vp),
        "dz": torch.empty_like(z), "dbeta_logit": torch.empty_like(beta_logit),
        "dconv_q": torch.empty_like(conv_q), "dconv_k": torch.empty_like(conv_k),
        "dconv_v": torch.empty_like(conv_v), "db_gate": torch.empty((H * dk_,), dtype=torch.float32, device=dev),
        "dA": torch.empty_like(A), "dconv_state": None,
    }
    if conv_state is not None and K > 1:
        out["dconv_state"] = torch.empty_like(conv_state)
    ws_bytes = lib().kda_prologue_bwd_workspace_bytes(B, T, H, dk_, dv_, K)
    ws = torch.empty((max(ws_bytes, 16),), dtype=torch.uint8, device=dev)
    rc = lib().kda_prologue_bwd(
        _ptr(qp), _ptr(kp), _ptr(vp), _ptr(z), _ptr(beta_logit), _ptr(conv_q), _ptr(conv_k), _ptr(conv_v),
        _ptr(b_gate), _ptr(A), float(g_min), _gate_kind(gate_kind), _ptr(conv_state), _ptr(cu), n_seqs, _ptr(rows),
        _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(dbeta), _ptr(out["dqp"]), _ptr(out["dkp"]),
        _ptr(out["dvp"]), _ptr(out["dz"]), _ptr(out["dbeta_logit"]), _ptr(out["dconv_q"]),
        _ptr(out["dconv_k"]), _ptr(out["dconv_v"]), _ptr(out["db_gate"]), _ptr(out["dA"]),
        _ptr(out["dconv_state"]), _ptr(ws), ws.numel(), B, T, H, dk_, dv_, K, _dt(qp, "qp"), _dt(dq, "dq"),
        _stream())
    check("kda_prologue_bwd", rc)
    return out


class _Prologue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, b_gate, H, g_min, gate_kind,
                cu_seqlens, out_rows):
        q, k, v, g, beta = prologue_fwd(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, H=H,
                                        b_gate=b_gate, g_min=g_min, gate_kind=gate_kind, cu_seqlens=cu_seqlens,
                                        out_rows=out_rows)
        ctx.save_for_backward(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, b_gate, cu_seqlens)
        ctx.cfg = (H, g_min, gate_kind, out_rows, q.shape[1])
        return q, k, v, g, beta

    @staticmethod
    def backward(ctx, dq, dk, dv, dg, dbeta):
        qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, b_gate, cu = ctx.saved_tensors
        H, g_min, gate_kind, out_rows, To = ctx.cfg
        grads = [dq, dk, dv, dg, dbeta]
        ref = (dq if dq is not None else dk)
        odt = qp.dtype if ref is None else ref.dtype
        B = qp.shape[0]
        shapes = ((B, To, H, qp.shape[2] // H),) * 2 + (
            (B, To, H, vp.shape[2] // H), (B, To, H, z.shape[2] // H), (B, To, H))
        grads = [torch.zeros(s, dtype=odt, device=qp.device) if x is None else x.to(odt).contiguous()
                 for x, s in zip(grads, shapes)]
        r = prologue_bwd(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, *grads, H=H, b_gate=b_gate,
                         g_min=g_min, gate_kind=gate_kind, cu_seqlens=cu, out_rows=out_rows)
        return (r["dqp"], r["dkp"], r["dvp"], r["dz"], r["dbeta_logit"], r["dconv_q"], r["dconv_k"],
                r["dconv_v"], r["dA"], None if b_gate is None else r["db_gate"], None, None, None, None, None)


def kda_prologue(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, *, H, b_gate=None, g_min=G_MIN,
                 gate_kind="sigmoid_min", cu_seqlens=None, out_rows=None):
    """Differentiable :func:`prologue_fwd` (no conv state): ``q, k, v, g, beta``."""
    if cu_seqlens is not None:
        cu_seqlens = cu_seqlens.to(device=qp.device, dtype=torch.int32)
    return _Prologue.apply(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, b_gate, H, g_min, gate_kind,
                           cu_seqlens, out_rows)


def _map(cu_seqlens, out_rows, device):
    if out_rows is None:
        return None, None, 0
    if cu_seqlens is None:
        raise ValueError("out_rows places packed sequences: cu_seqlens is required")
    cu = cu_seqlens.to(device=device, dtype=torch.int32).contiguous()
    rows, _ = _rows(out_rows, cu, cu.numel() - 1, 0, device)
    return cu, rows, cu.numel() - 1


def gated_rmsnorm_fwd(o, gate, *, eps=RMS_EPS, out_dtype=None, cu_seqlens=None, out_rows=None):
    """``sigmoid(gate) * o / sqrt(mean(o^2) + eps)`` per head: ``gate`` logits
    ``[..., N, H*dv]``, ``o [..., N, H, dv]`` -- or, with ``cu_seqlens`` and
    ``out_rows``, ``o`` in the chunk-aligned packed layout (``[1, T', H, dv]``)
    and ``gate`` packed (``[1, N, H*dv]``); returns the gate's shape."""
    _require_device("gated_rmsnorm")
    H, dv = o.shape[-2], o.shape[-1]
    N = gate.numel() // (H * dv)
    _check_tensor(o, "o", o.shape)
    if out_rows is None:
        _check_tensor(gate, "gate", tuple(o.shape[:-2]) + (H * dv,))
    cu, rows, n = _map(cu_seqlens, out_rows, o.device)
    y = torch.empty(gate.shape, dtype=out_dtype or gate.dtype, device=o.device)
    rc = lib().kda_gated_rmsnorm_fwd(_ptr(o), _ptr(gate), _ptr(y), _ptr(cu), _ptr(rows), n, N, H, dv, float(eps),
                                     _dt(o, "o"), _dt(gate, "gate"), _dt(y, "y"), _stream())
    check("kda_gated_rmsnorm_fwd", rc)
    return y


def gated_rmsnorm_bwd(o, gate, dy, *, eps=RMS_EPS, cu_seqlens=None, out_rows=None):
    """``(do, dgate)`` of :func:`gated_rmsnorm_fwd` (dtypes of ``o`` and ``gate``;
    ``do`` in ``o``'s rows, zero on the pad rows of a packed layout)."""
    _require_device("gated_rmsnorm_bwd")
    H, dv = o.shape[-2], o.shape[-1]
    N = gate.numel() // (H * dv)
    _check_tensor(dy, "dy", tuple(gate.shape))
    cu, rows, n = _map(cu_seqlens, out_rows, o.device)
    do = torch.empty_like(o)
    dgate = torch.empty_like(gate)
    rc = lib().kda_gated_rmsnorm_bwd(_ptr(o), _ptr(gate), _ptr(dy), _ptr(do), _ptr(dgate), _ptr(cu), _ptr(rows), n,
                                     N, H, dv, float(eps), _dt(o, "o"), _dt(gate, "gate"), _dt(dy, "dy"), _stream())
    check("kda_gated_rmsnorm_bwd", rc)
    return do, dgate


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, gate, eps, cu_seqlens, out_rows):
        ctx.save_for_backward(o, gate, cu_seqlens)
        ctx.eps, ctx.out_rows = eps, out_rows
        return gated_rmsnorm_fwd(o, gate, eps=eps, cu_seqlens=cu_seqlens, out_rows=out_rows)

    @staticmethod
    def backward(ctx, dy):
        o, gate, cu = ctx.saved_tensors
        do, dgate = gated_rmsnorm_bwd(o, gate, dy.to(gate.dtype).contiguous(), eps=ctx.eps, cu_seqlens=cu,
                                      out_rows=ctx.out_rows)
        return do, dgate, None, None, None


def gated_rmsnorm(o, gate, *, eps=RMS_EPS, cu_seqlens=None, out_rows=None):
    """Differentiable output gate (``_output_gate`` up to ``W_o``)."""
    if cu_seqlens is not None:
        cu_seqlens = cu_seqlens.to(device=o.device, dtype=torch.int32)
    return _GatedRMSNorm.apply(o, gate, eps, cu_seqlens, out_rows)


def decode_fused(S, conv_buf, qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, *, H, b_gate=None,
                 gate_logit=None, g_min=G_MIN, gate_kind="sigmoid_min", rms_eps=RMS_EPS, out_dtype=None):
    """One streaming token for ``N`` sequences; ``S [N, H, dk, dv]`` fp32 and
    ``conv_buf [N, K-1, H*(2dk+dv)]`` fp32 are updated in place.  Returns
    ``[N, H, dv]``: ``o = S^T q``, or its output gate when ``gate_logit``
    (``[N, H*dv]``) is given."""
    _require_device("decode_fused")
    N, HK = qp.shape
    dk, dv, K = HK // H, vp.shape[-1] // H, conv_q.shape[0]
    dt = qp.dtype
    _check_tensor(S, "S", (N, H, dk, dv), torch.float32)
    if K > 1:
        _check_tensor(conv_buf, "conv_buf", (N, K - 1, _state_width(H, dk, dv)), torch.float32)
    for x, n, s in ((kp, "kp", (N, H * dk)), (vp, "vp", (N, H * dv)), (z, "z", (N, H * dk)),
                    (beta_logit, "beta_logit", (N, H))):
        _check_tensor(x, n, s, dt)
    if gate_logit is not None:
        _check_tensor(gate_logit, "gate_logit", (N, H * dv), dt)
    out = torch.empty((N, H, dv), dtype=out_dtype or dt, device=S.device)
    rc = lib().kda_decode_fused(
        _ptr(S), _ptr(conv_buf if K > 1 else None), _ptr(qp), _ptr(kp), _ptr(vp), _ptr(z), _ptr(beta_logit),
        _ptr(gate_logit), _ptr(conv_q), _ptr(conv_k), _ptr(conv_v), _ptr(b_gate), _ptr(A), float(g_min),
        _gate_kind(gate_kind), float(rms_eps), _ptr(out), N, H, dk, dv, K, _dt(qp, "qp"), _dt(out, "out"),
        _stream())
    check("kda_decode_fused", rc)
    return out
