"""The KDA mixer layer on the B200 kernels: projections, fused prologue, KDA
core, output gate and output projection, differentiable end to end.

Mirrors the reference's layer function ``apply_kda(params, cfg, x,
chunk_size)`` (AXIOM ``net/kda.py:929-946``; :func:`apply_kda` takes its
arguments as they are, :func:`kda_layer` is the layer underneath; ``_project`` :157-191,
``_postprocess`` :194-203, ``_output_gate`` :206-214), with two additions the
mixer configuration needs: packed variable-length batches (``cu_seqlens``) and
the decay gate ``g = -exp(A_log) * softplus(z + b)`` beside the reference's
``g = g_min * sigmoid(exp(A) z)``.  The projection GEMMs are plain library
GEMMs (``torch.matmul``: cuBLAS); the per-token work and the KDA core run in
``libkda_b200.so``.  The reference's sliding-window branch (``_with_window``
:261-269) is outside this layer.  For inference, ``kda_layer_prefill`` runs N
prompts and returns a ``KDADecodeCache`` (recurrent state and short-conv
buffers, the reference's ``KDAState``) that ``kda_layer_decode`` advances one
token per call with the fused decode kernel.
"""

from __future__ import annotations

from dataclasses import dataclass, fields

import torch

from . import mixer
from .kda import CHUNK, chunk_kda, chunk_kda_varlen, kda_fwd, packing


@dataclass
class KDALayerParams:
    """Weights of one layer (the reference's ``KDAParams``, ``net/kda.py:63-80``;
    ``b_gate`` is its ``b_alpha``, ``A`` its ``A`` or the mixer's ``A_log``)."""

    W_q: torch.Tensor       # [d_model, H*dk]
    W_k: torch.Tensor       # [d_model, H*dk]
    W_v: torch.Tensor       # [d_model, H*dv]
    W_g: torch.Tensor       # [d_model, H*dv]   output gate
    W_beta: torch.Tensor    # [d_model, H]
    W_a_down: torch.Tensor  # [d_model, rank]
    W_a_up: torch.Tensor    # [rank, H*dk]
    b_gate: torch.Tensor    # [H*dk] fp32
    A: torch.Tensor         # [H] fp32
    conv_q: torch.Tensor    # [K, H*dk] fp32
    conv_k: torch.Tensor    # [K, H*dk] fp32
    conv_v: torch.Tensor    # [K, H*dv] fp32
    W_o: torch.Tensor       # [H*dv, d_model]

    def tensors(self):
        return [getattr(self, f.name) for f in fields(self)]


class _Projections(torch.autograd.Function):
    """``x @ W`` for several weights sharing the input ``x``.  The backward
    accumulates ``dx = sum_i dY_i W_i^T`` inside the GEMMs (``addmm_``, beta =
    1) instead of one GEMM per weight plus an elementwise add each."""

    @staticmethod
    def forward(ctx, x, *Ws):
        ctx.save_for_backward(x, *Ws)
        return tuple(x @ W for W in Ws)

    @staticmethod
    def backward(ctx, *dYs):
        x, *Ws = ctx.saved_tensors
        dx = None
        if ctx.needs_input_grad[0]:
            for dY, W in zip(dYs, Ws):
                if dY is None:
                    continue
                if dx is None:
                    dx = dY @ W.t()
                else:
                    dx.addmm_(dY, W.t())
        dWs = [(x.t() @ dY) if (dY is not None and ctx.needs_input_grad[1 + i]) else None
               for i, dY in enumerate(dYs)]
        return (dx, *dWs)


def init_params(d_model, H, dk, dv, *, rank=128, K=4, gate_kind="softplus", gate_bias="dt",
                dtype=torch.bfloat16, device="cuda", seed=0) -> KDALayerParams:
    """Random-init weights: projections N(0, 0.02) (the reference's ``_rand``
    scale, ``net/kda.py:110-127``), conv taps N(0, 0.1), ``A`` zero for the
    reference's gate (with ``b_alpha`` zero, ``net/kda.py:124-125``) or
    ``A_log ~ U(log 1, log 16)`` for the softplus gate.  The softplus gate's
    bias: ``gate_bias="dt"`` sets ``softplus(b)`` log-uniform in
    ``[1e-3, 1e-1]`` per channel (the usual time-step bias of this gate form),
    ``"zero"`` sets ``b = 0`` (per-token decay up to ``16 log 2``: every chunk
    then exceeds the tensor-core path's exponent budget).  Every tensor
    requires grad."""
    gen = torch.Generator(device="cpu").manual_seed(seed)

    def rnd(*shape, scale, dt=dtype):
        return (torch.randn(*shape, generator=gen) * scale).to(device=device, dtype=dt).requires_grad_(True)

    b = torch.zeros(H * dk)
    if gate_kind == "softplus":
        A = torch.empty(H).uniform_(0.0, float(torch.log(torch.tensor(16.0))), generator=gen)
        if gate_bias == "dt":
            lo, hi = float(torch.log(torch.tensor(1e-3))), float(torch.log(torch.tensor(1e-1)))
            dt_ = torch.exp(torch.empty(H * dk).uniform_(lo, hi, generator=gen))
            b = dt_ + torch.log(-torch.expm1(-dt_))  # softplus^-1(dt)
        elif gate_bias != "zero":
            raise ValueError(f"gate_bias={gate_bias!r}: expected 'dt' or 'zero'")
    else:
        A = torch.zeros(H)
    return KDALayerParams(
        W_q=rnd(d_model, H * dk, scale=0.02), W_k=rnd(d_model, H * dk, scale=0.02),
        W_v=rnd(d_model, H * dv, scale=0.02), W_g=rnd(d_model, H * dv, scale=0.02),
        W_beta=rnd(d_model, H, scale=0.02), W_a_down=rnd(d_model, rank, scale=0.02),
        W_a_up=rnd(rank, H * dk, scale=0.02), b_gate=b.to(device).requires_grad_(True),
        A=A.to(device).requires_grad_(True), conv_q=rnd(K, H * dk, scale=0.1, dt=torch.float32),
        conv_k=rnd(K, H * dk, scale=0.1, dt=torch.float32), conv_v=rnd(K, H * dv, scale=0.1, dt=torch.float32),
        W_o=rnd(H * dv, d_model, scale=0.02))


def kda_layer(p: KDALayerParams, x, *, H, cu_seqlens=None, gate_kind="softplus", g_min=mixer.G_MIN,
              chunk=CHUNK, S0=None, return_state=False):
    """One KDA mixer layer: ``x [T, d_model]`` (one sequence, or the packed
    sequences ``cu_seqlens`` delimits) -> ``[T, d_model]``.

    ``S0``/``S_T``: ``[n, H, dk, dv]`` fp32 (one state per sequence).
    """
    T, _ = x.shape
    dk = p.W_q.shape[1] // H
    dv = p.W_v.shape[1] // H
    # projections (_project, net/kda.py:157-191)
    qp, kp, vp, zd, bl, gl = _Projections.apply(x, p.W_q, p.W_k, p.W_v, p.W_a_down, p.W_beta, p.W_g)
    z = zd @ p.W_a_up
    if cu_seqlens is None:
        q, k, v, g, beta = mixer.kda_prologue(qp[None], kp[None], vp[None], z[None], bl[None], p.conv_q, p.conv_k,
                                              p.conv_v, p.A, H=H, b_gate=p.b_gate, g_min=g_min,
                                              gate_kind=gate_kind)
        o, s_t = chunk_kda(q, k, v, g, beta, S0, chunk=chunk)
        y = mixer.gated_rmsnorm(o, gl[None])
    else:
        offs, rows, _ = packing(cu_seqlens, chunk)
        cu = cu_seqlens if isinstance(cu_seqlens, torch.Tensor) else torch.tensor(list(cu_seqlens))
        cu = cu.to(device=x.device, dtype=torch.int32)
        q, k, v, g, beta = mixer.kda_prologue(qp[None], kp[None], vp[None], z[None], bl[None], p.conv_q, p.conv_k,
                                              p.conv_v, p.A, H=H, b_gate=p.b_gate, g_min=g_min,
                                              gate_kind=gate_kind, cu_seqlens=cu, out_rows=rows)
        o, s_t = chunk_kda_varlen(q, k, v, g, beta, offs, S0, chunk=chunk)
        y = mixer.gated_rmsnorm(o, gl[None], cu_seqlens=cu, out_rows=rows)
    out = y.squeeze(0) @ p.W_o  # a view both ways (indexing's backward would zero-fill y's shape)
    return (out, s_t) if return_state else out


def apply_kda(params, cfg, x, chunk_size=None):
    """The reference's layer entry point ``apply_kda(params, cfg, x, chunk_size)``
    (``net/kda.py:929-946``) on this library.

    ``params``: the reference's ``KDAParams`` fields as torch tensors (an object
    with those attributes, or a dict): ``W_q, W_k, W_v, W_o, W_g, W_beta,
    W_a_down, W_a_up, b_alpha, A, conv_q, conv_k, conv_v`` (the window fields are
    not read).  ``cfg``: its ``ModelConfig`` fields ``num_heads, kda_impl,
    kda_wyut_chunk, kda_g_min, swa_window, attn_dense_reference``.  ``x``:
    ``(T, hidden)`` as the reference takes it, or ``(B, T, hidden)``, which runs as
    one call over B packed sequences (where the reference maps the layer over
    the batch with ``vmap``, ``net/model.py:341-347``).

    The dispatch fails closed like the reference's: ``cfg.kda_impl`` must be
    ``chunked_cc`` (the form this library implements; ``chunked`` and ``wyut``
    are other algorithms, ``:929-946``), ``AXIOM_KDA_CC_IMPL`` must be ``b200``
    (``jax``, ``mosaic`` and ``persistent`` are the reference's JAX / Pallas
    bodies, not present here; an unknown value raises ``ValueError``), and the
    window branch must be off (``_with_window`` :261-269: ``attn_dense_reference``
    or ``swa_window == 0``, the reference's default).  The layer is then the
    reference's ``_apply_chunked_cc_persistent`` (:790-853): projections, short
    conv, Swish, L2 norm, sigmoid beta, the decay gate ``g = g_min sigmoid(exp(A)
    z)`` with ``z = x W_a_down W_a_up + b_alpha``, the chunked core, the
    head-wise RMSNorm times ``sigmoid(x W_g)`` and ``W_o``; differentiable."""
    from .kda import kda_cc_impl

    if cfg.kda_impl != "chunked_cc":
        raise NotImplementedError(
            f"kda_impl={cfg.kda_impl!r}: this library implements the chunked_cc form only")
    impl = kda_cc_impl()
    if impl != "b200":
        raise NotImplementedError(
            f"AXIOM_KDA_CC_IMPL={impl!r} selects a JAX / Pallas body of the reference; here only 'b200' runs")
    if not cfg.attn_dense_reference and cfg.swa_window > 0:
        raise NotImplementedError("the sliding-window branch (swa_window > 0) is not part of this library")
    get = (lambda n: params[n]) if isinstance(params, dict) else (lambda n: getattr(params, n))
    p = KDALayerParams(W_q=get("W_q"), W_k=get("W_k"), W_v=get("W_v"), W_g=get("W_g"), W_beta=get("W_beta"),
                       W_a_down=get("W_a_down"), W_a_up=get("W_a_up"), b_gate=get("b_alpha"), A=get("A"),
                       conv_q=get("conv_q"), conv_k=get("conv_k"), conv_v=get("conv_v"), W_o=get("W_o"))
    chunk = int(chunk_size or cfg.kda_wyut_chunk)
    kw = dict(H=cfg.num_heads, gate_kind="sigmoid_min", g_min=float(cfg.kda_g_min), chunk=chunk)
    if x.dim() == 2:
        return kda_layer(p, x, **kw)
    if x.dim() != 3:
        raise ValueError(f"x: expected (T, hidden) or (B, T, hidden), got {tuple(x.shape)}")
    B, T, hid = x.shape
    cu = [i * T for i in range(B + 1)]
    return kda_layer(p, x.reshape(B * T, hid), cu_seqlens=cu, **kw).reshape(B, T, -1)


@dataclass
class KDADecodeCache:
    """Per-layer streaming state of N sequences (the reference's ``KDAState``,
    ``net/kda.py:54-60``): the fp32 recurrent state and the short-conv buffers
    of the q, k, v projections (the last K-1 rows, side by side)."""

    S: torch.Tensor     # [N, H, dk, dv] fp32
    conv: torch.Tensor  # [N, K-1, H*(2dk+dv)] fp32


def _projections(p: KDALayerParams, x):
    return x @ p.W_q, x @ p.W_k, x @ p.W_v, (x @ p.W_a_down) @ p.W_a_up, x @ p.W_beta, x @ p.W_g


def kda_layer_prefill(p: KDALayerParams, x, *, H, gate_kind="softplus", g_min=mixer.G_MIN, chunk=CHUNK):
    """Inference over N prompts of one length: ``x [N, T, d_model]`` ->
    ``(out [N, T, d_model], cache)``.  The same kernels as :func:`kda_layer`
    (prologue with its conv state out, chunked core with its final state,
    output gate); the cache continues each sequence with
    :func:`kda_layer_decode`.  (The reference's ``generate``, ``net/infer.py``,
    re-runs the whole forward for every new token; this is the state cache
    that replaces that.)"""
    with torch.no_grad():
        qp, kp, vp, z, bl, gl = _projections(p, x)
        q, k, v, g, beta, conv = mixer.prologue_fwd(qp, kp, vp, z, bl, p.conv_q, p.conv_k, p.conv_v, p.A, H=H,
                                                    b_gate=p.b_gate, g_min=g_min, gate_kind=gate_kind,
                                                    return_state=True)
        o, S, _ = kda_fwd(q, k, v, g, beta, None, chunk=chunk)
        y = mixer.gated_rmsnorm_fwd(o, gl)
        out = y @ p.W_o
    if conv is None:  # K = 1: no buffers
        conv = torch.empty((x.shape[0], 0, 0), dtype=torch.float32, device=x.device)
    return out, KDADecodeCache(S=S, conv=conv)


def kda_layer_decode(p: KDALayerParams, x, cache: KDADecodeCache, *, H, gate_kind="softplus",
                     g_min=mixer.G_MIN):
    """One new token for each of the N cached sequences: ``x [N, d_model]`` ->
    ``[N, d_model]``; ``cache`` is updated in place.  The token's prologue, the
    recurrent step and the output gate are one kernel
    (``kda_decode_fused``); the projections are library GEMMs."""
    with torch.no_grad():
        qp, kp, vp, z, bl, gl = _projections(p, x)
        y = mixer.decode_fused(cache.S, cache.conv, qp, kp, vp, z, bl, p.conv_q, p.conv_k, p.conv_v, p.A, H=H,
                               b_gate=p.b_gate, gate_logit=gl, g_min=g_min, gate_kind=gate_kind)
        return y.reshape(x.shape[0], -1) @ p.W_o

