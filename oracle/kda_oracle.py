"""CPU oracle for the KDA hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped path (``axiom_b200``) runs the
CUDA library and fails loudly when it is missing; it never calls this file.

It is a NumPy restatement of the reference's KDA core (AXIOM, pure JAX), in
float64 by default (``dtype=np.float32`` reproduces the reference's fp32
arithmetic).  Every function cites the reference lines it follows.  The
restatement is pinned against golden vectors produced by running the
reference's own functions (``tests/golden/make_golden.py``), so parity is
pinned, not assumed.

Conventions (the BASELINE operand form of the reference interval):

* ``q, k``: ``[B, T, H, dk]``; ``v``: ``[B, T, H, dv]``;
* ``g``: ``[B, T, H, dk]`` per-channel log-decay (``alpha = exp(g)``, g <= 0),
  the reference passes ``alpha`` and takes ``log`` itself
  (``net/kernels/kda_cc_fused_bwd.py:157``); ``dg`` is therefore its ``dla``;
* ``beta``: ``[B, T, H]`` write gate (the reference's ``beta32`` is this value
  replicated over 32 columns, ``net/kernels/kda_cc_fused.py:275``);
* ``S``: ``[B, H, dk, dv]`` fp32 state.
"""

from __future__ import annotations

import numpy as np

#: Row-tile width of the tile-anchored decay factors (``net/kda.py:561``).
TILE = 16
#: Clamp of the column exponent (``net/kernels/kda_cc_fused_persist.py:224``).
COL_EXP_BUDGET = 80.0


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 (round-to-nearest-even) and return float32."""
    import ml_dtypes

    return np.asarray(x, np.float32).astype(ml_dtypes.bfloat16).astype(np.float32)


def scale_rel_err(got, ref) -> float:
    """``max|got - ref| / max|ref|`` -- the reference's tolerance convention
    (``net/tests/test_kda_cc_fused_bwd.py:88-106``)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    num = float(np.max(np.abs(got - ref))) if ref.size else 0.0
    return num / max(den, 1e-30)


def _logsigmoid(x):
    return -np.logaddexp(0.0, -x)


def make_inputs(B, T, H, dk, dv, seed=0, s0_std=None, decay="baseline"):
    """Seeded synthetic inputs with the BASELINE distributions.

    q, k ~ N(0,1) then L2-normalised per (token, head); v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = logsigmoid(N(3,1)) per key channel
    (``decay="strong"``: g = -5 sigmoid(3 N(0,1)), the reference's
    strong-decay test range ``net/tests/test_kda_chunked_cc.py:231``;
    ``decay="medium"``: g = -sigmoid(2 N(0,1)); ``decay="half_budget"``:
    g = -(1.6 + 0.4 sigmoid(N(0,1))), so a 64-token chunk sums past 80 while
    each 32-token half stays below it).
    S0 ~ N(0, s0_std) or zeros.  Returns float32 arrays.
    """
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, dk))
    k = rng.standard_normal((B, T, H, dk))
    q /= np.linalg.norm(q, axis=-1, keepdims=True) + 1e-12
    k /= np.linalg.norm(k, axis=-1, keepdims=True) + 1e-12
    v = rng.standard_normal((B, T, H, dv))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))
    if decay == "baseline":
        g = _logsigmoid(rng.normal(3.0, 1.0, (B, T, H, dk)))
    elif decay == "strong":
        z = rng.standard_normal((B, T, H, dk))
        g = -5.0 / (1.0 + np.exp(-3.0 * z))
    elif decay == "medium":
        g = -1.0 / (1.0 + np.exp(-2.0 * rng.standard_normal((B, T, H, dk))))
    elif decay == "half_budget":
        g = -(1.6 + 0.4 / (1.0 + np.exp(-rng.standard_normal((B, T, H, dk)))))
    else:
        raise ValueError(f"unknown decay {decay!r}")
    if s0_std is None:
        S0 = np.zeros((B, H, dk, dv))
    else:
        S0 = rng.normal(0.0, s0_std, (B, H, dk, dv))
    f = np.float32
    return dict(q=q.astype(f), k=k.astype(f), v=v.astype(f), g=g.astype(f),
                beta=beta.astype(f), S0=S0.astype(f))


def _to_heads(x):
    """[B, T, H, D] -> [B, H, T, D] (and [B, T, H] -> [B, H, T])."""
    return np.swapaxes(x, 1, 2)


# ---------------------------------------------------------------------------
# recurrence (secondary oracle) and decode step
# ---------------------------------------------------------------------------


def decode_step(S, q, k, v, g, beta, dtype=np.float64):
    """One token of the delta rule; returns ``(o, S_new)``.

    ``S <- diag(alpha) S - beta k ((alpha*k)^T S) + beta k v^T`` then
    ``o = S^T q`` with the *updated* S (``net/kda.py:298-310`` and ``:293``).
    Shapes: S ``[..., dk, dv]``; q, k, g ``[..., dk]``; v ``[..., dv]``;
    beta ``[...]``.
    """
    S = np.asarray(S, dtype)
    q, k, v, g = (np.asarray(a, dtype) for a in (q, k, v, g))
    beta = np.asarray(beta, dtype)
    alpha = np.exp(g)
    read = np.einsum("...d,...dv->...v", alpha * k, S)
    bk = beta[..., None] * k
    S_new = alpha[..., None] * S + bk[..., :, None] * (v - read)[..., None, :]
    o = np.einsum("...dv,...d->...v", S_new, q)
    return o, S_new


def recurrent(q, k, v, g, beta, S0=None, dtype=np.float64):
    """Token-by-token recurrence over ``[B, T, H, *]``; returns ``(o, S_T)``.

    ``apply_recurrent``'s ``lax.scan`` of ``_delta_step`` (``net/kda.py:313-317``).
    """
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    S = np.zeros((B, H, dk, dv), dtype) if S0 is None else np.asarray(S0, dtype).copy()
    o = np.zeros((B, T, H, dv), dtype)
    for t in range(T):
        o[:, t], S = decode_step(S, q[:, t], k[:, t], v[:, t], g[:, t], beta[:, t], dtype)
    return o, S


# ---------------------------------------------------------------------------
# chunked WY/UT forward (the ``chunked_cc`` form)
# ---------------------------------------------------------------------------


def cc_scores(row, col, G, tile=TILE, strict=False):
    """Decay-weighted ``C x C`` scores ``sum_d exp(G_c - G_i) row_c[d] col_i[d]``.

    Tile-anchored exactly like ``_cc_scores`` (``net/kda.py:588-631``): each
    row tile of ``tile`` positions measures the decay against its own first
    position ``p``, ``exp(G_c - G_i) = exp(G_c - G_p) exp(G_p - G_i)``; the
    column exponent is clamped at ``COL_EXP_BUDGET`` as the persistent kernel
    does (``net/kernels/kda_cc_fused_persist.py:482``; inert in-tile).
    Shapes ``[..., C, D]`` -> ``[..., C, C]``; mask keeps ``c >= i``
    (``strict``: ``c > i``).  ``tile=None`` takes the direct ratio instead,
    exact for any decay (the reference's anchor and clamp lose accuracy once a
    tile's summed decay passes the budget).
    """
    C = row.shape[-2]
    if tile is None:  # the direct ratio, exact for any decay (no anchor, no clamp)
        E = np.exp(np.minimum(G[..., :, None, :] - G[..., None, :, :], 0.0))
        mask = np.tril(np.ones((C, C), row.dtype), -1 if strict else 0)
        return mask * np.einsum("...cid,...cd,...id->...ci", E, row, col)
    out = np.zeros(row.shape[:-1] + (C,), row.dtype)
    for p in range(0, C, tile):
        b = min(tile, C - p)
        ref = G[..., p:p + 1, :]
        rows = row[..., p:p + b, :] * np.exp(G[..., p:p + b, :] - ref)
        cols = col[..., :p + b, :] * np.exp(np.minimum(ref - G[..., :p + b, :], COL_EXP_BUDGET))
        blk = rows @ np.swapaxes(cols, -1, -2)
        ri = np.arange(p, p + b)[:, None]
        ci = np.arange(p + b)[None, :]
        keep = (ri > ci) if strict else (ri >= ci)
        out[..., p:p + b, :p + b] = np.where(keep, blk, 0.0)
    return out


def _chunk_forward_parts(qc, kc, vc, gc, bc, S, tile=TILE):
    """All intermediates of one chunk (``net/kda.py:669-702``).

    ``qc, kc, gc``: ``[..., C, dk]``; ``vc``: ``[..., C, dv]``; ``bc``: ``[..., C]``;
    ``S``: ``[..., dk, dv]``.
    """
    C = qc.shape[-2]
    G = np.cumsum(gc, axis=-2)                      # _log_cumulative_decay :397-399
    aqk = cc_scores(qc, kc, G, tile, strict=False)  # :676
    akk = cc_scores(kc, kc, G, tile, strict=True)   # :677
    L = akk * bc[..., :, None]                      # :681 rows carry beta
    gam = np.exp(G)
    xw = gam * kc * bc[..., None]                   # :684-685
    vw = vc * bc[..., None]                         # :686
    M = np.eye(C, dtype=qc.dtype) + L
    W = np.linalg.solve(M, xw)                      # (I+L)^{-1} xw  (_solve_pair_jax :434-438)
    U = np.linalg.solve(M, vw)
    vt = U - W @ S                                  # :690
    o = (gam * qc) @ S + aqk @ vt                   # :693-696
    gC = gam[..., -1, :]                            # :699
    lam = np.exp(np.minimum(G[..., -1:, :] - G, 0.0))  # :700
    S_new = gC[..., :, None] * S + np.swapaxes(lam * kc, -1, -2) @ vt  # :701-702
    return dict(G=G, gam=gam, aqk=aqk, L=L, M=M, W=W, U=U, vt=vt, o=o,
                gC=gC, lam=lam, S_new=S_new)


def _pad_chunks(x, C, axis):
    T = x.shape[axis]
    n = -(-T // C)
    pad = n * C - T
    if pad:
        widths = [(0, 0)] * x.ndim
        widths[axis] = (0, pad)
        x = np.pad(x, widths)
    return x, n


def chunk_fwd(q, k, v, g, beta, S0=None, chunk=64, tile=TILE, dtype=np.float64,
              return_states=False):
    """Chunked KDA forward over ``[B, T, H, *]``; returns ``(o, S_T[, states])``.

    The ``chunked_cc`` scan (``net/kda.py:856-926`` with body ``cc_chunk_step``
    ``:634-705``; operand form ``net/kernels/kda_cc_fused.py:618-687`` scanned
    by ``net/kernels/kda_cc_fused_persist.py:768-791``).  A ragged tail is
    zero-padded (q = k = v = 0, beta = 0, g = 0), which leaves the state and
    the real rows untouched; ``states[:, :, c]`` is the state entering chunk c.
    """
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    C = int(chunk)
    Q, K, V, Gl = (_to_heads(np.asarray(a, dtype)) for a in (q, k, v, g))
    Bt = _to_heads(np.asarray(beta, dtype))
    Q, n = _pad_chunks(Q, C, 2)
    K, _ = _pad_chunks(K, C, 2)
    V, _ = _pad_chunks(V, C, 2)
    Gl, _ = _pad_chunks(Gl, C, 2)
    Bt, _ = _pad_chunks(Bt, C, 2)
    S = np.zeros((B, H, dk, dv), dtype) if S0 is None else np.asarray(S0, dtype).copy()
    O = np.zeros((B, H, n * C, dv), dtype)
    states = np.zeros((B, H, n, dk, dv), dtype) if return_states else None
    for c in range(n):
        sl = slice(c * C, (c + 1) * C)
        if return_states:
            states[:, :, c] = S
        parts = _chunk_forward_parts(Q[:, :, sl], K[:, :, sl], V[:, :, sl],
                                     Gl[:, :, sl], Bt[:, :, sl], S, tile)
        O[:, :, sl] = parts["o"]
        S = parts["S_new"]
    o = np.swapaxes(O[:, :, :T], 1, 2)
    if return_states:
        return o, S, states
    return o, S


# ---------------------------------------------------------------------------
# analytic adjoint (the fused backward) and the reverse chunk scan
# ---------------------------------------------------------------------------


def _chunk_backward(qc, kc, vc, gc, bc, S, do, dSn):
    """Adjoint of one chunk; returns ``(dq, dk, dv, dg, dbeta, dS_in)``.

    Restates ``reference_bwd`` (``net/kernels/kda_cc_fused_bwd.py:117-239``,
    equations ``:28-63``) with the decay taken as ``g = log alpha`` directly,
    so ``dg`` is its ``dla`` (``:224-226``) and no ``/alpha`` is applied.  The
    score adjoints use the direct ratio ``E = exp(min(G_c - G_i, 0))`` exactly
    like the reference (``:164-167``).
    """
    C = qc.shape[-2]
    T_ = np.swapaxes
    tri = np.tril(np.ones((C, C), qc.dtype))
    strict = np.tril(np.ones((C, C), qc.dtype), -1)
    G = np.cumsum(gc, axis=-2)
    gam = np.exp(G)
    E = np.exp(np.minimum(G[..., :, None, :] - G[..., None, :, :], 0.0))  # [..., C, C, dk]
    b1 = bc[..., :, None]
    aqk = tri * np.einsum("...cid,...cd,...id->...ci", E, qc, kc)
    L = strict * np.einsum("...cid,...cd,...id->...ci", E, kc * b1, kc)
    xw = gam * kc * b1
    vw = vc * b1
    SM = np.linalg.inv(np.eye(C, dtype=qc.dtype) + L)
    W = SM @ xw
    U = SM @ vw
    vt = U - W @ S
    gsum = G[..., -1, :]
    gcl = np.exp(gsum)
    lam = np.exp(np.minimum(gsum[..., None, :] - G, 0.0))
    y = lam * kc

    dS = gcl[..., :, None] * dSn
    dgc = np.sum(S * dSn, axis=-1)
    dY = vt @ T_(dSn, -1, -2)
    dvt = y @ dSn + T_(aqk, -1, -2) @ do
    daqk = (do @ T_(vt, -1, -2)) * tri
    dS = dS + T_(gam * qc, -1, -2) @ do
    dgq = do @ T_(S, -1, -2)
    dgam = dgq * qc
    dq = dgq * gam

    dU = dvt
    dW = -(dvt @ T_(S, -1, -2))
    dS = dS - T_(W, -1, -2) @ dvt
    Yw = T_(SM, -1, -2) @ dW
    Yu = T_(SM, -1, -2) @ dU
    dL = -(Yw @ T_(W, -1, -2) + Yu @ T_(U, -1, -2)) * strict
    dgam = dgam + Yw * (kc * b1)
    dk = Yw * (gam * b1)
    dv = Yu * b1
    db = np.sum(Yw * gam * kc, axis=-1) + np.sum(Yu * vc, axis=-1)

    dr_a = np.einsum("...ci,...cid,...id->...cd", daqk, E, kc)
    dc_a = np.einsum("...ci,...cid,...cd->...id", daqk, E, qc)
    dq = dq + dr_a
    dk = dk + dc_a
    dr_k = np.einsum("...ci,...cid,...id->...cd", dL, E, kc)
    dc_k = np.einsum("...ci,...cid,...cd->...id", dL, E, kc * b1)
    dk = dk + dr_k * b1 + dc_k
    db = db + np.sum(dr_k * kc, axis=-1)
    dG = (dr_a * qc - dc_a * kc) + (dr_k * (kc * b1) - dc_k * kc)
    dG = dG + dgam * gam

    dlam = dY * kc
    dk = dk + dY * lam
    dz = dlam * lam
    dG = dG - dz
    dsum = np.sum(dz, axis=-2)
    # tril^T @ dG == reverse cumulative sum over the chunk positions
    dla = np.flip(np.cumsum(np.flip(dG, -2), axis=-2), -2) + (dsum + gcl * dgc)[..., None, :]
    return dq, dk, dv, dla, db, dS


def chunk_bwd(q, k, v, g, beta, S0, do, dST=None, chunk=64, dtype=np.float64, tile=TILE):
    """Reverse chunk scan of the adjoint; returns ``(dq, dk, dv, dg, dbeta, dS0)``.

    ``reference_bwd_scan`` (``net/kernels/kda_cc_fused_persist.py:794-849``):
    a forward pass recomputes the incoming state of every chunk (``tile`` as in
    :func:`chunk_fwd`), then the chunks are walked in reverse carrying the state
    cotangent.
    """
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    C = int(chunk)
    Q, K, V, Gl, DO = (_to_heads(np.asarray(a, dtype)) for a in (q, k, v, g, do))
    Bt = _to_heads(np.asarray(beta, dtype))
    Q, n = _pad_chunks(Q, C, 2)
    K, _ = _pad_chunks(K, C, 2)
    V, _ = _pad_chunks(V, C, 2)
    Gl, _ = _pad_chunks(Gl, C, 2)
    Bt, _ = _pad_chunks(Bt, C, 2)
    DO, _ = _pad_chunks(DO, C, 2)
    S = np.zeros((B, H, dk, dv), dtype) if S0 is None else np.asarray(S0, dtype)
    s_ins = []
    for c in range(n):
        sl = slice(c * C, (c + 1) * C)
        s_ins.append(S)
        S = _chunk_forward_parts(Q[:, :, sl], K[:, :, sl], V[:, :, sl],
                                 Gl[:, :, sl], Bt[:, :, sl], S, tile)["S_new"]
    dS = np.zeros((B, H, dk, dv), dtype) if dST is None else np.asarray(dST, dtype)
    dQ, dK, dV, dGl = (np.zeros_like(a) for a in (Q, K, V, Gl))
    dB = np.zeros_like(Bt)
    for c in reversed(range(n)):
        sl = slice(c * C, (c + 1) * C)
        dq_c, dk_c, dv_c, dg_c, db_c, dS = _chunk_backward(
            Q[:, :, sl], K[:, :, sl], V[:, :, sl], Gl[:, :, sl], Bt[:, :, sl],
            s_ins[c], DO[:, :, sl], dS)
        dQ[:, :, sl], dK[:, :, sl], dV[:, :, sl] = dq_c, dk_c, dv_c
        dGl[:, :, sl], dB[:, :, sl] = dg_c, db_c
    back = lambda x: np.swapaxes(x[:, :, :T], 1, 2)  # noqa: E731
    return back(dQ), back(dK), back(dV), back(dGl), back(dB), dS


def recurrent_loss_grad_fd(q, k, v, g, beta, S0, do, dST, eps=1e-6, n_probe=8, seed=0):
    """Central finite differences of ``<o, do> + <S_T, dST>`` through the
    recurrence, at ``n_probe`` random coordinates of each input (float64).

    The reference's own float64 check (``net/tests/test_kda_chunked_cc.py:333-391``).
    Returns ``{name: (idx, fd_values)}``.
    """
    rng = np.random.default_rng(seed)
    args = dict(q=q, k=k, v=v, g=g, beta=beta, S0=S0)
    args = {n_: np.asarray(a, np.float64).copy() for n_, a in args.items()}

    def loss(a):
        o, S = recurrent(a["q"], a["k"], a["v"], a["g"], a["beta"], a["S0"])
        return float(np.sum(o * do) + np.sum(S * dST))

    out = {}
    for name in args:
        flat = args[name].reshape(-1)
        idx = rng.choice(flat.size, size=min(n_probe, flat.size), replace=False)
        vals = []
        for i in idx:
            old = flat[i]
            flat[i] = old + eps
            lp = loss(args)
            flat[i] = old - eps
            lm = loss(args)
            flat[i] = old
            vals.append((lp - lm) / (2 * eps))
        out[name] = (idx, np.array(vals))
    return out
