"""CPU oracle for the KDA mixer's prologue, epilogue and fused decode step --
TEST INFRASTRUCTURE ONLY.

Like ``kda_oracle`` this module is the checker, never the product: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` may
import it; the shipped path runs the CUDA library.

It restates, in NumPy (float64 by default), the per-token work the reference
does around the KDA core:

* the causal depthwise short convolution and its streaming step
  (``net/shortconv.py:14-30``, ``:33-53``);
* Swish and the guarded L2 norm with its derivative rule
  (``net/norm.py:15-17``, ``:20-61``) -- ``_postprocess`` ``net/kda.py:194-203``;
* the write gate ``beta = sigmoid(.)`` (``net/kda.py:169-171``) and the decay
  gate: the reference's ``g = g_min * sigmoid(exp(A) * z)`` with
  ``z = x W_down W_up + b_alpha`` (``net/kda.py:173-180``), or the
  ``g = -exp(A_log) * softplus(z + b)`` form of the mixer configuration;
* the output gate ``sigmoid(gate) * headwise_rms_norm(o)`` before ``W_o``
  (``net/kda.py:206-214``, ``net/norm.py:70-73``);
* one streaming decode step (``recurrent_step`` ``net/kda.py:277-295`` minus
  the projection GEMMs).

Backward rules are the analytic VJPs of these functions (the reference gets
them from ``jax.grad``); the tests pin them with float64 finite differences,
the reference's own check (``net/tests/test_kda_chunked_cc.py:333-391``), and
pin the forward functions against fixtures produced by executing the
reference's source (``tests/golden/make_golden_mixer.py``).

Layouts (this repo's): projections ``qp, kp, z : [B, T, H*dk]``,
``vp : [B, T, H*dv]``, ``beta_logit : [B, T, H]``; conv weights
``[K, H*d]`` (``w[i]`` weights the input ``i`` steps back); the conv state of a
sequence is ``[K-1, H*dk | H*dk | H*dv]`` (q, k and v buffers side by side,
oldest row first, as ``KDAState.q_buf/k_buf/v_buf``, ``net/kda.py:54-60``).
"""

from __future__ import annotations

import numpy as np

#: ``l2_norm``'s eps (``net/norm.py:51``)
L2_EPS = 1e-12
#: ``headwise_rms_norm``'s eps (``net/norm.py:70``)
RMS_EPS = 1e-6
#: the reference's lower bound of the log-decay (``net/config.py:131``)
G_MIN = -5.0

GATE_SIGMOID_MIN = 0  # g = g_min * sigmoid(exp(A) * (z + b))   net/kda.py:173-180
GATE_SOFTPLUS = 1     # g = -exp(A) * softplus(z + b)          (A = A_log)


def _sigmoid(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def _softplus(x):
    return np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))


# ---------------------------------------------------------------------------
# primitives
# ---------------------------------------------------------------------------


def _segments(T, cu_seqlens):
    """Sequence id of every token (all 0 without ``cu_seqlens``)."""
    if cu_seqlens is None:
        return np.zeros(T, np.int64)
    cu = np.asarray(cu_seqlens, np.int64)
    return np.searchsorted(cu, np.arange(T), side="right") - 1


def short_conv(x, w, state=None, cu_seqlens=None):
    """Causal depthwise convolution ``out[t] = sum_i w[i] x[t-i]``
    (``net/shortconv.py:14-30``).  ``x [T, D]``, ``w [K, D]``.  Inputs before
    the sequence start come from ``state`` (``[K-1, D]``, oldest first: row
    ``j`` is time ``j - (K-1)``) or are zero; with ``cu_seqlens`` every packed
    sequence starts from zeros."""
    x = np.asarray(x, np.float64)
    T, D = x.shape
    K = w.shape[0]
    seg = _segments(T, cu_seqlens)
    out = np.zeros_like(x)
    t = np.arange(T)
    for i in range(K):
        src = t - i
        inside = src >= 0
        same = np.zeros(T, bool)
        same[inside] = seg[src[inside]] == seg[inside]
        xs = np.zeros_like(x)
        xs[same] = x[src[same]]
        if state is not None and cu_seqlens is None:
            pre = (~inside) & (src + K - 1 >= 0)
            xs[pre] = np.asarray(state, np.float64)[src[pre] + K - 1]
        out += w[i][None, :] * xs
    return out


def short_conv_state_out(x, state, K):
    """The last ``K-1`` inputs after the sequence (the next call's state)."""
    x = np.asarray(x, np.float64)
    T, D = x.shape
    hist = np.zeros((K - 1 + T, D))
    if state is not None:
        hist[:K - 1] = state
    hist[K - 1:] = x
    return hist[T:]


def short_conv_step(x_t, w, buf):
    """Streaming form (``net/shortconv.py:33-53``): returns ``(out_t, new_buf)``."""
    K = w.shape[0]
    if K == 1:
        return w[0] * x_t, buf
    hist = np.einsum("kd,kd->d", w[:0:-1], buf)
    return w[0] * x_t + hist, np.concatenate([buf[1:], x_t[None, :]], axis=0)


def swish(x):
    """``x * sigmoid(x)`` (``net/norm.py:15-17``)."""
    return x * _sigmoid(x)


def swish_grad(x):
    s = _sigmoid(x)
    return s * (1.0 + x * (1.0 - s))


def l2_norm(x, eps=L2_EPS):
    """``x / (||x|| + eps)`` over the last axis (``net/norm.py:20-23``)."""
    return x / (np.linalg.norm(x, axis=-1, keepdims=True) + eps)


def l2_norm_vjp(x, dy, eps=L2_EPS):
    """Cotangent of ``l2_norm``: the reference's derivative rule
    (``net/norm.py:26-48``), whose Jacobian ``(I - x x^T / (|x| (|x|+eps))) /
    (|x|+eps)`` is symmetric, so the JVP formula applied to ``dy`` is the VJP;
    zero at ``x = 0``."""
    n = np.linalg.norm(x, axis=-1, keepdims=True)
    den = n + eps
    ok = n > 0.0
    unit = x / np.where(ok, n, 1.0)
    proj = np.sum(unit * dy, axis=-1, keepdims=True)
    return np.where(ok, (dy - x * proj / den) / den, 0.0)


def headwise_rms_norm(x, eps=RMS_EPS):
    """``x / sqrt(mean(x^2) + eps)`` over the last axis (``net/norm.py:70-73``)."""
    return x / np.sqrt(np.mean(np.square(x), axis=-1, keepdims=True) + eps)


def decay_gate(z, b, A, g_min=G_MIN, kind=GATE_SIGMOID_MIN):
    """Per-channel log-decay from the gate pre-activation ``z [..., H, dk]``,
    bias ``b [H, dk]`` and per-head ``A [H]``."""
    u = z + b
    a = np.exp(A)[:, None]
    if kind == GATE_SIGMOID_MIN:
        return g_min * _sigmoid(a * u)
    return -a * _softplus(u)


def decay_gate_vjp(z, b, A, dg, g_min=G_MIN, kind=GATE_SIGMOID_MIN):
    """``(dz, dA_per_element)``: ``dA`` is the per-element term summed by the
    caller over tokens and channels."""
    u = z + b
    a = np.exp(A)[:, None]
    if kind == GATE_SIGMOID_MIN:
        s = _sigmoid(a * u)
        t = dg * g_min * s * (1.0 - s)
        return t * a, t * a * u
    s = _sigmoid(u)
    return -dg * a * s, -dg * a * _softplus(u)


# ---------------------------------------------------------------------------
# fused prologue
# ---------------------------------------------------------------------------


def prologue_fwd(qp, kp, vp, z, beta_logit, wq, wk, wv, b_gate, A, H, dk, dv, g_min=G_MIN,
                 kind=GATE_SIGMOID_MIN, state=None, cu_seqlens=None):
    """The KDA core's inputs from the projections: ShortConv -> Swish -> L2 norm
    for q, k; ShortConv -> Swish for v (``net/kda.py:194-203``); sigmoid write
    gate; decay gate.  Returns ``q, k [B,T,H,dk]``, ``v [B,T,H,dv]``,
    ``g [B,T,H,dk]``, ``beta [B,T,H]`` and ``state_out [B,K-1,H*(2dk+dv)]``."""
    B, T = qp.shape[:2]
    K = wq.shape[0]
    nq = H * dk
    out = {n: [] for n in ("q", "k", "v", "state_out")}
    for b in range(B):
        st = None if state is None else np.asarray(state[b], np.float64)
        sq, sk, sv = (None, None, None) if st is None else (st[:, :nq], st[:, nq:2 * nq], st[:, 2 * nq:])
        cq = short_conv(qp[b], wq, sq, cu_seqlens)
        ck = short_conv(kp[b], wk, sk, cu_seqlens)
        cv = short_conv(vp[b], wv, sv, cu_seqlens)
        out["q"].append(l2_norm(swish(cq).reshape(T, H, dk)))
        out["k"].append(l2_norm(swish(ck).reshape(T, H, dk)))
        out["v"].append(swish(cv).reshape(T, H, dv))
        if K > 1:
            out["state_out"].append(np.concatenate(
                [short_conv_state_out(qp[b], sq, K), short_conv_state_out(kp[b], sk, K),
                 short_conv_state_out(vp[b], sv, K)], axis=1))
    res = {n: np.stack(vv) for n, vv in out.items() if vv}
    res["g"] = decay_gate(np.asarray(z, np.float64).reshape(B, T, H, dk), np.asarray(b_gate).reshape(H, dk),
                          np.asarray(A, np.float64), g_min, kind)
    res["beta"] = _sigmoid(np.asarray(beta_logit, np.float64))
    return res


def _conv_bwd(x, w, dc, state, cu_seqlens):
    """``(dx, dw, dstate)`` of ``short_conv`` for cotangent ``dc``."""
    T, D = x.shape
    K = w.shape[0]
    seg = _segments(T, cu_seqlens)
    t = np.arange(T)
    dx = np.zeros((T, D))
    dw = np.zeros((K, D))
    dstate = np.zeros((K - 1, D))
    for i in range(K):
        src = t - i
        inside = src >= 0
        same = np.zeros(T, bool)
        same[inside] = seg[src[inside]] == seg[inside]
        np.add.at(dx, src[same], w[i][None, :] * dc[same])
        dw[i] += np.sum(dc[same] * x[src[same]], axis=0)
        if cu_seqlens is None:
            pre = (~inside) & (src + K - 1 >= 0)
            if state is not None:
                dw[i] += np.sum(dc[pre] * state[src[pre] + K - 1], axis=0)
            np.add.at(dstate, src[pre] + K - 1, w[i][None, :] * dc[pre])
    return dx, dw, dstate


def prologue_bwd(qp, kp, vp, z, beta_logit, wq, wk, wv, b_gate, A, H, dk, dv, dq, dk_, dv_, dg,
                 dbeta, g_min=G_MIN, kind=GATE_SIGMOID_MIN, state=None, cu_seqlens=None):
    """Cotangents of ``prologue_fwd``'s inputs for output cotangents ``dq, dk_,
    dv_, dg, dbeta``: ``dqp, dkp, dvp, dz, dbeta_logit`` (input shapes),
    ``dwq, dwk, dwv [K, H*d]``, ``db_gate [H*dk]``, ``dA [H]`` and ``dstate``
    (``[B, K-1, H*(2dk+dv)]``)."""
    B, T = qp.shape[:2]
    K = wq.shape[0]
    nq = H * dk
    res = {n: [] for n in ("dqp", "dkp", "dvp", "dstate")}
    dws = [np.zeros((K, nq)), np.zeros((K, nq)), np.zeros((K, H * dv))]
    for b in range(B):
        st = None if state is None else np.asarray(state[b], np.float64)
        parts = (None, None, None) if st is None else (st[:, :nq], st[:, nq:2 * nq], st[:, 2 * nq:])
        grads = []
        for j, (x, w, dy, d) in enumerate(((qp[b], wq, dq[b], dk), (kp[b], wk, dk_[b], dk),
                                           (vp[b], wv, dv_[b], dv))):
            x = np.asarray(x, np.float64)
            c = short_conv(x, w, parts[j], cu_seqlens)
            s = swish(c)
            dy = np.asarray(dy, np.float64).reshape(T, H, d)
            ds = l2_norm_vjp(s.reshape(T, H, d), dy) if j < 2 else dy
            dc = ds.reshape(T, H * d) * swish_grad(c)
            dx, dw, dst = _conv_bwd(x, w, dc, parts[j], cu_seqlens)
            grads += [dx, dst]
            dws[j] += dw
        res["dqp"].append(grads[0])
        res["dkp"].append(grads[2])
        res["dvp"].append(grads[4])
        res["dstate"].append(np.concatenate([grads[1], grads[3], grads[5]], axis=1))
    out = {n: np.stack(vv) for n, vv in res.items()}
    out["dwq"], out["dwk"], out["dwv"] = dws
    zz = np.asarray(z, np.float64).reshape(B, T, H, dk)
    dz, da = decay_gate_vjp(zz, np.asarray(b_gate, np.float64).reshape(H, dk), np.asarray(A, np.float64),
                            np.asarray(dg, np.float64), g_min, kind)
    out["dz"] = dz.reshape(B, T, H * dk)
    out["db_gate"] = dz.sum(axis=(0, 1)).reshape(H * dk)
    out["dA"] = da.sum(axis=(0, 1, 3))
    bt = _sigmoid(np.asarray(beta_logit, np.float64))
    out["dbeta_logit"] = np.asarray(dbeta, np.float64) * bt * (1.0 - bt)
    return out


# ---------------------------------------------------------------------------
# output gate (epilogue)
# ---------------------------------------------------------------------------


def gated_rmsnorm(o, gate, eps=RMS_EPS):
    """``sigmoid(gate) * headwise_rms_norm(o)`` for ``o [..., H, dv]`` and
    gate logits of the same shape (``net/kda.py:206-214``)."""
    return _sigmoid(gate) * headwise_rms_norm(o, eps)


def gated_rmsnorm_bwd(o, gate, dy, eps=RMS_EPS):
    """``(do, dgate)`` of ``gated_rmsnorm``."""
    o = np.asarray(o, np.float64)
    r = 1.0 / np.sqrt(np.mean(o * o, axis=-1, keepdims=True) + eps)
    n = o * r
    s = _sigmoid(np.asarray(gate, np.float64))
    dgate = dy * n * s * (1.0 - s)
    dn = dy * s
    do = r * (dn - n * np.mean(dn * n, axis=-1, keepdims=True))
    return do, dgate


# ---------------------------------------------------------------------------
# fused decode step
# ---------------------------------------------------------------------------


def decode_fused_step(S, conv_buf, qp, kp, vp, z, beta_logit, wq, wk, wv, b_gate, A, H, dk, dv,
                      g_min=G_MIN, kind=GATE_SIGMOID_MIN, gate_logit=None):
    """One token for ``N`` sequences (``recurrent_step`` ``net/kda.py:277-295``
    without the projection GEMMs): ShortConv steps on the buffers, Swish, L2
    norm, gates, the delta-rule update and ``o = S^T q`` (then the output gate
    when ``gate_logit`` is given).  ``S [N,H,dk,dv]``, ``conv_buf
    [N,K-1,H*(2dk+dv)]``, ``qp, kp, z [N,H*dk]``, ``vp [N,H*dv]``,
    ``beta_logit [N,H]``.  Returns ``(S', conv_buf', out [N,H,dv])``."""
    from oracle.kda_oracle import decode_step

    N = S.shape[0]
    K = wq.shape[0]
    nq = H * dk
    Sn = np.array(S, np.float64)
    bufn = np.array(conv_buf, np.float64)
    out = np.zeros((N, H, dv))
    for n in range(N):
        bq, bk, bv = bufn[n][:, :nq], bufn[n][:, nq:2 * nq], bufn[n][:, 2 * nq:]
        cq, bq = short_conv_step(np.asarray(qp[n], np.float64), wq, bq)
        ck, bk = short_conv_step(np.asarray(kp[n], np.float64), wk, bk)
        cv, bv = short_conv_step(np.asarray(vp[n], np.float64), wv, bv)
        if K > 1:
            bufn[n] = np.concatenate([bq, bk, bv], axis=1)
        q = l2_norm(swish(cq).reshape(H, dk))
        k = l2_norm(swish(ck).reshape(H, dk))
        v = swish(cv).reshape(H, dv)
        g = decay_gate(np.asarray(z[n], np.float64).reshape(H, dk), np.asarray(b_gate).reshape(H, dk),
                       np.asarray(A, np.float64), g_min, kind)
        beta = _sigmoid(np.asarray(beta_logit[n], np.float64))
        o, s_new = decode_step(Sn[n], q, k, v, g, beta)
        Sn[n] = s_new
        out[n] = o if gate_logit is None else gated_rmsnorm(o, np.asarray(gate_logit[n], np.float64).reshape(H, dv))
    return Sn, bufn, out


# ---------------------------------------------------------------------------
# the whole layer: projections -> prologue -> core -> output gate -> W_o
# ---------------------------------------------------------------------------


def layer_fwd(P, x, H, cu_seqlens=None, kind=GATE_SOFTPLUS, g_min=G_MIN, chunk=64, tile="reference"):
    """``apply_kda`` of one layer (``net/kda.py:929-946`` with ``_project``
    :157-191, ``_postprocess`` :194-203 and ``_output_gate`` :206-214) over
    ``x [T, d_model]``, float64.  ``P`` maps the weight names of
    ``axiom_b200.layer.KDALayerParams`` to arrays.  Returns ``(out, cache)``;
    ``cache`` feeds :func:`layer_bwd`.  ``tile``: the core's score evaluation,
    the reference's tile-anchored one with its exponent clamp (default) or
    ``None`` for the direct decay ratio, exact for any decay (the clamp binds
    once a 16-token tile's summed decay passes 80, e.g. per-token decays of
    ~5 and more)."""
    from oracle.kda_oracle import TILE, chunk_fwd

    tile = TILE if tile == "reference" else tile

    x = np.asarray(x, np.float64)
    T = x.shape[0]
    dk = P["W_q"].shape[1] // H
    dv = P["W_v"].shape[1] // H
    a_down = x @ P["W_a_down"]
    proj = dict(qp=x @ P["W_q"], kp=x @ P["W_k"], vp=x @ P["W_v"], z=a_down @ P["W_a_up"], bl=x @ P["W_beta"],
                gl=x @ P["W_g"])
    pro = prologue_fwd(proj["qp"][None], proj["kp"][None], proj["vp"][None], proj["z"][None], proj["bl"][None],
                       P["conv_q"], P["conv_k"], P["conv_v"], P["b_gate"], P["A"], H, dk, dv, g_min=g_min, kind=kind,
                       cu_seqlens=cu_seqlens)
    cu = [0, T] if cu_seqlens is None else [int(c) for c in cu_seqlens]
    o = np.zeros((T, H, dv))
    for a, b in zip(cu[:-1], cu[1:]):
        if b > a:
            o[a:b] = chunk_fwd(*(pro[n][:, a:b] for n in ("q", "k", "v", "g", "beta")), None, chunk=chunk,
                               tile=tile)[0][0]
    y = gated_rmsnorm(o, proj["gl"].reshape(T, H, dv)).reshape(T, H * dv)
    cache = dict(x=x, a_down=a_down, proj=proj, pro=pro, o=o, y=y, cu=cu, H=H, dk=dk, dv=dv, kind=kind,
                 g_min=g_min, chunk=chunk, tile=tile, cu_seqlens=cu_seqlens)
    return y @ P["W_o"], cache


def layer_bwd(P, cache, dout):
    """Cotangents of :func:`layer_fwd`'s input and weights for ``dout``:
    ``{"x": ..., <weight name>: ...}`` -- the VJPs of the pieces composed."""
    from oracle.kda_oracle import chunk_bwd

    x, proj, pro, o, y, cu = (cache[n] for n in ("x", "proj", "pro", "o", "y", "cu"))
    H, dk, dv = cache["H"], cache["dk"], cache["dv"]
    T = x.shape[0]
    dout = np.asarray(dout, np.float64)
    g = {"W_o": y.T @ dout}
    dy = (dout @ P["W_o"].T).reshape(T, H, dv)
    do, dgl = gated_rmsnorm_bwd(o, proj["gl"].reshape(T, H, dv), dy)
    c = {n: np.zeros_like(pro[n]) for n in ("q", "k", "v", "g", "beta")}
    for a, b in zip(cu[:-1], cu[1:]):
        if b > a:
            r = chunk_bwd(*(pro[n][:, a:b] for n in ("q", "k", "v", "g", "beta")), None, do[a:b][None], None,
                          chunk=cache["chunk"], tile=cache["tile"])
            for n, d in zip(("q", "k", "v", "g", "beta"), r[:5]):
                c[n][:, a:b] = d
    pb = prologue_bwd(proj["qp"][None], proj["kp"][None], proj["vp"][None], proj["z"][None], proj["bl"][None],
                      P["conv_q"], P["conv_k"], P["conv_v"], P["b_gate"], P["A"], H, dk, dv, c["q"], c["k"], c["v"],
                      c["g"], c["beta"], g_min=cache["g_min"], kind=cache["kind"], cu_seqlens=cache["cu_seqlens"])
    d = dict(qp=pb["dqp"][0], kp=pb["dkp"][0], vp=pb["dvp"][0], z=pb["dz"][0], bl=pb["dbeta_logit"][0],
             gl=dgl.reshape(T, H * dv))
    da_down = d["z"] @ P["W_a_up"].T
    g.update(W_q=x.T @ d["qp"], W_k=x.T @ d["kp"], W_v=x.T @ d["vp"], W_g=x.T @ d["gl"], W_beta=x.T @ d["bl"],
             W_a_up=cache["a_down"].T @ d["z"], W_a_down=x.T @ da_down, conv_q=pb["dwq"], conv_k=pb["dwk"],
             conv_v=pb["dwv"], b_gate=pb["db_gate"], A=pb["dA"])
    g["x"] = (d["qp"] @ P["W_q"].T + d["kp"] @ P["W_k"].T + d["vp"] @ P["W_v"].T + d["gl"] @ P["W_g"].T
              + d["bl"] @ P["W_beta"].T + da_down @ P["W_a_down"].T)
    return g
