"""The mixer oracle (prologue, output gate, fused decode step) pinned against
fixtures made by executing the reference's own source
(``tests/golden/make_golden_mixer.py``), and its backward rules against
float64 finite differences (the reference's gradient check,
``net/tests/test_kda_chunked_cc.py:333-391``).  CPU only."""

import os

import numpy as np
import pytest

from oracle import mixer_oracle as M

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_mixer.npz"))


def _close(a, b, tol=1e-12):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.max(np.abs(a - b)) <= tol * max(1.0, float(np.max(np.abs(b)))), np.max(np.abs(a - b))


def test_short_conv_matches_reference_and_streaming_form():
    x, w = GOLDEN["conv/x"], GOLDEN["conv/w"]
    _close(M.short_conv(x, w), GOLDEN["conv/out"])
    buf = np.zeros((w.shape[0] - 1, x.shape[1]))
    steps = []
    for t in range(x.shape[0]):
        o, buf = M.short_conv_step(x[t], w, buf)
        steps.append(o)
    _close(np.stack(steps), GOLDEN["conv/steps"])
    _close(buf, GOLDEN["conv/buf"])
    _close(M.short_conv_state_out(x, None, w.shape[0]), GOLDEN["conv/buf"])


def test_short_conv_state_continues_a_sequence():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((20, 6))
    w = rng.standard_normal((4, 6))
    whole = M.short_conv(x, w)
    st = M.short_conv_state_out(x[:9], None, 4)
    _close(M.short_conv(x[9:], w, state=st), whole[9:])
    _close(M.short_conv_state_out(x[9:], st, 4), M.short_conv_state_out(x, None, 4))
    # a state longer than the sequence (T < K - 1)
    st2 = M.short_conv_state_out(x[9:11], st, 4)
    _close(st2, x[8:11])


def test_varlen_conv_restarts_every_sequence():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((30, 5))
    w = rng.standard_normal((4, 5))
    cu = [0, 7, 8, 19, 30]
    got = M.short_conv(x, w, cu_seqlens=cu)
    ref = np.concatenate([M.short_conv(x[a:b], w) for a, b in zip(cu[:-1], cu[1:])])
    _close(got, ref)


def test_norms_and_swish_match_reference():
    x = GOLDEN["norm/x"]
    _close(M.swish(x), GOLDEN["norm/swish"])
    _close(M.l2_norm(x), GOLDEN["norm/l2"])
    _close(M.headwise_rms_norm(x), GOLDEN["norm/rms"])
    # the reference's derivative rule; the Jacobian is symmetric, so it is the VJP
    _close(M.l2_norm_vjp(x, GOLDEN["norm/xdot"]), GOLDEN["norm/l2_tangent"])


def test_postprocess_and_gate_match_reference():
    H, dk, dv = 2, 16, 8
    qp, kp, vp = GOLDEN["post/qp"], GOLDEN["post/kp"], GOLDEN["post/vp"]
    one = lambda d: np.ones((1, H * d))  # noqa: E731  K = 1, identity conv
    T = qp.shape[0]
    res = M.prologue_fwd(qp[None], kp[None], vp[None], np.zeros((1, T, H * dk)), np.zeros((1, T, H)),
                         one(dk), one(dk), one(dv), np.zeros(H * dk), np.zeros(H), H, dk, dv)
    _close(res["q"][0], GOLDEN["post/q"])
    _close(res["k"][0], GOLDEN["post/k"])
    _close(res["v"][0], GOLDEN["post/v"])
    z, A = GOLDEN["gate/z"], GOLDEN["gate/A"]
    _close(M.decay_gate(z, np.zeros((H, dk)), A, -5.0, M.GATE_SIGMOID_MIN), GOLDEN["gate/g"])


def test_output_gate_matches_reference():
    o, gate = GOLDEN["ogate/o"], GOLDEN["ogate/gate"]
    logit = np.log(gate / (1.0 - gate)).reshape(o.shape)
    _close(M.gated_rmsnorm(o, logit).reshape(o.shape[0], -1), GOLDEN["ogate/y"], 1e-10)


def test_fused_decode_matches_reference_recurrent_step():
    G = {k.split("/", 1)[1]: GOLDEN[k] for k in GOLDEN.files if k.startswith("rec/")}
    H, dk, dv = 2, 16, 8
    S = G["S0"][None]
    buf = np.concatenate([G["q_buf0"], G["k_buf0"], G["v_buf0"]], axis=1)[None]
    outs = []
    for t in range(G["x"].shape[0]):
        x = G["x"][t][None]
        S, buf, y = M.decode_fused_step(
            S, buf, x @ G["W_q"], x @ G["W_k"], x @ G["W_v"], (x @ G["W_a_down"]) @ G["W_a_up"],
            x @ G["W_beta"], G["conv_q"], G["conv_k"], G["conv_v"], G["b_alpha"], G["A"], H, dk, dv,
            gate_logit=x @ G["W_g"])
        outs.append(y.reshape(1, H * dv) @ G["W_o"])
    _close(np.concatenate(outs), G["out"], 1e-10)
    _close(S[0], G["S"], 1e-10)
    nq = H * dk
    _close(buf[0][:, :nq], G["q_buf"])
    _close(buf[0][:, nq:2 * nq], G["k_buf"])
    _close(buf[0][:, 2 * nq:], G["v_buf"])


def _prologue_case(seed, kind, state, varlen):
    rng = np.random.default_rng(seed)
    B, T, H, dk, dv, K = (1 if varlen else 2), 13, 2, 8, 4, 4
    x = dict(qp=rng.standard_normal((B, T, H * dk)), kp=rng.standard_normal((B, T, H * dk)),
             vp=rng.standard_normal((B, T, H * dv)), z=rng.standard_normal((B, T, H * dk)),
             beta_logit=rng.standard_normal((B, T, H)))
    w = dict(wq=rng.standard_normal((K, H * dk)) * 0.5, wk=rng.standard_normal((K, H * dk)) * 0.5,
             wv=rng.standard_normal((K, H * dv)) * 0.5, b_gate=rng.standard_normal(H * dk) * 0.3,
             A=rng.standard_normal(H) * 0.3)
    st = rng.standard_normal((B, K - 1, H * (2 * dk + dv))) if state else None
    cu = [0, 4, 5, 13] if varlen else None
    cot = dict(dq=rng.standard_normal((B, T, H, dk)), dk_=rng.standard_normal((B, T, H, dk)),
               dv_=rng.standard_normal((B, T, H, dv)), dg=rng.standard_normal((B, T, H, dk)),
               dbeta=rng.standard_normal((B, T, H)))
    return x, w, st, cu, cot, (H, dk, dv)


@pytest.mark.parametrize("kind,state,varlen", [(M.GATE_SIGMOID_MIN, False, False),
                                               (M.GATE_SOFTPLUS, True, False),
                                               (M.GATE_SIGMOID_MIN, False, True)])
def test_prologue_bwd_matches_finite_differences(kind, state, varlen):
    x, w, st, cu, cot, (H, dk, dv) = _prologue_case(3, kind, state, varlen)

    def loss(xx, ww, ss):
        r = M.prologue_fwd(xx["qp"], xx["kp"], xx["vp"], xx["z"], xx["beta_logit"], ww["wq"], ww["wk"],
                           ww["wv"], ww["b_gate"], ww["A"], H, dk, dv, kind=kind, state=ss, cu_seqlens=cu)
        return (np.sum(r["q"] * cot["dq"]) + np.sum(r["k"] * cot["dk_"]) + np.sum(r["v"] * cot["dv_"])
                + np.sum(r["g"] * cot["dg"]) + np.sum(r["beta"] * cot["dbeta"]))

    g = M.prologue_bwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["wq"], w["wk"], w["wv"],
                       w["b_gate"], w["A"], H, dk, dv, cot["dq"], cot["dk_"], cot["dv_"], cot["dg"],
                       cot["dbeta"], kind=kind, state=st, cu_seqlens=cu)
    rng = np.random.default_rng(7)
    eps = 1e-6
    probes = [("x", n, d) for n, d in (("qp", "dqp"), ("kp", "dkp"), ("vp", "dvp"), ("z", "dz"),
                                       ("beta_logit", "dbeta_logit"))]
    probes += [("w", n, d) for n, d in (("wq", "dwq"), ("wk", "dwk"), ("wv", "dwv"), ("b_gate", "db_gate"),
                                        ("A", "dA"))]
    if state:
        probes.append(("s", None, "dstate"))
    for src, name, gname in probes:
        for _ in range(4):
            base = {"x": x, "w": w}.get(src)
            arr = st if src == "s" else base[name]
            idx = tuple(int(rng.integers(0, n)) for n in arr.shape)
            plus, minus = arr.copy(), arr.copy()
            plus[idx] += eps
            minus[idx] -= eps

            def ev(a):
                if src == "s":
                    return loss(x, w, a)
                nb = dict(base)
                nb[name] = a
                return loss(nb, w, st) if src == "x" else loss(x, nb, st)

            fd = (ev(plus) - ev(minus)) / (2 * eps)
            assert abs(fd - g[gname][idx]) < 1e-6 * max(1.0, abs(fd)), (gname, idx, fd, g[gname][idx])


def test_gated_rmsnorm_bwd_matches_finite_differences():
    rng = np.random.default_rng(4)
    o = rng.standard_normal((5, 2, 8))
    gl = rng.standard_normal((5, 2, 8))
    dy = rng.standard_normal((5, 2, 8))
    do, dgate = M.gated_rmsnorm_bwd(o, gl, dy)
    eps = 1e-6
    for arr, grad, which in ((o, do, 0), (gl, dgate, 1)):
        for _ in range(6):
            idx = tuple(int(rng.integers(0, n)) for n in arr.shape)
            p, m = arr.copy(), arr.copy()
            p[idx] += eps
            m[idx] -= eps
            f = (lambda a: np.sum(M.gated_rmsnorm(a, gl) * dy)) if which == 0 else (
                lambda a: np.sum(M.gated_rmsnorm(o, a) * dy))
            fd = (f(p) - f(m)) / (2 * eps)
            assert abs(fd - grad[idx]) < 1e-7 * max(1.0, abs(fd))


def _layer_case(seed):
    rng = np.random.default_rng(seed)
    d, H, dk, dv, r, K, T = 12, 2, 8, 4, 3, 4, 11
    P = dict(W_q=rng.standard_normal((d, H * dk)) * 0.3, W_k=rng.standard_normal((d, H * dk)) * 0.3,
             W_v=rng.standard_normal((d, H * dv)) * 0.3, W_g=rng.standard_normal((d, H * dv)) * 0.3,
             W_beta=rng.standard_normal((d, H)) * 0.3, W_a_down=rng.standard_normal((d, r)) * 0.3,
             W_a_up=rng.standard_normal((r, H * dk)) * 0.3, b_gate=rng.standard_normal(H * dk) * 0.2,
             A=rng.standard_normal(H) * 0.2, conv_q=rng.standard_normal((K, H * dk)) * 0.4,
             conv_k=rng.standard_normal((K, H * dk)) * 0.4, conv_v=rng.standard_normal((K, H * dv)) * 0.4,
             W_o=rng.standard_normal((H * dv, d)) * 0.3)
    return P, rng.standard_normal((T, d)), rng.standard_normal((T, d)), H


@pytest.mark.parametrize("cu,kind", [([0, 4, 4, 11], M.GATE_SOFTPLUS), (None, M.GATE_SIGMOID_MIN)])
def test_layer_bwd_matches_finite_differences(cu, kind):
    P, x, dout, H = _layer_case(0)
    out, cache = M.layer_fwd(P, x, H, cu, kind=kind, chunk=4)
    g = M.layer_bwd(P, cache, dout)

    def loss(P2, x2):
        return float(np.sum(M.layer_fwd(P2, x2, H, cu, kind=kind, chunk=4)[0] * dout))

    rng = np.random.default_rng(1)
    eps = 1e-6
    for name in list(P) + ["x"]:
        arr = x if name == "x" else P[name]
        for _ in range(2):
            idx = tuple(int(rng.integers(0, n)) for n in arr.shape)
            p, m = arr.copy(), arr.copy()
            p[idx] += eps
            m[idx] -= eps
            if name == "x":
                fd = (loss(P, p) - loss(P, m)) / (2 * eps)
            else:
                fd = (loss({**P, name: p}, x) - loss({**P, name: m}, x)) / (2 * eps)
            assert abs(fd - g[name][idx]) < 1e-6 * max(1.0, abs(fd)), (name, idx)
