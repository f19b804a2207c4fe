"""Parity of the mixer kernels (prologue, output gate, fused decode step) with
the oracle (``oracle/mixer_oracle.py``, pinned to the reference's source by
``tests/test_mixer_oracle.py``), through the C ABI of ``include/kda_mixer.h``.

Tolerances (scale-relative ``max|x - ref| / max|ref|``, the reference's
convention): fp32 tensors 1e-4; bf16 tensors 1e-2 (the BASELINE bound);
bf16 outputs are compared with the oracle run on the same bf16-rounded inputs.
"""

import numpy as np
import pytest
import torch

from oracle import mixer_oracle as M
from oracle.kda_oracle import bf16_round, scale_rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _tol(dt):
    return 1e-4 if dt == torch.float32 else 1e-2


def _t(x, dt):
    return torch.as_tensor(np.ascontiguousarray(x)).to(DEV).to(dt).contiguous()


def _np(x):
    return x.detach().float().cpu().numpy().astype(np.float64)


def _case(seed, B, T, H, dk, dv, K, dt, state=False):
    rng = np.random.default_rng(seed)
    r = (lambda a: bf16_round(a).astype(np.float64)) if dt == torch.bfloat16 else (lambda a: a.astype(np.float32).astype(np.float64))
    x = dict(qp=r(rng.standard_normal((B, T, H * dk))), kp=r(rng.standard_normal((B, T, H * dk))),
             vp=r(rng.standard_normal((B, T, H * dv))), z=r(rng.standard_normal((B, T, H * dk)) * 1.5),
             beta_logit=r(rng.standard_normal((B, T, H))))
    f32 = lambda a: a.astype(np.float32).astype(np.float64)  # noqa: E731
    w = dict(conv_q=f32(rng.standard_normal((K, H * dk)) * 0.5), conv_k=f32(rng.standard_normal((K, H * dk)) * 0.5),
             conv_v=f32(rng.standard_normal((K, H * dv)) * 0.5), b_gate=f32(rng.standard_normal(H * dk) * 0.3),
             A=f32(rng.standard_normal(H) * 0.3))
    st = f32(rng.standard_normal((B, K - 1, H * (2 * dk + dv)))) if state and K > 1 else None
    return x, w, st


def _run_fwd(x, w, st, H, dt, kind, cu=None, return_state=False):
    tx = {k: _t(v, dt) for k, v in x.items()}
    tw = {k: _t(v, torch.float32) for k, v in w.items()}
    from axiom_b200 import mixer

    return mixer.prologue_fwd(tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"], tw["conv_k"],
                              tw["conv_v"], tw["A"], H=H, b_gate=tw["b_gate"], gate_kind=kind,
                              conv_state=None if st is None else _t(st, torch.float32),
                              return_state=return_state,
                              cu_seqlens=None if cu is None else torch.tensor(cu, dtype=torch.int32))


KINDS = {"sigmoid_min": M.GATE_SIGMOID_MIN, "softplus": M.GATE_SOFTPLUS}


@pytest.mark.parametrize("B,T,H,dk,dv,K,dt,kind,state", [
    (2, 200, 2, 128, 128, 4, torch.bfloat16, "sigmoid_min", False),
    (1, 130, 3, 64, 128, 3, torch.float32, "softplus", True),
    (2, 64, 2, 128, 64, 2, torch.float32, "sigmoid_min", True),
    (1, 2, 2, 64, 64, 4, torch.float32, "softplus", True),     # T < K - 1: the state shifts through
    (1, 77, 1, 128, 128, 1, torch.bfloat16, "softplus", False),
    (1, 150, 2, 64, 64, 4, torch.bfloat16, "softplus", True),    # two channels per lane, bf16
])
def test_prologue_fwd_matches_oracle(B, T, H, dk, dv, K, dt, kind, state):
    x, w, st = _case(1, B, T, H, dk, dv, K, dt, state)
    q, k, v, g, beta, st_out = _run_fwd(x, w, st, H, dt, kind, return_state=True)
    ref = M.prologue_fwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                         w["b_gate"], w["A"], H, dk, dv, kind=KINDS[kind], state=st)
    for name, got in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        assert scale_rel_err(_np(got), ref[name]) <= _tol(dt), name
    if K > 1:
        assert scale_rel_err(_np(st_out), ref["state_out"]) <= 1e-6  # copies of the inputs


@pytest.mark.parametrize("cu,dt", [
    ([0, 5, 6, 70, 200, 300], torch.float32),
    # empty sequences inside the pack, two starting at the same token, and a
    # boundary inside an 8-token batch of a 256-token strip
    ([0, 5, 5, 70, 70, 70, 203, 300], torch.float32),
    ([0, 0, 1, 9, 9, 261, 300, 300], torch.bfloat16),
])
def test_prologue_varlen_restarts_each_sequence(cu, dt):
    H, dk, dv, K, T = 2, 128, 128, 4, 300
    x, w, _ = _case(2, 1, T, H, dk, dv, K, dt)
    q, k, v, g, beta = _run_fwd(x, w, None, H, dt, "sigmoid_min", cu=cu)
    ref = M.prologue_fwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                         w["b_gate"], w["A"], H, dk, dv, cu_seqlens=cu)
    for name, got in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        assert scale_rel_err(_np(got), ref[name]) <= (1e-4 if dt == torch.float32 else 1e-2), name


@pytest.mark.parametrize("B,T,H,dk,dv,K,dt,kind,state,cu", [
    (2, 200, 2, 128, 128, 4, torch.float32, "sigmoid_min", True, None),
    (1, 150, 2, 64, 128, 3, torch.float32, "softplus", False, None),
    (1, 260, 2, 128, 128, 4, torch.float32, "sigmoid_min", False, [0, 40, 41, 190, 260]),
    (1, 300, 2, 128, 128, 4, torch.bfloat16, "softplus", False, [0, 5, 5, 70, 70, 70, 203, 300]),
    (2, 130, 2, 128, 128, 4, torch.bfloat16, "sigmoid_min", False, None),
    (1, 3, 1, 64, 64, 4, torch.float32, "softplus", True, None),
    (1, 140, 2, 64, 64, 4, torch.bfloat16, "sigmoid_min", True, None),
    (1, 270, 2, 64, 64, 3, torch.bfloat16, "softplus", False, [0, 100, 100, 133, 270]),
])
def test_prologue_bwd_matches_oracle(B, T, H, dk, dv, K, dt, kind, state, cu):
    from axiom_b200 import mixer

    x, w, st = _case(3, B, T, H, dk, dv, K, dt, state)
    rng = np.random.default_rng(9)
    r = (lambda a: bf16_round(a).astype(np.float64)) if dt == torch.bfloat16 else (lambda a: a.astype(np.float32).astype(np.float64))
    cot = dict(dq=r(rng.standard_normal((B, T, H, dk))), dk=r(rng.standard_normal((B, T, H, dk))),
               dv=r(rng.standard_normal((B, T, H, dv))), dg=r(rng.standard_normal((B, T, H, dk))),
               dbeta=r(rng.standard_normal((B, T, H))))
    tx = {k_: _t(v_, dt) for k_, v_ in x.items()}
    tw = {k_: _t(v_, torch.float32) for k_, v_ in w.items()}
    tc = {k_: _t(v_, dt) for k_, v_ in cot.items()}
    got = mixer.prologue_bwd(tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"], tw["conv_k"],
                             tw["conv_v"], tw["A"], tc["dq"], tc["dk"], tc["dv"], tc["dg"], tc["dbeta"], H=H,
                             b_gate=tw["b_gate"], gate_kind=kind,
                             conv_state=None if st is None else _t(st, torch.float32),
                             cu_seqlens=None if cu is None else torch.tensor(cu, dtype=torch.int32))
    ref = M.prologue_bwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                         w["b_gate"], w["A"], H, dk, dv, cot["dq"], cot["dk"], cot["dv"], cot["dg"], cot["dbeta"],
                         kind=KINDS[kind], state=st, cu_seqlens=cu)
    pairs = [("dqp", "dqp"), ("dkp", "dkp"), ("dvp", "dvp"), ("dz", "dz"), ("dbeta_logit", "dbeta_logit"),
             ("dconv_q", "dwq"), ("dconv_k", "dwk"), ("dconv_v", "dwv"), ("db_gate", "db_gate"), ("dA", "dA")]
    if state:
        pairs.append(("dconv_state", "dstate"))
    for a, b in pairs:
        tol = _tol(dt) if a in ("dqp", "dkp", "dvp", "dz", "dbeta_logit") else (1e-4 if dt == torch.float32 else 1e-2)
        assert scale_rel_err(_np(got[a]), ref[b]) <= tol, a


def test_prologue_autograd_through_the_core_inputs():
    """kda_prologue's backward equals prologue_bwd fed with autograd's cotangents."""
    from axiom_b200 import mixer

    H, dk, dv, K, T = 2, 128, 128, 4, 96
    x, w, _ = _case(4, 1, T, H, dk, dv, K, torch.float32)
    tx = {k_: _t(v_, torch.float32).requires_grad_(True) for k_, v_ in x.items()}
    tw = {k_: _t(v_, torch.float32).requires_grad_(True) for k_, v_ in w.items()}
    outs = mixer.kda_prologue(tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"], tw["conv_k"],
                              tw["conv_v"], tw["A"], H=H, b_gate=tw["b_gate"])
    gen = torch.Generator(device=DEV).manual_seed(0)
    cots = [torch.randn(o.shape, device=DEV, generator=gen) for o in outs]
    torch.autograd.backward(outs, cots)
    ref = M.prologue_bwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                         w["b_gate"], w["A"], H, dk, dv, *[_np(c) for c in cots])
    for t_, name in ((tx["qp"], "dqp"), (tx["z"], "dz"), (tw["conv_k"], "dwk"), (tw["A"], "dA"),
                     (tw["b_gate"], "db_gate")):
        assert scale_rel_err(_np(t_.grad), ref[name]) <= 1e-4, name


@pytest.mark.parametrize("odt,gdt,dv", [(torch.float32, torch.float32, 128), (torch.bfloat16, torch.bfloat16, 128),
                                        (torch.float32, torch.bfloat16, 64)])
def test_gated_rmsnorm_matches_oracle(odt, gdt, dv):
    from axiom_b200 import mixer

    rng = np.random.default_rng(5)
    N, H = 333, 3
    r = lambda a, d: bf16_round(a).astype(np.float64) if d == torch.bfloat16 else a.astype(np.float32).astype(np.float64)  # noqa: E731
    o = r(rng.standard_normal((N, H, dv)) * 2.0, odt)
    gl = r(rng.standard_normal((N, H * dv)), gdt)
    dy = r(rng.standard_normal((N, H * dv)), gdt)
    y = mixer.gated_rmsnorm_fwd(_t(o, odt), _t(gl, gdt))
    ref = M.gated_rmsnorm(o, gl.reshape(N, H, dv)).reshape(N, H * dv)
    tol = 1e-4 if gdt == torch.float32 else 1e-2
    assert scale_rel_err(_np(y), ref) <= tol
    do, dgate = mixer.gated_rmsnorm_bwd(_t(o, odt), _t(gl, gdt), _t(dy, gdt))
    rdo, rdg = M.gated_rmsnorm_bwd(o, gl.reshape(N, H, dv), dy.reshape(N, H, dv))
    assert scale_rel_err(_np(do), rdo) <= (1e-4 if odt == torch.float32 and gdt == torch.float32 else 1e-2)
    assert scale_rel_err(_np(dgate).reshape(N, H, dv), rdg) <= tol


@pytest.mark.parametrize("dk,dv,K,dt,gated,kind", [
    (128, 128, 4, torch.float32, True, "sigmoid_min"),
    (64, 128, 3, torch.float32, False, "softplus"),
    (128, 64, 1, torch.float32, True, "softplus"),
    (128, 128, 4, torch.bfloat16, True, "sigmoid_min"),
])
def test_decode_fused_matches_oracle(dk, dv, K, dt, gated, kind):
    from axiom_b200 import mixer

    rng = np.random.default_rng(6)
    N, H, steps = 5, 3, 4
    r = (lambda a: bf16_round(a).astype(np.float64)) if dt == torch.bfloat16 else (lambda a: a.astype(np.float32).astype(np.float64))
    f32 = lambda a: a.astype(np.float32).astype(np.float64)  # noqa: E731
    w = dict(conv_q=f32(rng.standard_normal((K, H * dk)) * 0.5), conv_k=f32(rng.standard_normal((K, H * dk)) * 0.5),
             conv_v=f32(rng.standard_normal((K, H * dv)) * 0.5), b_gate=f32(rng.standard_normal(H * dk) * 0.3),
             A=f32(rng.standard_normal(H) * 0.3))
    S = f32(rng.standard_normal((N, H, dk, dv)) * 0.05)
    buf = f32(rng.standard_normal((N, K - 1, H * (2 * dk + dv))))
    tS, tb = _t(S, torch.float32), _t(buf, torch.float32)
    tw = {k_: _t(v_, torch.float32) for k_, v_ in w.items()}
    for _ in range(steps):
        x = dict(qp=r(rng.standard_normal((N, H * dk))), kp=r(rng.standard_normal((N, H * dk))),
                 vp=r(rng.standard_normal((N, H * dv))), z=r(rng.standard_normal((N, H * dk))),
                 beta_logit=r(rng.standard_normal((N, H))), gate=r(rng.standard_normal((N, H * dv))))
        tx = {k_: _t(v_, dt) for k_, v_ in x.items()}
        out = mixer.decode_fused(tS, tb, tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"],
                                 tw["conv_k"], tw["conv_v"], tw["A"], H=H, b_gate=tw["b_gate"],
                                 gate_logit=tx["gate"] if gated else None, gate_kind=kind,
                                 out_dtype=torch.float32)
        S, buf, ref = M.decode_fused_step(S, buf, x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"],
                                          w["conv_k"], w["conv_v"], w["b_gate"], w["A"], H, dk, dv, kind=KINDS[kind],
                                          gate_logit=x["gate"] if gated else None)
        assert scale_rel_err(_np(out), ref) <= 1e-4
    assert scale_rel_err(_np(tS), S) <= 1e-4
    if K > 1:
        assert scale_rel_err(_np(tb), buf) <= 1e-6


def test_decode_fused_matches_reference_recurrent_step():
    """The reference's own recurrent_step (golden, executed from its source)
    with its projections done by torch: one layer, a few tokens."""
    import os

    from axiom_b200 import mixer

    G0 = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_mixer.npz"))
    G = {k.split("/", 1)[1]: G0[k] for k in G0.files if k.startswith("rec/")}
    H, dk, dv = 2, 16, 8
    assert G["out"].shape == (G["x"].shape[0], H * dv)
    # the kernels take d in {64, 128}: the fixture's 16/8-wide heads are embedded
    # in 64-wide ones by zero columns, which is exact (zero projections and conv
    # weights give zero q, k, v channels; they add nothing to the L2 norms, the
    # state rows and columns they touch stay zero, and o's extra columns are zero)
    dkp, dvp = 64, 64
    f = lambda a: torch.as_tensor(a, dtype=torch.float32, device=DEV)  # noqa: E731

    def pad_cols(Wm, d, dp):  # [hid, H*d] -> [hid, H*dp]
        out = np.zeros((Wm.shape[0], H * dp))
        for h in range(H):
            out[:, h * dp:h * dp + d] = Wm[:, h * d:(h + 1) * d]
        return out

    S = np.zeros((1, H, dkp, dvp))
    S[0, :, :dk, :dv] = G["S0"]
    buf = np.zeros((1, 3, H * (2 * dkp + dvp)))
    buf[0][:, :H * dkp] = pad_cols(G["q_buf0"], dk, dkp)
    buf[0][:, H * dkp:2 * H * dkp] = pad_cols(G["k_buf0"], dk, dkp)
    buf[0][:, 2 * H * dkp:] = pad_cols(G["v_buf0"], dv, dvp)
    tS, tb = f(S), f(buf)
    conv = {n: f(pad_cols(G[n], d, dp)) for n, d, dp in (("conv_q", dk, dkp), ("conv_k", dk, dkp), ("conv_v", dv, dvp))}
    b_gate = f(pad_cols(G["b_alpha"][None], dk, dkp)[0])
    outs = []
    for t in range(G["x"].shape[0]):
        x = G["x"][t][None]
        qp = f(pad_cols(x @ G["W_q"], dk, dkp))
        kp = f(pad_cols(x @ G["W_k"], dk, dkp))
        vp = f(pad_cols(x @ G["W_v"], dv, dvp))
        z = f(pad_cols((x @ G["W_a_down"]) @ G["W_a_up"], dk, dkp))
        o = mixer.decode_fused(tS, tb, qp, kp, vp, z, f(x @ G["W_beta"]), conv["conv_q"], conv["conv_k"],
                               conv["conv_v"], f(G["A"]), H=H, b_gate=b_gate, out_dtype=torch.float32)
        o = _np(o)[0][:, :dv]  # the padded value channels are exactly zero
        y = M.gated_rmsnorm(o, (x @ G["W_g"]).reshape(H, dv))
        outs.append(y.reshape(1, H * dv) @ G["W_o"])
    assert scale_rel_err(np.concatenate(outs), G["out"]) <= 1e-4
    assert scale_rel_err(_np(tS)[0][:, :dk, :dv], G["S"]) <= 1e-4
