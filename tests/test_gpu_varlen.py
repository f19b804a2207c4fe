"""Packed (variable-length) sequences through the C ABI: the KDA core over the
chunk-aligned packed layout (``kda_fwd_varlen`` / ``kda_bwd_varlen``), the
prologue writing that layout (``out_rows``) and the output gate reading it.
Each sequence must equal the oracle run on that sequence alone; pad rows must
stay zero.  Tolerances are the scale-relative bounds of ``test_gpu_parity``:
bf16 1e-2, fp32 1e-4.
"""

import numpy as np
import pytest
import torch

from oracle import kda_oracle as K
from oracle import mixer_oracle as M

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
LENS = [100, 1, 64, 0, 200, 37]


def _pack(x, cu, rows, T_pad):
    """[n_tok, ...] packed rows -> [T_pad, ...] chunk-aligned rows (zero pads)."""
    out = np.zeros((T_pad,) + x.shape[1:], x.dtype)
    for s in range(len(cu) - 1):
        out[rows[s]:rows[s] + cu[s + 1] - cu[s]] = x[cu[s]:cu[s + 1]]
    return out


def _seq_inputs(seed, H, dk, dv, dt):
    from axiom_b200 import kda as KD

    cu = np.concatenate([[0], np.cumsum(LENS)]).astype(np.int64)
    n_tok = int(cu[-1])
    x = K.make_inputs(1, n_tok, H, dk, dv, seed=seed, s0_std=0.05)
    if dt == torch.bfloat16:
        x = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    rng = np.random.default_rng(seed + 1)
    S0 = (rng.standard_normal((len(LENS), H, dk, dv)) * 0.05).astype(np.float32)
    return cu, n_tok, x, S0


@pytest.mark.parametrize("dt,dk,dv,chunk", [(torch.bfloat16, 128, 128, 64), (torch.float32, 64, 32, 32)])
def test_varlen_core_matches_each_sequence(dt, dk, dv, chunk):
    from axiom_b200 import kda as KD

    H = 2
    cu, n_tok, x, S0 = _seq_inputs(3, H, dk, dv, dt)
    offs, rows, T_pad = KD.packing(cu.tolist(), chunk)
    t = {k: torch.as_tensor(_pack(x[k][0], cu, rows, T_pad)[None]).to(DEV).to(dt).contiguous()
         for k in ("q", "k", "v", "g", "beta")}
    S0_t = torch.as_tensor(S0).to(DEV)
    o, s_t, ckpt = KD.kda_fwd_varlen(t["q"], t["k"], t["v"], t["g"], t["beta"], offs, S0_t, chunk=chunk,
                                     o_dtype=torch.float32, need_ckpt=True)
    rng = np.random.default_rng(5)
    do_np = rng.standard_normal((n_tok, H, dv)).astype(np.float32)
    if dt == torch.bfloat16:
        do_np = K.bf16_round(do_np)
    dST = (rng.standard_normal((len(LENS), H, dk, dv)) * 0.1).astype(np.float32)
    do_t = torch.as_tensor(_pack(do_np, cu, rows, T_pad)[None]).to(DEV).to(dt).contiguous()
    grads = KD.kda_bwd_varlen(t["q"], t["k"], t["v"], t["g"], t["beta"], ckpt, do_t, offs,
                              torch.as_tensor(dST).to(DEV), chunk=chunk)
    o_np = o[0].float().cpu().numpy()
    tol = 1e-2 if dt == torch.bfloat16 else 1e-4
    for s, (a, b) in enumerate(zip(cu[:-1], cu[1:])):
        r0 = rows[s]
        ref_o, ref_s = K.chunk_fwd(*(x[k][:, a:b] for k in ("q", "k", "v", "g", "beta")), S0[s][None],
                                   chunk=chunk)
        if b > a:
            assert K.scale_rel_err(o_np[r0:r0 + b - a], ref_o[0]) <= tol, ("o", s)
        assert K.scale_rel_err(s_t[s].cpu().numpy(), ref_s[0]) <= tol, ("S_T", s)
        ref = K.chunk_bwd(*(x[k][:, a:b] for k in ("q", "k", "v", "g", "beta")), S0[s][None],
                          do_np[a:b][None], dST[s][None], chunk=chunk)
        for name, got, r in zip(("dq", "dk", "dv", "dg", "dbeta"), grads[:5], ref[:5]):
            if b > a:
                g_np = got[0].float().cpu().numpy()[r0:r0 + b - a]
                assert K.scale_rel_err(g_np, r[0]) <= tol, (name, s)
        assert K.scale_rel_err(grads[5][s].cpu().numpy(), ref[5][0]) <= tol, ("dS0", s)
    # the pad rows' outputs are the zero rows' outputs: zero
    real = np.zeros(T_pad, bool)
    for s in range(len(LENS)):
        real[rows[s]:rows[s] + LENS[s]] = True
    assert np.all(o_np[~real] == 0.0)


def test_prologue_writes_the_packed_layout_and_gate_reads_it():
    from axiom_b200 import kda as KD
    from axiom_b200 import mixer

    H, dk, dv, Kt = 2, 128, 128, 4
    cu = np.concatenate([[0], np.cumsum(LENS)]).astype(np.int64)
    n = int(cu[-1])
    offs, rows, T_pad = KD.packing(cu.tolist(), 64)
    rng = np.random.default_rng(7)
    f32 = lambda a: a.astype(np.float32).astype(np.float64)  # noqa: E731
    x = dict(qp=f32(rng.standard_normal((1, n, H * dk))), kp=f32(rng.standard_normal((1, n, H * dk))),
             vp=f32(rng.standard_normal((1, n, H * dv))), z=f32(rng.standard_normal((1, n, H * dk))),
             beta_logit=f32(rng.standard_normal((1, n, H))))
    w = dict(conv_q=f32(rng.standard_normal((Kt, H * dk)) * 0.5), conv_k=f32(rng.standard_normal((Kt, H * dk)) * 0.5),
             conv_v=f32(rng.standard_normal((Kt, H * dv)) * 0.5), b_gate=f32(rng.standard_normal(H * dk) * 0.3),
             A=f32(rng.standard_normal(H) * 0.3))
    tx = {k_: torch.as_tensor(v_, dtype=torch.float32, device=DEV) for k_, v_ in x.items()}
    tw = {k_: torch.as_tensor(v_, dtype=torch.float32, device=DEV) for k_, v_ in w.items()}
    cu_t = torch.as_tensor(cu, dtype=torch.int32)
    q, k, v, g, beta = mixer.prologue_fwd(tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"],
                                          tw["conv_k"], tw["conv_v"], tw["A"], H=H, b_gate=tw["b_gate"],
                                          cu_seqlens=cu_t, out_rows=rows)
    ref = M.prologue_fwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                         w["b_gate"], w["A"], H, dk, dv, cu_seqlens=cu)
    for name, got in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        want = _pack(ref[name][0], cu, rows, T_pad)
        assert K.scale_rel_err(got[0].cpu().numpy(), want) <= 1e-4, name
        pad = np.ones(T_pad, bool)
        for s in range(len(LENS)):
            pad[rows[s]:rows[s] + LENS[s]] = False
        assert np.all(got[0].cpu().numpy()[pad] == 0.0), name
    # backward: cotangents read from the packed rows
    cot = {nm: rng.standard_normal(t_.shape).astype(np.float32) for nm, t_ in
           (("dq", q), ("dk", k), ("dv", v), ("dg", g), ("dbeta", beta))}
    tc = {nm: torch.as_tensor(c, device=DEV) for nm, c in cot.items()}
    got = mixer.prologue_bwd(tx["qp"], tx["kp"], tx["vp"], tx["z"], tx["beta_logit"], tw["conv_q"], tw["conv_k"],
                             tw["conv_v"], tw["A"], tc["dq"], tc["dk"], tc["dv"], tc["dg"], tc["dbeta"], H=H,
                             b_gate=tw["b_gate"], cu_seqlens=cu_t, out_rows=rows)
    unpack = lambda a: np.concatenate([a[0][rows[s]:rows[s] + LENS[s]] for s in range(len(LENS))])[None]  # noqa: E731
    rb = M.prologue_bwd(x["qp"], x["kp"], x["vp"], x["z"], x["beta_logit"], w["conv_q"], w["conv_k"], w["conv_v"],
                        w["b_gate"], w["A"], H, dk, dv, unpack(cot["dq"]), unpack(cot["dk"]), unpack(cot["dv"]),
                        unpack(cot["dg"]), unpack(cot["dbeta"]), cu_seqlens=cu)
    for a_, b_ in (("dqp", "dqp"), ("dkp", "dkp"), ("dvp", "dvp"), ("dz", "dz"), ("dbeta_logit", "dbeta_logit"),
                   ("dconv_q", "dwq"), ("dconv_v", "dwv"), ("db_gate", "db_gate"), ("dA", "dA")):
        assert K.scale_rel_err(got[a_].cpu().numpy(), rb[b_]) <= 1e-4, a_
    # output gate over the packed o
    o_pad = rng.standard_normal((1, T_pad, H, dv)).astype(np.float32)
    gate = rng.standard_normal((1, n, H * dv)).astype(np.float32)
    dy = rng.standard_normal((1, n, H * dv)).astype(np.float32)
    to, tg, tdy = (torch.as_tensor(a_, device=DEV) for a_ in (o_pad, gate, dy))
    y = mixer.gated_rmsnorm_fwd(to, tg, cu_seqlens=cu_t, out_rows=rows)
    o_real = unpack(o_pad)[0]
    ref_y = M.gated_rmsnorm(o_real, gate[0].reshape(n, H, dv)).reshape(1, n, H * dv)
    assert K.scale_rel_err(y.cpu().numpy(), ref_y) <= 1e-4
    do, dgate = mixer.gated_rmsnorm_bwd(to, tg, tdy, cu_seqlens=cu_t, out_rows=rows)
    rdo, rdg = M.gated_rmsnorm_bwd(o_real, gate[0].reshape(n, H, dv), dy[0].reshape(n, H, dv))
    do_np = do.cpu().numpy()
    assert K.scale_rel_err(unpack(do_np)[0], rdo) <= 1e-4
    assert K.scale_rel_err(dgate.cpu().numpy().reshape(n, H, dv), rdg) <= 1e-4
    pad = np.ones(T_pad, bool)
    for s in range(len(LENS)):
        pad[rows[s]:rows[s] + LENS[s]] = False
    assert np.all(do_np[0][pad] == 0.0)


@pytest.mark.parametrize("n_seqs", [40, 300])
def test_varlen_many_sequences_any_order(n_seqs):
    """Many packed sequences with repeated lengths (ties) and empty ones: the
    per-sequence kernels take them longest first when there are at most 256,
    in order otherwise; every sequence must still equal the oracle run alone.
    O, S_T and dS0 are compared per sequence; the token gradients over all
    sampled sequences together (the bound's scale is the tensor's: a 1-token
    sequence with no state cotangent has dv = beta (q.k) do, whose score carries
    the bf16-operand rounding of q.k, ~1 % of a small number)."""
    from axiom_b200 import kda as KD

    H, dk, dv, chunk = 1, 128, 128, 64
    rng = np.random.default_rng(n_seqs)
    lens = rng.choice([0, 1, 17, 64, 65, 130], size=n_seqs).tolist()
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    n_tok = int(cu[-1])
    x = K.make_inputs(1, n_tok, H, dk, dv, seed=n_seqs, s0_std=None)
    x = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    S0 = (rng.standard_normal((n_seqs, H, dk, dv)) * 0.05).astype(np.float32)
    offs, rows, T_pad = KD.packing(cu.tolist(), chunk)
    t = {k: torch.as_tensor(_pack(x[k][0], cu, rows, T_pad)[None]).to(DEV).to(torch.bfloat16).contiguous()
         for k in ("q", "k", "v", "g", "beta")}
    do_np = K.bf16_round(rng.standard_normal((n_tok, H, dv)).astype(np.float32))
    do_t = torch.as_tensor(_pack(do_np, cu, rows, T_pad)[None]).to(DEV).to(torch.bfloat16).contiguous()
    o, s_t, ckpt = KD.kda_fwd_varlen(t["q"], t["k"], t["v"], t["g"], t["beta"], offs, torch.as_tensor(S0).to(DEV),
                                     chunk=chunk, o_dtype=torch.float32, need_ckpt=True)
    grads = KD.kda_bwd_varlen(t["q"], t["k"], t["v"], t["g"], t["beta"], ckpt, do_t, offs, None, chunk=chunk)
    o_np = o[0].float().cpu().numpy()
    g_np = [g_[0].float().cpu().numpy() for g_ in grads[:5]]
    ds0 = grads[5].cpu().numpy()
    got_rows = {n: [] for n in ("dq", "dk", "dv", "dg", "dbeta")}
    ref_rows = {n: [] for n in got_rows}
    for s in rng.choice(n_seqs, size=min(n_seqs, 24), replace=False):
        a, b = int(cu[s]), int(cu[s + 1])
        r0 = rows[s]
        xs = [x[k][:, a:b] for k in ("q", "k", "v", "g", "beta")]
        ref_o, ref_s = K.chunk_fwd(*xs, S0[s][None], chunk=chunk)
        assert K.scale_rel_err(s_t[s].cpu().numpy(), ref_s[0]) <= 1e-2, ("S_T", s)
        ref = K.chunk_bwd(*xs, S0[s][None], do_np[a:b][None], None, chunk=chunk)
        assert K.scale_rel_err(ds0[s], ref[5][0]) <= 1e-2, ("dS0", s)
        if b > a:
            assert K.scale_rel_err(o_np[r0:r0 + b - a], ref_o[0]) <= 1e-2, ("o", s)
            for name, gg, rf in zip(got_rows, g_np, ref[:5]):
                got_rows[name].append(gg[r0:r0 + b - a])
                ref_rows[name].append(rf[0])
    for name in got_rows:
        assert K.scale_rel_err(np.concatenate(got_rows[name]), np.concatenate(ref_rows[name])) <= 1e-2, name
