"""GPU parity of the tensor-core path (bf16 inputs, dk = dv = 128, chunk 64).

The oracle runs on the same bf16-rounded inputs in float64; the tolerance is
the BASELINE bf16 bar, scale-relative 1e-2 on O, the final state, the
chunk-boundary checkpoint and every gradient.
"""

import numpy as np
import pytest
import torch

from oracle import kda_oracle as K

pytestmark = pytest.mark.gpu

TOL = 1e-2
GRADS = ["dq", "dk", "dv", "dg", "dbeta", "dS0"]


def _dev(x, dtype):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32).cuda().to(dtype).contiguous()


def _np(x):
    return x.detach().float().cpu().numpy()


def _bf16_inputs(B, T, H, seed, s0_std=None, decay="baseline"):
    x = K.make_inputs(B, T, H, 128, 128, seed=seed, s0_std=s0_std, decay=decay)
    xr = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    dev = {k: _dev(v, torch.bfloat16 if k != "S0" else torch.float32) for k, v in x.items()}
    return xr, dev


@pytest.mark.parametrize("case", ["tc_scan_baseline", "tc_scan_medium"])
def test_tc_forward_matches_reference_golden(golden, case):
    """The tensor-core forward against the reference's own whole-sequence scan
    (kda_cc_fused_persist.reference, :768-791) at dk = dv = 128, C = 64, on inputs
    the fixture holds bf16-representable (tests/golden/make_golden.py, case 7)."""
    from axiom_b200 import kda_fwd

    d = golden[case]
    x = {n: _dev(d[n], torch.bfloat16) for n in ("q", "k", "v", "g", "beta")}
    o, s_t, _ = kda_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], _dev(d["S0"], torch.float32),
                        chunk=64, o_dtype=torch.float32)
    torch.cuda.synchronize()
    assert K.scale_rel_err(_np(o), d["o"]) <= TOL
    assert K.scale_rel_err(_np(s_t), d["S_T"]) <= TOL


@pytest.mark.parametrize("case", ["tc_bwd_scan_baseline", "tc_bwd_scan_medium"])
def test_tc_backward_matches_reference_golden(golden, case):
    """The tensor-core backward against the reference's reverse scan
    (kda_cc_fused_persist.reference_bwd_scan, :794-849) at dk = dv = 128, C = 64."""
    from axiom_b200 import kda_bwd, kda_fwd

    d = golden[case]
    x = {n: _dev(d[n], torch.bfloat16) for n in ("q", "k", "v", "g", "beta", "do")}
    _, _, ckpt = kda_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], _dev(d["S0"], torch.float32),
                         chunk=64, need_ckpt=True)
    grads = kda_bwd(x["q"], x["k"], x["v"], x["g"], x["beta"], ckpt, x["do"],
                    _dev(d["dST"], torch.float32), chunk=64)
    torch.cuda.synchronize()
    for name, gr in zip(GRADS, grads):
        assert K.scale_rel_err(_np(gr), d[name]) <= TOL, name


@pytest.mark.parametrize("B,T,H,s0,decay", [
    (2, 512, 4, 0.02, "baseline"),    # config-2 distributions at reduced size
    (1, 200, 2, 0.1, "baseline"),     # ragged tail
    (1, 5, 3, 0.1, "baseline"),       # shorter than one chunk
    (1, 256, 2, 0.1, "strong"),       # strong decay: exact score path (16-token block anchors)
    (1, 320, 2, 0.1, "half_budget"),  # chunk sums past 80, halves below: two-half anchored scores
    (1, 320, 2, 0.0, "medium"),
])
def test_tc_forward_matches_oracle(B, T, H, s0, decay):
    from axiom_b200 import kda_fwd
    from axiom_b200.kda import ckpt_states

    xr, d = _bf16_inputs(B, T, H, seed=T + H, s0_std=s0 if s0 else None, decay=decay)
    S0 = d["S0"] if s0 else None
    o, s_t, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], S0, chunk=64,
                           o_dtype=torch.float32, need_ckpt=True)
    torch.cuda.synchronize()
    o_ref, s_ref, states = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"],
                                       xr["S0"] if s0 else None, chunk=64, return_states=True)
    assert K.scale_rel_err(_np(o), o_ref) <= TOL
    assert K.scale_rel_err(_np(s_t), s_ref) <= TOL
    ck_states = _np(ckpt_states(ckpt, B, T, H, 128, 128, chunk=64))
    assert ck_states.shape == states.shape
    assert K.scale_rel_err(ck_states, states) <= TOL


def test_tc_forward_bf16_output_and_repeatability():
    from axiom_b200 import kda_fwd

    xr, d = _bf16_inputs(2, 384, 2, seed=3, s0_std=0.02)
    o1, s1, _ = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"])
    o2, s2, _ = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"])
    torch.cuda.synchronize()
    assert o1.dtype == torch.bfloat16
    assert torch.equal(o1, o2) and torch.equal(s1, s2)  # deterministic
    o_ref, s_ref = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64)
    assert K.scale_rel_err(_np(o1), o_ref) <= TOL


@pytest.mark.parametrize("T,decay", [(256, "baseline"), (130, "strong"), (200, "half_budget")])
def test_tc_training_step_matches_oracle(T, decay):
    from axiom_b200 import chunk_kda

    B, H = 1, 2
    xr, d = _bf16_inputs(B, T, H, seed=T, s0_std=0.05, decay=decay)
    rng = np.random.default_rng(T)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    leaves = {n: d[n].clone().requires_grad_() for n in ("q", "k", "v", "g", "beta", "S0")}
    o, s_t = chunk_kda(*(leaves[n] for n in ("q", "k", "v", "g", "beta", "S0")))
    (o.float() * _dev(do, torch.float32)).sum().backward(retain_graph=True)
    (s_t * _dev(dST, torch.float32)).sum().backward()
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64)
    for name, leaf, rf in zip(GRADS, ("q", "k", "v", "g", "beta", "S0"), ref):
        assert K.scale_rel_err(_np(leaves[leaf].grad), rf) <= TOL, name


def test_tc_backward_many_units_matches_oracle():
    """More (batch, head, chunk) units than SMs: bwd_par's persistent loop."""
    from axiom_b200 import kda_bwd, kda_fwd

    B, T, H = 2, 2048, 4
    xr, d = _bf16_inputs(B, T, H, seed=21, s0_std=0.02)
    rng = np.random.default_rng(22)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    o, s_t, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], need_ckpt=True)
    grads = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.bfloat16),
                    _dev(dST, torch.float32))
    torch.cuda.synchronize()
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64)
    for name, gr, rf in zip(GRADS, grads, ref):
        assert K.scale_rel_err(_np(gr), rf) <= TOL, name


def test_tc_forward_checkpoint_feeds_the_exact_backward():
    """A bf16 checkpoint from the tensor-core forward (operand-image states) read by
    the exact backward, which takes over when dO is fp32."""
    from axiom_b200 import kda_bwd, kda_fwd

    B, T, H = 1, 200, 2
    xr, d = _bf16_inputs(B, T, H, seed=31, s0_std=0.05)
    rng = np.random.default_rng(32)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    _, _, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], need_ckpt=True)
    exact = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.float32),
                    _dev(dST, torch.float32))
    tc = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.bfloat16),
                 _dev(dST, torch.float32))
    torch.cuda.synchronize()
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64)
    for name, ge, gt, rf in zip(GRADS, exact, tc, ref):
        assert K.scale_rel_err(_np(ge), rf) <= TOL, name
        assert K.scale_rel_err(_np(gt), rf) <= TOL, name


def test_tc_extreme_decay_is_exact():
    """Per-token decay up to 11 (BASELINE's mixer gate with b = 0): every chunk
    takes the exact score path.  The reference's tile-anchored chunk algorithm
    loses accuracy here (its column clamp binds inside a tile), so the forward is
    checked against the direct-ratio oracle and the token recurrence, the
    backward against the direct-ratio adjoint."""
    from axiom_b200 import chunk_kda

    B, T, H = 1, 200, 2
    x = K.make_inputs(B, T, H, 128, 128, seed=31, s0_std=0.05, decay="strong")
    x["g"] = x["g"] * 2.2
    xr = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    d = {k: _dev(v, torch.bfloat16 if k != "S0" else torch.float32) for k, v in xr.items()}
    rng = np.random.default_rng(32)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    leaves = {n: d[n].clone().requires_grad_() for n in ("q", "k", "v", "g", "beta", "S0")}
    o, s_t = chunk_kda(*(leaves[n] for n in ("q", "k", "v", "g", "beta", "S0")))
    o_rec, s_rec = K.recurrent(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"])
    o_ex, s_ex = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64, tile=None)
    assert K.scale_rel_err(o_ex, o_rec) <= 1e-10
    assert K.scale_rel_err(_np(o), o_rec) <= TOL
    assert K.scale_rel_err(_np(s_t), s_rec) <= TOL
    (o.float() * _dev(do, torch.float32)).sum().backward(retain_graph=True)
    (s_t * _dev(dST, torch.float32)).sum().backward()
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64, tile=None)
    for name, leaf, rf in zip(GRADS, ("q", "k", "v", "g", "beta", "S0"), ref):
        assert K.scale_rel_err(_np(leaves[leaf].grad), rf) <= TOL, name


def test_tc_backward_is_bitwise_repeatable():
    """Every reduction in the backward has a fixed order (the dbeta partials of the
    four channel quarters land in separate slots and are summed in order), so two
    calls on the same inputs give identical bits."""
    from axiom_b200 import kda_bwd, kda_fwd

    B, T, H = 2, 1024, 8
    _, d = _bf16_inputs(B, T, H, seed=41, s0_std=0.02)
    rng = np.random.default_rng(42)
    do = _dev(K.bf16_round(rng.standard_normal((B, T, H, 128))), torch.bfloat16)
    dST = _dev(rng.standard_normal((B, H, 128, 128)).astype(np.float32), torch.float32)
    _, _, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], need_ckpt=True)
    first = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, do, dST)
    for _ in range(3):
        again = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, do, dST)
        for name, a, b in zip(GRADS, first, again):
            assert torch.equal(a, b), name


@pytest.mark.parametrize("decay", ["baseline", "strong"])
def test_tc_fp32_checkpoint_states(decay):
    """The chunk-boundary states stored in fp32 (ckpt_dtype=float32) instead of
    their bf16 operand images: the backward reads them row-major and builds its
    operands itself.  Gradients against the oracle, at the bf16 bar."""
    from axiom_b200 import kda_bwd, kda_fwd
    from axiom_b200.kda import ckpt_states

    B, T, H = 1, 192, 2
    xr, d = _bf16_inputs(B, T, H, seed=51, s0_std=0.05, decay=decay)
    rng = np.random.default_rng(52)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    o, s_t, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], need_ckpt=True,
                           ckpt_dtype=torch.float32, o_dtype=torch.float32)
    grads = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.bfloat16),
                    _dev(dST, torch.float32))
    torch.cuda.synchronize()
    o_ref, s_ref, states = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64,
                                       return_states=True, tile=None)
    assert K.scale_rel_err(_np(o), o_ref) <= TOL
    assert ckpt.dtype == torch.float32
    st = _np(ckpt_states(ckpt, B, T, H, 128, 128, chunk=64))
    assert K.scale_rel_err(st, states) <= TOL
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64, tile=None)
    for name, gr, rf in zip(GRADS, grads, ref):
        assert K.scale_rel_err(_np(gr), rf) <= TOL, name


def test_tc_mixed_decay_regimes_in_one_call():
    """Heads in one launch on three score paths at once: head 0 within the single
    anchor's budget, head 1 past it with each 32-token half within it (two-half
    anchors), head 2 past both (16-token block anchors).  Forward and backward
    against the direct-ratio oracle."""
    from axiom_b200 import kda_bwd, kda_fwd

    B, T = 1, 256
    parts = [K.make_inputs(B, T, 1, 128, 128, seed=61 + i, s0_std=0.05, decay=dcy)
             for i, dcy in enumerate(("baseline", "half_budget", "strong"))]
    x = {k: np.concatenate([p_[k] for p_ in parts], axis=2 if k != "S0" else 1) for k in parts[0]}
    xr = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    d = {k: _dev(v, torch.bfloat16 if k != "S0" else torch.float32) for k, v in x.items()}
    rng = np.random.default_rng(64)
    do = K.bf16_round(rng.standard_normal((B, T, 3, 128)))
    dST = rng.standard_normal((B, 3, 128, 128)).astype(np.float32)
    o, s_t, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], need_ckpt=True,
                           o_dtype=torch.float32)
    grads = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.bfloat16),
                    _dev(dST, torch.float32))
    torch.cuda.synchronize()
    o_ref, s_ref = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64, tile=None)
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64, tile=None)
    for h in range(3):
        assert K.scale_rel_err(_np(o)[:, :, h], o_ref[:, :, h]) <= TOL, ("o", h)
        assert K.scale_rel_err(_np(s_t)[:, h], s_ref[:, h]) <= TOL, ("S_T", h)
        for name, gr, rf in zip(GRADS, grads, ref):
            g_, r_ = (_np(gr)[:, h], rf[:, h]) if name == "dS0" else (_np(gr)[:, :, h], rf[:, :, h])
            assert K.scale_rel_err(g_, r_) <= TOL, (name, h)


@pytest.mark.parametrize("schedule", ["split", "fused"])
@pytest.mark.parametrize("B,T,H,ck,slices", [
    (1, 200, 2, torch.bfloat16, "8"),   # 2 (sequence, head) pairs, forced 8 state slices of 16 columns
    (1, 130, 32, torch.bfloat16, None),  # 32 pairs: 4 slices of 32 columns
    (2, 128, 32, torch.float32, None),   # 64 pairs: 2 slices of 64 columns, fp32 checkpoint
    (2, 64, 64, torch.bfloat16, "1"),   # 128 pairs, forced: one CTA per pair, whole state
])
def test_tc_training_forward_schedules_match_oracle(monkeypatch, schedule, B, T, H, ck, slices):
    """The training forward (checkpoint written) on both schedules: the split
    one (chunk-parallel prep + state scan sliced by columns, the slice count
    following the number of (sequence, head) pairs or KDA_SCAN_SLICES) and the
    fused one; outputs, states and the backward (whose state-cotangent scan is
    sliced the same way) from each checkpoint against the oracle."""
    from axiom_b200 import kda_bwd, kda_fwd
    from axiom_b200.kda import ckpt_states

    monkeypatch.setenv("KDA_FWD_SCHEDULE", schedule)
    if slices:
        monkeypatch.setenv("KDA_SCAN_SLICES", slices)
    xr, d = _bf16_inputs(B, T, H, seed=B * 1000 + T + H, s0_std=0.05)
    rng = np.random.default_rng(T + H)
    do = K.bf16_round(rng.standard_normal((B, T, H, 128)))
    dST = rng.standard_normal((B, H, 128, 128)).astype(np.float32)
    o, s_t, ckpt = kda_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], chunk=64,
                           o_dtype=torch.float32, need_ckpt=True, ckpt_dtype=ck)
    # the backward's state-cotangent scan is sliced the same way (2, 4, 8 slices here)
    grads = kda_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], ckpt, _dev(do, torch.bfloat16),
                    _dev(dST, torch.float32), chunk=64)
    torch.cuda.synchronize()
    o_ref, s_ref, states = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64,
                                       return_states=True)
    assert K.scale_rel_err(_np(o), o_ref) <= TOL
    assert K.scale_rel_err(_np(s_t), s_ref) <= TOL
    assert K.scale_rel_err(_np(ckpt_states(ckpt, B, T, H, 128, 128, chunk=64)), states) <= TOL
    ref = K.chunk_bwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], do, dST, chunk=64)
    for name, gr, rf in zip(GRADS, grads, ref):
        assert K.scale_rel_err(_np(gr), rf) <= TOL, name
