"""The CPU oracle against the reference's golden vectors and its own relations.

These pin the oracle before any kernel is compared with it:
* every golden case (outputs of the reference's own functions, see
  ``tests/golden/make_golden.py``) is reproduced to fp32 rounding;
* chunked == recurrent in float64 for several chunk widths and decays
  (``net/tests/test_kda_chunked_cc.py:189-218``);
* the adjoint == central finite differences of the recurrence
  (``net/tests/test_kda_chunked_cc.py:333-391``).
"""

import numpy as np
import pytest

from oracle import kda_oracle as K

FWD_CASES = ["chunk_a", "chunk_b", "chunk_c", "scan_a", "scan_b", "scan_c", "scan_d",
             "tc_scan_baseline", "tc_scan_medium"]
BWD_CASES = ["bwd_chunk", "bwd_scan", "bwd_scan_strong", "bwd_scan_medium",
             "tc_bwd_scan_baseline", "tc_bwd_scan_medium"]
GRADS = ["dq", "dk", "dv", "dg", "dbeta", "dS0"]


@pytest.mark.parametrize("case", FWD_CASES)
def test_oracle_forward_matches_reference_golden(golden, case):
    d = golden[case]
    o, S = K.chunk_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], chunk=int(d["chunk"]))
    assert K.scale_rel_err(o, d["o"]) <= 1e-5
    assert K.scale_rel_err(S, d["S_T"]) <= 1e-5


@pytest.mark.parametrize("case", BWD_CASES)
def test_oracle_adjoint_matches_reference_golden(golden, case):
    d = golden[case]
    got = K.chunk_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], d["do"], d["dST"],
                      chunk=int(d["chunk"]))
    for name, x in zip(GRADS, got):
        assert K.scale_rel_err(x, d[name]) <= 1e-5, name


def test_oracle_recurrence_matches_reference_golden(golden):
    d = golden["recurrent"]
    o, S = K.recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"])
    assert K.scale_rel_err(o, d["o"]) <= 1e-5
    assert K.scale_rel_err(S, d["S_T"]) <= 1e-5


@pytest.mark.parametrize("strict", [False, True])
def test_oracle_tile_scores_match_reference_golden(golden, strict):
    d = golden["scores"]
    got = K.cc_scores(d["row"].astype(np.float64), d["col"].astype(np.float64),
                      d["G"].astype(np.float64), 16, strict=strict)
    assert K.scale_rel_err(got, d["strict" if strict else "lower"]) <= 1e-5


def test_tile_scores_equal_direct_ratio_under_strong_decay():
    """The tile-anchored scores equal the brute (C, C, dk) ratio form
    (``net/tests/test_kda_chunked_cc.py:221-247``), here at C = 64."""
    rng = np.random.default_rng(4)
    C, dk = 64, 16
    g = -5.0 / (1.0 + np.exp(-3.0 * rng.standard_normal((2, C, dk))))
    G = np.cumsum(g, axis=1)
    row, col = rng.standard_normal((2, C, dk)), rng.standard_normal((2, C, dk))
    E = np.exp(np.minimum(G[:, :, None, :] - G[:, None, :, :], 0.0))
    brute = np.einsum("hcid,hcd,hid->hci", E, row, col)
    for strict in (False, True):
        mask = np.tril(np.ones((C, C)), -1 if strict else 0)
        got = K.cc_scores(row, col, G, 16, strict=strict)
        assert np.all(np.isfinite(got))
        assert K.scale_rel_err(got, brute * mask) <= 1e-12


@pytest.mark.parametrize("chunk", [16, 32, 64])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_chunked_equals_recurrent(chunk, seed):
    x = K.make_inputs(2, 100, 2, 16, 8, seed=seed, s0_std=0.1)
    o_r, s_r = K.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"])
    o_c, s_c = K.chunk_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk=chunk)
    assert K.scale_rel_err(o_c, o_r) <= 1e-10
    assert K.scale_rel_err(s_c, s_r) <= 1e-10


@pytest.mark.parametrize("T", [5, 40, 127])
def test_oracle_ragged_and_short_sequences(T):
    """T below the chunk and ragged tails (``test_kda_chunked_cc.py:271-288``)."""
    x = K.make_inputs(1, T, 2, 16, 16, seed=T, decay="strong")
    o_r, s_r = K.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"])
    o_c, s_c = K.chunk_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk=64)
    assert o_c.shape == o_r.shape
    assert K.scale_rel_err(o_c, o_r) <= 1e-10
    assert K.scale_rel_err(s_c, s_r) <= 1e-10


def test_oracle_adjoint_matches_finite_differences():
    x = K.make_inputs(1, 40, 2, 8, 8, seed=3, s0_std=0.1)
    rng = np.random.default_rng(5)
    do = rng.standard_normal((1, 40, 2, 8))
    dST = rng.standard_normal((1, 2, 8, 8))
    grads = K.chunk_bwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], do, dST, chunk=16)
    fd = K.recurrent_loss_grad_fd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], do, dST,
                                  n_probe=6)
    for name, gr in zip(["q", "k", "v", "g", "beta", "S0"], grads):
        idx, vals = fd[name]
        assert np.max(np.abs(gr.reshape(-1)[idx] - vals)) <= 1e-6 * max(1.0, np.max(np.abs(vals))), name


def test_oracle_zero_rows_stay_finite():
    """Explicit zero rows (``test_kda_chunked_cc.py:301-306``) give finite outputs and grads."""
    x = K.make_inputs(1, 96, 2, 16, 16, seed=6)
    for key in ("q", "k", "v"):
        x[key][:, 64:] = 0.0
    o, S = K.chunk_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk=64)
    grads = K.chunk_bwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], np.ones_like(o),
                        np.ones_like(S), chunk=64)
    assert np.all(np.isfinite(o)) and np.all(np.isfinite(S))
    assert all(np.all(np.isfinite(gr)) for gr in grads)


def test_decode_step_is_one_token_of_the_recurrence():
    x = K.make_inputs(3, 1, 4, 32, 16, seed=9, s0_std=0.02)
    o1, s1 = K.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"])
    o2, s2 = K.decode_step(x["S0"], x["q"][:, 0], x["k"][:, 0], x["v"][:, 0], x["g"][:, 0],
                           x["beta"][:, 0])
    assert np.allclose(o1[:, 0], o2) and np.allclose(s1, s2)
