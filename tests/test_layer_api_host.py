"""``axiom_b200.layer.apply_kda``: the reference's dispatch contract
(``net/kda.py:708-729, 929-946``, ``_with_window`` :261-269), checked on the host:
every refusal happens before any tensor is touched."""

from types import SimpleNamespace

import pytest

from axiom_b200.layer import apply_kda


def _cfg(**kw):
    base = dict(num_heads=2, kda_dk=128, kda_dv=128, kda_g_min=-5.0, kda_impl="chunked_cc", kda_wyut_chunk=64,
                swa_window=128, attn_dense_reference=True)
    base.update(kw)
    return SimpleNamespace(**base)


@pytest.mark.parametrize("impl", ["chunked", "wyut"])
def test_other_kda_forms_are_refused(impl, monkeypatch):
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "b200")
    with pytest.raises(NotImplementedError, match="chunked_cc"):
        apply_kda(None, _cfg(kda_impl=impl), None)


@pytest.mark.parametrize("body", ["jax", "mosaic", "persistent"])
def test_reference_bodies_are_refused(body, monkeypatch):
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", body)
    with pytest.raises(NotImplementedError, match="b200"):
        apply_kda(None, _cfg(), None)


def test_unknown_impl_value_raises(monkeypatch):
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "bogus")
    with pytest.raises(ValueError):
        apply_kda(None, _cfg(), None)


def test_window_branch_is_refused(monkeypatch):
    monkeypatch.setenv("AXIOM_KDA_CC_IMPL", "b200")
    with pytest.raises(NotImplementedError, match="window"):
        apply_kda(None, _cfg(attn_dense_reference=False, swa_window=128), None)
