"""Generate the golden fixtures by executing the reference's own KDA functions.

The reference (AXIOM) is pure JAX and JAX is not installed in the build
container, so its functions are run under ``jaxshim`` (NumPy stand-ins for the
handful of ``jax`` calls they make).  The functions are loaded unmodified from
the reference checkout given by ``--reference``:

* ``net/kernels/kda_cc_fused.py:618-687``        ``reference``      (one chunk, operand form)
* ``net/kernels/kda_cc_fused_persist.py:768-791`` ``reference``      (whole-sequence chunk scan)
* ``net/kernels/kda_cc_fused_bwd.py:117-239``     ``reference_bwd``  (analytic adjoint, one chunk)
* ``net/kernels/kda_cc_fused_persist.py:794-849`` ``reference_bwd_scan`` (reverse scan)
* ``net/kda.py:298-310``                          ``_delta_step``    (the recurrence), ``o = S^T q`` :293
* ``net/kda.py:588-631``                          ``_cc_scores``     (tile-anchored scores)

The ``tc_*`` cases run the scan and its reverse scan at the tensor-core shape
(dk = dv = 128, C = 64) on inputs that are exactly representable in bfloat16,
so the bf16 kernels can be checked against the reference's own outputs.

The reference's operand-form replica (``kda_cc_fused.reference``) builds the
column factor ``exp(anchor - G)`` over the whole chunk before masking it, which
overflows to ``inf * 0 = nan`` once the decay summed over a chunk passes ~88
(strong decay at C >= 32); the reference's Mosaic kernel clamps that exponent
(``COL_EXP_BUDGET``).  Strong-decay fixtures therefore use C = 16, where the
replica is finite, and a medium decay covers C = 64.

Inputs are drawn with NumPy seeds and converted between the reference's
operand form (``(T, H*D)``, ``alpha = exp(g)``, ``beta32``) and this repo's
``[B, T, H, D]`` form (``g``, ``beta``); the fixtures store this repo's form,
with ``g = log(alpha)`` evaluated in float64 on the exact fp32 ``alpha`` the
reference saw, ``dg = dalpha * alpha`` and ``dbeta = sum of dbeta32``.

Usage::

    python tests/golden/make_golden.py --reference <path to the reference checkout>
"""

from __future__ import annotations

import argparse
import ast
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import jaxshim  # noqa: E402


def _load_kernels(ref_root):
    """Import ``net/kernels/*`` as package ``refk`` (skips ``net/__init__``)."""
    pkg = types.ModuleType("refk")
    pkg.__path__ = [os.path.join(ref_root, "net", "kernels")]
    sys.modules["refk"] = pkg
    mods = {}
    for name in ("kda_cc_fused", "kda_cc_fused_bwd", "kda_cc_fused_persist"):
        path = os.path.join(ref_root, "net", "kernels", name + ".py")
        spec = importlib.util.spec_from_file_location("refk." + name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["refk." + name] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def _load_kda_functions(ref_root, names):
    """Execute selected top-level functions of ``net/kda.py`` from its source."""
    path = os.path.join(ref_root, "net", "kda.py")
    src = open(path).read()
    tree = ast.parse(src)
    import jax
    import jax.numpy as jnp

    ns = {"jax": jax, "jnp": jnp}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            code = compile(ast.Module(body=[node], type_ignores=[]), path, "exec")
            exec(code, ns)
    return {n: ns[n] for n in names}


def _inputs(rng, T, H, dk, dv, decay, s0_std):
    q = rng.standard_normal((T, H, dk))
    k = rng.standard_normal((T, H, dk))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, H, dv))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((T, H))))
    if decay == "baseline":
        g = -np.logaddexp(0.0, -rng.normal(3.0, 1.0, (T, H, dk)))
    elif decay == "medium":
        g = -1.0 / (1.0 + np.exp(-2.0 * rng.standard_normal((T, H, dk))))
    else:
        g = -5.0 / (1.0 + np.exp(-3.0 * rng.standard_normal((T, H, dk))))
    alpha = np.exp(g).astype(np.float32)
    S = (rng.standard_normal((H, dk, dv)) * s0_std).astype(np.float32)
    f = np.float32
    return dict(q=q.astype(f), k=k.astype(f), v=v.astype(f), alpha=alpha,
                beta=beta.astype(f), S=S)


def _bf16(a):
    """Round to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _bf16_inputs(x):
    """The same draw made bf16-representable: q, k, v, beta rounded; alpha = exp(g)
    of the rounded log-decay (so log(alpha) rounds back to it); S stays fp32."""
    g = _bf16(np.log(x["alpha"].astype(np.float64)))
    return dict(q=_bf16(x["q"]), k=_bf16(x["k"]), v=_bf16(x["v"]),
                alpha=np.exp(g.astype(np.float64)).astype(np.float32), beta=_bf16(x["beta"]), S=x["S"])


def _ref_form(x):
    T, H = x["q"].shape[:2]
    b32 = np.broadcast_to(x["beta"][:, :, None], (T, H, 32)).reshape(T, H * 32)
    A = lambda a: np.ascontiguousarray(a.reshape(T, -1)).view(jaxshim.Arr)  # noqa: E731
    return (A(x["q"]), A(x["k"]), A(x["v"]), A(x["alpha"]),
            np.ascontiguousarray(b32).view(jaxshim.Arr), x["S"].view(jaxshim.Arr))


def _our_inputs(x):
    return dict(q=x["q"][None], k=x["k"][None], v=x["v"][None],
                g=np.log(x["alpha"].astype(np.float64))[None],
                beta=x["beta"][None].astype(np.float64), S0=x["S"][None])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()

    jaxshim.install()
    mods = _load_kernels(args.reference)
    fused, fbwd, persist = mods["kda_cc_fused"], mods["kda_cc_fused_bwd"], mods["kda_cc_fused_persist"]
    kfn = _load_kda_functions(args.reference, ["_delta_step", "_cc_scores"])

    out = {}

    def put(prefix, dct):
        for k_, v_ in dct.items():
            out[f"{prefix}/{k_}"] = np.asarray(v_)

    # 1. one chunk, operand form (kda_cc_fused.reference)
    for name, (C, H, dk, dv, decay, seed) in {
        "chunk_a": (32, 2, 32, 16, "baseline", 0),
        "chunk_b": (64, 2, 64, 64, "medium", 1),
        "chunk_c": (16, 2, 32, 32, "strong", 10),
    }.items():
        x = _inputs(np.random.default_rng(seed), C, H, dk, dv, decay, 0.1)
        o, s_new = fused.reference(*_ref_form(x), tile=16)
        put(name, _our_inputs(x))
        put(name, dict(o=np.asarray(o).reshape(1, C, H, dv), S_T=np.asarray(s_new)[None],
                       chunk=np.array(C)))

    # 2. whole-sequence scan (persist.reference)
    for name, (T, C, H, dk, dv, decay, s0, seed) in {
        "scan_a": (128, 32, 2, 32, 32, "baseline", 0.0, 2),
        "scan_b": (192, 64, 1, 64, 64, "baseline", 0.02, 3),
        "scan_c": (128, 16, 2, 32, 16, "strong", 0.1, 4),
        "scan_d": (256, 64, 2, 64, 32, "medium", 0.1, 11),
    }.items():
        x = _inputs(np.random.default_rng(seed), T, H, dk, dv, decay, s0)
        o, s_new = persist.reference(*_ref_form(x), tile=16, chunk=C)
        put(name, _our_inputs(x))
        put(name, dict(o=np.asarray(o).reshape(1, T, H, dv), S_T=np.asarray(s_new)[None],
                       chunk=np.array(C)))

    # 3. adjoint of one chunk and 4. the reverse scan
    for name, (T, C, H, dk, dv, decay, seed, scan) in {
        "bwd_chunk": (32, 32, 2, 32, 16, "baseline", 5, False),
        "bwd_scan": (128, 32, 2, 32, 32, "baseline", 6, True),
        "bwd_scan_strong": (128, 16, 1, 32, 32, "strong", 7, True),
        "bwd_scan_medium": (192, 64, 2, 32, 32, "medium", 12, True),
    }.items():
        rng = np.random.default_rng(seed)
        x = _inputs(rng, T, H, dk, dv, decay, 0.1)
        do = rng.standard_normal((T, H * dv)).astype(np.float32)
        dS = rng.standard_normal((H, dk, dv)).astype(np.float32)
        ref = _ref_form(x)
        if scan:
            res = persist.reference_bwd_scan(*ref, do.view(jaxshim.Arr), dS.view(jaxshim.Arr),
                                             tile=16, chunk=C)
        else:
            res = fbwd.reference_bwd(*ref, do.view(jaxshim.Arr), dS.view(jaxshim.Arr), tile=16)
        dq, dk_, dv_, dalpha, dbeta32, dS_in = (np.asarray(r) for r in res)
        put(name, _our_inputs(x))
        put(name, dict(
            do=do.reshape(1, T, H, dv), dST=dS[None], chunk=np.array(C),
            dq=dq.reshape(1, T, H, dk), dk=dk_.reshape(1, T, H, dk), dv=dv_.reshape(1, T, H, dv),
            dg=(dalpha.astype(np.float64) * x["alpha"].reshape(T, H * dk)).reshape(1, T, H, dk),
            dbeta=dbeta32.astype(np.float64).reshape(T, H, 32).sum(-1)[None],
            dS0=dS_in[None]))

    # 5. the recurrence (_delta_step, o = S^T q with the updated state)
    T, H, dk, dv = 48, 2, 16, 8
    x = _inputs(np.random.default_rng(8), T, H, dk, dv, "baseline", 0.1)
    S = x["S"].view(jaxshim.Arr)
    o = np.zeros((T, H, dv), np.float32)
    for t in range(T):
        S = kfn["_delta_step"](S, x["k"][t].view(jaxshim.Arr), x["v"][t].view(jaxshim.Arr),
                               x["beta"][t].view(jaxshim.Arr), x["alpha"][t].view(jaxshim.Arr))
        o[t] = np.einsum("hdv,hd->hv", np.asarray(S), x["q"][t])
    put("recurrent", _our_inputs(x))
    put("recurrent", dict(o=o[None], S_T=np.asarray(S)[None]))

    # 6. tile-anchored scores under strong decay (net/kda.py:_cc_scores)
    rng = np.random.default_rng(9)
    C, H, dk = 32, 2, 16
    g = -5.0 / (1.0 + np.exp(-3.0 * rng.standard_normal((H, C, dk))))
    G = np.cumsum(g.astype(np.float32), axis=1).astype(np.float32)
    row = rng.standard_normal((H, C, dk)).astype(np.float32)
    col = rng.standard_normal((H, C, dk)).astype(np.float32)
    for strict in (False, True):
        sc = kfn["_cc_scores"](row.view(jaxshim.Arr), col.view(jaxshim.Arr),
                               G.view(jaxshim.Arr), 16, strict)
        out[f"scores/{'strict' if strict else 'lower'}"] = np.asarray(sc)
    out["scores/row"], out["scores/col"], out["scores/G"] = row, col, G

    # 7. the tensor-core shape (dk = dv = 128, C = 64) on bf16-representable inputs:
    # q, k, v, beta, dO and the log-decay are rounded to bf16 before the reference
    # sees them (alpha = exp of the rounded g, in fp32), so a bf16 caller passes
    # exactly the values the reference computed with.
    for name, (T, H, decay, s0, seed, bwd) in {
        "tc_scan_baseline": (192, 1, "baseline", 0.02, 13, False),
        "tc_scan_medium": (192, 1, "medium", 0.1, 14, False),
        "tc_bwd_scan_baseline": (128, 1, "baseline", 0.02, 15, True),
        "tc_bwd_scan_medium": (128, 1, "medium", 0.1, 16, True),
    }.items():
        rng = np.random.default_rng(seed)
        x = _bf16_inputs(_inputs(rng, T, H, 128, 128, decay, s0))
        ref = _ref_form(x)
        put(name, _our_inputs(x))
        if not bwd:
            o, s_new = persist.reference(*ref, tile=16, chunk=64)
            put(name, dict(o=np.asarray(o).reshape(1, T, H, 128), S_T=np.asarray(s_new)[None],
                           chunk=np.array(64)))
            continue
        do = _bf16(rng.standard_normal((T, H * 128)))
        dS = rng.standard_normal((H, 128, 128)).astype(np.float32)
        dq, dk_, dv_, dalpha, dbeta32, dS_in = (np.asarray(r) for r in persist.reference_bwd_scan(
            *ref, do.view(jaxshim.Arr), dS.view(jaxshim.Arr), tile=16, chunk=64))
        put(name, dict(
            do=do.reshape(1, T, H, 128), dST=dS[None], chunk=np.array(64),
            dq=dq.reshape(1, T, H, 128), dk=dk_.reshape(1, T, H, 128), dv=dv_.reshape(1, T, H, 128),
            dg=(dalpha.astype(np.float64) * x["alpha"].reshape(T, H * 128)).reshape(1, T, H, 128),
            dbeta=dbeta32.astype(np.float64).reshape(T, H, 32).sum(-1)[None],
            dS0=dS_in[None]))

    path = os.path.join(args.out, "reference_kda.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
