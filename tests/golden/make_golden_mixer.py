"""Generate the mixer fixtures by executing the reference's own source.

Like ``make_golden.py`` this runs the reference's functions under ``jaxshim``
(no JAX in the build container), loaded unmodified from the checkout given by
``--reference``:

* ``net/shortconv.py:14-30, :33-53``  ``short_conv``, ``short_conv_step``
* ``net/norm.py:15-73``               ``swish``, ``l2_norm`` (and its derivative
                                      rule ``_l2_norm_guarded_jvp``), ``headwise_rms_norm``
* ``net/kda.py:194-203``              ``_postprocess``
* ``net/kda.py:179``                  the decay-gate expression of ``_project``
* ``net/kda.py:206-214``              ``_output_gate``
* ``net/kda.py:277-295``              ``recurrent_step`` (with ``_project``,
                                      ``_delta_step``, ``KDAState``)

``compute_dtype.gemm`` (the projection GEMM with its precision policy, outside
the path) is replaced by a float64 matmul; every other operation is the
reference's own code.

Usage::

    python tests/golden/make_golden_mixer.py --reference <path to the reference checkout>
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


def _load_module(ref_root, rel, name):
    path = os.path.join(ref_root, *rel.split("/"))
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _kda_namespace(ref_root, names, ns):
    """Execute the named top-level definitions of ``net/kda.py`` into ``ns``."""
    path = os.path.join(ref_root, "net", "kda.py")
    tree = ast.parse(open(path).read())
    nodes = {}
    for node in tree.body:
        if isinstance(node, (ast.FunctionDef, ast.ClassDef)) and node.name in names:
            exec(compile(ast.Module(body=[node], type_ignores=[]), path, "exec"), ns)
            nodes[node.name] = node
    return nodes, path


def _gate_expression(project_node, path):
    """The ``g = ...`` assignment of ``_project``, compiled as an expression."""
    for st in ast.walk(project_node):
        if isinstance(st, ast.Assign) and len(st.targets) == 1 and getattr(st.targets[0], "id", "") == "g":
            return compile(ast.Expression(body=st.value), path, "eval"), st.lineno
    raise RuntimeError("decay-gate assignment not found in _project")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()

    jax = jaxshim.install()
    import jax.numpy as jnp

    sc = _load_module(args.reference, "net/shortconv.py", "ref_shortconv")
    nm = _load_module(args.reference, "net/norm.py", "ref_norm")

    class _Gemm(types.ModuleType):
        @staticmethod
        def gemm(x, w, fp8=False):  # noqa: ARG004 - the precision policy is outside the path
            return (np.asarray(x, np.float64) @ np.asarray(w, np.float64)).view(jaxshim.Arr)

    from typing import NamedTuple

    ns = {"jax": jax, "jnp": jnp, "NamedTuple": NamedTuple, "compute_dtype": _Gemm("compute_dtype"),
          "swish": nm.swish, "l2_norm": nm.l2_norm, "headwise_rms_norm": nm.headwise_rms_norm,
          "short_conv": sc.short_conv, "short_conv_step": sc.short_conv_step}
    ns["KDAParams"] = object
    ns["ModelConfig"] = object
    nodes, kda_path = _kda_namespace(
        args.reference, {"KDAState", "_project", "_postprocess", "_output_gate", "_delta_step",
                         "recurrent_step"}, ns)
    gate_expr, gate_line = _gate_expression(nodes["_project"], kda_path)

    A_ = lambda a: np.ascontiguousarray(a, np.float64).view(jaxshim.Arr)  # noqa: E731
    out = {}
    rng = np.random.default_rng(20)

    # 1. short conv: whole-sequence and streaming forms
    T, D, K = 37, 24, 4
    x = rng.standard_normal((T, D))
    w = rng.standard_normal((K, D)) * 0.5
    out["conv/x"], out["conv/w"] = x, w
    out["conv/out"] = np.asarray(sc.short_conv(A_(x), A_(w)))
    buf = A_(np.zeros((K - 1, D)))
    steps = []
    for t in range(T):
        o_t, buf = sc.short_conv_step(A_(x[t]), A_(w), buf)
        steps.append(np.asarray(o_t))
    out["conv/steps"], out["conv/buf"] = np.stack(steps), np.asarray(buf)

    # 2. norms and Swish (a zero row exercises the guarded L2 norm)
    xs = rng.standard_normal((9, 3, 16)) * 2.0
    xs[4, 1] = 0.0
    xd = rng.standard_normal(xs.shape)
    out["norm/x"], out["norm/xdot"] = xs, xd
    out["norm/swish"] = np.asarray(nm.swish(A_(xs)))
    out["norm/l2"] = np.asarray(nm.l2_norm(A_(xs)))
    _, tangent = nm._l2_norm_guarded.jvp_rule(1e-12, -1, (A_(xs),), (A_(xd),))
    out["norm/l2_tangent"] = np.asarray(tangent)
    out["norm/rms"] = np.asarray(nm.headwise_rms_norm(A_(xs)))

    # 3. _postprocess and the decay gate of _project
    H, dk, dv = 2, 16, 8
    cfg = types.SimpleNamespace(num_heads=H, kda_dk=dk, kda_dv=dv, kda_g_min=-5.0)
    qp, kp = rng.standard_normal((5, H * dk)), rng.standard_normal((5, H * dk))
    vp = rng.standard_normal((5, H * dv))
    q, k, v = ns["_postprocess"](A_(qp), A_(kp), A_(vp), cfg)
    out.update({"post/qp": qp, "post/kp": kp, "post/vp": vp, "post/q": np.asarray(q),
                "post/k": np.asarray(k), "post/v": np.asarray(v)})
    z = rng.standard_normal((5, H, dk)) * 2.0
    Ah = rng.standard_normal(H) * 0.5
    g = eval(gate_expr, {"jax": jax, "jnp": jnp}, {"cfg": cfg, "params": types.SimpleNamespace(A=A_(Ah)),
                                                   "z": A_(z)})
    out.update({"gate/z": z, "gate/A": Ah, "gate/g": np.asarray(g), "gate/line": np.array(gate_line)})

    # 4. _output_gate with W_o = I (the gated RMSNorm before the projection)
    o = rng.standard_normal((6, H, dv))
    gate = 1.0 / (1.0 + np.exp(-rng.standard_normal((6, H * dv))))
    y = ns["_output_gate"](A_(o), A_(gate), types.SimpleNamespace(W_o=A_(np.eye(H * dv))))
    out.update({"ogate/o": o, "ogate/gate": gate, "ogate/y": np.asarray(y)})

    # 5. recurrent_step: the streaming decode of one layer, a few tokens
    hid, r, Tn = H * dv, 8, 6
    P = dict(W_q=rng.standard_normal((hid, H * dk)) * 0.3, W_k=rng.standard_normal((hid, H * dk)) * 0.3,
             W_v=rng.standard_normal((hid, H * dv)) * 0.3, W_o=rng.standard_normal((H * dv, hid)) * 0.3,
             W_g=rng.standard_normal((hid, hid)) * 0.3, W_beta=rng.standard_normal((hid, H)) * 0.3,
             W_a_down=rng.standard_normal((hid, r)) * 0.3, W_a_up=rng.standard_normal((r, H * dk)) * 0.3,
             b_alpha=rng.standard_normal(H * dk) * 0.5, A=rng.standard_normal(H) * 0.3,
             conv_q=rng.standard_normal((K, H * dk)) * 0.4, conv_k=rng.standard_normal((K, H * dk)) * 0.4,
             conv_v=rng.standard_normal((K, H * dv)) * 0.4)
    params = types.SimpleNamespace(**{n: A_(a) for n, a in P.items()})
    carry = ns["KDAState"](A_(rng.standard_normal((H, dk, dv)) * 0.1), A_(rng.standard_normal((K - 1, H * dk))),
                           A_(rng.standard_normal((K - 1, H * dk))), A_(rng.standard_normal((K - 1, H * dv))))
    for n_, a in zip(("S", "q_buf", "k_buf", "v_buf"), carry):
        out[f"rec/{n_}0"] = np.asarray(a)
    xr = rng.standard_normal((Tn, hid))
    outs = []
    for t in range(Tn):
        carry, o_t = ns["recurrent_step"](params, cfg, carry, A_(xr[t]))
        outs.append(np.asarray(o_t))
    for n_, a in P.items():
        out[f"rec/{n_}"] = a
    out["rec/x"], out["rec/out"] = xr, np.stack(outs)
    for n_, a in zip(("S", "q_buf", "k_buf", "v_buf"), carry):
        out[f"rec/{n_}"] = np.asarray(a)

    path = os.path.join(args.out, "reference_mixer.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
