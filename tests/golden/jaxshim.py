"""A minimal NumPy stand-in for the parts of ``jax`` that the reference's KDA
reference functions use, so that those functions can be *executed* from the
reference's own source files in a container that has no JAX.

Used only by ``make_golden.py`` and ``make_golden_mixer.py`` (fixture
generation); nothing at test or run time imports it.  It covers exactly what
the generating scripts call: ``jax.numpy`` (delegated to NumPy, with the
``x.at[idx].set/add`` functional update JAX arrays have), ``jax.lax.scan`` (a
Python loop), ``jax.custom_vjp`` and ``jax.jit`` as pass-throughs, and
``jax.custom_jvp``, which keeps the registered derivative rule callable.  The arithmetic is NumPy's; the algorithm --
operation order, tiling, clamps, dtype casts -- is the reference's own code.
"""

from __future__ import annotations

import sys
import types

import ml_dtypes
import numpy as np


class Arr(np.ndarray):
    """ndarray with JAX's ``.at[idx].set(v)`` / ``.add(v)`` functional updates."""

    def __array_finalize__(self, obj):  # noqa: D401 - numpy hook
        pass

    @property
    def at(self):
        arr = self

        class _At:
            def __getitem__(self, idx):
                class _Upd:
                    def set(self, val):
                        out = np.array(arr, copy=True).view(Arr)
                        out[idx] = val
                        return out

                    def add(self, val):
                        out = np.array(arr, copy=True).view(Arr)
                        out[idx] += val
                        return out

                return _Upd()

        return _At()


def _wrap(x):
    if isinstance(x, np.ndarray) and not isinstance(x, Arr):
        return x.view(Arr)
    if isinstance(x, tuple):
        return tuple(_wrap(e) for e in x)
    if isinstance(x, list):
        return [_wrap(e) for e in x]
    return x


def _wrapfn(fn):
    def inner(*a, **k):
        return _wrap(fn(*a, **k))

    return inner


def _make_jnp():
    jnp = types.ModuleType("jax.numpy")
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.float32 = np.float32
    jnp.float64 = np.float64
    jnp.int32 = np.int32
    jnp.bool_ = np.bool_
    jnp.ndarray = np.ndarray

    def dtype(x):
        if isinstance(x, str) and x == "bfloat16":
            return np.dtype(ml_dtypes.bfloat16)
        return np.dtype(x)

    jnp.dtype = dtype
    linalg = types.ModuleType("jax.numpy.linalg")
    linalg.inv = _wrapfn(np.linalg.inv)
    linalg.solve = _wrapfn(np.linalg.solve)
    linalg.norm = _wrapfn(np.linalg.norm)
    jnp.linalg = linalg

    def asarray(x, dtype=None):
        return np.asarray(x, dtype=dtype).view(Arr)

    jnp.asarray = asarray
    jnp.array = lambda x, dtype=None: np.array(x, dtype=dtype).view(Arr)

    def __getattr__(name):
        fn = getattr(np, name)
        return _wrapfn(fn) if callable(fn) else fn

    jnp.__getattr__ = __getattr__
    return jnp


def _scan(f, init, xs, length=None, reverse=False):
    if xs is None:
        n = int(length)
        leaves = None
    else:
        leaves = xs if isinstance(xs, tuple) else (xs,)
        n = leaves[0].shape[0]
    order = range(n - 1, -1, -1) if reverse else range(n)
    carry = init
    ys = [None] * n
    for i in order:
        x = None if leaves is None else (tuple(l[i] for l in leaves) if isinstance(xs, tuple) else xs[i])
        carry, y = f(carry, x)
        ys[i] = y
    if ys and ys[0] is None:
        return carry, None
    if isinstance(ys[0], tuple):
        stacked = tuple(np.stack([y[j] for y in ys]).view(Arr) for j in range(len(ys[0])))
    else:
        stacked = np.stack(ys).view(Arr)
    return carry, stacked


class _CustomJvp:
    """``jax.custom_jvp`` stand-in: calling it runs the primal; ``defjvp``
    records the rule, which ``jvp_rule`` exposes so that a fixture can evaluate
    the reference's own derivative."""

    def __init__(self, fn, nondiff_argnums=()):
        self.fn = fn
        self.nondiff_argnums = tuple(nondiff_argnums)
        self.jvp_rule = None

    def __call__(self, *a, **k):
        return self.fn(*a, **k)

    def defjvp(self, rule):
        self.jvp_rule = rule
        return rule


def install():
    """Register the stand-in as ``jax`` / ``jax.numpy`` / ``jax.lax`` / ``jax.nn``."""
    jax = types.ModuleType("jax")
    jnp = _make_jnp()
    lax = types.ModuleType("jax.lax")
    lax.scan = _scan
    nn = types.ModuleType("jax.nn")
    nn.sigmoid = _wrapfn(lambda x: 1.0 / (1.0 + np.exp(-x)))
    jax.numpy = jnp
    jax.lax = lax
    jax.nn = nn
    jax.jit = lambda f, *a, **k: f
    jax.custom_vjp = lambda f, *a, **k: f
    jax.custom_jvp = _CustomJvp
    jax.devices = lambda *a, **k: []
    sys.modules["jax"] = jax
    sys.modules["jax.numpy"] = jnp
    sys.modules["jax.lax"] = lax
    sys.modules["jax.nn"] = nn
    return jax
