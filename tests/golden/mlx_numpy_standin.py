"""A numpy stand-in for the handful of MLX APIs that alloy's Mamba-2 block uses.

MLX (``mlx>=0.22.0``) is not installable in this environment, so the golden
vectors are produced by executing the reference's own source files
(``alloy/models/mamba_block.py``, ``alloy/models/cache.py``) with
``sys.modules['mlx']`` pointing at this module.  Only the operations those
files call are provided, with MLX's dtype conventions: Python floats and
default-constructed arrays are float32 (numpy would use float64).

This module is test infrastructure: ``make_golden.py`` runs the reference
under it, and ``tests/test_gpu_bridge.py`` installs it as ``mlx`` so that
the MLX bridge's wrappers can be driven with the reference's recorded calls
on a machine without MLX.  Nothing in the product imports it.
"""

from __future__ import annotations

import sys
import types

import numpy as np

float32 = np.float32
float16 = np.float16
bfloat16 = np.float32  # numpy has no bf16; goldens run fp32 on bf16-rounded inputs


def _f32(a):
    a = np.asarray(a)
    return a.astype(np.float32) if a.dtype == np.float64 else a


def array(v, dtype=None):
    a = np.asarray(v, dtype=dtype)
    return a if dtype is not None else _f32(a)


def zeros(shape, dtype=np.float32):
    return np.zeros(shape, dtype=dtype)


def ones(shape, dtype=np.float32):
    return np.ones(shape, dtype=dtype)


def zeros_like(a):
    return np.zeros_like(a)


def exp(a):
    return np.exp(a)


def log(a):
    return np.log(a)


def clip(a, a_min=None, a_max=None):
    lo = None if a_min is None else np.asarray(a_min, a.dtype)
    hi = None if a_max is None else np.asarray(a_max, a.dtype)
    return np.clip(a, lo, hi)


def cumsum(a, axis=None):
    return np.cumsum(a, axis=axis, dtype=a.dtype)


def where(cond, a, b):
    return np.where(cond, _f32(a), _f32(b))


def tril(a, k=0):
    return np.tril(a, k)


def concatenate(arrs, axis=0):
    return np.concatenate(arrs, axis=axis)


def stack(arrs, axis=0):
    return np.stack(arrs, axis=axis)


def pad(a, pad_width, constant_values=0):
    return np.pad(a, pad_width, constant_values=constant_values)


def repeat(a, repeats, axis=None):
    return np.repeat(a, repeats, axis=axis)


def sigmoid(a):
    one = a.dtype.type(1)
    return one / (one + np.exp(-a))


def eval(*_a, **_k):  # noqa: A001 - MLX name
    return None


class _Random(types.SimpleNamespace):
    _rng = np.random.default_rng(1234)

    def seed(self, s):
        _Random._rng = np.random.default_rng(s)

    def normal(self, shape=(), dtype=np.float32):
        return _Random._rng.standard_normal(shape).astype(dtype)

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=np.float32):
        return _Random._rng.uniform(low, high, shape).astype(dtype)


random = _Random()


# ---- mlx.nn ---------------------------------------------------------------

class Module:
    def __init__(self):
        pass


class Linear(Module):
    def __init__(self, in_dims, out_dims, bias=True):
        super().__init__()
        self.weight = random.normal((out_dims, in_dims)) * np.float32(0.02)
        self.bias = zeros((out_dims,)) if bias else None

    def __call__(self, x):
        y = x @ self.weight.T
        return y if self.bias is None else y + self.bias


class RMSNorm(Module):
    def __init__(self, dims, eps=1e-5):
        super().__init__()
        self.weight = ones((dims,))
        self.eps = eps

    def __call__(self, x):
        ms = np.mean(x * x, axis=-1, keepdims=True)
        return self.weight * x / np.sqrt(ms + np.float32(self.eps))


def silu(a):
    return a * sigmoid(a)


def softplus(a):
    return np.logaddexp(a, a.dtype.type(0)).astype(a.dtype, copy=False)


class AtArray(np.ndarray):
    """An ndarray with MLX's functional scatter, ``a.at[idx].add(v)`` (a new
    array with v added at idx), for the code paths that use it."""

    @property
    def at(self):
        return _At(self)


class _At:
    def __init__(self, a):
        self._a = a

    def __getitem__(self, idx):
        a = self._a

        class _Idx:
            @staticmethod
            def add(v):
                r = a.copy()
                r[idx] += v
                return r

        return _Idx()


def custom_function(f):
    """``mx.custom_function``: calls f; ``.vjp`` registers and returns the VJP."""

    class _Custom:
        def __init__(self):
            self.vjp_fn = None

        def __call__(self, *args):
            return f(*args)

        def vjp(self, g):
            self.vjp_fn = g
            return g

    return _Custom()


def install():
    """Register this module as ``mlx``, ``mlx.core`` and ``mlx.nn``."""
    me = sys.modules[__name__]
    nn = types.ModuleType("mlx.nn")
    for name in ("Module", "Linear", "RMSNorm", "silu", "softplus", "sigmoid"):
        setattr(nn, name, getattr(me, name))
    pkg = types.ModuleType("mlx")
    pkg.core = me
    pkg.nn = nn
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = me
    sys.modules["mlx.nn"] = nn
