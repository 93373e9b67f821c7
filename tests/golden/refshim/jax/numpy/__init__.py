"""numpy standing in for ``jax.numpy`` (test infrastructure: golden-vector generation only).

Arrays are numpy arrays viewed as ``JArray``, which adds jax's functional ``.at[idx].set/add/get``.
Every function of numpy is reachable under its jax name; keyword arguments that only steer XLA
(``precision``, ``preferred_element_type``) are dropped. ``einsum`` runs with numpy's contraction
optimiser, which changes the order of the sums but not the value beyond float64 rounding.
"""

from __future__ import annotations

import numpy as _np


class _AtIndexer:
    def __init__(self, arr, idx):
        self._arr, self._idx = arr, idx

    def set(self, v):
        out = _np.array(self._arr, copy=True)
        out[self._idx] = v
        return out.view(JArray)

    def add(self, v):
        out = _np.array(self._arr, copy=True)
        _np.add.at(out, self._idx, v)
        return out.view(JArray)

    def multiply(self, v):
        out = _np.array(self._arr, copy=True)
        out[self._idx] = out[self._idx] * v
        return out.view(JArray)

    def get(self, **_kw):
        return _np.asarray(self._arr)[self._idx]


class _At:
    def __init__(self, arr):
        self._arr = arr

    def __getitem__(self, idx):
        return _AtIndexer(self._arr, idx)


class JArray(_np.ndarray):
    """A numpy array with jax's ``.at`` update syntax."""

    @property
    def at(self):
        return _At(self)


_DROP = ("precision", "preferred_element_type")


def _wrap(x):
    if isinstance(x, _np.ndarray) and not isinstance(x, JArray):
        return x.view(JArray)
    if isinstance(x, tuple):
        return tuple(_wrap(v) for v in x)
    if isinstance(x, list):
        return [_wrap(v) for v in x]
    return x


def _fn(f):
    def g(*args, **kw):
        for k in _DROP:
            kw.pop(k, None)
        return _wrap(f(*args, **kw))

    g.__name__ = getattr(f, "__name__", "fn")
    return g


ndarray = _np.ndarray
dtype = _np.dtype
float16 = _np.float16
float32 = _np.float32
float64 = _np.float64
complex64 = _np.complex64
complex128 = _np.complex128
int32 = _np.int32
int64 = _np.int64
bool_ = _np.bool_
pi = _np.pi
inf = _np.inf
nan = _np.nan
newaxis = None
finfo = _np.finfo
iinfo = _np.iinfo
issubdtype = _np.issubdtype
floating = _np.floating
complexfloating = _np.complexfloating
integer = _np.integer
bfloat16 = _np.float32  # only named in dtype lists; never computed with here


def einsum(eq, *ops, **kw):
    for k in _DROP:
        kw.pop(k, None)
    kw.setdefault("optimize", True)
    return _wrap(_np.einsum(eq, *ops, **kw))


def asarray(x, dtype=None, **_kw):
    return _wrap(_np.asarray(x, dtype=dtype))


def array(x, dtype=None, copy=True, **_kw):
    return _wrap(_np.array(x, dtype=dtype, copy=copy))


def iscomplexobj(x):
    return _np.iscomplexobj(x)


class _Linalg:
    def __getattr__(self, name):
        return _fn(getattr(_np.linalg, name))


linalg = _Linalg()


class _Fft:
    def __getattr__(self, name):
        return _fn(getattr(_np.fft, name))


fft = _Fft()


def __getattr__(name):
    f = getattr(_np, name)
    if callable(f) and not isinstance(f, type):
        return _fn(f)
    return f
