"""Truncated tensor algebra on level lists (signax 0.2.1's ``tensor_ops``, restated; numpy stand-in).
A group-like element is [S_1, ..., S_n] with S_k of shape (..., d, ..., d) (k tensor axes) and an
implicit S_0 = 1."""

from __future__ import annotations

import numpy as _np


def _wrap(x):
    from jax.numpy import JArray

    return _np.asarray(x).view(JArray)


def _outer(a, b, ka, kb):
    """Tensor product over the last ka axes of a and the last kb axes of b (shared leading axes)."""
    a = _np.asarray(a)
    b = _np.asarray(b)
    lead = a.shape[: a.ndim - ka]
    ea = a.reshape(a.shape + (1,) * kb)
    eb = b.reshape(b.shape[: b.ndim - kb] + (1,) * ka + b.shape[b.ndim - kb :])
    out = ea * eb
    return out.reshape(lead + out.shape[len(lead) :])


def mult(X, Y):
    """(1 + X) (x) (1 + Y) truncated at len(X): level k = X_k + Y_k + sum_{i+j=k} X_i (x) Y_j."""
    n = len(X)
    out = []
    for k in range(1, n + 1):
        z = _np.asarray(X[k - 1]) + _np.asarray(Y[k - 1])
        for i in range(1, k):
            z = z + _outer(X[i - 1], Y[k - i - 1], i, k - i)
        out.append(_wrap(z))
    return out


def mult_nonunit(X, Y):
    """Product of two elements with zero level 0: level k = sum_{i+j=k, i,j>=1} X_i (x) Y_j."""
    n = len(X)
    out = []
    for k in range(1, n + 1):
        z = _np.zeros_like(_np.asarray(X[k - 1]))
        for i in range(1, k):
            z = z + _outer(X[i - 1], Y[k - i - 1], i, k - i)
        out.append(z)
    return out


def log(X):
    """Tensor logarithm of 1 + X: sum_{m>=1} (-1)^{m+1} X^m / m, truncated at len(X)."""
    n = len(X)
    acc = [_np.asarray(x).astype(_np.result_type(_np.asarray(x), _np.float64)) for x in X]
    power = [_np.asarray(x) for x in X]
    for m in range(2, n + 1):
        power = mult_nonunit(power, X)
        sign = 1.0 if m % 2 == 1 else -1.0
        acc = [a + sign * p / m for a, p in zip(acc, power)]
    return [_wrap(a) for a in acc]
