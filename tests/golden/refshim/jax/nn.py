"""``jax.nn`` activations on numpy (stand-in)."""

import numpy as _np

from .numpy import JArray


def _w(x):
    return _np.asarray(x).view(JArray)


def sigmoid(x):
    return _w(1.0 / (1.0 + _np.exp(-_np.asarray(x))))


def softplus(x):
    x = _np.asarray(x)
    return _w(_np.logaddexp(0.0, x))


def relu(x):
    return _w(_np.maximum(_np.asarray(x), 0))


def gelu(x, approximate=True):
    x = _np.asarray(x)
    return _w(0.5 * x * (1.0 + _np.tanh(_np.sqrt(2.0 / _np.pi) * (x + 0.044715 * x**3))))
