"""``jax.scipy.linalg`` on scipy (stand-in; both evaluate expm by Pade scaling and squaring)."""

import numpy as _np
import scipy.linalg as _sl

from ..numpy import JArray


def expm(A, **_kw):
    A = _np.asarray(A)
    if A.ndim == 2:
        return _sl.expm(A).view(JArray)
    flat = A.reshape((-1,) + A.shape[-2:])
    return _np.stack([_sl.expm(a) for a in flat]).reshape(A.shape).view(JArray)


def block_diag(*arrs):
    return _sl.block_diag(*[_np.asarray(a) for a in arrs]).view(JArray)


def solve(a, b, **_kw):
    return _np.linalg.solve(_np.asarray(a), _np.asarray(b)).view(JArray)


def inv(a, **_kw):
    return _np.linalg.inv(_np.asarray(a)).view(JArray)
