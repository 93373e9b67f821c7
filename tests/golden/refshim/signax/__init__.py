"""A numpy restatement of the parts of signax 0.2.1 (third-party, not installed) that the reference's
EWS path calls: ``tensor_ops.mult`` (truncated tensor product of group-like elements with implicit
level 0), ``signature`` of a piecewise-linear path (Chen products of the segments' tensor
exponentials), ``signature_to_logsignature`` (tensor logarithm, then the coefficients of the Lyndon
words in Duval order) and ``utils.lyndon_words``. Written from the published definitions; test
infrastructure for golden-vector generation only."""

from __future__ import annotations

import numpy as _np

from . import tensor_ops, utils  # noqa: F401
from .tensor_ops import _wrap, mult


def _segment_exp(delta, depth):
    out = [delta]
    for k in range(2, depth + 1):
        out.append(_np.multiply.outer(out[-1], delta) / k)
    return out


def signature(path, depth, stream=False, flatten=True, num_chunks=1):
    path = _np.asarray(path)
    if path.ndim != 2:
        raise ValueError("signature stand-in: one path (length, dim) at a time")
    incs = path[1:] - path[:-1]
    S = _segment_exp(incs[0], depth)
    trace = [S]
    for dlt in incs[1:]:
        S = mult(S, _segment_exp(dlt, depth))
        trace.append(S)
    if stream:
        res = [_np.stack([t[k] for t in trace]) for k in range(depth)]
        if flatten:
            return _wrap(_np.concatenate([r.reshape(r.shape[0], -1) for r in res], axis=1))
        return [_wrap(r) for r in res]
    if flatten:
        return _wrap(_np.concatenate([s.ravel() for s in S]))
    return [_wrap(s) for s in S]


def signature_to_logsignature(signature, stream=False, flatten=False):
    if not isinstance(signature, (list, tuple)):
        raise ValueError("signature_to_logsignature stand-in takes the level list")
    depth = len(signature)
    dim = _np.shape(signature[0])[-1]
    log = tensor_ops.log(list(signature))
    words = utils.lyndon_words(depth, dim)
    out = []
    for k, (lv, w) in enumerate(zip(log, words), start=1):
        flat = _np.asarray(lv).reshape(_np.shape(lv)[: _np.ndim(lv) - k] + (dim**k,))
        idx = _np.zeros(w.shape[0], dtype=_np.int64)
        for j in range(k):
            idx = idx * dim + w[:, j]
        out.append(_wrap(flat[..., idx]))
    if flatten:
        return _wrap(_np.concatenate([o.reshape(o.shape[:-1] + (-1,)) for o in out], axis=-1))
    return out
