"""signax 0.2.1 ``utils`` (restated): Lyndon words by Duval's algorithm, grouped by length."""

from __future__ import annotations

import numpy as _np


def _duval(depth, dim):
    """All Lyndon words over {0..dim-1} of length <= depth, in Duval's generation order."""
    words = []
    w = [-1]
    while w:
        w[-1] += 1
        words.append(list(w))
        m = len(w)
        while len(w) < depth:
            w.append(w[len(w) - m])
        while w and w[-1] == dim - 1:
            w.pop()
    return words


def lyndon_words(depth, dim):
    """Level k: an int array (W_k, k) of the Lyndon words of length k."""
    ws = _duval(depth, dim)
    out = []
    for k in range(1, depth + 1):
        lv = [w for w in ws if len(w) == k]
        out.append(_np.asarray(lv, dtype=_np.int64).reshape(len(lv), k))
    return out


def unravel_signature(flat, dim, depth):
    flat = _np.asarray(flat)
    out, i = [], 0
    for k in range(1, depth + 1):
        n = dim**k
        out.append(flat[..., i : i + n].reshape(flat.shape[:-1] + (dim,) * k))
        i += n
    return out
