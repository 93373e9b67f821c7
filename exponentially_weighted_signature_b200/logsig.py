"""Log-signature epilogue of LogEWS: truncated tensor log and the Lyndon-word compression.

signax 0.2.1 (``signature_to_logsignature``, used at ews/layer.py:494,502 of the reference) returns the
coefficients of the Lyndon words of the expanded log, grouped by length; ``lyndon_words`` follows
its published generation order (Duval's algorithm, lexicographic within each length).
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import torch


@lru_cache(maxsize=None)
def lyndon_words(depth: int, dim: int):
    """Lyndon words of lengths 1..depth over {0..dim-1}: a tuple of (W_k, k) int arrays."""
    groups = [[] for _ in range(depth)]
    w = [-1]
    while w:
        w[-1] += 1
        groups[len(w) - 1].append(tuple(w))
        m = len(w)
        while len(w) < depth:
            w.append(w[len(w) - m])
        while w and w[-1] == dim - 1:
            w.pop()
    return tuple(np.asarray(g, dtype=np.int64).reshape(len(g), k + 1) for k, g in enumerate(groups))


def log_level_sizes(d: int, N: int):
    """Witt numbers W_d(1..N) (ews/layer.py:417-420)."""
    return [int(w.shape[0]) for w in lyndon_words(N, d)]


def log_signature_dim(d: int, N: int) -> int:
    return int(sum(log_level_sizes(d, N)))


@lru_cache(maxsize=None)
def _flat_indices(depth: int, dim: int):
    out = []
    for k, wk in enumerate(lyndon_words(depth, dim), start=1):
        idx = np.zeros(wk.shape[0], dtype=np.int64)
        for j in range(k):
            idx = idx * dim + wk[:, j]
        out.append(idx)
    return out


def _mult_nonscalar(X, Y):
    n = len(X)
    Z = [torch.zeros_like(x) for x in X]
    for i in range(1, n + 1):
        for j in range(1, n + 1 - i):
            o = X[i - 1][..., :, None] * Y[j - 1][..., None, :]
            Z[i + j - 1] = Z[i + j - 1] + o.reshape(o.shape[:-2] + (o.shape[-2] * o.shape[-1],))
    return Z


def tensor_log(levels):
    """log(1 + X) truncated at len(levels): sum_j (-1)^{j+1} X^{(x) j} / j."""
    n = len(levels)
    out = list(levels)
    P = list(levels)
    for j in range(2, n + 1):
        P = _mult_nonscalar(P, levels)
        sign = -1.0 if j % 2 == 0 else 1.0
        out = [o + (sign / j) * p for o, p in zip(out, P)]
    return out


@lru_cache(maxsize=None)
def flat_index_tensors(depth: int, dim: int, device: str):
    """The Lyndon-word gather indices of every level as int64 tensors on ``device``, made once per
    (depth, dim, device) so that a forward issues no host-to-device copy."""
    return tuple(torch.as_tensor(ix, device=device) for ix in _flat_indices(depth, dim))


def compress(log_levels, dim: int):
    """Lyndon-word coordinates (..., sum_k W_d(k)) of an expanded log."""
    idx = flat_index_tensors(len(log_levels), dim, str(log_levels[0].device))
    return torch.cat([lv[..., ix] for lv, ix in zip(log_levels, idx)], dim=-1)


def split_levels(flat, dim: int, depth: int):
    """Flat levels 1..depth (without the level-0 column) -> list of (..., dim**k)."""
    out, start = [], 0
    for k in range(1, depth + 1):
        out.append(flat[..., start : start + dim**k])
        start += dim**k
    return out
