"""``jax.lax`` control flow as the plain loops it is defined as (numpy stand-in)."""

from __future__ import annotations

import numpy as _np

from .numpy import JArray
from .tree_util import tree_flatten, tree_unflatten


class Precision:
    DEFAULT = "default"
    HIGH = "high"
    HIGHEST = "highest"


def _stack_trees(items):
    leaves0, d = tree_flatten(items[0])
    per = [tree_flatten(t)[0] for t in items]
    return tree_unflatten(d, [_np.stack([_np.asarray(p[j]) for p in per]).view(JArray) for j in range(len(leaves0))])


def scan(f, init, xs=None, length=None, reverse=False, unroll=1, **_kw):
    """carry, y_t = f(carry, x_t) over the leading axis of xs; ys stacked."""
    if xs is None:
        n = int(length)
        xs_at = lambda i: None  # noqa: E731
    else:
        leaves, d = tree_flatten(xs)
        n = int(_np.shape(leaves[0])[0]) if length is None else int(length)
        xs_at = lambda i: tree_unflatten(d, [l[i] for l in leaves])  # noqa: E731
    order = range(n - 1, -1, -1) if reverse else range(n)
    carry = init
    ys = [None] * n
    for i in order:
        carry, y = f(carry, xs_at(i))
        ys[i] = y
    if n == 0 or ys[0] is None:
        return carry, None
    return carry, _stack_trees(ys)


def cond(pred, true_fun, false_fun, *operands, operand=None):
    ops = operands if operands else (operand,)
    return true_fun(*ops) if bool(pred) else false_fun(*ops)


def fori_loop(lower, upper, body, init):
    v = init
    for i in range(int(lower), int(upper)):
        v = body(i, v)
    return v


def while_loop(cond_fun, body_fun, init):
    v = init
    while bool(cond_fun(v)):
        v = body_fun(v)
    return v


def complex(re, im):  # noqa: A001 - jax's name
    return (_np.asarray(re) + 1j * _np.asarray(im)).view(JArray)


def stop_gradient(x):
    return x


def _ix(ndim, axis, sl):
    idx = [slice(None)] * ndim
    idx[axis] = sl
    return tuple(idx)


def associative_scan(fn, elems, reverse=False, axis=0):
    """Inclusive scan with jax's documented odd/even recursion: combine adjacent pairs, scan those,
    then combine the pair prefixes with the remaining even-position elements and interleave. ``fn``
    receives whole slices along ``axis`` (it is written batched, as under jax)."""
    leaves, d = tree_flatten(elems)
    leaves = [_np.asarray(l) for l in leaves]
    axis = axis % leaves[0].ndim
    if reverse:
        leaves = [_np.flip(l, axis=axis) for l in leaves]

    def sl(ls, s):
        return [l[_ix(l.ndim, axis, s)] for l in ls]

    def combine(a, b):
        if a[0].shape[axis] == 0:
            return [x.copy() for x in b]
        out = fn(tree_unflatten(d, a), tree_unflatten(d, b))
        return [_np.asarray(x) for x in tree_flatten(out)[0]]

    def rec(ls):
        n = ls[0].shape[axis]
        if n < 2:
            return ls
        reduced = combine(sl(ls, slice(0, -1, 2)), sl(ls, slice(1, None, 2)))
        odd = rec(reduced)
        if n % 2 == 0:
            even = combine(sl(odd, slice(0, -1)), sl(ls, slice(2, None, 2)))
        else:
            even = combine(odd, sl(ls, slice(2, None, 2)))
        even = [_np.concatenate([l[_ix(l.ndim, axis, slice(0, 1))], e], axis=axis) for l, e in zip(ls, even)]
        out = []
        for e, o in zip(even, odd):
            shape = list(e.shape)
            shape[axis] = n
            res = _np.empty(shape, dtype=_np.result_type(e, o))
            res[_ix(res.ndim, axis, slice(0, None, 2))] = e
            res[_ix(res.ndim, axis, slice(1, None, 2))] = o
            out.append(res)
        return out

    res = rec(leaves)
    if reverse:
        res = [_np.flip(l, axis=axis) for l in res]
    return tree_unflatten(d, [_np.ascontiguousarray(r).view(JArray) for r in res])


def slice_in_dim(x, start, limit, stride=1, axis=0):
    x = _np.asarray(x)
    axis = axis % x.ndim
    return x[_ix(x.ndim, axis, slice(start, limit, stride))].view(JArray)


def index_in_dim(x, index, axis=0, keepdims=True):
    x = _np.asarray(x)
    axis = axis % x.ndim
    out = _np.take(x, [index] if keepdims else index, axis=axis)
    return _np.asarray(out).view(JArray)
