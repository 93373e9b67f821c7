"""A numpy stand-in for the few jax entry points the reference's ``ews/core`` and ``ews/layer.py`` use.

Test infrastructure only: ``tests/golden/make_golden.py`` puts this directory first on ``sys.path``
so that the reference's own, unmodified modules import and run on numpy in float64, and writes their
outputs as golden fixtures. jax itself cannot be installed on these machines (no wheel offline).

What is restated here is jax's published behaviour, not its code:
* ``jit`` / ``checkpoint`` are the identity (tracing changes no value);
* ``vmap`` maps a function over a leading (or given) axis of every pytree leaf with a Python loop and
  stacks the results;
* ``lax.scan`` / ``lax.cond`` / ``lax.fori_loop`` are the plain loops and branches they are defined as;
* ``lax.associative_scan`` is the odd/even recursion jax documents (combine adjacent pairs, scan the
  pair results, combine them with the even elements, interleave), so the reference's Chen operator is
  applied in the same grouping as under jax;
* ``scipy.linalg.expm`` is scipy's (both are Pade scaling-and-squaring);
* ``custom_vjp`` keeps the primal function (only forward values are generated);
* ``jvp`` is not provided: the fixtures need no forward-mode derivative.
"""

from __future__ import annotations

import numpy as _np

from . import flatten_util, lax, nn, numpy, random, scipy, tree_util  # noqa: F401
from .tree_util import tree_flatten, tree_map, tree_unflatten

Array = _np.ndarray


class _Config:
    def update(self, *_a, **_k):
        return None

    def __getattr__(self, name):
        return None


config = _Config()


def jit(fun=None, **_kw):
    if fun is None:
        return lambda f: f
    return fun


def checkpoint(fun=None, **_kw):
    if fun is None:
        return lambda f: f
    return fun


remat = checkpoint


def _axes_for(in_axes, args):
    if isinstance(in_axes, (list, tuple)):
        if len(in_axes) != len(args):
            raise ValueError("vmap in_axes length mismatch")
        return list(in_axes)
    return [in_axes] * len(args)


def vmap(fun, in_axes=0, out_axes=0, **_kw):
    """Loop over the mapped axis; every leaf of a mapped argument is sliced, unmapped (None) ones are
    passed whole; outputs are stacked leaf by leaf along ``out_axes`` (0 or a negative axis)."""

    def mapped(*args):
        axes = _axes_for(in_axes, args)
        n = None
        flat_args = []
        for a, ax in zip(args, axes):
            leaves, treedef = tree_flatten(a)
            flat_args.append((leaves, treedef, ax))
            if ax is not None:
                for leaf in leaves:
                    size = _np.shape(leaf)[ax]
                    if n is None:
                        n = size
                    elif n != size:
                        raise ValueError("vmap: inconsistent mapped sizes")
        if n is None:
            raise ValueError("vmap: nothing to map over")
        if n == 0:
            # jax gives empty results of the mapped function's output shapes: probe with a zero slice
            call = []
            for leaves, treedef, ax in flat_args:
                if ax is None:
                    call.append(tree_unflatten(treedef, leaves))
                else:
                    call.append(tree_unflatten(treedef, [
                        _np.zeros(_np.delete(_np.shape(l), ax), dtype=_np.asarray(l).dtype) for l in leaves]))
            probe = fun(*call)
            pl, pd = tree_flatten(probe)
            return tree_unflatten(pd, [_np.zeros((0,) + _np.shape(x), dtype=_np.asarray(x).dtype).view(numpy.JArray) for x in pl])
        outs = []
        for i in range(n):
            call = []
            for leaves, treedef, ax in flat_args:
                if ax is None:
                    call.append(tree_unflatten(treedef, leaves))
                else:
                    call.append(tree_unflatten(treedef, [_np.take(_np.asarray(l), i, axis=ax) for l in leaves]))
            outs.append(fun(*call))
        leaves0, treedef0 = tree_flatten(outs[0])
        per_leaf = [tree_flatten(o)[0] for o in outs]
        stacked = []
        for j in range(len(leaves0)):
            st = _np.stack([_np.asarray(p[j]) for p in per_leaf], axis=0)
            if out_axes not in (0, None):
                st = _np.moveaxis(st, 0, out_axes)
            stacked.append(st.view(numpy.JArray))
        return tree_unflatten(treedef0, stacked)

    return mapped


class custom_vjp:
    """Keeps the primal function; ``defvjp`` records nothing (no gradients are traced here)."""

    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.nondiff_argnums = nondiff_argnums

    def defvjp(self, fwd, bwd, **_kw):
        return None

    def __call__(self, *args, **kw):
        return self.fun(*args, **kw)


class custom_jvp(custom_vjp):
    def defjvp(self, jvp_fn, **_kw):
        return None


def jvp(*_a, **_k):
    raise NotImplementedError("the numpy stand-in has no forward-mode derivatives")


def grad(*_a, **_k):
    raise NotImplementedError("the numpy stand-in has no derivatives; fixtures use central differences")


value_and_grad = grad


class default_matmul_precision:  # noqa: N801 - jax's name; a context manager that changes nothing here
    def __init__(self, *_a):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def devices():
    return ["cpu"]


def block_until_ready(x):
    return x
