"""Pytrees over tuples, lists, dicts and None (the containers the reference's core code passes)."""

from __future__ import annotations


class _Def:
    __slots__ = ("kind", "children", "meta")

    def __init__(self, kind, children=(), meta=None):
        self.kind, self.children, self.meta = kind, children, meta


def tree_flatten(tree):
    leaves = []

    def rec(t):
        if t is None:
            return _Def("none")
        if isinstance(t, tuple) and not hasattr(t, "_fields"):
            return _Def("tuple", tuple(rec(c) for c in t))
        if isinstance(t, tuple):
            return _Def("namedtuple", tuple(rec(c) for c in t), type(t))
        if isinstance(t, list):
            return _Def("list", tuple(rec(c) for c in t))
        if isinstance(t, dict):
            keys = sorted(t)
            return _Def("dict", tuple(rec(t[k]) for k in keys), keys)
        leaves.append(t)
        return _Def("leaf")

    d = rec(tree)
    return leaves, d


def tree_unflatten(treedef, leaves):
    it = iter(leaves)

    def rec(d):
        if d.kind == "leaf":
            return next(it)
        if d.kind == "none":
            return None
        kids = [rec(c) for c in d.children]
        if d.kind == "tuple":
            return tuple(kids)
        if d.kind == "namedtuple":
            return d.meta(*kids)
        if d.kind == "list":
            return kids
        return dict(zip(d.meta, kids))

    return rec(treedef)


def tree_leaves(tree):
    return tree_flatten(tree)[0]


def tree_map(f, tree, *rest):
    leaves, d = tree_flatten(tree)
    others = [tree_flatten(r)[0] for r in rest]
    return tree_unflatten(d, [f(l, *[o[i] for o in others]) for i, l in enumerate(leaves)])


def tree_structure(tree):
    return tree_flatten(tree)[1]
