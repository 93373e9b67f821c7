"""A minimal ``equinox`` stand-in: ``Module`` is a dataclass-like base class (numpy stand-in for
golden-vector generation; no filtering, no tree flattening of modules)."""

from __future__ import annotations

import dataclasses


def field(*, static=False, converter=None, **kw):
    md = dict(kw.pop("metadata", {}) or {})
    md["static"] = static
    return dataclasses.field(metadata=md, **kw)


def _has_custom_init(cls):
    for k in cls.__mro__:
        if k is Module or k is object:
            return False
        if "__init__" in k.__dict__ and not getattr(k.__dict__["__init__"], "_eqx_generated", False):
            return True
    return False


class Module:
    def __init_subclass__(cls, **kw):
        super().__init_subclass__(**kw)
        if not _has_custom_init(cls):
            dataclasses.dataclass(cls, init=True, repr=False, eq=False)
            if "__init__" in cls.__dict__:
                cls.__init__._eqx_generated = True


def static_field(**kw):
    return field(static=True, **kw)


def filter_jit(fun=None, **_kw):
    if fun is None:
        return lambda f: f
    return fun


def is_array(x):
    import numpy as np

    return isinstance(x, np.ndarray)


class nn:  # noqa: N801 - equinox's namespace
    pass
