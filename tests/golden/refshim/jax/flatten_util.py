"""``jax.flatten_util.ravel_pytree`` on numpy (stand-in)."""

import numpy as _np

from .numpy import JArray
from .tree_util import tree_flatten, tree_unflatten


def ravel_pytree(tree):
    leaves, d = tree_flatten(tree)
    shapes = [_np.shape(l) for l in leaves]
    flat = _np.concatenate([_np.ravel(_np.asarray(l)) for l in leaves]) if leaves else _np.zeros(0)

    def unravel(v):
        out, i = [], 0
        for s in shapes:
            n = int(_np.prod(s))
            out.append(_np.asarray(v[i : i + n]).reshape(s))
            i += n
        return tree_unflatten(d, out)

    return flat.view(JArray), unravel
