"""Import the reference's own ``ews`` modules, unmodified, on the numpy stand-ins in ``refshim/``.

Test infrastructure for ``make_golden.py`` (fixture generation in the development container, where
the reference checkout exists). The package object ``ews`` is created directly so that its
``__init__`` (which pulls in the training scaffold) does not run; ``ews.layer``, ``ews.params`` and
``ews.core.*`` then import from the reference tree as they are.
"""

from __future__ import annotations

import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
SHIM = os.path.join(HERE, "refshim")


def import_reference(root: str):
    if not os.path.isdir(os.path.join(root, "ews")):
        raise FileNotFoundError(f"no reference checkout at {root}")
    if SHIM not in sys.path:
        sys.path.insert(0, SHIM)
    if "jax" in sys.modules and not getattr(sys.modules["jax"], "__file__", "").startswith(SHIM):
        raise RuntimeError("a real jax is already imported; run the fixture generator in a fresh process")
    if "ews" not in sys.modules:
        pkg = types.ModuleType("ews")
        pkg.__path__ = [os.path.join(root, "ews")]
        sys.modules["ews"] = pkg
    import ews.layer as layer  # noqa: E402
    import ews.params as params  # noqa: E402

    return layer, params
