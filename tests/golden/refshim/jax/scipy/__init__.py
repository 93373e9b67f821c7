"""``jax.scipy`` stand-in."""

from . import linalg  # noqa: F401
