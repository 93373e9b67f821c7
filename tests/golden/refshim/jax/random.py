"""``jax.random`` is named by the reference's parameter builders only; the fixtures pass explicit arrays."""


def PRNGKey(seed):  # noqa: N802 - jax's name
    raise NotImplementedError("the numpy stand-in has no jax PRNG; pass explicit parameter arrays")


key = PRNGKey


def split(*_a, **_k):
    raise NotImplementedError("the numpy stand-in has no jax PRNG")


normal = uniform = split
