"""Pallas names imported at module load by the reference's kernels; calling any of them raises."""


def pallas_call(kernel, *, out_shape=None, grid=None, in_specs=None, out_specs=None, backend=None, **_kw):
    raise NotImplementedError("Pallas kernels do not run on the numpy stand-in")


class BlockSpec:
    def __init__(self, *_a, **_k):
        raise NotImplementedError("Pallas kernels do not run on the numpy stand-in")


def program_id(*_a, **_k):
    raise NotImplementedError("Pallas kernels do not run on the numpy stand-in")


def dot(*_a, **_k):
    raise NotImplementedError("Pallas kernels do not run on the numpy stand-in")


load = store = num_programs = dot
