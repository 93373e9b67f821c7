"""Look-back timeouts reach the caller as Python exceptions (failure detection without a GPU fault).

The failure is injected with EWS_F_TEST_WITHHOLD: the chunk every other chunk waits for never
publishes, so their bounded waits run out (a short spin limit keeps that fast), the kernels set the
workspace's error word and return. The layer folds every call's error word into a device-side sticky
word and copies it to pinned host memory without synchronising; the next engine call raises
EWSLookbackTimeout, and ``configure(check_status=True)`` raises at once. The reference raises its
errors as Python exceptions (ews/layer.py:112-152); this is the runtime counterpart.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


@pytest.fixture
def withheld():
    from exponentially_weighted_signature_b200 import _lib, engine, layer

    engine.reset_status()
    old = (layer._EXTRA_FLAGS, engine.SPIN_LIMIT, engine.CHECK_SYNC)
    layer._EXTRA_FLAGS = _lib.EWS_F_TEST_WITHHOLD
    engine.SPIN_LIMIT = 2000
    yield
    layer._EXTRA_FLAGS, engine.SPIN_LIMIT, engine.CHECK_SYNC = old
    torch.cuda.synchronize()
    engine.reset_status()


def _diag_layer(N=16):
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    lam = torch.exp(torch.linspace(-3, 1, N))
    return EWS(AParamDiag(lam).to(DEV), N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=4, combine="b200", combine_chunk=8)


def _inputs(B=2, T=256, d=16):
    g = torch.Generator().manual_seed(0)
    path = torch.cumsum(torch.randn(B, T + 1, d, generator=g) / T**0.5, 1).to(DEV)
    clock = (torch.arange(T + 1, dtype=torch.float32) / T).expand(B, T + 1).contiguous().to(DEV)
    return path, clock


def test_timeout_raises_at_once_with_check_status(withheld):
    _require_gpu()
    from exponentially_weighted_signature_b200 import _lib, configure

    layer = _diag_layer()
    path, clock = _inputs()
    configure(check_status=True)
    try:
        with pytest.raises(_lib.EWSLookbackTimeout):
            layer(path, clock, readout="prefix")
    finally:
        configure(check_status=False)


def test_timeout_raises_on_the_next_call(withheld):
    _require_gpu()
    from exponentially_weighted_signature_b200 import _lib, layer as layer_mod

    layer = _diag_layer()
    path, clock = _inputs()
    layer(path, clock, readout="prefix")  # fails on the device; returns without waiting
    torch.cuda.synchronize()
    layer_mod._EXTRA_FLAGS = 0
    with pytest.raises(_lib.EWSLookbackTimeout):
        layer(path, clock, readout="prefix")
    # raised once: the following calls run normally
    out = layer(path, clock, readout="prefix")
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("engine_kind", ["block"])
def test_timeout_in_other_engines(withheld, engine_kind):
    """The block engine's chains look back like the diagonal engine's. (The dense engine takes its carries
    from scans over precomputed chunk aggregates and has no device-side waits.)"""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamBlockDiag, _lib, configure

    rng = np.random.default_rng(0)
    T = 256
    if engine_kind == "block":
        N, d = 8, 8
        blocks = [torch.tensor([[0.3, 1.0], [-1.0, 0.3]], dtype=torch.float32) for _ in range(N // 2)]
        layer = EWS(AParamBlockDiag(blocks, (2,) * (N // 2)).to(DEV), N=3, reweighting_mode="displacement",
                    leaf="series", series_q=4, combine="b200", combine_chunk=8)
    else:
        N, d = 32, 32
        A = torch.tensor(0.5 * np.eye(N) - 0.1 * rng.normal(size=(N, N)) / N**0.5, dtype=torch.float32)
        layer = EWS(A.to(DEV), N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=3, combine="b200", combine_chunk=8)
    path, clock = _inputs(B=2, T=T, d=d)
    path.requires_grad_(True)
    configure(check_status=True)
    try:
        with pytest.raises(_lib.EWSLookbackTimeout):
            layer(path, clock, readout="prefix").sum().backward()
    finally:
        configure(check_status=False)
