"""Parity of the diagonal engine's per-interval clock mode (the reference's default reweighting mode
"displacement") with the float64 CPU oracle, through the layer and the C ABI.

Every interval has its own clock step, so its own flow and series tables (ews/core/chen_scan.py:155-168
with cached=False, ews/core/series_leaf.py:72-127 per interval). Inputs are rounded to float32 for both
sides; the oracle runs the reference's algorithm on them in float64.

Tolerances (as in tests/test_gpu_diag.py): global relative error max|a-b| / max|b| <= 1e-5 for the
forward and for the gradients of the path, the clock, the diagonal of A and the lift; for paths of at most
256 intervals the forward also elementwise: |out - ref| <= 1e-6 max(1, max|ref|) + 1e-5 |ref|.
"""

import numpy as np
import pytest
import torch

from oracle import ews_oracle as O
from tests.conftest import relerr

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _f32(a):
    return None if a is None else np.asarray(a, dtype=np.float32).astype(np.float64)


def _case(B, T, N, d_in, seed=0, lam_lo=-3.0, lam_hi=1.0, zero_first=False, scale=1.0):
    """C4-style data: AR(1)-like channels, A = diag(e^u), and a per-sample clock with positive steps of
    varying size (softplus of a random gate over T, the shape of a learned input-dependent clock)."""
    rng = np.random.default_rng(seed)
    inc = rng.normal(size=(B, T, d_in)) / np.sqrt(T)
    path = np.concatenate([np.zeros((B, 1, d_in)), np.cumsum(inc, 1)], 1)
    lam = np.exp(rng.uniform(lam_lo, lam_hi, N))
    lift = rng.normal(size=(N, d_in)) / np.sqrt(d_in)
    gate = rng.normal(size=(B, T))
    steps = scale * np.log1p(np.exp(gate)) / T
    if zero_first:
        steps[:, 0] = 0.0
    clock = np.concatenate([np.zeros((B, 1)), np.cumsum(steps, 1)], 1)
    return _f32(path), _f32(clock), _f32(lam), _f32(lift)


def _oracle(path, clock, lam, lift, readout, q, w=None):
    p = torch.tensor(path, requires_grad=True)
    ck = torch.tensor(clock, requires_grad=True)
    L = torch.tensor(lam, requires_grad=True)
    Bm = torch.tensor(lift, requires_grad=True)
    out = O.ews_layer(O.lift(p, Bm), ck, torch.diag(L), 2, leaf="series", series_q=q, reweighting_mode="displacement", readout=readout)
    if w is None:
        return out.detach(), None
    (out * w.double()).sum().backward()
    return out.detach(), (p.grad, ck.grad, L.grad, Bm.grad)


def _kernel(path, clock, lam, lift, readout, q, w=None, chunk=0):
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    A = AParamDiag(torch.tensor(lam, dtype=torch.float32)).to(DEV)
    layer = EWS(A, N=2, reweighting_mode="displacement", leaf="series", series_q=q, combine="b200", combine_chunk=chunk)
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    ck = torch.tensor(clock, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, ck, readout=readout, lift=Bm)
    if w is None:
        return out.detach().cpu().double(), None
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    grads = (p.grad, ck.grad, A.values.grad, Bm.grad)
    return out.detach().cpu().double(), tuple(g.cpu().double() for g in grads)


def _assert_fwd(out, ref, elementwise=True):
    assert out.shape == ref.shape
    e = relerr(out, ref)
    assert e <= 1e-5, f"forward relerr {e:.2e}"
    if elementwise:
        err = (out - ref).abs()
        bound = 1e-6 * max(1.0, float(ref.abs().max())) + 1e-5 * ref.abs()
        assert bool((err <= bound).all()), f"max excess {float((err - bound).max()):.3e}"


def _assert_grads(got, ref):
    for name, g, r in zip(("path", "clock", "lambda", "lift"), got, ref):
        e = relerr(g, r)
        assert e <= 1e-5, f"d/d{name}: relerr {e:.2e}"


@pytest.mark.parametrize("N", [4, 8, 16, 24, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_forward_matches_oracle(N, readout):
    _require_gpu()
    path, clock, lam, lift = _case(3, 60, N, d_in=5, seed=N)
    ref, _ = _oracle(path, clock, lam, lift, readout, q=8)
    out, _ = _kernel(path, clock, lam, lift, readout, q=8, chunk=16)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("chunk", [1, 9, 32, 0])
def test_chunking_and_lookback(chunk):
    _require_gpu()
    path, clock, lam, lift = _case(4, 150, 16, d_in=6, seed=2)
    ref, _ = _oracle(path, clock, lam, lift, "prefix", q=6)
    out, _ = _kernel(path, clock, lam, lift, "prefix", q=6, chunk=chunk)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("q", [0, 1, 3, 8])
def test_series_orders(q):
    """Large clock steps (x up to ~e) make the series order visible in the output."""
    _require_gpu()
    path, clock, lam, lift = _case(2, 40, 8, d_in=3, seed=5, scale=20.0)
    ref, _ = _oracle(path, clock, lam, lift, "prefix", q=q)
    out, _ = _kernel(path, clock, lam, lift, "prefix", q=q, chunk=8)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("N", [8, 16, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_gradients_match_oracle(N, readout):
    _require_gpu()
    path, clock, lam, lift = _case(3, 70, N, d_in=4, seed=10 + N)
    w_shape = (3, 70, 1 + N + N * N) if readout == "prefix" else (3, 1 + N + N * N)
    w = torch.randn(w_shape, generator=torch.Generator().manual_seed(N), dtype=torch.float64)
    ref, gref = _oracle(path, clock, lam, lift, readout, q=8, w=w)
    out, gout = _kernel(path, clock, lam, lift, readout, q=8, w=w, chunk=16)
    _assert_fwd(out, ref)
    _assert_grads(gout, gref)


def test_zero_first_step_and_large_steps():
    """A zero clock step (the identity flow, Q1 = 1, Q2 = 1/2) and steps of order one."""
    _require_gpu()
    path, clock, lam, lift = _case(2, 50, 16, d_in=4, seed=7, zero_first=True, scale=8.0)
    w = torch.randn((2, 50, 1 + 16 + 256), generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    ref, gref = _oracle(path, clock, lam, lift, "prefix", q=8, w=w)
    out, gout = _kernel(path, clock, lam, lift, "prefix", q=8, w=w, chunk=8)
    _assert_fwd(out, ref)
    _assert_grads(gout, gref)


def test_config4_block_shape():
    """One EWS block of config 4's shape (B = 128 -> 16 here, T = 1440, N = 16, lifted 16 -> 16), gradients
    included; global relative errors only (long path)."""
    _require_gpu()
    path, clock, lam, lift = _case(4, 1440, 16, d_in=16, seed=11)
    w = torch.randn((4, 1440, 1 + 16 + 256), generator=torch.Generator().manual_seed(4), dtype=torch.float64)
    ref, gref = _oracle(path, clock, lam, lift, "prefix", q=8, w=w)
    out, gout = _kernel(path, clock, lam, lift, "prefix", q=8, w=w)
    _assert_fwd(out, ref, elementwise=False)
    _assert_grads(gout, gref)
