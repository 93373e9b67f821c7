"""Parity of the diagonal engine (CUDA, fp32) with the float64 CPU oracle, through the C ABI.

Tolerance (fp32 kernel against the float64 restatement of the reference): forward elementwise
|out - ref| <= 1e-6 + 1e-5 |ref| (the north star's rel 1e-5 / abs 1e-6), gradients by the reference's
global relative error max|a-b|/max|b| <= 1e-5, plus the reference's own f32 acceptance rule
(tests/test_engines.py:131-164: relerr < 2e-3).
"""

import numpy as np
import pytest
import torch

from oracle import ews_oracle as O
from tests.conftest import relerr

pytestmark = pytest.mark.gpu

DEV = "cuda"
Q = 8


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _case(B, T, N, d_in=None, seed=0, lam_lo=-3.0, lam_hi=1.0, h=None):
    """C1-style data: Brownian channels + time channel lifted by B ~ N(0, 1/d_in), A = diag(e^u)."""
    rng = np.random.default_rng(seed)
    d_in = d_in or N
    inc = rng.normal(size=(B, T, d_in)) / np.sqrt(T)
    path = np.concatenate([np.zeros((B, 1, d_in)), np.cumsum(inc, 1)], 1)
    lam = np.exp(rng.uniform(lam_lo, lam_hi, N))
    lift = rng.normal(size=(N, d_in)) / np.sqrt(d_in)
    h = h if h is not None else 1.0 / T
    clock = np.broadcast_to(np.arange(T + 1) * h, (B, T + 1)).copy()
    return path, clock, lam, lift


def _oracle(path, clock, lam, lift, readout, mode="displacement_uniform", w=None):
    p = torch.tensor(path, dtype=torch.float64, requires_grad=True)
    L = torch.tensor(lam, dtype=torch.float64, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=torch.float64, requires_grad=True)
    y = p if Bm is None else O.lift(p, Bm)
    out = O.ews_layer(y, torch.tensor(clock, dtype=torch.float64), torch.diag(L), 2, series_q=Q, reweighting_mode=mode, readout=readout)
    if w is None:
        return out.detach(), None
    (out * w).sum().backward()
    return out.detach(), (p.grad, L.grad, None if Bm is None else Bm.grad)


def _kernel(path, clock, lam, lift, readout, mode="displacement_uniform", w=None, chunk=0):
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    A = AParamDiag(torch.tensor(lam, dtype=torch.float32)).to(DEV)
    layer = EWS(A, N=2, reweighting_mode=mode, series_q=Q, combine_chunk=chunk)
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
    if w is None:
        return out.detach().cpu().double(), None
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    return out.detach().cpu().double(), (p.grad.cpu().double(), A.values.grad.cpu().double(), None if Bm is None else Bm.grad.cpu().double())


def _assert_fwd(out, ref):
    assert out.shape == ref.shape
    err = (out - ref).abs()
    bound = 1e-6 + 1e-5 * ref.abs()
    assert bool((err <= bound).all()), f"max excess {float((err - bound).max()):.3e}, relerr {relerr(out, ref):.2e}"


@pytest.mark.parametrize("N", [4, 8, 12, 16, 24, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean", "max"])
def test_forward_matches_oracle(N, readout):
    _require_gpu()
    path, clock, lam, lift = _case(3, 50, N, d_in=5, seed=N)
    ref, _ = _oracle(path, clock, lam, lift, readout)
    out, _ = _kernel(path, clock, lam, lift, readout, chunk=16)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("chunk", [1, 7, 16, 64, 0])
def test_chunking_and_lookback(chunk):
    """Many chunks per sample exercise the decoupled look-back; chunk=1 is one interval per tile."""
    _require_gpu()
    path, clock, lam, lift = _case(5, 130, 16, d_in=4, seed=3)
    ref, _ = _oracle(path, clock, lam, lift, "prefix")
    out, _ = _kernel(path, clock, lam, lift, "prefix", chunk=chunk)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("N", [8, 16, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_gradients_match_oracle(N, readout):
    _require_gpu()
    path, clock, lam, lift = _case(3, 70, N, d_in=6, seed=10 + N)
    ref, _ = _oracle(path, clock, lam, lift, readout)
    w = torch.tensor(np.random.default_rng(3).normal(size=ref.shape))
    _, (gp_r, gl_r, gb_r) = _oracle(path, clock, lam, lift, readout, w=w)
    _, (gp_n, gl_n, gb_n) = _kernel(path, clock, lam, lift, readout, w=w, chunk=16)
    for name, a, b in [("path", gp_n, gp_r), ("lambda", gl_n, gl_r), ("lift", gb_n, gb_r)]:
        e = relerr(a, b)
        assert e < 1e-5, f"{name} grad relerr {e:.2e}"


def test_identity_lift_and_basepoint_mode():
    _require_gpu()
    rng = np.random.default_rng(7)
    B, T, N = 2, 40, 8
    path = np.cumsum(rng.normal(size=(B, T + 1, N)) * 0.2, 1)
    path[:, 0] = path[:, 1]  # basepoint knot: zero first increment
    clock = np.broadcast_to(np.concatenate([[0.0], np.arange(T) * 0.05]), (B, T + 1)).copy()
    lam = rng.uniform(0.1, 2.0, N)
    for readout in ("prefix", "terminal"):
        ref, _ = _oracle(path, clock, lam, None, readout, mode="displacement_uniform_basepoint")
        out, _ = _kernel(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", chunk=8)
        _assert_fwd(out, ref)
        w = torch.tensor(rng.normal(size=ref.shape))
        _, (gp_r, gl_r, _) = _oracle(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", w=w)
        _, (gp_n, gl_n, _) = _kernel(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", w=w, chunk=8)
        assert relerr(gp_n, gp_r) < 1e-5 and relerr(gl_n, gl_r) < 1e-5


def test_config1_full_size():
    """B=4, T=4096, 3 Brownian channels + time, lift 4 -> 16, A = diag(e^u), u~U(-3,1)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import workloads

    case = workloads.config1(seed=0)
    ref, _ = _oracle(case["path"], case["clock"], case["lam"], case["lift"], "prefix")
    out, _ = _kernel(case["path"], case["clock"], case["lam"], case["lift"], "prefix")
    _assert_fwd(out, ref)
    w = torch.tensor(np.random.default_rng(3).normal(size=ref.shape))
    _, (gp_r, gl_r, gb_r) = _oracle(case["path"], case["clock"], case["lam"], case["lift"], "prefix", w=w)
    _, (gp_n, gl_n, gb_n) = _kernel(case["path"], case["clock"], case["lam"], case["lift"], "prefix", w=w)
    for name, a, b in [("path", gp_n, gp_r), ("lambda", gl_n, gl_r), ("lift", gb_n, gb_r)]:
        e = relerr(a, b)
        assert e < 1e-5, f"{name} grad relerr {e:.2e}"


def test_backward_is_deterministic_and_status_clean():
    _require_gpu()
    path, clock, lam, lift = _case(4, 300, 16, d_in=4, seed=5)
    w = torch.tensor(np.random.default_rng(9).normal(size=(4, 300, 273)))
    _, g1 = _kernel(path, clock, lam, lift, "prefix", w=w, chunk=16)
    _, g2 = _kernel(path, clock, lam, lift, "prefix", w=w, chunk=16)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_bf16_increments():
    """bf16 increments, fp32 accumulation (config 5's variant): tolerance relerr <= 1e-2 against the f64
    oracle on the unrounded increments, and 1e-5 against the oracle on the bf16-rounded increments."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    rng = np.random.default_rng(11)
    B, T, N = 4, 200, 32
    inc = rng.normal(size=(B, T, N)) / np.sqrt(T)
    lam = np.exp(rng.uniform(-4, 0, N))
    clock = np.broadcast_to(np.arange(T + 1) / T, (B, T + 1)).copy()
    inc_bf = torch.tensor(inc, dtype=torch.float32).to(torch.bfloat16)
    layer = EWS(AParamDiag(torch.tensor(lam, dtype=torch.float32)).to(DEV), N=2, reweighting_mode="displacement_uniform", series_q=Q)
    out = layer(inc_bf.to(DEV), torch.tensor(clock, dtype=torch.float32, device=DEV), readout="terminal", increments=True).cpu().double()
    path_exact = np.concatenate([np.zeros((B, 1, N)), np.cumsum(inc, 1)], 1)
    path_round = np.concatenate([np.zeros((B, 1, N)), np.cumsum(inc_bf.double().numpy(), 1)], 1)
    ref_exact, _ = _oracle(path_exact, clock, lam, None, "terminal")
    ref_round, _ = _oracle(path_round, clock, lam, None, "terminal")
    assert relerr(out, ref_exact) < 1e-2
    _assert_fwd(out, ref_round)
