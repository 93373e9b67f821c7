"""Parity of the block engine (2x2 generator blocks, depth 3, per-interval clock; CUDA, fp32) with the
float64 CPU oracle, through the layer and the C ABI.

The generator is config 3's: rotation-decay blocks [[a, w], [-w, a]] (the reference's A_ref = -A_cfg),
an input-dependent clock, the series leaf, the lift inside the kernel. Inputs are rounded to float32 for
both sides; the oracle evaluates the reference's algorithm on them in float64.

Tolerances (as in tests/test_gpu_diag.py): global relative error max|a-b| / max|b| <= 1e-5 for the
forward and every gradient; for paths of at most 256 intervals the forward also elementwise:
|out - ref| <= 1e-6 max(1, M) + 1e-5 |ref|, with M the largest magnitude of the prefix stream (for a
terminal or mean readout too: a float32 scan's absolute error is set by the largest values it carried,
and these rotation-decay states pass through values ten times their final size).
"""

import math

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
    return np.asarray(a, dtype=np.float32).astype(np.float64)


def _case(B, T, N, d_in=4, seed=0, rot=True, step_scale=1.0):
    """Config-3 data at a small size: AR(1) channels, lift d_in -> N, 2x2 blocks, softplus clock steps.
    rot=False draws general 2x2 blocks whose symmetric part is positive definite (decaying flows): a
    rotation-decay block plus a random symmetric perturbation."""
    rng = np.random.default_rng(seed)
    x = np.zeros((B, T + 1, d_in))
    eps = rng.normal(size=(B, T + 1, d_in))
    for t in range(1, T + 1):
        x[:, t] = 0.9 * x[:, t - 1] + eps[:, t]
    A = np.zeros((N, N))
    for j in range(N // 2):
        a, w = rng.uniform(0.05, 1.0), rng.uniform(0.0, math.pi)
        blk = np.array([[a, w], [-w, a]])
        if not rot:
            e = rng.normal(size=3) * a / 3
            blk = blk + np.array([[e[0], e[1]], [e[1], e[2]]])
        A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = blk
    lift = rng.normal(size=(N, d_in)) / math.sqrt(d_in)
    wc = rng.normal(size=d_in) / 2.0
    dtau = step_scale * np.log1p(np.exp(x[:, :-1] @ wc)) / T
    clock = np.concatenate([np.zeros((B, 1)), np.cumsum(dtau, 1)], 1)
    return _f32(x), _f32(clock), _f32(A), _f32(lift)


def _oracle(path, clock, A, lift, readout, q, w=None):
    p = torch.tensor(path, requires_grad=True)
    ck = torch.tensor(clock, requires_grad=True)
    At = torch.tensor(A, requires_grad=True)
    Bm = torch.tensor(lift, requires_grad=True)
    out = O.ews_layer(O.lift(p, Bm), ck, At, 3, leaf="series", series_q=q, reweighting_mode="displacement", readout=readout)
    if w is None:
        return out.detach(), None
    (out * w.double()).sum().backward()
    # the generator's parameters are its 2x2 diagonal blocks: compare the gradient there
    N = At.shape[0]
    mask = torch.block_diag(*[torch.ones(2, 2, dtype=torch.float64)] * (N // 2))
    return out.detach(), (p.grad, ck.grad, At.grad * mask, Bm.grad)


def _kernel(path, clock, A, lift, readout, q, w=None, chunk=0):
    from exponentially_weighted_signature_b200 import EWS, AParamBlockDiag

    N = A.shape[0]
    blocks = [torch.tensor(A[2 * k : 2 * k + 2, 2 * k : 2 * k + 2], dtype=torch.float32) for k in range(N // 2)]
    Ap = AParamBlockDiag(blocks, (2,) * (N // 2)).to(DEV)
    layer = EWS(Ap, N=3, reweighting_mode="displacement", leaf="series", series_q=q, combine="b200", combine_chunk=chunk)
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    ck = torch.tensor(clock, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, ck, readout=readout, lift=Bm)
    if w is None:
        return out.detach().cpu().double(), None
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    gA = torch.block_diag(*[b.grad for b in Ap.blocks])
    grads = (p.grad, ck.grad, gA, Bm.grad)
    return out.detach().cpu().double(), tuple(g.cpu().double() for g in grads)


def _assert_fwd(out, ref, elementwise=True, scale=None):
    assert out.shape == ref.shape
    e = relerr(out, ref)
    assert e <= 1e-5, f"forward relerr {e:.2e}"
    if elementwise:
        err = (out - ref).abs()
        M = float(ref.abs().max()) if scale is None else scale
        bound = 1e-6 * max(1.0, M) + 1e-5 * ref.abs()
        assert bool((err <= bound).all()), f"max excess {float((err - bound).max()):.3e}"


@pytest.mark.parametrize("N", [2, 4, 6, 8])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_forward_matches_oracle(N, readout):
    _require_gpu()
    path, clock, A, lift = _case(3, 40, N, seed=N)
    ref, _ = _oracle(path, clock, A, lift, readout, q=5)
    out, _ = _kernel(path, clock, A, lift, readout, q=5, chunk=8)
    scale = float(_oracle(path, clock, A, lift, "prefix", q=5)[0].abs().max())
    _assert_fwd(out, ref, scale=scale)


@pytest.mark.parametrize("chunk", [1, 5, 16, 0])
def test_chunking_and_lookback(chunk):
    _require_gpu()
    path, clock, A, lift = _case(3, 100, 8, seed=1)
    ref, _ = _oracle(path, clock, A, lift, "prefix", q=5)
    out, _ = _kernel(path, clock, A, lift, "prefix", q=5, chunk=chunk)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("q", [0, 1, 3, 8])
def test_series_orders_and_general_blocks(q):
    """Large clock steps make the series order visible; general (non-rotation) 2x2 blocks."""
    _require_gpu()
    path, clock, A, lift = _case(2, 30, 8, seed=3, rot=False, step_scale=20.0)
    ref, _ = _oracle(path, clock, A, lift, "prefix", q=q)
    out, _ = _kernel(path, clock, A, lift, "prefix", q=q, chunk=8)
    _assert_fwd(out, ref)


def _assert_grads(got, ref):
    for name, g, r in zip(("path", "clock", "A", "lift"), got, ref):
        e = relerr(g, r)
        assert e <= 1e-5, f"d/d{name}: relerr {e:.2e}"


@pytest.mark.parametrize("N", [2, 4, 8])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_gradients_match_oracle(N, readout):
    _require_gpu()
    path, clock, A, lift = _case(3, 40, N, seed=20 + N)
    D = N + N * N + N * N * N
    w_shape = (3, 40, 1 + D) if readout == "prefix" else (3, 1 + D)
    w = torch.randn(w_shape, generator=torch.Generator().manual_seed(N), dtype=torch.float64)
    ref, gref = _oracle(path, clock, A, lift, readout, q=5, w=w)
    out, gout = _kernel(path, clock, A, lift, readout, q=5, w=w, chunk=8)
    assert relerr(out, ref) <= 1e-5
    _assert_grads(gout, gref)


@pytest.mark.parametrize("chunk", [1, 7, 0])
def test_gradients_chunking_general_blocks(chunk):
    _require_gpu()
    path, clock, A, lift = _case(2, 60, 8, seed=31, rot=False, step_scale=4.0)
    w = torch.randn((2, 60, 1 + 8 + 64 + 512), generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    ref, gref = _oracle(path, clock, A, lift, "prefix", q=6, w=w)
    out, gout = _kernel(path, clock, A, lift, "prefix", q=6, w=w, chunk=chunk)
    assert relerr(out, ref) <= 1e-5
    _assert_grads(gout, gref)


@pytest.mark.parametrize("chunk", [1, 7, 0])
def test_terminal_gradients_recompute_the_chunks(chunk):
    """Terminal readout with gradients: the backward re-runs every chunk from the forward's saved chunk
    start into per-worker scratch rows (as the reference's block_terminal_vjp, pallas_combine.py:1911-2027)
    instead of reading a prefix stream. One-interval chunks, a ragged last chunk (60 = 7 x 8 + 4) and the
    engine's own chunk length."""
    _require_gpu()
    path, clock, A, lift = _case(2, 60, 8, seed=32, rot=False, step_scale=4.0)
    w = torch.randn((2, 1 + 8 + 64 + 512), generator=torch.Generator().manual_seed(6), dtype=torch.float64)
    ref, gref = _oracle(path, clock, A, lift, "terminal", q=6, w=w)
    out, gout = _kernel(path, clock, A, lift, "terminal", q=6, w=w, chunk=chunk)
    assert relerr(out, ref) <= 1e-5
    _assert_grads(gout, gref)


def test_terminal_training_step_keeps_no_prefix_stream():
    """What autograd keeps for a terminal fwd+bwd is the (B, 1 + D) terminal row, not a (B, T, 1 + D)
    prefix stream, and the gradients equal the prefix path's (its last row's cotangent)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamBlockDiag

    B, T, N = 3, 200, 8
    W = 1 + N + N * N + N * N * N
    path, clock, A, lift = _case(B, T, N, seed=41)
    blocks = [torch.tensor(A[2 * k : 2 * k + 2, 2 * k : 2 * k + 2], dtype=torch.float32) for k in range(N // 2)]
    w = torch.randn((B, W), generator=torch.Generator().manual_seed(7)).to(DEV)
    grads = {}
    for readout in ("terminal", "prefix"):
        Ap = AParamBlockDiag(blocks, (2,) * (N // 2)).to(DEV)
        layer = EWS(Ap, N=3, reweighting_mode="displacement", leaf="series", series_q=5)
        p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
        ck = torch.tensor(clock, dtype=torch.float32, device=DEV, requires_grad=True)
        Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
        shapes = []

        def pack(t):
            shapes.append(tuple(t.shape))
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            out = layer(p, ck, readout=readout, lift=Bm)
        last = out if readout == "terminal" else out[:, -1]
        (last * w).sum().backward()
        torch.cuda.synchronize()
        if readout == "terminal":
            assert (B, T, W) not in shapes, shapes
        gA = torch.block_diag(*[b.grad for b in Ap.blocks])
        grads[readout] = (p.grad, ck.grad, gA, Bm.grad)
    for name, a, b in zip(("path", "clock", "A", "lift"), grads["terminal"], grads["prefix"]):
        e = relerr(a.double().cpu(), b.double().cpu())
        assert e <= 1e-5, f"d/d{name}: terminal vs prefix relerr {e:.2e}"


def test_config3_terminal_full_length():
    """Config 3 at full length (T = 2048, N = 8, depth 3, the softplus clock), batch 2: the terminal readout
    with gradients (every chunk re-run from its carry in the backward) against the oracle."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import workloads

    case = workloads.config3(B=2)
    path, clock, A, lift = (_f32(case[k]) for k in ("path", "clock", "A", "lift"))
    w = torch.randn((2, 1 + 8 + 64 + 512), generator=torch.Generator().manual_seed(11), dtype=torch.float64)
    ref, gref = _oracle(path, clock, A, lift, "terminal", q=5, w=w)
    out, gout = _kernel(path, clock, A, lift, "terminal", q=5, w=w)
    assert relerr(out, ref) <= 1e-5
    _assert_grads(gout, gref)
