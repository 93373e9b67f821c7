"""Parity of the diagonal engine (CUDA, fp32) with the float64 CPU oracle, through the C ABI.

Both sides see the same inputs: every array is rounded to float32 first (the kernel's input type), and
the oracle evaluates the reference's algorithm on those values in float64.

Tolerances (written here, applied below):
* every forward and gradient: the reference's global relative error max|a-b| / max|b|
  (tests/test_engines.py:31-33) at most 1e-5 against the float64 oracle, and at most 4x the error of
  the reference's own algorithm run in float32 plus 1e-5 (its f32 acceptance rule, :131-164);
* paths of at most 256 intervals, forward elementwise: |out - ref| <= 1e-6 max(1, max|ref|) + 1e-5 |ref|
  (the north star's abs 1e-6 / rel 1e-5, the absolute part taken relative to outputs of unit scale).
For long paths the elementwise form is out of reach of any float32 scan: the reference's own float32
path misses it on 59% of the config-1 entries (relerr 8e-5), this kernel stays near 2e-6.
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
    return _f32(path), _f32(clock), _f32(lam), _f32(lift)


def _f32(a):
    """Round to float32 (the kernel's inputs) and keep as float64 for the oracle."""
    return None if a is None else np.asarray(a, dtype=np.float32).astype(np.float64)


def _oracle(path, clock, lam, lift, readout, mode="displacement_uniform", w=None, dtype=torch.float64):
    p = torch.tensor(path, dtype=dtype, requires_grad=True)
    L = torch.tensor(lam, dtype=dtype, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=dtype, requires_grad=True)
    y = p if Bm is None else O.lift(p, Bm)
    out = O.ews_layer(y, torch.tensor(clock, dtype=dtype), torch.diag(L), 2, leaf="series", series_q=Q, reweighting_mode=mode, readout=readout)
    if w is None:
        return out.detach().double(), None
    (out * w.to(dtype)).sum().backward()
    grads = (p.grad.double(), L.grad.double(), None if Bm is None else Bm.grad.double())
    return out.detach().double(), grads


def _kernel(path, clock, lam, lift, readout, mode="displacement_uniform", w=None, chunk=0):
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    A = AParamDiag(torch.tensor(lam, dtype=torch.float32)).to(DEV)
    layer = EWS(A, N=2, reweighting_mode=mode, leaf="series", series_q=Q, combine="b200", combine_chunk=chunk)
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
    if w is None:
        return out.detach().cpu().double(), None
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    return out.detach().cpu().double(), (p.grad.cpu().double(), A.values.grad.cpu().double(), None if Bm is None else Bm.grad.cpu().double())


def _assert_close(name, out, ref, ref32=None):
    """Global relerr <= 1e-5 and, when the float32 reference run is given, <= 4x its error + 1e-5."""
    assert out.shape == ref.shape, name
    e = relerr(out, ref)
    assert e <= 1e-5, f"{name}: relerr {e:.2e}"
    if ref32 is not None:
        e32 = relerr(ref32, ref)
        assert e <= 4 * e32 + 1e-5, f"{name}: relerr {e:.2e} vs float32 reference {e32:.2e}"


def _assert_fwd(out, ref, ref32=None, elementwise=True):
    _assert_close("forward", out, ref, ref32)
    if elementwise:
        err = (out - ref).abs()
        bound = 1e-6 * max(1.0, float(ref.abs().max())) + 1e-5 * ref.abs()
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
        _assert_close(f"{name} grad", a, b)


def test_identity_lift_and_basepoint_mode():
    _require_gpu()
    rng = np.random.default_rng(7)
    B, T, N = 2, 40, 8
    path = np.cumsum(rng.normal(size=(B, T + 1, N)) * 0.2, 1)
    path[:, 0] = path[:, 1]  # basepoint knot: zero first increment
    clock = np.broadcast_to(np.concatenate([[0.0], np.arange(T) * 0.05]), (B, T + 1)).copy()
    lam = rng.uniform(0.1, 2.0, N)
    path, clock, lam = _f32(path), _f32(clock), _f32(lam)
    for readout in ("prefix", "terminal"):
        ref, _ = _oracle(path, clock, lam, None, readout, mode="displacement_uniform_basepoint")
        out, _ = _kernel(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", chunk=8)
        _assert_fwd(out, ref)
        w = torch.tensor(rng.normal(size=ref.shape))
        _, (gp_r, gl_r, _) = _oracle(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", w=w)
        _, (gp_n, gl_n, _) = _kernel(path, clock, lam, None, readout, mode="displacement_uniform_basepoint", w=w, chunk=8)
        _assert_close("path grad", gp_n, gp_r)
        _assert_close("lambda grad", gl_n, gl_r)


def test_config1_full_size():
    """B=4, T=4096, 3 Brownian channels + time, lift 4 -> 16, A = diag(e^u), u~U(-3,1)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import workloads

    case = {k: (_f32(v) if isinstance(v, np.ndarray) else v) for k, v in workloads.config1(seed=0).items()}
    args = (case["path"], case["clock"], case["lam"], case["lift"], "prefix")
    ref, _ = _oracle(*args)
    ref32, _ = _oracle(*args, dtype=torch.float32)
    out, _ = _kernel(*args)
    _assert_fwd(out, ref, ref32, elementwise=False)
    w = torch.tensor(np.random.default_rng(3).normal(size=ref.shape))
    _, g64 = _oracle(*args, w=w)
    _, g32 = _oracle(*args, w=w, dtype=torch.float32)
    _, gk = _kernel(*args, w=w)
    for name, a, b, c in zip(("path", "lambda", "lift"), gk, g64, g32):
        _assert_close(f"{name} grad", a, b, c)


def test_deterministic_mode_is_bit_reproducible():
    """configure(deterministic=True): carries are left folds of the chunk aggregates, so two runs agree bit
    for bit (forward and every gradient); the default decoupled look-back agrees within tolerance."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import configure

    path, clock, lam, lift = _case(4, 300, 16, d_in=4, seed=5)
    w = torch.tensor(np.random.default_rng(9).normal(size=(4, 300, 273)))
    configure(deterministic=True)
    try:
        o1, g1 = _kernel(path, clock, lam, lift, "prefix", w=w, chunk=8)
        o2, g2 = _kernel(path, clock, lam, lift, "prefix", w=w, chunk=8)
    finally:
        configure(deterministic=False)
    assert torch.equal(o1, o2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)
    o3, g3 = _kernel(path, clock, lam, lift, "prefix", w=w, chunk=8)
    _assert_close("forward", o3, o1)
    for a, b in zip(g3, g1):
        _assert_close("grad", a, b)


def test_lookback_timeout_reports_status():
    """Failure detection without a GPU fault: the chunk all others wait for withholds its flag, their
    bounded waits run out, the call returns and the device status reads EWS_ERR_LOOKBACK_TIMEOUT; a
    following normal call on the same context succeeds."""
    _require_gpu()
    import ctypes

    from exponentially_weighted_signature_b200 import _lib, series

    lib = _lib.load()
    B, T, N = 2, 256, 16
    dev = torch.device(DEV)
    path = torch.randn(B, T + 1, N, device=dev)
    x = torch.full((B, N), -1e-3, device=dev)
    q1, q2 = series.diag_tables(x, 4)
    out = torch.empty(B, T, 1 + N + N * N, device=dev)
    a = _lib.DiagArgs()
    a.batch, a.steps, a.d_in, a.dim, a.depth, a.chunk = B, T, N, N, 2, 8
    a.readout, a.flags, a.spin_limit = 0, _lib.EWS_F_UNIFORM | _lib.EWS_F_TEST_WITHHOLD, 2000
    fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.ews_diag_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)) == 0
    ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
    q1, q2 = q1.contiguous(), q2.contiguous()
    a.path, a.tab_x, a.tab_q1, a.tab_q2, a.out = (ctypes.c_void_p(t.data_ptr()) for t in (path, x, q1, q2, out))
    a.fwd_ws, a.fwd_ws_bytes = ctypes.c_void_p(ws.data_ptr()), fb.value
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.ews_diag_fwd(ctypes.byref(a), stream) == 0
    assert _lib.read_device_status(ws.data_ptr(), torch.cuda.current_stream().cuda_stream) == _lib.EWS_ERR_LOOKBACK_TIMEOUT
    a.flags, a.spin_limit = _lib.EWS_F_UNIFORM, 0
    assert lib.ews_diag_fwd(ctypes.byref(a), stream) == 0
    assert _lib.read_device_status(ws.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()


def test_bf16_increments():
    """bf16 increments, fp32 accumulation (config 5's variant): tolerance relerr <= 1e-2 against the f64
    oracle on the unrounded increments, and 1e-5 against the oracle on the bf16-rounded increments."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamDiag

    rng = np.random.default_rng(11)
    B, T, N = 4, 200, 32
    inc = rng.normal(size=(B, T, N)) / np.sqrt(T)
    lam = _f32(np.exp(rng.uniform(-4, 0, N)))
    clock = _f32(np.broadcast_to(np.arange(T + 1) / T, (B, T + 1)).copy())
    inc_bf = torch.tensor(inc, dtype=torch.float32).to(torch.bfloat16)
    layer = EWS(AParamDiag(torch.tensor(lam, dtype=torch.float32)).to(DEV), N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=Q)
    out = layer(inc_bf.to(DEV), torch.tensor(clock, dtype=torch.float32, device=DEV), readout="terminal", increments=True).detach().cpu().double()
    path_exact = np.concatenate([np.zeros((B, 1, N)), np.cumsum(inc, 1)], 1)
    path_round = np.concatenate([np.zeros((B, 1, N)), np.cumsum(inc_bf.double().numpy(), 1)], 1)
    ref_exact, _ = _oracle(path_exact, clock, lam, None, "terminal")
    ref_round, _ = _oracle(path_round, clock, lam, None, "terminal")
    assert relerr(out, ref_exact) < 1e-2
    _assert_fwd(out, ref_round)
