"""Parity of the dense engine (CUDA, fp32) with the float64 CPU oracle, through the C ABI.

Same inputs on both sides (float32-rounded, evaluated by the oracle in float64), same tolerances as
tests/test_gpu_diag.py: global relerr <= 1e-5 against the float64 oracle and <= 4x the reference
algorithm's own float32 error + 1e-5 for outputs and gradients; for paths of at most 256 intervals the
forward also elementwise |out - ref| <= 1e-6 max(1, max|ref|) + 1e-5 |ref|.
"""

import numpy as np
import pytest
import torch

from oracle import ews_oracle as O
from tests.conftest import relerr

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _f32(a):
    return None if a is None else np.asarray(a, dtype=np.float32).astype(np.float64)


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _case(B, T, N, d_in, seed=0, scale=0.1):
    """Config-2 style: Brownian channels (N(0, 1/T) increments), A = 0.5 I - scale G / sqrt(N)."""
    rng = np.random.default_rng(seed)
    inc = rng.normal(size=(B, T, d_in)) / np.sqrt(T)
    path = np.concatenate([np.zeros((B, 1, d_in)), np.cumsum(inc, 1)], 1)
    A = 0.5 * np.eye(N) - scale * rng.normal(size=(N, N)) / np.sqrt(N)
    lift = rng.normal(size=(N, d_in)) / np.sqrt(d_in)
    clock = np.broadcast_to(np.arange(T + 1) / T, (B, T + 1)).copy()
    return _f32(path), _f32(clock), _f32(A), _f32(lift)


def _oracle(path, clock, A, lift, readout, q, w=None, dtype=torch.float64):
    p = torch.tensor(path, dtype=dtype, requires_grad=True)
    Am = torch.tensor(A, dtype=dtype, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=dtype, requires_grad=True)
    y = p if Bm is None else O.lift(p, Bm)
    out = O.ews_layer(y, torch.tensor(clock, dtype=dtype), Am, 2, leaf="series", series_q=q, reweighting_mode="displacement_uniform", readout=readout)
    if w is None:
        return out.detach().double(), None
    (out * w.to(dtype)).sum().backward()
    return out.detach().double(), (p.grad.double(), Am.grad.double(), None if Bm is None else Bm.grad.double())


def _kernel(path, clock, A, lift, readout, q, w=None, chunk=0):
    from exponentially_weighted_signature_b200 import EWS, AParamGeneral

    Ap = AParamGeneral(torch.tensor(A, dtype=torch.float32)).to(DEV)
    layer = EWS(Ap, N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=q, combine="b200", combine_chunk=chunk)
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = None if lift is None else torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
    if w is None:
        return out.detach().cpu().double(), None
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    return out.detach().cpu().double(), (p.grad.cpu().double(), Ap.matrix.grad.cpu().double(), None if Bm is None else Bm.grad.cpu().double())


def _assert_close(name, out, ref, ref32=None):
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


@pytest.mark.parametrize("N", [5, 16, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal", "mean"])
def test_forward_matches_oracle(N, readout):
    _require_gpu()
    path, clock, A, lift = _case(3, 60, N, d_in=7, seed=N)
    ref, _ = _oracle(path, clock, A, lift, readout, 6)
    out, _ = _kernel(path, clock, A, lift, readout, 6, chunk=16)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("chunk", [1, 7, 64, 0])
def test_chunking_and_lookback(chunk):
    _require_gpu()
    path, clock, A, lift = _case(3, 130, 32, d_in=7, seed=3)
    ref, _ = _oracle(path, clock, A, lift, "prefix", 5)
    out, _ = _kernel(path, clock, A, lift, "prefix", 5, chunk=chunk)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("N", [8, 32])
@pytest.mark.parametrize("readout", ["prefix", "terminal"])
def test_gradients_match_oracle(N, readout):
    _require_gpu()
    path, clock, A, lift = _case(2, 70, N, d_in=7, seed=20 + N)
    ref, _ = _oracle(path, clock, A, lift, readout, 6)
    w = torch.tensor(np.random.default_rng(3).normal(size=ref.shape))
    _, (gp_r, ga_r, gb_r) = _oracle(path, clock, A, lift, readout, 6, w=w)
    _, (gp_n, ga_n, gb_n) = _kernel(path, clock, A, lift, readout, 6, w=w, chunk=16)
    for name, a, b in [("path", gp_n, gp_r), ("A", ga_n, ga_r), ("lift", gb_n, gb_r)]:
        _assert_close(f"{name} grad", a, b)


@pytest.mark.parametrize("N,d_in,q,T,chunk", [(32, 7, 6, 75, 7), (5, 3, 2, 33, 5), (16, 11, 8, 40, 8), (8, 4, 0, 30, 6), (12, 8, 1, 37, 9)])
def test_gradients_odd_chunks_and_table_sizes(N, d_in, q, T, chunk):
    """Odd chunk lengths, a padded state (N = 5), large series tables (q = 8, d_in = 11) and the register
    table-gradient kernel's sizes (q + 1 <= 4 with d_in <= 8: 3, 5, 7 and 9 table rows per lane)."""
    _require_gpu()
    path, clock, A, lift = _case(2, T, N, d_in=d_in, seed=40 + N)
    ref, _ = _oracle(path, clock, A, lift, "prefix", q)
    w = torch.tensor(np.random.default_rng(5).normal(size=ref.shape))
    _, (gp_r, ga_r, gb_r) = _oracle(path, clock, A, lift, "prefix", q, w=w)
    _, (gp_n, ga_n, gb_n) = _kernel(path, clock, A, lift, "prefix", q, w=w, chunk=chunk)
    for name, a, b in [("path", gp_n, gp_r), ("A", ga_n, ga_r), ("lift", gb_n, gb_r)]:
        _assert_close(f"{name} grad", a, b)


def test_identity_lift():
    _require_gpu()
    path, clock, A, _ = _case(2, 40, 12, d_in=12, seed=4, scale=0.5)
    ref, _ = _oracle(path, clock, A, None, "prefix", 6)
    out, _ = _kernel(path, clock, A, None, "prefix", 6, chunk=8)
    _assert_fwd(out, ref)


@pytest.mark.parametrize("readout,q", [("prefix", 3), ("prefix", 4), ("terminal", 3)])
def test_config2_full_length(readout, q):
    """BASELINE config 2 at full length (T = 17984, N = 32, d = 7), batch reduced to 2 for the oracle's
    memory; forward and gradients at the bench's series order (q = 3, from the truncation bound) and one
    above it (terminal: the backward re-runs the chunks from the forward's carries instead of reading a
    prefix stream)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import workloads

    case = workloads.config2(B=2)
    path, clock, A, lift = (_f32(case[k]) for k in ("path", "clock", "A", "lift"))
    args = (path, clock, A, lift, readout, q)
    T = path.shape[1] - 1
    shape = (2, T, 1 + 32 + 32 * 32) if readout == "prefix" else (2, 1 + 32 + 32 * 32)
    w = torch.tensor(np.random.default_rng(3).normal(size=shape))
    ref, g64 = _oracle(*args, w=w)
    ref32, g32 = _oracle(*args, w=w, dtype=torch.float32)
    out, gk = _kernel(*args, w=w)
    _assert_fwd(out, ref, ref32, elementwise=False)
    for name, a, b, c in zip(("path", "A", "lift"), gk, g64, g32):
        _assert_close(f"{name} grad", a, b, c)


def _plane_case(B, T, K, d_in, seed=5, hmax=0.4):
    """2x2 planes with general blocks [[a, w], [v, b]] (the plane leaf reads only a and w of each block),
    uniform clock with ||h A_planes|| below the leaf's series range."""
    rng = np.random.default_rng(seed)
    N = 2 * K
    inc = rng.normal(size=(B, T, d_in)) / np.sqrt(T)
    path = np.concatenate([np.zeros((B, 1, d_in)), np.cumsum(inc, 1)], 1)
    A = np.zeros((N, N))
    for j in range(K):
        a, b = rng.uniform(0.05, 1.0, size=2)
        w, v = rng.uniform(-3.0, 3.0, size=2)
        A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = [[a, w], [v, b]]
    lift = rng.normal(size=(N, d_in)) / np.sqrt(d_in)
    planes = np.abs([A[2 * j, 2 * j] for j in range(K)]) + np.abs([A[2 * j, 2 * j + 1] for j in range(K)])
    h = hmax / planes.max()
    clock = np.broadcast_to(np.arange(T + 1) * h, (B, T + 1)).copy()
    return _f32(path), _f32(clock), _f32(A), _f32(lift)


@pytest.mark.parametrize("readout", ["prefix", "terminal"])
def test_plane_closed_leaf_matches_oracle(readout):
    """leaf='plane_closed' (ews/core/kernels/plane_engine.py:134-155, via ews/core/leaf.py:116-136) against the
    oracle's closed form (complex phi and divided differences) in float64: outputs and the gradients of the
    path, the generator and the lift."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamGeneral

    path, clock, A, lift = _plane_case(2, 96, 4, 3)
    rng = np.random.default_rng(9)
    L, N = path.shape[1], A.shape[0]
    D = 1 + N + N * N
    w = torch.tensor(rng.normal(size=(2, L - 1, D) if readout == "prefix" else (2, D)))
    p64 = torch.tensor(path, requires_grad=True)
    A64 = torch.tensor(A, requires_grad=True)
    B64 = torch.tensor(lift, requires_grad=True)
    ref = O.ews_layer(O.lift(p64, B64), torch.tensor(clock), A64, 2, leaf="plane_closed",
                      reweighting_mode="displacement_uniform", readout=readout)
    (ref * w).sum().backward()
    Ap = AParamGeneral(torch.tensor(A, dtype=torch.float32)).to(DEV)
    layer = EWS(Ap, N=2, reweighting_mode="displacement_uniform", leaf="plane_closed", combine="b200")
    assert layer.engine == "dense"
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    _assert_close("forward", out.detach().cpu().double(), ref.detach())
    _assert_close("d path", p.grad.cpu().double(), p64.grad)
    _assert_close("d A", Ap.matrix.grad.cpu().double(), A64.grad)
    _assert_close("d lift", Bm.grad.cpu().double(), B64.grad)


def test_plane_closed_range_guard_raises_on_the_next_call():
    """Outside ||h A|| <= PLANE_X_MAX the series evaluation of the plane leaf is not the closed form: the
    device-side check records it and an engine call raises at the latest on the next call (no host
    synchronisation in the call itself)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamGeneral, engine

    path, clock, A, lift = _plane_case(1, 32, 2, 2, hmax=3.0)
    Ap = AParamGeneral(torch.tensor(A, dtype=torch.float32)).to(DEV)
    layer = EWS(Ap, N=2, reweighting_mode="displacement_uniform", leaf="plane_closed", combine="b200")
    p = torch.tensor(path, dtype=torch.float32, device=DEV)
    c = torch.tensor(clock, dtype=torch.float32, device=DEV)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV)
    try:
        with pytest.raises(NotImplementedError, match="plane_closed"):
            layer(p, c, readout="prefix", lift=Bm)  # may already raise: the flag's copy can land before the call
            torch.cuda.synchronize()
            layer(p, c, readout="prefix", lift=Bm)
    finally:
        for slot in engine._GUARD.values():
            slot[0].zero_()
            slot[1].zero_()


def _jordan_case(B, T, chain, K, d_in, seed=7, hmax=0.4, extra=0.2):
    """K uniform Jordan chains (ews/params.py:412-460) plus `extra`-sized entries inside each chain's block that
    the Jordan leaf does not read (it rebuilds the chains from their first rows) but the flows do; uniform
    clock with ||h J|| (the chain generator) at most hmax."""
    kind, size = chain
    rng = np.random.default_rng(seed)
    N = K * size
    inc = rng.normal(size=(B, T, d_in)) / np.sqrt(T)
    path = np.concatenate([np.zeros((B, 1, d_in)), np.cumsum(inc, 1)], 1)
    A = np.zeros((N, N))
    for f in range(0, N, size):
        if kind == "real":
            blk = rng.uniform(0.1, 2.0) * np.eye(size) + rng.uniform(0.5, 1.5) * np.eye(size, k=1)
            blk += extra * np.tril(rng.normal(size=(size, size)), -1)
        else:
            a, b, e = rng.uniform(0.1, 1.5), rng.uniform(-2.0, 2.0), rng.uniform(0.5, 1.5)
            k = size // 2
            blk = np.kron(np.eye(k), [[a, -b], [b, a]]) + e * np.kron(np.eye(k, k=1), np.eye(2))
            blk += extra * np.tril(rng.normal(size=(size, size)), -2)
        A[f : f + size, f : f + size] = blk
    lift = rng.normal(size=(N, d_in)) / np.sqrt(d_in)
    import torch as _t
    from exponentially_weighted_signature_b200 import series as _s

    J = _s.jordan_generator(_t.tensor(A), kind, size).numpy()
    h = hmax / np.abs(J).sum(-1).max()
    clock = np.broadcast_to(np.arange(T + 1) * h, (B, T + 1)).copy()
    return _f32(path), _f32(clock), _f32(A), _f32(lift)


def _jordan_param(A, chain):
    """An AParamJordanRepeated (the layer reads the chains from the class) that materialises the given matrix."""
    from exponentially_weighted_signature_b200 import AParamJordanRepeated

    class JordanMatrix(AParamJordanRepeated):
        def forward(self):
            return self.matrix

    kind, size = chain
    K = A.shape[0] // size
    ap = JordanMatrix([size] * K, [kind] * K, [torch.zeros(1 if kind == "real" else 2)] * K)
    ap.matrix = torch.nn.Parameter(torch.tensor(A, dtype=torch.float32))
    return ap


@pytest.mark.parametrize("chain,K,readout", [(("real", 4), 8, "prefix"), (("real", 2), 4, "terminal"),
                                             (("complex", 4), 4, "prefix"), (("complex", 8), 2, "terminal"),
                                             (("real", 3), 3, "prefix")])
def test_jordan_closed_leaf_matches_oracle(chain, K, readout):
    """leaf='jordan_closed' (ews/core/kernels/jordan_engine.py:324-353, via ews/core/leaf.py:173-192) against the
    oracle's restatement of the reference's float64 / complex128 table forms: outputs and the gradients of the
    path, the generator (flows from the whole A, the leaf from the chains' first rows) and the lift."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS

    path, clock, A, lift = _jordan_case(2, 80, chain, K, 3)
    rng = np.random.default_rng(11)
    L, N = path.shape[1], A.shape[0]
    D = 1 + N + N * N
    w = torch.tensor(rng.normal(size=(2, L - 1, D) if readout == "prefix" else (2, D)))
    p64 = torch.tensor(path, requires_grad=True)
    A64 = torch.tensor(A, requires_grad=True)
    B64 = torch.tensor(lift, requires_grad=True)
    ref = O.ews_layer(O.lift(p64, B64), torch.tensor(clock), A64, 2, leaf="jordan_closed",
                      reweighting_mode="displacement_uniform", readout=readout, jordan_chain=chain)
    (ref * w).sum().backward()
    Ap = _jordan_param(A, chain).to(DEV)
    layer = EWS(Ap, N=2, reweighting_mode="displacement_uniform", leaf="jordan_closed", combine="b200")
    assert layer.engine == "dense" and layer._jordan_chain == chain
    p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
    out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
    (out * w.to(DEV, torch.float32)).sum().backward()
    torch.cuda.synchronize()
    _assert_close("forward", out.detach().cpu().double(), ref.detach())
    _assert_close("d path", p.grad.cpu().double(), p64.grad)
    _assert_close("d A", Ap.matrix.grad.cpu().double(), A64.grad)
    _assert_close("d lift", Bm.grad.cpu().double(), B64.grad)


def test_jordan_closed_range_guard_raises_on_the_next_call():
    """The Jordan leaf outside ||h J|| <= CLOSED_X_MAX: recorded on the device, raised on the next call."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, engine

    chain = ("complex", 4)
    path, clock, A, lift = _jordan_case(1, 32, chain, 2, 2, hmax=3.0)
    layer = EWS(_jordan_param(A, chain).to(DEV), N=2, reweighting_mode="displacement_uniform", leaf="jordan_closed",
                combine="b200")
    p = torch.tensor(path, dtype=torch.float32, device=DEV)
    c = torch.tensor(clock, dtype=torch.float32, device=DEV)
    Bm = torch.tensor(lift, dtype=torch.float32, device=DEV)
    try:
        with pytest.raises(NotImplementedError, match="jordan_closed"):
            layer(p, c, readout="prefix", lift=Bm)  # may already raise: the flag's copy can land before the call
            torch.cuda.synchronize()
            layer(p, c, readout="prefix", lift=Bm)
    finally:
        for slot in engine._GUARD.values():
            slot[0].zero_()
            slot[1].zero_()


@pytest.mark.parametrize("B,T,N,chunk", [(2, 2000, 8, 1), (3, 75, 32, 7), (2, 130, 5, 0)])
def test_terminal_gradients_in_windows(B, T, N, chunk):
    """Terminal readout with gradients: the backward re-runs windows of chunk groups from the forward's carries
    (the output pass into scratch rows, then the exact pass on them), as the reference's block_terminal_vjp
    (pallas_combine.py:1911-2027) recomputes each chunk from its saved start. 2000 one-interval chunks make
    several windows (the window holds one output-pass grid of tiles); a ragged last chunk; a padded state."""
    _require_gpu()
    path, clock, A, lift = _case(B, T, N, d_in=4, seed=60 + N)
    w = torch.tensor(np.random.default_rng(8).normal(size=(B, 1 + N + N * N)))
    ref, (gp_r, ga_r, gb_r) = _oracle(path, clock, A, lift, "terminal", 4, w=w)
    out, (gp_n, ga_n, gb_n) = _kernel(path, clock, A, lift, "terminal", 4, w=w, chunk=chunk)
    _assert_close("forward", out, ref)
    for name, a, b in [("path", gp_n, gp_r), ("A", ga_n, ga_r), ("lift", gb_n, gb_r)]:
        _assert_close(f"{name} grad", a, b)


def test_terminal_training_step_keeps_no_prefix_stream():
    """What autograd keeps for a terminal fwd+bwd is the (B, 1 + D) terminal row, not a (B, T, 1 + D) prefix
    stream, and the gradients equal the prefix path's with the cotangent on its last row."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import EWS, AParamGeneral

    B, T, N, d_in = 2, 300, 32, 7
    W = 1 + N + N * N
    path, clock, A, lift = _case(B, T, N, d_in=d_in, seed=9)
    w = torch.tensor(np.random.default_rng(9).normal(size=(B, W)), dtype=torch.float32, device=DEV)
    grads = {}
    for readout in ("terminal", "prefix"):
        Ap = AParamGeneral(torch.tensor(A, dtype=torch.float32)).to(DEV)
        layer = EWS(Ap, N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=4)
        p = torch.tensor(path, dtype=torch.float32, device=DEV, requires_grad=True)
        Bm = torch.tensor(lift, dtype=torch.float32, device=DEV, requires_grad=True)
        shapes = []

        def pack(t):
            shapes.append(tuple(t.shape))
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            out = layer(p, torch.tensor(clock, dtype=torch.float32, device=DEV), readout=readout, lift=Bm)
        last = out if readout == "terminal" else out[:, -1]
        (last * w).sum().backward()
        torch.cuda.synchronize()
        if readout == "terminal":
            assert (B, T, W) not in shapes, shapes
        grads[readout] = (p.grad, Ap.matrix.grad, Bm.grad)
    for name, a, b in zip(("path", "A", "lift"), grads["terminal"], grads["prefix"]):
        e = relerr(a.double().cpu(), b.double().cpu())
        assert e <= 1e-5, f"d/d{name}: terminal vs prefix relerr {e:.2e}"
