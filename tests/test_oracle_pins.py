"""Pins for the CPU oracle (oracle/ews_oracle.py) against the reference's own known answers.

Each test names the reference test it restates. They run in float64 on the CPU and need no GPU.
"""

import math

import numpy as np
import pytest
import torch
from scipy.linalg import expm as scipy_expm

from oracle import ews_oracle as O
from tests.conftest import relerr

DT = torch.float64


def _general_A(m, seed=0):
    """tests/test_engines.py:36-40 (reference): skew part + positive diagonal."""
    rng = np.random.default_rng(seed)
    A0 = rng.normal(size=(m, m)) * 0.2
    A0 = (A0 - A0.T) / 2 + np.diag(rng.uniform(0.05, 0.3, m))
    return torch.tensor(A0, dtype=DT)


def _blockdiag_A(sizes, seed=0):
    """tests/test_engines.py:43-46 (reference)."""
    rng = np.random.default_rng(seed)
    m = sum(sizes)
    A = np.zeros((m, m))
    o = 0
    for s in sizes:
        A[o : o + s, o : o + s] = rng.normal(size=(s, s)) * 0.3
        o += s
    return torch.tensor(A, dtype=DT)


def _planes_A(K, seed=0):
    """Canonical planes [[d, w], [-w, d]] (tests/test_engines.py:49-56 of the reference)."""
    rng = np.random.default_rng(seed)
    A = np.zeros((2 * K, 2 * K))
    for j in range(K):
        d, w = rng.uniform(0.05, 0.4), rng.uniform(-1.0, 1.0)
        A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = [[d, w], [-w, d]]
    return torch.tensor(A, dtype=DT)


def _data(L, m, seed=1, uniform=False):
    """tests/test_engines.py:66-77 (reference): cumulative N(0, 0.09) path, log-normal clock steps."""
    rng = np.random.default_rng(seed)
    path = torch.tensor(np.cumsum(rng.normal(size=(L + 1, m)) * 0.3, 0), dtype=DT)
    if uniform:
        clock = torch.tensor(np.arange(L + 1) * 0.7, dtype=DT)
    else:
        clock = torch.tensor(np.cumsum(rng.lognormal(0, 0.3, L + 1)), dtype=DT)
    return path, clock


def _planes_param(A):
    """(K, 2) [d, w] parameters of canonical planes and the builder back to A (the rotation parametrisations
    of the reference differentiate w.r.t. these, not w.r.t. the full matrix)."""
    K = A.shape[0] // 2
    dw = torch.stack([A[0::2, 0::2].diagonal(), A[0::2, 1::2].diagonal()], -1)

    def build(p):
        out = torch.zeros((2 * K, 2 * K), dtype=p.dtype)
        idx = torch.arange(K) * 2
        out = out.index_put((idx, idx), p[:, 0]).index_put((idx + 1, idx + 1), p[:, 0])
        out = out.index_put((idx, idx + 1), p[:, 1]).index_put((idx + 1, idx), -p[:, 1])
        return out

    return dw, build


def _value_and_grads(path, clock, A, N, readout, w, A_param=None, **kw):
    path = path.clone().requires_grad_(True)
    if A_param is None:
        P = A.clone().requires_grad_(True)
        build = lambda p: p
    else:
        P, build = A_param
        P = P.clone().requires_grad_(True)
    out = O.ews_layer(path, clock, build(P), N, readout=readout, **kw)
    v = (out * w).sum()
    gp, ga = torch.autograd.grad(v, (path, P))
    return out.detach(), v.detach(), gp, ga


def _compare(path, clock, A, N, readouts, tol, ref_kw, new_kw, grads=True, A_param=None):
    """The reference's _compare (tests/test_engines.py:107-122): forward and path/A gradients of sum(w out)."""
    for readout in readouts:
        out_r = O.ews_layer(path, clock, A, N, readout=readout, **ref_kw)
        out_n = O.ews_layer(path, clock, A, N, readout=readout, **new_kw)
        assert out_r.shape == out_n.shape
        assert relerr(out_n, out_r) < tol, readout
        if grads:
            w = torch.tensor(np.random.default_rng(3).normal(size=out_r.shape), dtype=DT)
            _, v_r, gp_r, ga_r = _value_and_grads(path, clock, A, N, readout, w, A_param, **ref_kw)
            _, v_n, gp_n, ga_n = _value_and_grads(path, clock, A, N, readout, w, A_param, **new_kw)
            assert relerr(v_n, v_r) < tol
            assert relerr(gp_n, gp_r) < tol, f"{readout}: path grad"
            assert relerr(ga_n, ga_r) < tol, f"{readout}: A grad"


# ------------------------------------------------------------------------- series coefficients


def test_series_coefficients_closed_form():
    """c_m from the simplex integrals of monomials (ews/core/series_leaf.py:8-20 of the reference)."""
    C1, C2, C3 = O.series_coeffs(3, 4)
    for p in range(5):
        assert C1[p] == pytest.approx(1.0 / (p + 1))
    for a in range(5):
        for b in range(5 - a):
            assert C2[a, b] == pytest.approx(1.0 / ((a + b + 2) * (b + 1)))
    assert C3[1, 1, 1] == pytest.approx(1.0 / (6 * 4 * 2))
    assert C2[3, 2] == 0.0  # |m| > q


def test_series_error_bound_and_suggest_q():
    """suggest_series_q returns the smallest q under the bound (ews/core/leaf.py:201-215 of the reference)."""
    for x, k, tol in [(1e-3, 2, 1e-14), (0.05, 3, 1e-10), (0.5, 2, 1e-6)]:
        q = O.suggest_series_q(x, k, tol)
        assert O.series_error_bound(x, k, q) < tol
        assert q == 1 or O.series_error_bound(x, k, q - 1) >= tol * 0.999
    assert O.suggest_series_q(0.0, 2) == 1


def test_series_truncation_error_within_bound():
    """The series at q against q=30 stays inside series_error_bound (ews/core/series_leaf.py:139-143)."""
    rng = np.random.default_rng(5)
    d, L = 3, 6
    A = torch.tensor(rng.normal(size=(d, d)) * 0.5, dtype=DT)
    path, clock = _data(L, d, seed=4)
    x = float(torch.linalg.matrix_norm(A, 2)) * float((clock[1:] - clock[:-1]).max())
    exact = O.series_local_signatures(path, clock, A, 3, 30)
    for q in (3, 5, 8):
        approx = O.series_local_signatures(path, clock, A, 3, q)
        for k in range(1, 4):
            err = float((approx[k - 1] - exact[k - 1]).abs().max())
            dxn = float((path[1:] - path[:-1]).norm(dim=-1).max())
            assert err <= O.series_error_bound(x, k, q) * dxn**k * 1.01 + 1e-13


# ------------------------------------------------------------------------------- known answers


@pytest.mark.parametrize("L", [6, 9])
def test_depth_one_is_the_augmented_exponential_recursion(L):
    """tests/test_block.py:565-596 (reference): at depth 1 the layer is S <- E S + G dx with
    exp([[-dtheta A, dx], [0, 0]]) = [[E, G dx], [0, 1]]."""
    H = 4
    rng = np.random.default_rng(36)
    x = rng.standard_normal((L, H))
    S0 = rng.normal(size=(H, H)) * 0.1
    A = torch.tensor(S0 - S0.T, dtype=DT)
    theta = np.arange(L) / (L - 1)
    out = O.ews_layer(torch.tensor(x), torch.tensor(theta), A, 1, leaf="series", series_q=30, readout="prefix")
    S = np.zeros(H)
    expected = []
    for j in range(1, L):
        aug = np.zeros((H + 1, H + 1))
        aug[:H, :H] = -(theta[j] - theta[j - 1]) * A.numpy()
        aug[:H, H] = x[j] - x[j - 1]
        Mv = scipy_expm(aug)
        S = Mv[:H, :H] @ S + Mv[:H, H]
        expected.append(S)
    np.testing.assert_allclose(out[:, 1:].numpy(), np.stack(expected), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(out[:, 0].numpy(), 1.0)


def _classical_signature(path, n):
    """Chen product of straight-segment signatures exp(dx) (A = 0), independent of the EWS code."""
    d = path.shape[-1]
    S = [torch.zeros((d**k,), dtype=DT) for k in range(1, n + 1)]
    for t in range(1, path.shape[0]):
        seg = O.tensor_exp([path[t] - path[t - 1]] + [torch.zeros((d**k,), dtype=DT) for k in range(2, n + 1)])
        S = O.tensor_mult(S, seg)
    return torch.cat(S)


@pytest.mark.parametrize("n", [1, 2, 3])
def test_zero_generator_gives_the_signature(n):
    """tests/test_log_ews.py:82-96 (reference): A = 0 makes the EWS the signature."""
    d, L = 3, 8
    path, _ = _data(L - 1, d, seed=2)
    clock = torch.linspace(0.0, 1.0, L, dtype=DT)
    got = O.ews_layer(path, clock, torch.zeros((d, d), dtype=DT), n, series_q=4, readout="terminal")
    ref = _classical_signature(path, n)
    assert float((got[1:] - ref).abs().max()) < 1e-12
    assert got[0] == 1.0


def test_zero_generator_log_is_the_log_signature():
    """tests/test_log_ews.py:82-96: with A = 0, log(EWS) equals log of the classical signature."""
    d, L, n = 3, 8, 3
    path, _ = _data(L - 1, d, seed=1)
    clock = torch.linspace(0.0, 1.0, L, dtype=DT)
    got = O.log_ews_layer(path, clock, torch.zeros((d, d), dtype=DT), n, series_q=4, readout="terminal")
    sig = O.unpack(_classical_signature(path, n), d, n)
    ref = O.compress_log(O.tensor_log(sig), d)
    assert got.shape == (14,)
    assert float((got - ref).abs().max()) < 1e-12
    # level 1 of the log is the increment; level 2 on Lyndon words (i<j) is the Levy area
    assert float((got[:3] - (path[-1] - path[0])).abs().max()) < 1e-12


def test_exp_of_log_recovers_the_ews():
    """tests/test_log_ews.py:99-109 (reference): exp(log(EWS)) = EWS for a general A."""
    d, n, L = 3, 3, 8
    path, _ = _data(L - 1, d, seed=2)
    clock = torch.linspace(0.0, 1.0, L, dtype=DT)
    A = torch.tensor(np.random.default_rng(3).normal(size=(d, d)) * 0.5, dtype=DT)
    flat = O.ews_layer(path, clock, A, n, series_q=20, readout="terminal")
    levels = O.unpack(flat[1:], d, n)
    rt = O.tensor_exp(O.tensor_log(levels))
    assert max(float((a - b).abs().max()) for a, b in zip(levels, rt)) < 1e-12


def test_witt_dimensions():
    """tests/test_log_ews.py:112-122 (reference): flat log length is the Witt dimension."""
    for d, n, expect in [(3, 3, 14), (4, 2, 4 + 6), (2, 4, 2 + 1 + 2 + 3), (32, 2, 32 + 496)]:
        assert sum(O.witt_dims(d, n)) == expect
    w2 = O.lyndon_words(2, 3)[1]
    assert [tuple(r) for r in w2] == [(0, 1), (0, 2), (1, 2)]


# ------------------------------------------------------------------------- engine agreement


@pytest.mark.parametrize("N", [1, 2, 3])
@pytest.mark.parametrize("mode", list(O.MODES))
def test_sequential_matches_assoc(N, mode):
    """tests/test_engines.py:198-214 (reference: lean = assoc at 1e-10): the sequential recursion equals the
    associative scan for every readout and reweighting mode."""
    m, L = 4, 13
    A = _general_A(m)
    uniform = mode != "displacement"
    path, clock = _data(L, m, uniform=uniform)
    if mode == "displacement_uniform_basepoint":
        clock = torch.tensor(np.concatenate([[0.0], np.arange(L) * 0.7]), dtype=DT)
        path = path.clone()
        path[0] = path[1]
    kw = dict(series_q=12, reweighting_mode=mode)
    _compare(path, clock, A, N, ["prefix", "terminal", "mean", "max"], 1e-10, dict(kw, combine="assoc", terminal_reduce="assoc"), dict(kw, combine="seq"), grads=N < 3)


def test_terminal_tree_matches_assoc():
    """tests/test_engines.py:217-224 (reference)."""
    m, L = 3, 10
    A = _general_A(m)
    path, clock = _data(L, m)
    _compare(path, clock, A, 2, ["terminal"], 1e-10, dict(series_q=12, terminal_reduce="tree"), dict(series_q=12, combine="seq"))


@pytest.mark.parametrize("N", [1, 2])
def test_plane_closed_leaf_matches_series(N):
    """tests/test_engines.py:227-237 (reference, tol 1e-7 against series q=24)."""
    K, L = 3, 17
    A = _planes_A(K)
    path, clock = _data(L, 2 * K)
    _compare(
        path, clock, A, N, ["prefix", "terminal", "mean"], 1e-7, dict(leaf="series", series_q=24), dict(leaf="plane_closed"),
        A_param=_planes_param(A),
    )


@pytest.mark.parametrize("N", [1, 2])
@pytest.mark.parametrize("sizes", [(2, 2, 2), (2, 3, 1), (4, 4), (3, 4), (1,) * 6])
def test_block_series_leaf_matches_series(N, sizes):
    """tests/test_engines.py:240-248 (reference, tol 1e-7); sizes (1,)*m is the free diagonal."""
    L = 11
    A = _blockdiag_A(sizes)
    path, clock = _data(L, sum(sizes))
    _compare(path, clock, A, N, ["prefix", "terminal"], 1e-7, dict(leaf="series", series_q=24), dict(leaf="block_series", series_q=24))


def test_depth3_closed_leaves_fail_fast():
    """tests/test_engines.py:266-272 (reference)."""
    A = _planes_A(2)
    path, clock = _data(6, 4)
    with pytest.raises(NotImplementedError):
        O.ews_layer(path, clock, A, 3, leaf="plane_closed")
    with pytest.raises(NotImplementedError):
        O.ews_layer(path, clock, A, 3, leaf="block_series", series_q=4)


def test_gradients_match_finite_differences():
    """tests/test_log_ews.py:149 (reference): autograd gradients of the oracle match central differences."""
    d, N, L = 3, 3, 6
    path, clock = _data(L, d, seed=7)
    A0 = torch.tensor(np.random.default_rng(8).normal(size=(d, d)) * 0.2, dtype=DT)

    def loss(A):
        return (O.log_ews_layer(path, clock, A, N, series_q=16, readout="terminal") ** 2).sum()

    A = A0.clone().requires_grad_(True)
    (g,) = torch.autograd.grad(loss(A), A)
    eps = 1e-6
    fd = torch.zeros_like(A0)
    for i in range(d):
        for j in range(d):
            E = torch.zeros_like(A0)
            E[i, j] = eps
            fd[i, j] = (loss(A0 + E) - loss(A0 - E)) / (2 * eps)
    assert relerr(g, fd) < 1e-7
    assert float(g.abs().max()) > 0


def test_flow_semantics_diagonal_closed_form():
    """For diagonal A the level-2 local term is dx_i dx_j D(-h l_i, -h l_j) with D the divided difference of
    phi (ews/core/kernels/plane_engine.py:1-11, 65-78): the series at high order reproduces it."""
    lam = torch.tensor([0.3, 1.2, 2.5], dtype=DT)
    A = torch.diag(lam)
    path, clock = _data(5, 3, seed=9)
    lv = O.series_local_signatures(path, clock, A, 2, 40)
    dx = path[1:] - path[:-1]
    h = clock[1:] - clock[:-1]
    x = -h[:, None] * lam[None, :]
    s1 = O.phi(x) * dx
    D = O.divdiff_phi(x[:, :, None], x[:, None, :])
    s2 = (dx[:, :, None] * dx[:, None, :] * D).reshape(5, 9)
    assert float((lv[0] - s1).abs().max()) < 1e-12
    assert float((lv[1] - s2).abs().max()) < 1e-10
    assert math.isclose(float(O.phi(torch.tensor(0.0, dtype=DT))), 1.0)
