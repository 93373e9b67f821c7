"""The dense engine's flow exponential (ews_expm_batched) and its VJP (ews_expm_adjoint_batched) against
torch.linalg.matrix_exp and scipy.linalg.expm_frechet in float64.

The reference builds the dense flow with expm_matrix(-h A, "exact") = jax.scipy.linalg.expm
(ews/core/chen_scan.py:155-168, ews/core/expm_approx.py:34-41). Tolerance (written here): relative
error max|a-b| / max|b| <= 1e-12 for the exponential and for the adjoint against scipy's Frechet
derivative L(X^T, G), over matrices of 1-norm from 1e-6 to 40 (no scaling up to several squarings) and
sizes 1..64 (adjoint 1..32); torch's own autograd of matrix_exp, which exponentiates the unscaled block
matrix, agrees to 1e-10.
"""

import numpy as np
import pytest
import scipy.linalg
import torch

from tests.conftest import relerr

pytestmark = pytest.mark.gpu


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _mats(B, n, scale, seed):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(B, n, n, generator=g, dtype=torch.float64)
    X = X / X.abs().sum(-2).amax(-1)[:, None, None]  # unit 1-norm
    return X * torch.logspace(-6, 0, B, dtype=torch.float64)[:, None, None] * scale


@pytest.mark.parametrize("n", [1, 2, 5, 16, 31, 32, 33, 48, 64])
@pytest.mark.parametrize("scale", [1.0, 40.0])
def test_expm_matches_torch(n, scale):
    _require_gpu()
    from exponentially_weighted_signature_b200.engine import Expm

    X = _mats(7, n, scale, seed=n).cuda()
    got = Expm.apply(X)
    ref = torch.linalg.matrix_exp(X)
    for b in range(X.shape[0]):
        assert relerr(got[b].cpu(), ref[b].cpu()) <= 1e-12, (b, relerr(got[b].cpu(), ref[b].cpu()))


@pytest.mark.parametrize("n", [1, 3, 8, 32])
@pytest.mark.parametrize("scale", [1.0, 40.0])
def test_expm_adjoint_matches_autograd(n, scale):
    _require_gpu()
    from exponentially_weighted_signature_b200.engine import Expm

    X = _mats(5, n, scale, seed=100 + n).cuda()
    G = torch.randn(X.shape, generator=torch.Generator().manual_seed(n), dtype=torch.float64).cuda() * 1e3
    Xa = X.clone().requires_grad_(True)
    (Expm.apply(Xa) * G).sum().backward()
    Xr = X.clone().requires_grad_(True)
    (torch.linalg.matrix_exp(Xr) * G).sum().backward()
    for b in range(X.shape[0]):
        ref = scipy.linalg.expm_frechet(X[b].cpu().numpy().T, G[b].cpu().numpy(), compute_expm=False)
        assert relerr(Xa.grad[b].cpu(), torch.from_numpy(np.ascontiguousarray(ref))) <= 1e-12
        assert relerr(Xa.grad[b].cpu(), Xr.grad[b].cpu()) <= 1e-10


def test_expm_zero_and_identity_cases():
    _require_gpu()
    from exponentially_weighted_signature_b200.engine import Expm

    Z = torch.zeros(3, 32, 32, dtype=torch.float64, device="cuda")
    assert torch.equal(Expm.apply(Z), torch.eye(32, dtype=torch.float64, device="cuda").expand(3, 32, 32))
    Xa = Z.clone().requires_grad_(True)
    Expm.apply(Xa).sum().backward()
    assert torch.allclose(Xa.grad, torch.ones_like(Z))  # L(0, G) = G
    Xz = torch.randn(2, 8, 8, dtype=torch.float64, device="cuda").requires_grad_(True)
    (Expm.apply(Xz) * 0.0).sum().backward()
    assert torch.equal(Xz.grad, torch.zeros_like(Xz))


@pytest.mark.parametrize("n,d,q,lifted", [(32, 7, 3, True), (5, 3, 0, True), (16, 16, 11, False), (32, 32, 8, True), (9, 4, 6, False)])
def test_series_tables_match_torch(n, d, q, lifted):
    """ews_series_tables / _adjoint (the dense engine's series-leaf tables in one kernel each way) against
    series.dense_leaf_tables in float64 torch, forward and VJP: relative error <= 1e-6 (float32 outputs;
    the VJP's cotangents are float32 too)."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import series
    from exponentially_weighted_signature_b200.engine import SeriesTables

    if not lifted:
        d = n
    g = torch.Generator().manual_seed(n * 100 + q)
    X = (0.3 * torch.randn(3, n, n, generator=g, dtype=torch.float64)).cuda().requires_grad_(True)
    W = (torch.randn(n, d, generator=g, dtype=torch.float64) / np.sqrt(d)).cuda().requires_grad_(True) if lifted else None
    c1, c2 = series._leaf_coeffs(q, "cuda")
    F, G, H = SeriesTables.apply(X, W, c1, c2)
    Fr, Gr, Hr = series.dense_leaf_tables(X, q, W, (c1, c2))
    for a, b2 in ((F, Fr), (G, Gr), (H, Hr)):
        assert relerr(a.double().detach().cpu(), b2.detach().cpu()) <= 1e-6
    wF = torch.randn(F.shape, generator=g, dtype=torch.float64).cuda()
    wG = torch.randn(G.shape, generator=g, dtype=torch.float64).cuda()
    wH = torch.randn(H.shape, generator=g, dtype=torch.float64).cuda()
    ins = [X] + ([W] if lifted else [])
    got = torch.autograd.grad((F * wF.float()).sum() + (G * wG.float()).sum() + (H * wH.float()).sum(), ins)
    # q = 0: the tables do not depend on X (P_0 = I), so the reference graph does not reach it
    ref = torch.autograd.grad((Fr * wF.float().double()).sum() + (Gr * wG.float().double()).sum()
                              + (Hr * wH.float().double()).sum(), ins, allow_unused=True)
    for a, b2, t in zip(got, ref, ins):
        b2 = torch.zeros_like(t) if b2 is None else b2
        if float(b2.abs().max()) == 0.0:
            assert float(a.abs().max()) == 0.0
        else:
            assert relerr(a.detach().cpu(), b2.detach().cpu()) <= 1e-6


@pytest.mark.parametrize(
    "B,n,d,q,lifted,own_leaf",
    [(4, 32, 7, 3, True, False), (1, 5, 3, 0, True, True), (33, 16, 16, 11, False, False), (6, 32, 32, 8, True, True),
     (3, 9, 4, 6, False, True)],
)
def test_dense_leaf_matches_the_torch_composition(B, n, d, q, lifted, own_leaf):
    """ews_dense_leaf / _adjoint (the flow complement D = I - expm(-h_b A) and the series tables of
    -h_b A_l in one launch each way, with dA, dh, dA_l and dW summed over samples on the device) against
    the same composition in float64 torch (matrix_exp, series.dense_leaf_tables): relative error <= 1e-6
    for every output and gradient (float32 outputs and cotangents). The clock steps span 1e-5 .. 3, so
    the flows run from no squaring to several."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import series
    from exponentially_weighted_signature_b200.engine import DenseLeaf

    if not lifted:
        d = n
    g = torch.Generator().manual_seed(B * 1000 + n * 10 + q)
    A = (0.5 * torch.eye(n, dtype=torch.float64) - torch.randn(n, n, generator=g, dtype=torch.float64) / np.sqrt(n))
    A = A.float().cuda().requires_grad_(True)
    h = torch.logspace(-5, 0.5, B, dtype=torch.float64).float().cuda().requires_grad_(True)
    Al = (torch.randn(n, n, generator=g, dtype=torch.float64) / np.sqrt(n)).float().cuda().requires_grad_(True) if own_leaf else None
    W = (torch.randn(n, d, generator=g, dtype=torch.float64) / np.sqrt(d)).float().cuda().requires_grad_(True) if lifted else None
    c1, c2 = series._leaf_coeffs(q, "cuda")
    Dc, F, G, H = DenseLeaf.apply(A, h, Al, W, c1, c2)

    A64 = A.detach().double().requires_grad_(True)
    h64 = h.detach().double().requires_grad_(True)
    Al64 = None if Al is None else Al.detach().double().requires_grad_(True)
    W64 = None if W is None else W.detach().double().requires_grad_(True)
    X = -h64[:, None, None] * A64
    Dr = torch.eye(n, dtype=torch.float64, device="cuda") - torch.linalg.matrix_exp(X)
    Xl = X if Al64 is None else -h64[:, None, None] * Al64
    Fr, Gr, Hr = series.dense_leaf_tables(Xl, q, W64, (c1, c2))
    for a, b2 in ((Dc, Dr), (F, Fr), (G, Gr), (H, Hr)):
        assert a.dtype == torch.float32
        assert relerr(a.double().detach().cpu(), b2.detach().cpu()) <= 1e-6

    ws = [torch.randn(t.shape, generator=g, dtype=torch.float32).cuda() for t in (Dc, F, G, H)]
    ins = [A, h] + ([Al] if Al is not None else []) + ([W] if W is not None else [])
    ins64 = [A64, h64] + ([Al64] if Al64 is not None else []) + ([W64] if W64 is not None else [])
    got = torch.autograd.grad(sum((t * w).sum() for t, w in zip((Dc, F, G, H), ws)), ins)
    ref = torch.autograd.grad(sum((t * w.double()).sum() for t, w in zip((Dr, Fr, Gr, Hr), ws)), ins64, allow_unused=True)
    for a, b2, t in zip(got, ref, ins):
        assert a.dtype == torch.float32 and a.shape == t.shape
        b2 = torch.zeros_like(t, dtype=torch.float64) if b2 is None else b2
        if float(b2.abs().max()) == 0.0:
            assert float(a.abs().max()) == 0.0
        else:
            assert relerr(a.double().detach().cpu(), b2.detach().cpu()) <= 1e-6


def test_dense_leaf_partial_cotangents():
    """Only some of the tables reach the loss: the missing cotangents count as zeros (flows only, series
    tables only), and the gradients match the float64 composition as above."""
    _require_gpu()
    from exponentially_weighted_signature_b200 import series
    from exponentially_weighted_signature_b200.engine import DenseLeaf

    g = torch.Generator().manual_seed(7)
    n, d, q, B = 12, 5, 4, 3
    A = (torch.randn(n, n, generator=g) / np.sqrt(n)).cuda().requires_grad_(True)
    h = torch.tensor([0.01, 0.3, 2.0]).cuda()
    W = (torch.randn(n, d, generator=g) / np.sqrt(d)).cuda().requires_grad_(True)
    c1, c2 = series._leaf_coeffs(q, "cuda")
    for use in ("flow", "tables"):
        Dc, F, G, H = DenseLeaf.apply(A, h, None, W, c1, c2)
        A64 = A.detach().double().requires_grad_(True)
        W64 = W.detach().double().requires_grad_(True)
        X = -h.double()[:, None, None] * A64
        if use == "flow":
            loss = (Dc * Dc.detach()).sum()
            loss64 = ((torch.eye(n, dtype=torch.float64, device="cuda") - torch.linalg.matrix_exp(X)) * Dc.detach().double()).sum()
        else:
            Fr, Gr, Hr = series.dense_leaf_tables(X, q, W64, (c1, c2))
            loss = F.sum() + (H * 0.5).sum()
            loss64 = Fr.sum() + (Hr * 0.5).sum()
        got = torch.autograd.grad(loss, [A, W], allow_unused=True)
        ref = torch.autograd.grad(loss64, [A64, W64], allow_unused=True)
        for a, b2, t in zip(got, ref, (A, W)):
            a = torch.zeros_like(t) if a is None else a
            b2 = torch.zeros_like(t, dtype=torch.float64) if b2 is None else b2
            if float(b2.abs().max()) == 0.0:
                assert float(a.abs().max()) == 0.0
            else:
                assert relerr(a.double().detach().cpu(), b2.detach().cpu()) <= 1e-6
