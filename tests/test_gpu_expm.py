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
