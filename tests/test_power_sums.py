"""The identity behind the dense engine's zero-carry adjoints (bagg_kernel in csrc/ews_dense.cu), on the CPU.

The reverse recursion of one chunk run from a zero cotangent (the adjoint of the modified-Chen step
S2' = M S2 M^T + u s1^T + ..., S1' = M S1 + s1 of ews/core/chen_scan.py:124-152 with a uniform flow M),
    l2 <- M^T l2 M + G_j,   l1 <- M^T (l1 + l2 s1_j) + g1_j     (j from the chunk's end to its start),
equals the power sums
    mu2 = sum_j P_j^T G_j P_j,   mu1 = sum_j P_j^T (g1_j + G_j s^_j),   P_j = M^(j+1),
with s^_j = M s^_(j-1) + s1_j the chunk's level 1 from a zero start. The kernel evaluates the right-hand
sides with P_j = I - E_(j+1) from the forward's power complements; this test checks the algebra in float64.
"""

import numpy as np
import pytest


def _chain(M, G, g1, s1):
    L, N = g1.shape
    l2 = np.zeros((N, N))
    l1 = np.zeros(N)
    for j in range(L - 1, -1, -1):
        l2 = l2 + G[j]
        l1 = l1 + g1[j]
        v = l1 + l2 @ s1[j]
        l2 = M.T @ l2 @ M
        l1 = M.T @ v
    return l1, l2


def _power_sums(M, G, g1, s1):
    L, N = g1.shape
    E = [np.eye(N) - np.linalg.matrix_power(M, j) for j in range(L + 1)]  # the power complements
    mu2 = np.zeros((N, N))
    mu1 = np.zeros(N)
    shat = np.zeros(N)
    for j in range(L):
        shat = M @ shat + s1[j]
        P = np.eye(N) - E[j + 1]
        H = G[j] - G[j] @ E[j + 1]          # G P
        mu2 += H - E[j + 1].T @ H           # P^T G P
        w = g1[j] + G[j] @ shat
        mu1 += w - E[j + 1].T @ w           # P^T w
        assert np.allclose(P, np.linalg.matrix_power(M, j + 1))
    return mu1, mu2


@pytest.mark.parametrize("N,L,scale", [(5, 1, 0.3), (8, 17, 0.2), (32, 40, 0.05)])
def test_zero_carry_adjoint_is_the_power_sums(N, L, scale):
    rng = np.random.default_rng(N + L)
    M = np.eye(N) - scale * rng.normal(size=(N, N)) / np.sqrt(N)
    G = rng.normal(size=(L, N, N))
    g1 = rng.normal(size=(L, N))
    s1 = rng.normal(size=(L, N))
    c1, c2 = _chain(M, G, g1, s1)
    p1, p2 = _power_sums(M, G, g1, s1)
    np.testing.assert_allclose(p2, c2, rtol=1e-11, atol=1e-11 * np.abs(c2).max())
    np.testing.assert_allclose(p1, c1, rtol=1e-11, atol=1e-11 * np.abs(c1).max())
