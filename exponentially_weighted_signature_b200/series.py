"""Series-leaf coefficients and the per-sample local tables of the engines.

The series leaf (ews/core/series_leaf.py:1-25 of the reference) writes the depth-k local term of one
linear interval (increment dy, clock step h) as

    s_k = sum_{|m| <= q} c_m  b_{m1} (x) ... (x) b_{mk},    b_p = ((-h A)^p / p!) dy,
    c_m = prod_j 1 / (M_j + k - j + 1),   M_j = m_j + ... + m_k.

For a diagonal A = diag(lambda) every letter is a scaled copy of dy, so the local terms collapse to
tables in x = -h lambda:  s1_i = Q1_i dy_i,  s2_ij = Q2_ij dy_i dy_j  with
Q1_i = sum_p c_p x_i^p / p!  and  Q2_ij = sum_{a+b<=q} c_ab x_i^a x_j^b / (a! b!).
"""

from __future__ import annotations

import math
from fractions import Fraction
from functools import lru_cache
from itertools import product as _iproduct

import numpy as np
import torch


def coeff_exact(m) -> Fraction:
    """c_m as an exact rational (ews/core/series_leaf.py:45-52)."""
    k = len(m)
    out = Fraction(1)
    for j in range(1, k + 1):
        out /= sum(m[j - 1 :]) + k - j + 1
    return out


@lru_cache(maxsize=None)
def series_coeffs(depth: int, q: int):
    """Level-k coefficient tensors (q+1,)*k, zero where |m| > q (ews/core/series_leaf.py:55-66)."""
    out = []
    for k in range(1, depth + 1):
        C = np.zeros((q + 1,) * k, dtype=np.float64)
        for m in _iproduct(range(q + 1), repeat=k):
            if sum(m) <= q:
                C[m] = float(coeff_exact(m))
        out.append(C)
    return tuple(out)


def series_error_bound(x: float, k: int, q: int) -> float:
    """Per-interval relative error bound at level k (ews/core/series_leaf.py:139-143)."""
    return (k * x) ** (q + 1) / math.factorial(q + 1) * math.exp(k * x)


def suggest_series_q(x, trunc, tol=1e-6, q_max=200):
    """Smallest q whose level-``trunc`` bound is below tol (ews/core/leaf.py:201-215)."""
    if x <= 0.0:
        return 1
    lx, ltol = math.log(trunc * x), math.log(tol)
    for q in range(1, q_max):
        if (q + 1) * lx - math.lgamma(q + 2) + trunc * x < ltol:
            return q
    return q_max


def check_series_q(A, dtheta_max, trunc, series_q, tol=1e-6, where=""):
    """Warns when series_q is too small for x = ||A||_op max dtheta (ews/core/leaf.py:218-238)."""
    import warnings

    x = float(torch.linalg.matrix_norm(torch.as_tensor(A, dtype=torch.float64), 2)) * float(dtheta_max)
    bound = series_error_bound(x, int(trunc), int(series_q))
    need = suggest_series_q(x, int(trunc), tol=tol)
    if bound > tol:
        warnings.warn(
            f"[series leaf{' ' + where if where else ''}] series_q={series_q} gives a per-interval error bound "
            f"of {bound:.2e} at x={x:.3f} (||A||*max dtheta), above tol={tol:.0e}. series_q={need} would suffice.",
            RuntimeWarning,
            stacklevel=2,
        )
    return x, bound, need


@lru_cache(maxsize=None)
def _scaled_coeffs(q: int, device: str, dtype: torch.dtype):
    """c1_p / p!  (q+1,)  and  c2_ab / (a! b!)  (q+1, q+1), the polynomial coefficients of Q1, Q2 in x."""
    C1, C2 = series_coeffs(2, q)
    fact = np.array([math.factorial(p) for p in range(q + 1)], dtype=np.float64)
    c1 = C1 / fact
    c2 = C2 / np.outer(fact, fact)
    return (torch.tensor(c1, dtype=dtype, device=device), torch.tensor(c2, dtype=dtype, device=device))


def diag_tables(x: torch.Tensor, q: int):
    """Q1 (..., N) and Q2 (..., N, N) of the diagonal series leaf at log-flows x (..., N), differentiable.

    Evaluated in float64 and returned in x's dtype: the tables are tiny (B x N^2) and exact tables keep
    the kernel's only rounding in the scan itself."""
    xd = x.to(torch.float64)
    c1, c2 = _scaled_coeffs(int(q), str(x.device), torch.float64)
    pw = [torch.ones_like(xd)]
    for _ in range(q):
        pw.append(pw[-1] * xd)  # products, so the gradient at x = 0 stays finite
    powers = torch.stack(pw, dim=-1)  # (..., N, q+1)
    q1 = powers @ c1
    q2 = torch.einsum("...ia,ab,...jb->...ij", powers, c2, powers)
    return q1.to(x.dtype), q2.to(x.dtype)


@lru_cache(maxsize=None)
def _leaf_coeffs(q: int, device: str):
    """c_p (q+1,) and c_ab (q+1, q+1) of the depth-2 series leaf as float64 tensors on ``device``, made
    once per (q, device) so that building the tables issues no host-to-device copy."""
    C1, C2 = series_coeffs(2, q)
    return (torch.tensor(C1, dtype=torch.float64, device=device), torch.tensor(C2, dtype=torch.float64, device=device))


def dense_leaf_tables(X: torch.Tensor, q: int, lift=None):
    """The series-leaf tables of the dense engine at X = -h A (B, N, N), float64: F = K1 W, G_a = P_a W,
    H_a = K2_a W with P_a = X^a / a!, K1 = sum_p c_p P_p, K2_a = sum_b c_ab P_b (the series leaf with
    shared letters, ews/core/series_leaf.py:72-113) and the lift W (identity when None). Differentiable."""
    N = X.shape[-1]
    eye = torch.eye(N, dtype=X.dtype, device=X.device).expand_as(X)
    P = [eye]
    for a in range(1, q + 1):
        P.append(P[-1] @ X / a)
    P = torch.stack(P, dim=1)  # (B, q+1, N, N)
    c1, c2 = _leaf_coeffs(int(q), str(X.device))
    K1 = torch.einsum("p,bpij->bij", c1, P)
    K2 = torch.einsum("ab,zbij->zaij", c2, P)
    W = torch.eye(N, dtype=X.dtype, device=X.device) if lift is None else lift.to(X.dtype)
    return K1 @ W, P @ W, K2 @ W


def dense_tables(A: torch.Tensor, h: torch.Tensor, q: int, lift=None):
    """Per-sample tables of the dense engine for generator A (N, N), clock steps h (B,) and lift W (N, d_in):
    the flow complement D = I - expm(-hA) and the series-leaf tables F, G, H (dense_leaf_tables).
    Differentiable; evaluated in float64 and returned in float32. The exponential
    (ews/core/chen_scan.py:155-168) and its VJP run in the library's expm kernels (CUDA tensors only)."""
    from .engine import Expm

    X = -h.to(torch.float64)[:, None, None] * A.to(torch.float64)  # (B, N, N)
    N = A.shape[-1]
    Dc = torch.eye(N, dtype=torch.float64, device=A.device) - Expm.apply(X)
    F, G, H = dense_leaf_tables(X, q, lift)
    return Dc.float(), F.float(), G.float(), H.float()
