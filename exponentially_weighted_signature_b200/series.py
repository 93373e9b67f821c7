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

import numpy as np
import torch


def level_coefficient(m) -> float:
    """c_m for the multi-index m = (m_1, ..., m_k): with the suffix sums M_j = m_j + ... + m_k, the k
    nested integrals over the simplex contribute the factors 1 / (M_j + k - j + 1)."""
    k = len(m)
    suffix = 0
    out = 1.0
    for j in range(k, 0, -1):  # innermost integral first
        suffix += m[j - 1]
        out /= suffix + (k - j + 1)
    return out


@lru_cache(maxsize=None)
def coefficient_tables(q: int):
    """The depth-1 and depth-2 coefficients the engines use, as float64 arrays with zeros where the
    order exceeds q: c1[p] = 1 / (p + 1) and c2[a, b] = 1 / ((a + b + 2) (b + 1))."""
    p = np.arange(q + 1, dtype=np.float64)
    c1 = 1.0 / (p + 1.0)
    a, b = np.meshgrid(p, p, indexing="ij")
    c2 = np.where(a + b <= q, 1.0 / ((a + b + 2.0) * (b + 1.0)), 0.0)
    return c1, c2


def series_error_bound(x: float, k: int, q: int) -> float:
    """Per-interval relative error of the level-k series truncated at order q, for x = ||A|| dtheta: the
    first omitted term of exp(k x), (k x)^(q+1) / (q+1)!, times the tail factor e^{k x}."""
    kx = k * x
    term = 1.0
    for n in range(1, q + 2):
        term *= kx / n
    return term * math.exp(kx)


def suggest_series_q(x, trunc, tol=1e-6, q_max=200):
    """The smallest order q >= 1 whose level-``trunc`` error bound is below ``tol`` (the reference's
    ``ews.core.leaf.suggest_series_q``). The bound's terms are followed as logarithms, so large x does not
    overflow."""
    if x <= 0.0:
        return 1
    log_kx = math.log(trunc * x)
    log_term = log_kx  # log of (k x)^(q+1) / (q+1)! at q = 0
    target = math.log(tol) - trunc * x
    for q in range(1, q_max):
        log_term += log_kx - math.log(q + 1)
        if log_term < target:
            return q
    return q_max


def check_series_q(A, dtheta_max, trunc, series_q, tol=1e-6, where=""):
    """Warns (RuntimeWarning) when ``series_q`` leaves a per-interval error bound above ``tol`` at the
    observed x = ||A||_2 max dtheta; returns (x, bound, the order that would meet tol), like the
    reference's ``ews.core.leaf.check_series_q``."""
    import warnings

    x = float(torch.linalg.matrix_norm(torch.as_tensor(A, dtype=torch.float64), 2)) * float(dtheta_max)
    bound = series_error_bound(x, int(trunc), int(series_q))
    need = suggest_series_q(x, int(trunc), tol=tol)
    if bound > tol:
        tag = f" ({where})" if where else ""
        warnings.warn(
            f"series leaf{tag}: order {series_q} bounds the local error by {bound:.2e} at "
            f"x = ||A|| max dtheta = {x:.3f}, above {tol:.0e}; order {need} meets it (the order is fixed "
            "when the layer is built)",
            RuntimeWarning,
            stacklevel=2,
        )
    return x, bound, need


@lru_cache(maxsize=None)
def _scaled_coeffs(q: int, device: str, dtype: torch.dtype):
    """c1_p / p!  (q+1,)  and  c2_ab / (a! b!)  (q+1, q+1), the polynomial coefficients of Q1, Q2 in x."""
    C1, C2 = coefficient_tables(q)
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
    C1, C2 = coefficient_tables(q)
    return (torch.tensor(C1, dtype=torch.float64, device=device), torch.tensor(C2, dtype=torch.float64, device=device))


def vanloan_series_coeffs(M: int, method: str, q: int):
    """The Van Loan leaf in the series leaf's normalisation: c1_p = k1_p p! and c_ab = k2_ab a! b! (the
    coefficients of b_p = (X^p / p!) dy), so the series leaf's dense tables evaluate it unchanged."""
    k1, k2 = vanloan_poly_coeffs(int(M), method, int(q))
    fact = np.array([math.factorial(p) for p in range(q + 1)], dtype=np.float64)
    return k1 * fact, k2 * np.outer(fact, fact)


@lru_cache(maxsize=None)
def vanloan_device_coeffs(M: int, method: str, q: int, device: str):
    """``vanloan_series_coeffs`` as float64 tensors on ``device``, made once per key (no copy per call)."""
    c1, c2 = vanloan_series_coeffs(M, method, q)
    return (torch.tensor(c1, dtype=torch.float64, device=device), torch.tensor(c2, dtype=torch.float64, device=device))


def dense_leaf_tables(X: torch.Tensor, q: int, lift=None, coeffs=None):
    """The series-leaf tables of the dense engine at X = -h A (B, N, N), float64: F = K1 W, G_a = P_a W,
    H_a = K2_a W with P_a = X^a / a!, K1 = sum_p c_p P_p, K2_a = sum_b c_ab P_b (the series leaf with
    shared letters, ews/core/series_leaf.py:72-113) and the lift W (identity when None). Differentiable."""
    N = X.shape[-1]
    eye = torch.eye(N, dtype=X.dtype, device=X.device).expand_as(X)
    P = [eye]
    for a in range(1, q + 1):
        P.append(P[-1] @ X / a)
    P = torch.stack(P, dim=1)  # (B, q+1, N, N)
    if coeffs is None:
        c1, c2 = _leaf_coeffs(int(q), str(X.device))
    else:
        c1, c2 = coeffs
    K1 = torch.einsum("p,bpij->bij", c1, P)
    K2 = torch.einsum("ab,zbij->zaij", c2, P)
    W = torch.eye(N, dtype=X.dtype, device=X.device) if lift is None else lift.to(X.dtype)
    return K1 @ W, P @ W, K2 @ W


def dense_tables(A: torch.Tensor, h: torch.Tensor, q: int, lift=None, coeffs=None, A_leaf=None):
    """Per-sample tables of the dense engine for generator A (N, N), clock steps h (B,) and lift W (N, d_in):
    the flow complement D = I - expm(-hA) (ews/core/chen_scan.py:155-168) and the series-leaf tables F, G, H
    (dense_leaf_tables), the latter of ``A_leaf`` when given (a leaf that reads its own generator from A,
    e.g. the plane leaf). Differentiable in A, h, A_leaf and W; evaluated in float64 by one library launch
    each way (CUDA tensors only) and returned in float32."""
    from .engine import DenseLeaf

    c1, c2 = _leaf_coeffs(int(q), str(A.device)) if coeffs is None else coeffs
    return DenseLeaf.apply(A, h, A_leaf, lift, c1, c2)


# ------------------------------------------------------------------------------ plane leaf


# The series order at which the plane leaf is evaluated, and the largest ||h A_planes||_inf for which that
# order reproduces the closed form to float32 rounding: the truncation error of the level-2 local terms is
# below series_error_bound(x, 2, q) = (2x)^(q+1) / (q+1)! e^(2x), 5.7e-9 relative at q = 11, x = 0.5.
PLANE_Q = 11
PLANE_X_MAX = 0.5
# The Jordan leaf is evaluated the same way (the closed forms of ews/core/kernels/jordan_engine.py are the
# series leaf's limit for the chain generator), at the same order and range.
CLOSED_Q = PLANE_Q
CLOSED_X_MAX = PLANE_X_MAX


def plane_generator(A: torch.Tensor) -> torch.Tensor:
    """The generator whose local terms the plane leaf computes (ews/core/leaf.py:116-136 reads
    d = A[2j, 2j] and w = A[2j, 2j+1] of each 2x2 plane and treats the plane as [[d, w], [-w, d]]): a
    block-diagonal matrix of those rotation-scaling blocks. Differentiable in A."""
    N = A.shape[-1]
    ii = torch.arange(0, N, 2, device=A.device)
    d = A[ii, ii]
    w = A[ii, ii + 1]
    P = torch.zeros_like(A)
    P[ii, ii] = d
    P[ii + 1, ii + 1] = d
    P[ii, ii + 1] = w
    P[ii + 1, ii] = -w
    return P


def jordan_generator(A: torch.Tensor, kind: str, size: int) -> torch.Tensor:
    """The generator whose local terms the Jordan leaf computes: its chains' parameters read off the first
    rows of each chain of A (ews/core/kernels/jordan_engine.py:324-353) and the chains rebuilt,
    J_j = D_j + eps_j Nil with Nil the shift by one coordinate (real chain, D = lam I; lam = A[f, f],
    eps = A[f, f+1]) or by one 2x2 slot (complex chain, D = diag(C, .., C), C = [[a, -b], [b, a]];
    a = A[f, f], b = A[f+1, f], eps = A[f, f+2]); f is the chain's first index. Equals A when A is the
    Jordan-structured matrix itself. Differentiable in A."""
    m = A.shape[-1]
    size = int(size)
    if m % size:
        raise ValueError(f"the Jordan leaf needs chains of size {size} that tile A; dimension {m}")
    first = torch.arange(0, m, size, device=A.device)
    K = first.numel()
    if kind == "real":
        lam, eps = A[first, first], A[first, first + 1]
        eye = torch.eye(size, dtype=A.dtype, device=A.device)
        nil = torch.diag(torch.ones(size - 1, dtype=A.dtype, device=A.device), 1)
        blocks = lam[:, None, None] * eye + eps[:, None, None] * nil  # (K, n, n)
    else:
        k = size // 2
        a, b, eps = A[first, first], A[first + 1, first], A[first, first + 2]
        C = torch.stack([torch.stack([a, -b], -1), torch.stack([b, a], -1)], -2)  # (K, 2, 2)
        eye_k = torch.eye(k, dtype=A.dtype, device=A.device)
        shift = torch.diag(torch.ones(k - 1, dtype=A.dtype, device=A.device), 1)
        eye2 = torch.eye(2, dtype=A.dtype, device=A.device)
        blocks = (torch.einsum("ij,nab->niajb", eye_k, C)
                  + eps[:, None, None, None, None] * torch.einsum("ij,ab->iajb", shift, eye2)[None]).reshape(K, size, size)
    return torch.block_diag(*blocks.unbind(0))


# ------------------------------------------------------------------------------ Van Loan leaf tables


def _vanloan_step(z: torch.Tensor, method: str):
    """For the augmented step matrix X = [[z, v], [0, 0]] of one coordinate (z = a dtheta / M, a the
    generator's diagonal entry, v the increment / M), the chosen exponential gives
    E(X) = [[c, g v], [0, 1]]; returns (c, g). Derived per method from the reference's formulas
    (ews/core/expm_approx.py:13-41): exact c = e^z, g = (e^z - 1) / z; euler c = 1 + z, g = 1;
    cayley (I - X/2)^{-1} (I + X/2): c = (1 + z/2) / (1 - z/2), g = 1 / (1 - z/2); pade (2, 2):
    c = (1 + z/2 + z^2/12) / (1 - z/2 + z^2/12), g = 1 / (1 - z/2 + z^2/12)."""
    if method == "exact":
        c = torch.exp(z)
        small = z.abs() < 1e-8
        zs = torch.where(small, torch.ones_like(z), z)
        g = torch.where(small, 1.0 + z / 2, torch.expm1(zs) / zs)
        return c, g
    if method == "euler":
        return 1.0 + z, torch.ones_like(z)
    if method == "cayley":
        den = 1.0 - z / 2
        return (1.0 + z / 2) / den, 1.0 / den
    if method == "pade":
        z2 = z * z / 12.0
        den = 1.0 - z / 2 + z2
        return (1.0 + z / 2 + z2) / den, 1.0 / den
    raise ValueError(f"unknown expm method {method!r}")


def vanloan_diag_tables(lam: torch.Tensor, h: torch.Tensor, M: int, method: str = "cayley", eps: float = 1e-12):
    """Q1 (B, N), Q2 (B, N, N) of the Van Loan leaf (the reference's default local terms,
    ews/core/van_loan.py:91-144 and ews/core/signature.py:19-36) for a diagonal generator
    A = diag(lam) under a uniform clock step h (B,), so that s1_i = Q1_i dy_i and s2_ij = Q2_ij dy_i dy_j
    as in the series tables. Differentiable; float64 in, float64 out.

    With A diagonal the augmented exponential acts coordinate by coordinate. The leaf's M + 1 knots
    k_m = E_A^{-M} (sum_{j<m} E_A^j) g v are those of a piecewise-linear path whose m-th segment is
    p_m dy with p_m = g c^{m-1-M} / M (m = 1..M); the depth-2 signature of M segments is
    level 1 = sum_m p_m dy and level 2 = (sum_{m<n} p_m (x) p_n + 1/2 sum_m p_m (x) p_m) dy (x) dy.
    A step below ``eps`` is the reference's jump case (linear interpolation): Q1 = 1, Q2 = 1/2."""
    lam = lam.to(torch.float64)
    h = h.to(torch.float64)
    z = (h[:, None] * lam[None, :]) / M  # (B, N)
    c, g = _vanloan_step(z, method)
    m = torch.arange(1, M + 1, dtype=torch.float64, device=lam.device)
    P = (g[..., None] / M) * c[..., None] ** (m - 1 - M)  # (B, N, M)
    jump = (h <= eps)[:, None, None]
    P = torch.where(jump, torch.full_like(P, 1.0 / M), P)
    q1 = P.sum(-1)
    # R[j, m] = 1/2 p_{m,j} + sum_{n>m} p_{n,j}
    tail = torch.flip(torch.cumsum(torch.flip(P, [-1]), -1), [-1]) - P
    R = 0.5 * P + tail
    q2 = torch.einsum("bim,bjm->bij", P, R)
    return q1, q2


def _ps_mul(a, b, n):
    out = [Fraction(0)] * (n + 1)
    for i, ai in enumerate(a):
        if ai == 0:
            continue
        for j in range(n + 1 - i):
            out[i + j] += ai * b[j]
    return out


def _ps_inv(a, n):
    """1 / a as a power series (a[0] != 0)."""
    out = [Fraction(0)] * (n + 1)
    out[0] = 1 / a[0]
    for k in range(1, n + 1):
        acc = Fraction(0)
        for j in range(1, k + 1):
            if j < len(a):
                acc += a[j] * out[k - j]
        out[k] = -acc / a[0]
    return out


def _ps_pow(a, e, n):
    base = a if e >= 0 else _ps_inv(a, n)
    out = [Fraction(1)] + [Fraction(0)] * n
    for _ in range(abs(e)):
        out = _ps_mul(out, base, n)
    return out


@lru_cache(maxsize=None)
def vanloan_poly_coeffs(M: int, method: str, degree: int):
    """Polynomial coefficients, in the log-flow x = -dtheta a, of the Van Loan leaf's diagonal tables:
    Q1(x) = sum_a k1[a] x^a and Q2(x_i, x_j) = sum_{a,b} k2[a, b] x_i^a x_j^b, truncated at ``degree`` in
    each variable (float64 arrays).

    The leaf's m-th segment is p_m(x) dy with p_m(x) = g(z) c(z)^{m-1-M} / M, z = -x / M (c, g the
    chosen exponential of the augmented step, ``_vanloan_step``), so Q1 = sum_m p_m and
    Q2 = sum_{m<n} p_m(x_i) p_n(x_j) + 1/2 sum_m p_m(x_i) p_m(x_j). For a generator that is not diagonal
    the same coefficients apply to the powers of X = -dtheta A (every factor is a function of one
    matrix), i.e. they are the series leaf's coefficients c_p / p! and c_ab / (a! b!) with the Van Loan
    leaf's values. The power series are exact rationals; the truncation error is of order
    |x|^(degree+1) / (degree+1)! relative."""
    n = degree
    half = Fraction(1, 2)
    if method == "exact":
        ez = [Fraction(1, math.factorial(k)) for k in range(n + 2)]
        c = ez[: n + 1]
        g = [Fraction(1, math.factorial(k + 1)) for k in range(n + 1)]  # (e^z - 1) / z
    elif method == "euler":
        c = [Fraction(1), Fraction(1)] + [Fraction(0)] * (n - 1)
        g = [Fraction(1)] + [Fraction(0)] * n
    elif method == "cayley":
        den = _ps_inv([Fraction(1), -half], n)
        c = _ps_mul([Fraction(1), half], den, n)
        g = den
    elif method == "pade":
        den = _ps_inv([Fraction(1), -half, Fraction(1, 12)], n)
        c = _ps_mul([Fraction(1), half, Fraction(1, 12)], den, n)
        g = den
    else:
        raise ValueError(f"unknown expm method {method!r}")
    c = (c + [Fraction(0)] * (n + 1))[: n + 1]
    g = (g + [Fraction(0)] * (n + 1))[: n + 1]
    # series in z -> series in x (z = -x / M): coefficient k scales by (-1/M)^k
    scale = [Fraction(-1, M) ** k for k in range(n + 1)]
    segs = []
    for m in range(1, M + 1):
        pz = _ps_mul(g, _ps_pow(c, m - 1 - M, n), n)
        segs.append([pz[k] * scale[k] / M for k in range(n + 1)])
    k1 = [sum(s[a] for s in segs) for a in range(n + 1)]
    # tails[m][b] = sum_{n > m} p_n[b]
    tails = [[Fraction(0)] * (n + 1) for _ in range(M)]
    run = [Fraction(0)] * (n + 1)
    for m in range(M - 1, -1, -1):
        tails[m] = list(run)
        run = [run[b] + segs[m][b] for b in range(n + 1)]
    k2 = [[sum(segs[m][a] * (tails[m][b] + half * segs[m][b]) for m in range(M)) for b in range(n + 1)]
          for a in range(n + 1)]
    return np.array([float(v) for v in k1]), np.array([[float(v) for v in row] for row in k2])
