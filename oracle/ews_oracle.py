"""CPU restatement of the reference's EWS hot path (test infrastructure only; see ``oracle/__init__``).

Every function restates, in torch on the CPU, the reference function named in its docstring
(paths inside the reference project alexandre-bloch/exponentially-weighted-signature). All
functions broadcast over leading batch axes: a path is ``(..., L, d)`` knots, a clock ``(..., L)``;
time is the second-to-last path axis. Levels are kept flat, level k as ``(..., d**k)`` row-major,
which is the reference's packed layout (``ews/core/chen_scan.py:34-47``).

Sign convention: the reference's flow is ``exp(-dtheta * A)`` (``ews/core/chen_scan.py:155-168``).
Generators here are the reference's ``A``; a configuration written as ``expm(A_cfg * dtau)`` is
called with ``A = -A_cfg``.
"""

from __future__ import annotations

import math
from fractions import Fraction
from functools import lru_cache
from itertools import product as _iproduct

import numpy as np
import torch

# ----------------------------------------------------------------------------------- series leaf


def coeff_exact(m) -> Fraction:
    """c_m = prod_j 1/(M_j + k - j + 1), M_j = m_j + ... + m_k (``ews/core/series_leaf.py:45-52``)."""
    k = len(m)
    out = Fraction(1)
    for j in range(1, k + 1):
        out /= sum(m[j - 1 :]) + k - j + 1
    return out


@lru_cache(maxsize=None)
def series_coeffs(depth: int, q: int):
    """Level-k coefficient tensors C^k of shape (q+1,)*k, zero beyond |m| > q
    (``ews/core/series_leaf.py:55-66``)."""
    out = []
    for k in range(1, depth + 1):
        C = np.zeros((q + 1,) * k, dtype=np.float64)
        for m in _iproduct(range(q + 1), repeat=k):
            if sum(m) <= q:
                C[m] = float(coeff_exact(m))
        out.append(C)
    return tuple(out)


def series_letters(delta_x, delta_theta, A, q: int):
    """Letters b_0 = dx, b_p = (-dtheta/p) A b_{p-1}: (..., L, q+1, d) (``ews/core/series_leaf.py:72-86``)."""
    bs = [delta_x]
    for p in range(1, q + 1):
        bs.append((-delta_theta / p)[..., None] * torch.einsum("...ij,...lj->...li", A, bs[-1]))
    return torch.stack(bs, dim=-2)


def _level_einsum(k: int) -> str:
    coeff = "abcdefgh"[:k]
    outs = "ABCDEFGH"[:k]
    factors = [f"...n{coeff[j]}{outs[j]}" for j in range(k)]
    return coeff + "," + ",".join(factors) + "->...n" + outs


def assemble_from_letters(b, depth: int, q: int):
    """Level k = sum_m c_m b_{m1} (x) ... (x) b_{mk}, flat (..., L, d**k) (``ews/core/series_leaf.py:100-113``)."""
    coeffs = series_coeffs(depth, q)
    lead, L, d = b.shape[:-3], b.shape[-3], b.shape[-1]
    levels = []
    for k in range(1, depth + 1):
        C = torch.as_tensor(coeffs[k - 1], dtype=b.dtype)
        lvl = torch.einsum(_level_einsum(k), C, *([b] * k))
        levels.append(lvl.reshape(lead + (L, d**k)))
    return levels


def series_local_signatures(path, clock, A, depth: int, q: int):
    """Per-interval local terms from the series (``ews/core/series_leaf.py:116-126``)."""
    delta_x = path[..., 1:, :] - path[..., :-1, :]
    delta_theta = clock[..., 1:] - clock[..., :-1]
    return assemble_from_letters(series_letters(delta_x, delta_theta, A, q), depth, q)


def series_error_bound(x: float, k: int, q: int) -> float:
    """(k x)^(q+1)/(q+1)! e^(k x) (``ews/core/series_leaf.py:139-143``)."""
    return (k * x) ** (q + 1) / math.factorial(q + 1) * math.exp(k * x)


def suggest_series_q(x, trunc, tol=1e-6, q_max=200):
    """Smallest q with the level-``trunc`` bound below tol, in log space (``ews/core/leaf.py:201-215``)."""
    if x <= 0.0:
        return 1
    lx, ltol = math.log(trunc * x), math.log(tol)
    for q in range(1, q_max):
        if (q + 1) * lx - math.lgamma(q + 2) + trunc * x < ltol:
            return q
    return q_max


# ------------------------------------------------------------------------ plane closed forms


def _guarded(x, closed, series, tol):
    small = x.abs() < tol
    xs = torch.where(small, torch.ones_like(x), x)
    return torch.where(small, series(x), closed(xs))


def phi(x):
    """(e^x - 1)/x with a Taylor guard below 1e-3 (``ews/core/kernels/plane_engine.py:29-35``)."""
    return _guarded(
        x,
        lambda x: torch.expm1(x) / x,
        lambda x: 1 + x * (1 / 2 + x * (1 / 6 + x * (1 / 24 + x * (1 / 120 + x / 720)))),
        1e-3,
    )


def dphi(x):
    """phi'(x) (``ews/core/kernels/plane_engine.py:38-44``)."""
    return _guarded(
        x,
        lambda x: (torch.exp(x) * (x - 1) + 1) / x**2,
        lambda x: 1 / 2 + x * (1 / 3 + x * (1 / 8 + x * (1 / 30 + x * (1 / 144 + x / 840)))),
        3e-2,
    )


def d2phi(x):
    """phi''(x) (``ews/core/kernels/plane_engine.py:47-53``)."""
    return _guarded(
        x,
        lambda x: (torch.exp(x) * (x**2 - 2 * x + 2) - 2) / x**3,
        lambda x: 1 / 3 + x * (1 / 4 + x * (1 / 10 + x * (1 / 36 + x * (1 / 168 + x / 960)))),
        1e-1,
    )


def d3phi(x):
    """phi'''(x) (``ews/core/kernels/plane_engine.py:56-62``)."""
    return _guarded(
        x,
        lambda x: (torch.exp(x) * (x**3 - 3 * x**2 + 6 * x - 6) + 6) / x**4,
        lambda x: 1 / 4 + x * (1 / 5 + x * (1 / 12 + x * (1 / 42 + x * (1 / 192 + x / 1080)))),
        2.5e-1,
    )


def divdiff_phi(x, delta, tol=None):
    """(phi(x + delta) - phi(x))/delta with a third-order Taylor guard in delta
    (``ews/core/kernels/plane_engine.py:65-78``)."""
    if tol is None:
        real = x.real if x.is_complex() else x
        tol = 4e-4 if real.dtype == torch.float64 else 5e-2
    small = delta.abs() < tol
    ds = torch.where(small, torch.ones_like(delta), delta)
    direct = (phi(x + ds) - phi(x)) / ds
    series = dphi(x) + delta * (d2phi(x) / 2 + delta * d3phi(x) / 6)
    return torch.where(small, series, direct)


def to_complex_planes(v):
    """(..., m) real, plane j at (2j, 2j+1) -> (..., K) complex (``plane_engine.py:84-87``)."""
    v = v.reshape(v.shape[:-1] + (-1, 2))
    return torch.complex(v[..., 0], v[..., 1])


def from_complex_planes(p):
    """(..., K) complex -> (..., m) interleaved (``plane_engine.py:90-92``)."""
    return torch.stack([p.real, p.imag], -1).reshape(p.shape[:-1] + (-1,))


def _blocks_from_AB(A, B):
    """Real 2x2 blocks of u w^T from A = u conj(w), B = u w (``plane_engine.py:111-116``)."""
    q00 = (A.real + B.real) / 2
    q11 = (A.real - B.real) / 2
    q01 = (B.imag - A.imag) / 2
    q10 = (A.imag + B.imag) / 2
    return torch.stack([torch.stack([q00, q01], -1), torch.stack([q10, q11], -1)], -2)


def blocks_to_flat(Q):
    """(..., K, K, n, n) -> (..., m*m) row-major (``plane_engine.py:119-122``, ``blockdiag_engine.py:176-179``)."""
    K, n = Q.shape[-3], Q.shape[-1]
    return Q.transpose(-3, -2).reshape(Q.shape[:-4] + (K * n * K * n,))


def plane_local_terms(v, dw, dtheta, N):
    """Closed-form local terms of canonical planes [[d, w], [-w, d]], depths 1-2
    (``ews/core/kernels/plane_engine.py:134-152``). v (..., L, m), dw (K, 2), dtheta (..., L)."""
    z = torch.complex(dw[:, 0], dw[:, 1])
    zc = z.conj()
    h = dtheta[..., None].to(z.dtype)
    rho = torch.exp(-h * zc)
    p = to_complex_planes(v)
    s1 = phi(-h * zc) * p
    if N == 1:
        return rho, s1, None
    x = -h[..., None] * zc[:, None]
    IA = divdiff_phi(x, -h[..., None] * z[None, :])
    IB = divdiff_phi(x, -h[..., None] * zc[None, :])
    A = IA * p[..., :, None] * p.conj()[..., None, :]
    B = IB * p[..., :, None] * p[..., None, :]
    return rho, s1, _blocks_from_AB(A, B)


# ---------------------------------------------------------------------------- exponentials


def _expm_taylor(X):
    """Matrix exponential by scaling and squaring with a degree-16 Taylor polynomial, in torch ops (so
    autograd differentiates it): X is scaled by 2^-s until ||X||_1 <= 1/64, where the truncation error
    is below 1e-40, then squared s times. The reference's ``jax.scipy.linalg.expm`` is accurate to
    float64 rounding; torch.linalg.matrix_exp is not (3e-11 on a diagonal matrix of norm 0.04), which
    would leave the oracle's flows ~1e-11 off after a few steps."""
    with torch.no_grad():
        norm = torch.linalg.matrix_norm(X.detach(), ord=1)
        nmax = float(norm.max()) if norm.numel() else 0.0
    s = 0 if nmax <= 1.0 / 64 else int(math.ceil(math.log2(nmax * 64)))
    Y = X / (2.0**s)
    eye = torch.eye(X.shape[-1], dtype=X.dtype, device=X.device).expand(X.shape)
    term = eye
    out = eye
    for k in range(1, 17):
        term = term @ Y / k
        out = out + term
    for _ in range(s):
        out = out @ out
    return out


def expm_matrix(X, method="exact"):
    """exact / euler / cayley / pade exponentials (``ews/core/expm_approx.py:13-41``)."""
    method = method.lower()
    if method in {"pade_lite", "pade-lite"}:
        method = "pade"
    if method == "exact":
        return _expm_taylor(X)
    eye = torch.eye(X.shape[-1], dtype=X.dtype).expand(X.shape)
    if method == "euler":
        return eye + X
    if method == "cayley":
        return torch.linalg.solve(eye - 0.5 * X, eye + 0.5 * X)
    if method == "pade":
        X2 = X @ X
        return torch.linalg.solve(eye - 0.5 * X + X2 / 12.0, eye + 0.5 * X + X2 / 12.0)
    raise ValueError(f"Unknown expm method: {method}")


def block_series_local_terms(path, clock, A, N, q):
    """``leaf='block_series'``: level 1 = G v with [[E, G], [0, I]] = exp([[-hA, I], [0, 0]]), level 2 = the
    series letters assembled blockwise (``ews/core/kernels/blockdiag_engine.py:88-155``). For a block-diagonal A
    the augmented exponential of the whole A is block-diagonal in the same blocks, so this equals the
    reference's per-block evaluation."""
    v = path[..., 1:, :] - path[..., :-1, :]
    dth = clock[..., 1:] - clock[..., :-1]
    d = A.shape[-1]
    aug = torch.zeros(dth.shape + (2 * d, 2 * d), dtype=A.dtype)
    aug[..., :d, :d] = -dth[..., None, None] * A
    aug[..., :d, d:] = torch.eye(d, dtype=A.dtype)
    G = torch.linalg.matrix_exp(aug)[..., :d, d:]
    levels = [torch.einsum("...ab,...b->...a", G, v)]
    if N == 2:
        b = series_letters(v, dth, A, q)
        levels.append(assemble_from_letters(b, 2, q)[1])
    return levels


def plane_closed_local_terms(path, clock, A, N):
    """``leaf='plane_closed'`` (``ews/core/leaf.py:116-136``)."""
    v = path[..., 1:, :] - path[..., :-1, :]
    dth = clock[..., 1:] - clock[..., :-1]
    d = A.shape[-1]
    ii = torch.arange(0, d, 2)
    dw = torch.stack([A[ii, ii], A[ii, ii + 1]], -1)
    _rho, s1, s2 = plane_local_terms(v, dw, dth, N)
    levels = [from_complex_planes(s1)]
    if N == 2:
        levels.append(blocks_to_flat(s2))
    return levels


# ------------------------------------------------------------------------ Jordan closed forms
# Restatement of the float64 / complex128 table forms of ews/core/kernels/jordan_engine.py:159-320 (the
# leaves "jordan_closed" and "jordan_closed_tables"; the fast forms of :46-157 compute the same closed
# forms by forward-mode derivatives, which agree to rounding).
J_PHI_TERMS, J_PHI_SWITCH = 64, 8.0
J_PAIR_TERMS, J_PAIR_SWITCH, J_PAIR_S, J_PAIR_DELTA0 = 24, 1.5, 10, 0.25


def _cplx(x):
    return torch.is_complex(x)


def phi_derivative_table(y, r_max, n_terms=J_PHI_TERMS, switch=J_PHI_SWITCH):
    """phi^(r)(y), r = 0..r_max, phi(y) = (e^y - 1)/y, real or complex y with Re y <= 0 (``jordan_engine.py:175-199``):
    the entire series sum_j y^j / ((j + r + 1) j!) for |y| <= switch, else phi^(r) = (e^y - r phi^(r-1)) / y from
    expm1(y)/y. y (...) -> (..., r_max + 1)."""
    small = y.abs() <= switch
    ys = torch.where(small, y, torch.zeros_like(y))
    yl = torch.where(small, torch.full_like(y, -2.0 * switch), y)
    j = torch.arange(int(n_terms), dtype=torch.float64)
    ratios = torch.where(j == 0, torch.ones_like(ys[..., None]), ys[..., None] / torch.clamp(j, min=1.0))
    ypow = torch.cumprod(ratios, dim=-1)  # y^j / j!
    r = torch.arange(r_max + 1, dtype=torch.float64)
    C = 1.0 / (j[None, :] + r[:, None] + 1.0)  # (R, J)
    series = ypow @ (C.T.to(ypow.dtype))
    ey = torch.exp(yl)
    cols = [torch.expm1(yl) / yl]
    for rr in range(1, r_max + 1):
        cols.append((ey - rr * cols[-1]) / yl)
    return torch.where(small[..., None], series, torch.stack(cols, dim=-1))


def pair_integral_derivatives(x, delta, p_max, q_max):
    """d_x^p d_delta^q of D(x, delta) = (phi(x + delta) - phi(x)) / delta on the chain-pair grid, x (L, K), delta (L, K)
    -> {(p, q): (L, K, K)} (``jordan_engine.py:202-243``): the delta expansion below J_PAIR_DELTA0, Leibniz on
    F(delta) / delta above."""
    if _cplx(x) != _cplx(delta):
        x, delta = x.to(torch.complex128), delta.to(torch.complex128)
    small = delta.abs() < J_PAIR_DELTA0
    ds = torch.where(small, delta, torch.zeros_like(delta))
    dl = torch.where(small, torch.full_like(delta, -1.0), delta)
    tab_x = phi_derivative_table(x, p_max + q_max + 1 + J_PAIR_S)  # (L, K_j, R)
    s_idx = torch.arange(J_PAIR_S, dtype=torch.float64)
    ratios = torch.where(s_idx == 0, torch.ones_like(ds[..., None]), ds[..., None] / torch.clamp(s_idx, min=1.0))
    dpow = torch.cumprod(ratios, dim=-1)  # delta^s / s!
    tab_xd = phi_derivative_table(x[:, :, None] + dl[:, None, :], p_max + q_max, J_PAIR_TERMS, J_PAIR_SWITCH)
    inv = 1.0 / dl
    out = {}
    for pp in range(p_max + 1):
        for qq in range(q_max + 1):
            base = pp + qq + 1
            ser = torch.einsum("njs,nks->njk", tab_x[:, :, base : base + J_PAIR_S], dpow / (qq + s_idx + 1.0))
            lei = 0.0
            for ss in range(qq + 1):
                F = tab_xd[..., pp + ss] - (tab_x[:, :, None, pp] if ss == 0 else 0.0)
                coef = math.comb(qq, ss) * (-1.0) ** (qq - ss) * math.factorial(qq - ss)
                lei = lei + coef * F * inv[:, None, :] ** (qq - ss + 1)
            out[(pp, qq)] = torch.where(small[:, None, :], ser, lei)
    return out


def _jordan_shifted(P, eps, n):
    """[(eps Nil)^p P for p < n]; P (L, K, n), eps (K,) (``jordan_engine.py:246-252``)."""
    L, K, _ = P.shape
    e = eps.to(P.real.dtype if _cplx(P) else P.dtype)[None, :, None]
    return [torch.cat([P[:, :, p:], torch.zeros((L, K, p), dtype=P.dtype)], -1) * e**p for p in range(n)]


def _jordan_real(v, lam, eps, dtheta, N, n):
    """Real chains of length n (``jordan_engine.py:255-285``). v (L, m), lam, eps (K,), dtheta (L,)."""
    L, m = v.shape
    K = m // n
    h = dtheta[:, None]
    x = -h * lam[None, :]
    shifted = _jordan_shifted(v.reshape(L, K, n), eps, n)
    tab = phi_derivative_table(x, n - 1)
    s1 = torch.zeros((L, K, n), dtype=v.dtype)
    for p in range(n):
        s1 = s1 + ((-h) ** p * tab[:, :, p] / math.factorial(p))[:, :, None] * shifted[p]
    s1 = s1.reshape(L, m)
    if N == 1:
        return [s1]
    D = pair_integral_derivatives(x, x, n - 1, n - 1)
    Q = torch.zeros((L, K, K, n, n), dtype=v.dtype)
    for p in range(n):
        for q in range(n):
            coef = (-h[:, :, None]) ** (p + q) * D[(p, q)] / (math.factorial(p) * math.factorial(q))
            Q = Q + coef[..., None, None] * shifted[p][:, :, None, :, None] * shifted[q][:, None, :, None, :]
    return [s1, Q.transpose(2, 3).reshape(L, m, m)]


def _jordan_complex(v, c, eps, dtheta, N, k):
    """Complex chains of k complex coordinates (``jordan_engine.py:288-320``); c (K,) = a + ib."""
    L, m = v.shape
    K = m // (2 * k)
    h = dtheta[:, None].to(torch.float64)
    x = -h * c[None, :]
    vv = v.reshape(L, K, k, 2)
    shifted = _jordan_shifted(torch.complex(vv[..., 0], vv[..., 1]), eps, k)
    tab = phi_derivative_table(x, k - 1)
    s1c = torch.zeros((L, K, k), dtype=torch.complex128)
    for p in range(k):
        s1c = s1c + ((-h) ** p * tab[:, :, p] / math.factorial(p))[:, :, None] * shifted[p]
    s1 = torch.stack([s1c.real, s1c.imag], -1).reshape(L, m)
    if N == 1:
        return [s1]
    DA = pair_integral_derivatives(x, torch.conj(x), k - 1, k - 1)
    DB = pair_integral_derivatives(x, x, k - 1, k - 1)
    Ab = torch.zeros((L, K, K, k, k), dtype=torch.complex128)
    Bb = torch.zeros((L, K, K, k, k), dtype=torch.complex128)
    for p in range(k):
        for q in range(k):
            scale = (-h[:, :, None]) ** (p + q) / (math.factorial(p) * math.factorial(q))
            Pj = shifted[p][:, :, None, :, None]
            Pk = shifted[q][:, None, :, None, :]
            Ab = Ab + (scale * DA[(p, q)])[..., None, None] * Pj * torch.conj(Pk)
            Bb = Bb + (scale * DB[(p, q)])[..., None, None] * Pj * Pk
    # real 2x2 blocks of the complex coordinate pairs (``jordan_engine.py:79-91``)
    q00 = (Ab.real + Bb.real) / 2
    q11 = (Ab.real - Bb.real) / 2
    q01 = (Bb.imag - Ab.imag) / 2
    q10 = (Ab.imag + Bb.imag) / 2
    Qb = torch.stack([torch.stack([q00, q01], -1), torch.stack([q10, q11], -1)], -2)  # (L, Kj, Kk, ki, kl, 2, 2)
    Qb = Qb.permute(0, 1, 3, 5, 2, 4, 6)
    return [s1, Qb.reshape(L, m, m)]


def jordan_local_terms(path, clock, A, trunc, chain):
    """``leaf='jordan_closed'`` / ``'jordan_closed_tables'`` (``ews/core/leaf.py:173-192``,
    ``ews/core/kernels/jordan_engine.py:324-353``): the chains' eigenvalue and coupling read off A's first rows.
    path (..., L, d) knots, clock (..., L); broadcast over leading axes."""
    if trunc > 2:
        raise NotImplementedError("the closed-form Jordan leaf exists for depths 1 and 2")
    kind, size = chain
    lead = path.shape[:-2]
    v_all = (path[..., 1:, :] - path[..., :-1, :]).reshape(-1, path.shape[-2] - 1, path.shape[-1])
    dth_all = (clock[..., 1:] - clock[..., :-1]).reshape(-1, clock.shape[-1] - 1)
    m = A.shape[-1]
    first = torch.arange(0, m, size)
    outs = []
    for i in range(v_all.shape[0]):
        v, dth = v_all[i], dth_all[i]
        if kind == "real":
            lv = _jordan_real(v, A[first, first], A[first, first + 1], dth, trunc, size)
        else:
            c = torch.complex(A[first, first].to(torch.float64), A[first + 1, first].to(torch.float64))
            lv = _jordan_complex(v, c, A[first, first + 2], dth, trunc, size // 2)
        outs.append([lv[0]] + ([lv[1].reshape(lv[1].shape[0], -1)] if trunc == 2 else []))
    L1 = v_all.shape[1]
    return [torch.stack([o[k] for o in outs]).reshape(lead + (L1, -1)) for k in range(trunc)]


def local_signatures(path, clock, A, trunc, kind="series", series_q=None, jordan_chain=None):
    """Leaf dispatcher for the exact leaves (``ews/core/leaf.py:50-198``)."""
    if kind in ("jordan_closed", "jordan_closed_tables"):
        if jordan_chain is None:
            raise ValueError(f"leaf={kind!r} needs jordan_chain (uniform Jordan chains)")
        return jordan_local_terms(path, clock, A, trunc, jordan_chain)
    if kind == "series":
        if series_q is None:
            raise ValueError("kind='series' requires series_q (see check_series_q).")
        return series_local_signatures(path, clock, A, trunc, int(series_q))
    if kind == "plane_closed":
        if trunc > 2:
            raise NotImplementedError("leaf='plane_closed': closed-form local terms exist for depths 1 and 2")
        return plane_closed_local_terms(path, clock, A, trunc)
    if kind == "block_series":
        if trunc > 2:
            raise NotImplementedError("leaf='block_series': blockwise series local terms exist for depths 1 and 2")
        if trunc == 2 and series_q is None:
            raise ValueError("leaf='block_series' at depth 2 requires series_q (see check_series_q).")
        return block_series_local_terms(path, clock, A, trunc, series_q)
    raise ValueError(f"unsupported oracle leaf {kind!r}")


# ------------------------------------------------------------------------------- Chen algebra


def level_sizes(d, n):
    return [d**k for k in range(1, n + 1)]


def unpack(packed, d, n):
    """(..., sum d^k) -> [(..., d^k)] (``ews/core/chen_scan.py:64-78``)."""
    out, start = [], 0
    for s in level_sizes(d, n):
        out.append(packed[..., start : start + s])
        start += s
    return out


def pack(levels):
    """(``ews/core/chen_scan.py:33-46``)."""
    return torch.cat(levels, dim=-1)


def apply_flow(M, level, k, d):
    """M applied along every axis of a flat level-k tensor (``ews/core/chen_scan.py:98-111``), one axis at a
    time (the contraction order jnp.einsum's path optimiser picks: d^{k+1} per tensor)."""
    lead = level.shape[:-1]
    T = level.reshape(lead + (d,) * k)
    for ax in range(k):
        # contract axis ax of T with M's second index, put the new index back in place
        T = torch.movedim(torch.einsum("...ij,...j->...i", M[(...,) + (None,) * (k - 1) + (slice(None), slice(None))], torch.movedim(T, len(lead) + ax, -1)), -1, len(lead) + ax)
    return T.reshape(lead + (d**k,))


def tensor_mult(X, Y):
    """Truncated tensor product with implicit level 0 (signax 0.2.1 ``tensor_ops.mult``):
    Z_k = X_k + Y_k + sum_{i+j=k} X_i (x) Y_j."""
    n = len(X)
    Z = []
    for k in range(1, n + 1):
        z = X[k - 1] + Y[k - 1]
        for i in range(1, k):
            o = X[i - 1][..., :, None] * Y[k - i - 1][..., None, :]
            z = z + o.reshape(o.shape[:-2] + (o.shape[-2] * o.shape[-1],))
        Z.append(z)
    return Z


def chen_op(left, right, d, n):
    """(packed, h, M) pairs -> (mult(flow_{M_R}(S_L), S_R), h_L + h_R, M_L @ M_R)
    (``ews/core/chen_scan.py:124-152``)."""
    pL, hL, ML = left
    pR, hR, MR = right
    SL = unpack(pL, d, n)
    SR = unpack(pR, d, n)
    flowed = [apply_flow(MR, SL[k - 1], k, d) for k in range(1, n + 1)]
    return pack(tensor_mult(flowed, SR)), hL + hR, ML @ MR


def _interleave(a, b):
    """a[0], b[0], a[1], b[1], ... along dim 0 (len(a) == len(b) or len(b) + 1)."""
    m = b.shape[0]
    pairs = torch.stack([a[:m], b], dim=1).reshape((2 * m,) + a.shape[1:])
    if a.shape[0] > m:
        pairs = torch.cat([pairs, a[m:]], dim=0)
    return pairs


def associative_scan(op, elems):
    """Inclusive parallel prefix scan along dim 0 with the odd/even recursion of
    ``jax.lax.associative_scan`` (the scan the reference runs at ``ews/core/chen_scan.py:211``)."""
    n = elems[0].shape[0]
    if n < 2:
        return elems
    reduced = op(tuple(e[0:-1:2] for e in elems), tuple(e[1::2] for e in elems))
    odd = associative_scan(op, reduced)
    if n % 2 == 0:
        even = op(tuple(e[:-1] for e in odd), tuple(e[2::2] for e in elems))
    else:
        even = op(odd, tuple(e[2::2] for e in elems))
    even = tuple(torch.cat([e[0:1], r], dim=0) for e, r in zip(elems, even))
    return tuple(_interleave(e, o) for e, o in zip(even, odd))


def chen_M_per_interval(interval_times, A, expm_method="exact", cached=False, basepoint=False):
    """Flows M_t = exp(-dtheta_t A) (``ews/core/chen_scan.py:155-168``). interval_times (..., L)."""
    if not cached:
        return expm_matrix(-interval_times[..., None, None] * A, expm_method)
    L = interval_times.shape[-1]
    h = interval_times[..., 1] if basepoint else interval_times[..., 0]
    M1 = expm_matrix(-h[..., None, None] * A, expm_method)
    M = M1[..., None, :, :].expand(M1.shape[:-2] + (L,) + M1.shape[-2:])
    if basepoint:
        eye = torch.eye(A.shape[-1], dtype=A.dtype).expand(M1.shape[:-2] + (1,) + M1.shape[-2:])
        M = torch.cat([eye, M[..., 1:, :, :]], dim=-3)
    return M


def _time_first(x, nd_tail):
    """Move the time axis (just before ``nd_tail`` trailing axes) to dim 0."""
    return x.movedim(x.dim() - 1 - nd_tail, 0)


def _time_back(x, nd_tail):
    return x.movedim(0, x.dim() - 1 - nd_tail)


def chen_prefix_assoc(levels, interval_times, M, d, n):
    """Packed associative prefix scan carrying (h, M) (``ews/core/chen_scan.py:171-214``):
    levels [(..., L, d^k)], interval_times (..., L), M (..., L, d, d) -> (..., L, D)."""
    packed = pack(levels)
    elems = (_time_first(packed, 1), _time_first(interval_times, 0), _time_first(M, 2))
    out = associative_scan(lambda l, r: chen_op(l, r, d, n), elems)
    return _time_back(out[0], 1)


def chen_prefix_sequential(levels, M, d, n):
    """Sequential recursion S_t = flow_{M_t}(S_{t-1}) (x) p_t (``ews/core/kernels/pallas_combine.py:1804-1834``)."""
    packed = pack(levels)
    L = packed.shape[-2]
    S = torch.zeros_like(packed[..., 0, :])
    eye = torch.eye(d, dtype=packed.dtype)
    rows = []
    for t in range(L):
        S = chen_op((S, 0.0, eye), (packed[..., t, :], 0.0, M[..., t, :, :]), d, n)[0]
        rows.append(S)
    return torch.stack(rows, dim=-2)


def chen_tree_final(levels, interval_times, M, d, n):
    """Power-of-two pairwise reduction, identity padding (``ews/core/chen_scan.py:244-298``)."""
    packed = _time_first(pack(levels), 1)
    times = _time_first(interval_times, 0)
    Ms = _time_first(M, 2)
    L = packed.shape[0]
    if L > 1:
        target = 1 << int(math.ceil(math.log2(L)))
        if target != L:
            pad = target - L
            packed = torch.cat([packed, torch.zeros((pad,) + packed.shape[1:], dtype=packed.dtype)], 0)
            times = torch.cat([times, torch.zeros((pad,) + times.shape[1:], dtype=times.dtype)], 0)
            eye = torch.eye(d, dtype=Ms.dtype).expand((pad,) + Ms.shape[1:])
            Ms = torch.cat([Ms, eye], 0)
    while packed.shape[0] > 1:
        packed, times, Ms = chen_op((packed[0::2], times[0::2], Ms[0::2]), (packed[1::2], times[1::2], Ms[1::2]), d, n)
    return packed[0]


# -------------------------------------------------------------------------------- the layer

READOUTS = ("terminal", "prefix", "mean", "max")
MODES = ("displacement", "displacement_uniform", "displacement_uniform_basepoint")


def ews_layer(
    path,
    clock,
    A,
    N,
    *,
    leaf="series",
    series_q=None,
    reweighting_mode="displacement",
    readout="prefix",
    terminal_reduce="tree",
    combine="assoc",
    chen_expm="exact",
    a_scale=1.0,
    jordan_chain=None,
):
    """``EWS._single_path`` for exact leaves, broadcast over leading batch axes (``ews/layer.py:154-265``).

    path (..., L, d) knots, clock (..., L), A (d, d). Returns the flat layout with level 0:
    prefix (..., L-1, 1+D), terminal / mean / max (..., 1+D). ``combine``: 'assoc' (the reference's
    associative scan) or 'seq' (the sequential recursion; identical in exact arithmetic).
    """
    if readout not in READOUTS:
        raise ValueError("readout must be 'terminal', 'prefix', 'mean', or 'max'")
    if reweighting_mode not in MODES:
        raise ValueError(f"unknown reweighting_mode {reweighting_mode!r}")
    A = A * a_scale
    d = A.shape[-1]
    interval_times = clock[..., 1:] - clock[..., :-1]
    levels = local_signatures(path, clock, A, N, kind=leaf, series_q=series_q, jordan_chain=jordan_chain)
    cached = reweighting_mode in ("displacement_uniform", "displacement_uniform_basepoint")
    basepoint = reweighting_mode == "displacement_uniform_basepoint"
    if readout == "terminal":
        if terminal_reduce == "tree" and combine == "assoc":
            # the default tree ignores the uniform-clock caching (ews/layer.py:218-220)
            M = chen_M_per_interval(interval_times, A, chen_expm, False, False)
            final = chen_tree_final(levels, interval_times, M, d, N)
        else:
            M = chen_M_per_interval(interval_times, A, chen_expm, cached, basepoint)
            if combine == "seq":
                final = chen_prefix_sequential(levels, M, d, N)[..., -1, :]
            else:
                final = chen_prefix_assoc(levels, interval_times, M, d, N)[..., -1, :]
        one = torch.ones(final.shape[:-1] + (1,), dtype=final.dtype)
        return torch.cat([one, final], dim=-1)
    M = chen_M_per_interval(interval_times, A, chen_expm, cached, basepoint)
    if combine == "seq":
        prefix = chen_prefix_sequential(levels, M, d, N)
    else:
        prefix = chen_prefix_assoc(levels, interval_times, M, d, N)
    one = torch.ones(prefix.shape[:-1] + (1,), dtype=prefix.dtype)
    flat = torch.cat([one, prefix], dim=-1)
    if readout == "mean":
        return flat.mean(dim=-2)
    if readout == "max":
        return flat.max(dim=-2).values
    return flat


def lift(path, B, preserve_first_channel=False):
    """``B.__call__`` (``ews/params.py:1181-1192``): path @ B^T, optionally keeping channel 0."""
    if preserve_first_channel:
        return torch.cat([path[..., :1], path[..., 1:] @ B.T], dim=-1)
    return path @ B.T


# ------------------------------------------------------------------------- log-signature


def lyndon_words(depth, dim):
    """Lyndon words of lengths 1..depth over {0..dim-1}, grouped by length, each group in the
    lexicographic order Duval's algorithm generates (signax 0.2.1 ``utils.lyndon_words``)."""
    groups = [[] for _ in range(depth)]
    w = [-1]
    while w:
        w[-1] += 1
        groups[len(w) - 1].append(tuple(w))
        m = len(w)
        while len(w) < depth:
            w.append(w[len(w) - m])
        while w and w[-1] == dim - 1:
            w.pop()
    return [np.asarray(g, dtype=np.int64).reshape(len(g), k + 1) for k, g in enumerate(groups)]


def witt_dims(dim, depth):
    return [int(w.shape[0]) for w in lyndon_words(depth, dim)]


def tensor_log(levels):
    """Truncated log(1 + X) = sum_{j>=1} (-1)^{j+1} X^{(x) j} / j for a group-like element."""
    n = len(levels)
    zero = [torch.zeros_like(x) for x in levels]

    def mult_nonscalar(X, Y):
        Z = [z.clone() for z in zero]
        for i in range(1, n + 1):
            for j in range(1, n + 1 - i):
                o = X[i - 1][..., :, None] * Y[j - 1][..., None, :]
                Z[i + j - 1] = Z[i + j - 1] + o.reshape(o.shape[:-2] + (o.shape[-2] * o.shape[-1],))
        return Z

    out = [x.clone() for x in levels]
    P = list(levels)
    for j in range(2, n + 1):
        P = mult_nonscalar(P, levels)
        sign = -1.0 if j % 2 == 0 else 1.0
        out = [o + sign * p / j for o, p in zip(out, P)]
    return out


def tensor_exp(ell):
    """Truncated exp of a level list with zero scalar part (``tests/test_log_ews.py:36-58``)."""
    n = len(ell)
    zero = [torch.zeros_like(x) for x in ell]

    def mult_nonscalar(X, Y):
        Z = [z.clone() for z in zero]
        for i in range(1, n + 1):
            for j in range(1, n + 1 - i):
                o = X[i - 1][..., :, None] * Y[j - 1][..., None, :]
                Z[i + j - 1] = Z[i + j - 1] + o.reshape(o.shape[:-2] + (o.shape[-2] * o.shape[-1],))
        return Z

    out = [x.clone() for x in ell]
    P = list(ell)
    for k in range(2, n + 1):
        P = mult_nonscalar(P, ell)
        out = [o + p / math.factorial(k) for o, p in zip(out, P)]
    return out


def compress_log(log_levels, dim):
    """Coefficients of the Lyndon words in the expanded log (the compression of
    signax 0.2.1 ``signature_to_logsignature``): flat (..., sum_k W_d(k))."""
    n = len(log_levels)
    words = lyndon_words(n, dim)
    cols = []
    for k, wk in enumerate(words, start=1):
        flat_idx = np.zeros(wk.shape[0], dtype=np.int64)
        for j in range(k):
            flat_idx = flat_idx * dim + wk[:, j]
        cols.append(log_levels[k - 1][..., torch.as_tensor(flat_idx)])
    return torch.cat(cols, dim=-1)


def log_ews_layer(path, clock, A, N, *, readout="terminal", **kw):
    """``LogEWS._single_path`` (``ews/layer.py:488-517``): log of each EWS element, Lyndon-compressed."""
    d = A.shape[-1]
    if readout == "terminal":
        flat = ews_layer(path, clock, A, N, readout="terminal", **kw)
        return compress_log(tensor_log(unpack(flat[..., 1:], d, N)), d)
    flat = ews_layer(path, clock, A, N, readout="prefix", **kw)
    feat = compress_log(tensor_log(unpack(flat[..., 1:], d, N)), d)
    if readout == "prefix":
        return feat
    if readout == "mean":
        return feat.mean(dim=-2)
    return feat.max(dim=-2).values
