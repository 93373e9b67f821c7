"""Seeded inputs of the token-cached scan's golden cases (shared by make_token_golden.py and the tests).

A case is a vocabulary of per-token displacements (already lifted) and clock increments, a generator A,
and a batch of token sequences with a padding mask (ews/core/token_scan.py:55-118, ews/block.py:787-803).
Inputs are float32 (both sides see identical values); the fixture stores their SHA-256 digests.
"""

from __future__ import annotations

import hashlib
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _inputs(spec):
    rng = np.random.default_rng(spec["seed"])
    V, d, L, B = spec["V"], spec["d"], spec["L"], spec["B"]
    vdx = rng.normal(size=(V, d)) * 0.3
    vdt = rng.uniform(0.005, 0.05, size=V)
    if spec["a"] == "diag":
        A = np.diag(np.exp(rng.uniform(-2.0, 1.5, d)))
    else:  # 2x2 rotation-decay blocks
        A = np.zeros((d, d))
        for j in range(d // 2):
            a, w = rng.uniform(0.05, 1.0), rng.uniform(0.0, math.pi)
            A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = [[a, w], [-w, a]]
    tok = rng.integers(0, V, size=(B, L))
    mask = np.ones((B, L), dtype=bool)
    mask[1, L - 5 :] = False  # a padded tail
    f32 = lambda x: np.asarray(x, dtype=np.float32)
    return dict(vdx=f32(vdx), vdt=f32(vdt), A=f32(A), tok=tok.astype(np.int64), mask=mask)


CASES = {
    "token_diag_series": dict(seed=70, V=11, d=8, L=96, B=2, N=2, a="diag", leaf="series", series_q=8),
    "token_block_series": dict(seed=71, V=9, d=4, L=64, B=2, N=3, a="block2", leaf="series", series_q=6),
}


def case_inputs(name):
    return _inputs(CASES[name])


def directions(name):
    spec = CASES[name]
    inp = case_inputs(name)
    rng = np.random.default_rng(1000 + spec["seed"])
    out = {"vdx": rng.normal(size=inp["vdx"].shape) * 0.3, "vdt": rng.normal(size=inp["vdt"].shape) * 0.01}
    S = rng.normal(size=inp["A"].shape)
    if spec["a"] == "diag":
        S = np.diag(np.diag(S))
    else:
        S = S * np.kron(np.eye(spec["d"] // 2), np.ones((2, 2)))
    out["A"] = S
    return out


def weights(shape, salt=0.0):
    idx = np.indices(shape).astype(np.float64)
    arg = 0.3 * salt
    for k, ax in enumerate(idx):
        arg = arg + (0.7 + 1.2 * k) * ax
    return np.cos(arg)


def fixture_path(name):
    return os.path.join(HERE, f"{name}.npz")
