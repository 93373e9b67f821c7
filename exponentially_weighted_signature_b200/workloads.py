"""Seeded synthetic inputs of the benchmark configurations (no dataset is involved in any of them).

Generators are given as the reference calls them: a configuration written as expm(A_cfg dtau) with
A_cfg = -diag(exp(u)) becomes the reference generator A = -A_cfg = diag(exp(u)) (its flow is
exp(-dtheta A), ews/core/chen_scan.py:155-168). Data seed 0, parameter seed 1.
"""

from __future__ import annotations

import math

import numpy as np


def _brownian(rng, B, T, channels):
    inc = rng.normal(size=(B, T, channels)) / math.sqrt(T)
    return inc


def _knots_with_time(inc, T):
    B = inc.shape[0]
    time = np.broadcast_to(np.arange(T + 1, dtype=np.float64)[None, :, None] / T, (B, T + 1, 1))
    knots = np.concatenate([np.zeros((B, 1, inc.shape[2])), np.cumsum(inc, 1)], 1)
    return np.concatenate([knots, time], -1)


def uniform_clock(B, T):
    return np.broadcast_to(np.arange(T + 1, dtype=np.float64) / T, (B, T + 1)).copy()


def config1(seed=0, B=4, T=4096):
    """Single EWS layer, depth 2: 3 Brownian channels + time (d=4), lift 4 -> 16 ~ N(0, 1/4),
    A = diag(e^u), u ~ U(-3, 1), uniform clock dtau = 1/T, prefix readout."""
    rng = np.random.default_rng(seed)
    prng = np.random.default_rng(seed + 1)
    path = _knots_with_time(_brownian(rng, B, T, 3), T)
    lam = np.exp(prng.uniform(-3.0, 1.0, 16))
    lift = prng.normal(size=(16, 4)) / math.sqrt(4)
    return dict(name="config1", path=path, clock=uniform_clock(B, T), lam=lam, lift=lift, B=B, T=T, N=16, depth=2)


def config2(seed=0, B=32, T=17984):
    """Dense A, N=32, depth 2: 6 Brownian channels + time (d=7), lift 7 -> 32 ~ N(0, 1/7),
    A = 0.5 I - 0.1 G / sqrt(32), G ~ N(0, 1), uniform clock, prefix readout."""
    rng = np.random.default_rng(seed)
    prng = np.random.default_rng(seed + 1)
    path = _knots_with_time(_brownian(rng, B, T, 6), T)
    A = 0.5 * np.eye(32) - 0.1 * prng.normal(size=(32, 32)) / math.sqrt(32)
    lift = prng.normal(size=(32, 7)) / math.sqrt(7)
    return dict(name="config2", path=path, clock=uniform_clock(B, T), A=A, lift=lift, B=B, T=T, N=32, depth=2)


def config3(seed=0, B=64, T=2048):
    """2x2 rotation-decay blocks, N=8, depth 3: 4 AR(1) channels (0.9, unit noise), lift 4 -> 8 ~ N(0, 1/4),
    A blocks [[a, w], [-w, a]] (a ~ U(0.05, 1), w ~ U(0, pi)), clock steps softplus(w_c . x_t)/T with
    w_c ~ N(0, 1/4), prefix readout."""
    rng = np.random.default_rng(seed)
    prng = np.random.default_rng(seed + 1)
    x = np.zeros((B, T + 1, 4))
    eps = rng.normal(size=(B, T + 1, 4))
    for t in range(1, T + 1):
        x[:, t] = 0.9 * x[:, t - 1] + eps[:, t]
    A = np.zeros((8, 8))
    for j in range(4):
        a, w = prng.uniform(0.05, 1.0), prng.uniform(0.0, math.pi)
        A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = [[a, w], [-w, a]]
    lift = prng.normal(size=(8, 4)) / math.sqrt(4)
    wc = prng.normal(size=4) / 2.0
    dtau = np.log1p(np.exp(x[:, :-1] @ wc)) / T
    clock = np.concatenate([np.zeros((B, 1)), np.cumsum(dtau, 1)], 1)
    return dict(name="config3", path=x, clock=clock, A=A, lift=lift, B=B, T=T, N=8, depth=3)


def config4(seed=0, B=128, T=1440):
    """StackedEWS training data: 21 channels of Gaussian AR(1) with coefficient 0.95 and unit-variance noise;
    the model reads positions 0..T-1 and predicts the next value of every channel (MSE)."""
    rng = np.random.default_rng(seed)
    x = np.zeros((B, T + 1, 21), dtype=np.float64)
    eps = rng.normal(size=(B, T + 1, 21))
    for t in range(1, T + 1):
        x[:, t] = 0.95 * x[:, t - 1] + eps[:, t]
    return dict(name="config4", inputs=x[:, :T].astype(np.float32), targets=x[:, 1:].astype(np.float32),
                B=B, T=T, N=16, depth=2, hidden=128, blocks=4)


def config5(seed=0, B=1024, T=8192):
    """LogEWS depth 2, diagonal N=32, A = diag(e^u), u ~ U(-4, 0): 16 channels of i.i.d. N(0, 1/T)
    increments (stored as increments), lift 16 -> 32 ~ N(0, 1/16), uniform clock, terminal readout."""
    rng = np.random.default_rng(seed)
    prng = np.random.default_rng(seed + 1)
    inc = (rng.standard_normal(size=(B, T, 16), dtype=np.float32) / np.float32(math.sqrt(T))).astype(np.float32)
    lam = np.exp(prng.uniform(-4.0, 0.0, 32))
    lift = prng.normal(size=(32, 16)) / 4.0
    return dict(name="config5", increments=inc, clock=uniform_clock(B, T), lam=lam, lift=lift, B=B, T=T, N=32, depth=2)
