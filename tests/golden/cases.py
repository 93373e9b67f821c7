"""The golden cases: seeded inputs shared by the fixture generator and the tests that read the fixtures.

Each case names the reference layer it runs (``EWS`` or ``LogEWS`` of ews/layer.py with the listed
options), its generator, its inputs and the readouts to record. Inputs are regenerated here from
their seeds (float32, so both sides see identical bits) and checked against the SHA-256 digests the
fixture stores, so a fixture never silently pairs with other inputs.

Generators are the reference's ``A`` (flow ``exp(-dtheta A)``, ews/core/chen_scan.py:155-168); a
configuration written as ``expm(A_cfg dtau)`` has ``A = -A_cfg``.
"""

from __future__ import annotations

import hashlib
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _f32(a):
    return np.asarray(a, dtype=np.float32)


def _bf16_round(a32):
    """Round float32 values to bfloat16 (round to nearest even), returned as float32."""
    u = np.ascontiguousarray(a32, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _brownian_knots(rng, B, T, channels, with_time=True):
    inc = rng.normal(size=(B, T, channels)) / math.sqrt(T)
    knots = np.concatenate([np.zeros((B, 1, channels)), np.cumsum(inc, 1)], 1)
    if with_time:
        t = np.broadcast_to(np.arange(T + 1, dtype=np.float64)[None, :, None] / T, (B, T + 1, 1))
        knots = np.concatenate([knots, t], -1)
    return knots


def _uniform_clock(B, T):
    return np.broadcast_to(np.arange(T + 1, dtype=np.float64) / T, (B, T + 1)).copy()


def _random_clock(rng, B, T):
    steps = rng.uniform(0.2, 1.8, size=(B, T)) / T
    return np.concatenate([np.zeros((B, 1)), np.cumsum(steps, 1)], 1)


def _basepoint_clock(B, T):
    """Interval 0 is a basepoint jump (dtheta = 0), the rest uniform (ews/core/chen_scan.py:160-166)."""
    c = np.zeros((B, T + 1))
    c[:, 1:] = np.arange(T, dtype=np.float64)[None, :] / (T - 1)
    return c


def _diag_generator(prng, N, lo, hi):
    return np.diag(np.exp(prng.uniform(lo, hi, N)))


def _dense_generator(prng, N):
    return 0.5 * np.eye(N) - 0.1 * prng.normal(size=(N, N)) / math.sqrt(N)


def _block_generator(prng, N):
    A = np.zeros((N, N))
    for j in range(N // 2):
        a, w = prng.uniform(0.05, 1.0), prng.uniform(0.0, math.pi)
        A[2 * j : 2 * j + 2, 2 * j : 2 * j + 2] = [[a, w], [-w, a]]
    return A


def _jordan_generator(prng, N, chain):
    """A Jordan-repeated A (the reference's AParamJordanRepeated, ews/params.py:412-460): real chains lam I + Nil,
    lam ~ U(0.2, 2); complex chains of [[a, -b], [b, a]] slots with the 2x2 identity above, a ~ U(0.2, 1.5),
    b ~ U(0, 1.2)."""
    kind, size = chain
    A = np.zeros((N, N))
    for f in range(0, N, size):
        if kind == "real":
            A[f : f + size, f : f + size] = prng.uniform(0.2, 2.0) * np.eye(size) + np.eye(size, k=1)
        else:
            a, b = prng.uniform(0.2, 1.5), prng.uniform(0.0, 1.2)
            k = size // 2
            A[f : f + size, f : f + size] = np.kron(np.eye(k), [[a, -b], [b, a]]) + np.kron(np.eye(k, k=1), np.eye(2))
    return A


def _ar1(rng, B, T, channels, phi):
    x = np.zeros((B, T + 1, channels))
    eps = rng.normal(size=(B, T + 1, channels))
    for t in range(1, T + 1):
        x[:, t] = phi * x[:, t - 1] + eps[:, t]
    return x


def _build(spec):
    """Inputs of a case: knots (B, T+1, d_in), clock (B, T+1), A (N, N), lift (N, d_in), float32 (config 5's
    knots: float64 sums of its float32 increments)."""
    rng = np.random.default_rng(spec["seed"])
    prng = np.random.default_rng(spec["seed"] + 1)
    B, T, N, kind = spec["B"], spec["T"], spec["N"], spec["family"]
    if kind == "c1":  # 3 Brownian channels + time, lift 4 -> N, A = diag(e^u), u ~ U(-3, 1)
        x = _brownian_knots(rng, B, T, 3)
        A = _diag_generator(prng, N, -3.0, 1.0)
        lift = prng.normal(size=(N, 4)) / 2.0
    elif kind == "c2":  # 6 Brownian channels + time, lift 7 -> 32, dense A
        x = _brownian_knots(rng, B, T, 6)
        A = _dense_generator(prng, N)
        lift = prng.normal(size=(N, 7)) / math.sqrt(7)
    elif kind == "c3":  # 4 AR(1) channels (0.9), lift 4 -> 8, 2x2 rotation-decay blocks, softplus clock
        x = _ar1(rng, B, T, 4, 0.9)
        A = _block_generator(prng, N)
        lift = prng.normal(size=(N, 4)) / 2.0
        wc = prng.normal(size=4) / 2.0
        dtau = np.log1p(np.exp(x[:, :-1] @ wc)) / T
        clock = np.concatenate([np.zeros((B, 1)), np.cumsum(dtau, 1)], 1)
    elif kind == "c5":  # 16 channels of N(0, 1/T) increments, lift 16 -> 32, A = diag(e^u), u ~ U(-4, 0)
        inc = rng.standard_normal(size=(B, T, 16)) / math.sqrt(T)
        inc = _f32(inc)
        if spec.get("bf16"):
            inc = _bf16_round(inc)
        x = np.concatenate([np.zeros((B, 1, 16)), np.cumsum(inc.astype(np.float64), 1)], 1)
        A = _diag_generator(prng, N, -4.0, 0.0)
        lift = prng.normal(size=(N, 16)) / 4.0
    elif kind == "jordan":  # 3 Brownian channels + time, lift 4 -> N, Jordan chains, clock of total time 8
        x = _brownian_knots(rng, B, T, 3)
        A = _jordan_generator(prng, N, spec["jordan"])
        lift = prng.normal(size=(N, 4)) / 2.0
        clock = 8.0 * _uniform_clock(B, T)
    else:
        raise ValueError(kind)
    mode = spec["mode"]
    if kind not in ("c3", "jordan"):
        if mode == "displacement_uniform":
            clock = _uniform_clock(B, T)
        elif mode == "displacement_uniform_basepoint":
            clock = _basepoint_clock(B, T)
        else:
            clock = _random_clock(rng, B, T)
    out = dict(x=_f32(x), clock=_f32(clock), A=_f32(A), lift=_f32(lift))
    if kind == "c5":
        # the engines take the float32 (or bf16-rounded) increments themselves; the knots the reference
        # reads are their float64 running sum, so both sides see the same increments
        out["increments"] = inc
        out["x"] = x
    return out


def _rows(T, n=16):
    return np.unique(np.round(np.linspace(0, T - 1, n)).astype(np.int64))


# name -> spec. ``layer``: the reference class; ``kw``: its options; ``readouts``: recorded readouts;
# ``grads``: the readouts whose loss <w, out> gets directional derivatives; ``dirs``: the inputs those
# derivatives move (A moves inside its structure: diagonal, 2x2 blocks, or dense).
CASES = {
    # config 1 family: diagonal generator, depth 2
    "c1_uniform_short": dict(family="c1", seed=10, B=2, T=64, N=16, depth=2, layer="EWS", mode="displacement_uniform",
                             kw=dict(leaf="series", series_q=8), a_struct="diag",
                             readouts=("prefix", "terminal", "mean", "max"), grads=("prefix", "terminal"),
                             dirs=("x", "A", "lift")),
    "c1_clock_short": dict(family="c1", seed=11, B=2, T=64, N=16, depth=2, layer="EWS", mode="displacement",
                           kw=dict(leaf="series", series_q=8), a_struct="diag",
                           readouts=("prefix", "terminal"), grads=("prefix", "terminal"),
                           dirs=("x", "clock", "A", "lift")),
    "c1_basepoint_short": dict(family="c1", seed=12, B=2, T=64, N=16, depth=2, layer="EWS",
                               mode="displacement_uniform_basepoint", kw=dict(leaf="series", series_q=8),
                               a_struct="diag", readouts=("prefix", "terminal"), grads=("prefix",),
                               dirs=("x", "A", "lift")),
    "c1_full": dict(family="c1", seed=13, B=1, T=4096, N=16, depth=2, layer="EWS", mode="displacement_uniform",
                    kw=dict(leaf="series", series_q=8), a_struct="diag", readouts=("prefix", "terminal"),
                    grads=("prefix",), dirs=("x", "A", "lift")),
    "c1_vanloan_short": dict(family="c1", seed=14, B=2, T=64, N=16, depth=2, layer="EWS", mode="displacement_uniform",
                             kw=dict(leaf="van_loan", M=20, van_loan_expm="cayley"), a_struct="diag",
                             readouts=("prefix", "terminal"), grads=("prefix",), dirs=("x", "A", "lift")),
    "c1_vanloan_clock_short": dict(family="c1", seed=15, B=2, T=64, N=16, depth=2, layer="EWS", mode="displacement",
                                   kw=dict(leaf="van_loan", M=20, van_loan_expm="cayley"), a_struct="diag",
                                   readouts=("prefix", "terminal"), grads=("prefix",),
                                   dirs=("x", "clock", "A", "lift")),
    # config 2 family: dense generator, depth 2
    "c2_q3_short": dict(family="c2", seed=20, B=2, T=64, N=32, depth=2, layer="EWS", mode="displacement_uniform",
                        kw=dict(leaf="series", series_q=3), a_struct="dense", readouts=("prefix", "terminal"),
                        grads=("prefix", "terminal"), dirs=("x", "A", "lift")),
    "c2_q4_short": dict(family="c2", seed=21, B=2, T=64, N=32, depth=2, layer="EWS", mode="displacement_uniform",
                        kw=dict(leaf="series", series_q=4), a_struct="dense", readouts=("prefix",),
                        grads=("prefix",), dirs=("x", "A", "lift")),
    "c2_full": dict(family="c2", seed=22, B=1, T=17984, N=32, depth=2, layer="EWS", mode="displacement_uniform",
                    kw=dict(leaf="series", series_q=3), a_struct="dense", readouts=("prefix",), grads=("prefix",),
                    dirs=("x", "A", "lift")),
    "c2_vanloan_short": dict(family="c2", seed=23, B=2, T=64, N=32, depth=2, layer="EWS", mode="displacement_uniform",
                             kw=dict(leaf="van_loan", M=20, van_loan_expm="cayley"), a_struct="dense",
                             readouts=("prefix", "terminal"), grads=("prefix",), dirs=("x", "A", "lift")),
    # config 3 family: 2x2 blocks, depth 3, input-dependent clock
    "c3_short": dict(family="c3", seed=30, B=2, T=64, N=8, depth=3, layer="EWS", mode="displacement",
                     kw=dict(leaf="series", series_q=4), a_struct="block2", readouts=("prefix", "terminal", "mean"),
                     grads=("prefix", "terminal"), dirs=("x", "clock", "A", "lift")),
    "c3_full": dict(family="c3", seed=31, B=1, T=2048, N=8, depth=3, layer="EWS", mode="displacement",
                    kw=dict(leaf="series", series_q=4), a_struct="block2", readouts=("prefix", "terminal"),
                    grads=("prefix",), dirs=("x", "clock", "A", "lift")),
    # config 5 family: LogEWS, diagonal N = 32, terminal readout, increments
    "c5_short": dict(family="c5", seed=50, B=2, T=128, N=32, depth=2, layer="LogEWS", mode="displacement_uniform",
                     kw=dict(leaf="series", series_q=4), a_struct="diag", readouts=("terminal", "prefix"),
                     grads=("terminal",), dirs=("x", "A", "lift")),
    "c5_full": dict(family="c5", seed=51, B=1, T=8192, N=32, depth=2, layer="LogEWS", mode="displacement_uniform",
                    kw=dict(leaf="series", series_q=4), a_struct="diag", readouts=("terminal",), grads=("terminal",),
                    dirs=("x", "A", "lift")),
    # Jordan chains (AParamJordanRepeated), depth 2, uniform clock: the closed-form Jordan leaf
    "jordan_real2_short": dict(family="jordan", seed=60, B=2, T=64, N=8, depth=2, layer="EWS",
                               mode="displacement_uniform", jordan=("real", 2), kw=dict(leaf="jordan_closed_tables"),
                               a_struct="jordan", readouts=("prefix", "terminal"), grads=("prefix",),
                               dirs=("x", "A", "lift")),
    "jordan_real3_short": dict(family="jordan", seed=61, B=2, T=64, N=9, depth=2, layer="EWS",
                               mode="displacement_uniform", jordan=("real", 3), kw=dict(leaf="jordan_closed"),
                               a_struct="jordan", readouts=("prefix", "terminal"), grads=("prefix",),
                               dirs=("x", "A", "lift")),
    "jordan_complex4_short": dict(family="jordan", seed=62, B=2, T=64, N=8, depth=2, layer="EWS",
                                  mode="displacement_uniform", jordan=("complex", 4),
                                  kw=dict(leaf="jordan_closed_tables"), a_struct="jordan",
                                  readouts=("prefix", "terminal"), grads=("prefix",), dirs=("x", "A", "lift")),
    "c5_bf16_full": dict(family="c5", seed=51, B=1, T=8192, N=32, depth=2, layer="LogEWS", mode="displacement_uniform",
                         bf16=True, kw=dict(leaf="series", series_q=4), a_struct="diag", readouts=("terminal",),
                         grads=(), dirs=()),
}


def case_inputs(name):
    return _build(CASES[name])


def prefix_rows(name):
    return _rows(CASES[name]["T"])


def weights(shape, salt=0.0):
    """The loss cotangent w of a readout output: a fixed formula (no RNG), so every machine builds the same w."""
    idx = np.indices(shape).astype(np.float64)
    arg = 0.3 * salt
    for k, ax in enumerate(idx):
        arg = arg + (0.7 + 1.2 * k) * ax
    return np.cos(arg)


def directions(name):
    """Seeded perturbation directions for the directional derivatives (float64)."""
    spec = CASES[name]
    inp = case_inputs(name)
    rng = np.random.default_rng(1000 + spec["seed"])
    B, T, N = spec["B"], spec["T"], spec["N"]
    d_in = inp["x"].shape[-1]
    out = {}
    if spec["family"] == "c5":
        out["x"] = rng.normal(size=(B, T, d_in)) / math.sqrt(T)  # over the increments
    else:
        out["x"] = rng.normal(size=(B, T + 1, d_in)) * float(np.std(inp["x"]))
    steps = np.diff(inp["clock"].astype(np.float64), axis=1)
    out["clock"] = np.concatenate([np.zeros((B, 1)), np.cumsum(rng.uniform(-0.5, 0.5, (B, T)) * steps, 1)], 1)
    S = rng.normal(size=(N, N))
    if spec["a_struct"] == "diag":
        S = np.diag(np.diag(S))
    elif spec["a_struct"] == "block2":
        mask = np.kron(np.eye(N // 2), np.ones((2, 2)))
        S = S * mask
    elif spec["a_struct"] == "jordan":  # within the family: each chain's eigenvalue (and frequency)
        kind, size = spec["jordan"]
        S = np.zeros((N, N))
        for f in range(0, N, size):
            if kind == "real":
                S[f : f + size, f : f + size] = rng.normal() * np.eye(size)
            else:
                da, db = rng.normal(size=2)
                S[f : f + size, f : f + size] = np.kron(np.eye(size // 2), [[da, -db], [db, da]])
    out["A"] = S * float(np.max(np.abs(inp["A"])))
    out["lift"] = rng.normal(size=inp["lift"].shape) * float(np.std(inp["lift"]))
    return out


def fixture_path(name):
    return os.path.join(HERE, f"{name}.npz")


def load_fixture(name):
    """Loads a fixture and regenerates its inputs, checking their digests."""
    fx = dict(np.load(fixture_path(name), allow_pickle=False))
    inp = case_inputs(name)
    for k, v in inp.items():
        key = f"sha_{k}"
        if key in fx and str(fx[key]) != sha(v):
            raise AssertionError(f"golden {name}: regenerated input {k!r} differs from the one the fixture was made from")
    return fx, inp


def jordan_params(A, chain):
    """(block_sizes, block_kinds, block_params) of an AParamJordanRepeated that materialises A (ews/params.py:412-460):
    the softplus inverse of each chain's eigenvalue (real) or real part (complex, with the frequency b)."""
    kind, size = chain
    N = A.shape[0]
    sizes, kinds, ps = [], [], []
    for f in range(0, N, size):
        v = float(np.log(np.expm1(float(A[f, f]))))
        sizes.append(size)
        kinds.append(kind)
        ps.append(np.array([v]) if kind == "real" else np.array([v, float(A[f + 1, f])]))
    return sizes, kinds, ps
