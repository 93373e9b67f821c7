"""Pins the CPU oracle to the REFERENCE's own outputs (the fixtures of tests/golden/).

The fixtures were written by tests/golden/make_golden.py, which runs the reference's unmodified
ews/layer.py and ews/core modules (float64, on numpy stand-ins for jax / equinox / signax). Here the
oracle (oracle/ews_oracle.py, float64 torch) evaluates the same inputs and must agree:

* outputs: max|oracle - reference| <= 1e-10 max(1, max|reference|) (both float64; the rest is the
  order of the sums);
* gradients: for every recorded direction v, <grad oracle, v> against the reference's directional
  derivative (a fourth-order central difference of its forward) within 1e-7 of sum|grad_i v_i|.

Cases whose leaf the oracle does not restate are only checked for presence.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from oracle import ews_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import cases  # noqa: E402

ORACLE_LEAVES = ("series", "block_series", "plane_closed", "jordan_closed", "jordan_closed_tables")
# full-length cases the oracle finishes in seconds on the CPU; the others are checked on the GPU only
CPU_CASES = [n for n, s in cases.CASES.items() if s["T"] <= 256 or n in ("c1_full", "c3_full")]


def oracle_forward(name, b, readout, inp, requires_grad=False):
    """The oracle's evaluation of one sample of a golden case: returns (out, leaf tensors)."""
    spec = cases.CASES[name]
    f64 = torch.float64
    if spec["family"] == "c5":
        inc = torch.tensor(inp["increments"][b], dtype=f64, requires_grad=requires_grad)
        x = torch.cat([torch.zeros((1, inc.shape[1]), dtype=f64), torch.cumsum(inc, 0)], 0)
        leaf_x = inc
    else:
        x = torch.tensor(inp["x"][b], dtype=f64, requires_grad=requires_grad)
        leaf_x = x
    clock = torch.tensor(inp["clock"][b], dtype=f64, requires_grad=requires_grad)
    A = torch.tensor(inp["A"], dtype=f64, requires_grad=requires_grad)
    lift = torch.tensor(inp["lift"], dtype=f64, requires_grad=requires_grad)
    kw = dict(spec["kw"])
    path = O.lift(x, lift)
    fn = O.log_ews_layer if spec["layer"] == "LogEWS" else O.ews_layer
    out = fn(path, clock, A, spec["depth"], readout=readout, reweighting_mode=spec["mode"],
             leaf=kw.get("leaf", "series"), series_q=kw.get("series_q"), combine="assoc", terminal_reduce="assoc",
             **({"jordan_chain": spec["jordan"]} if "jordan" in spec else {}))
    return out, dict(x=leaf_x, clock=clock, A=A, lift=lift)


def _have(name):
    return os.path.exists(cases.fixture_path(name))


def test_every_case_has_a_fixture():
    missing = [n for n in cases.CASES if not _have(n)]
    assert not missing, f"golden fixtures missing: {missing} (run tests/golden/make_golden.py)"


@pytest.mark.parametrize("name", list(cases.CASES))
def test_fixture_inputs_regenerate(name):
    """The seeded inputs rebuild bit for bit (their digests match the ones the fixture was made from)."""
    fx, inp = cases.load_fixture(name)
    for k in inp:
        assert f"sha_{k}" in fx


@pytest.mark.parametrize("name", CPU_CASES)
def test_oracle_matches_reference(name):
    spec = cases.CASES[name]
    if spec["kw"].get("leaf", "series") not in ORACLE_LEAVES:
        pytest.skip(f"leaf {spec['kw']['leaf']!r}: checked on the device engines")
    fx, inp = cases.load_fixture(name)
    for b in range(spec["B"]):
        for r in spec["readouts"]:
            out, leaves = oracle_forward(name, b, r, inp, requires_grad=r in spec["grads"])
            ref = fx[f"out_{r}"][b]
            got = out.detach().numpy()
            if r == "prefix":
                got = got[fx["rows"]]
            scale = max(1.0, float(np.max(np.abs(ref))))
            assert np.max(np.abs(got - ref)) <= 1e-10 * scale, (name, b, r, float(np.max(np.abs(got - ref))))
            if r not in spec["grads"]:
                continue
            w = torch.tensor(cases.weights(tuple(out.shape), salt=b))
            loss = (out * w).sum()
            assert abs(float(loss) - fx[f"loss_{r}"][b]) <= 1e-10 * max(1.0, abs(fx[f"loss_{r}"][b]))
            dirs = cases.directions(name)
            grads = torch.autograd.grad(loss, [leaves[d] for d in spec["dirs"]])
            for d, g in zip(spec["dirs"], grads):
                v = dirs[d][b] if d in ("x", "clock") else dirs[d]
                proj = float((g.numpy() * v).sum())
                mag = float(np.abs(g.numpy() * v).sum())
                ref_dd = float(fx[f"dd_{r}_{d}"][b])
                assert abs(proj - ref_dd) <= 1e-7 * mag + 1e-12, (name, b, r, d, proj, ref_dd, mag)


def test_token_cached_scan_is_the_gathered_per_interval_scan():
    """The reference's token-cached scan (ews/core/token_scan.py:55-118, fixtures tests/golden/token_*.npz) equals
    the oracle's per-interval-clock scan of the gathered path (segment t: the token's displacement and clock
    step; padded steps: zero and zero), which is how token_scan.token_cached_prefix runs it on the engines."""
    import token_cases as tc

    for name, spec in tc.CASES.items():
        fx = dict(np.load(tc.fixture_path(name), allow_pickle=False))
        inp = tc.case_inputs(name)
        for k, v in inp.items():
            assert str(fx[f"sha_{k}"]) == tc.sha(v)
        for b in range(spec["B"]):
            m = inp["mask"][b].astype(np.float64)
            dx = inp["vdx"].astype(np.float64)[inp["tok"][b]] * m[:, None]
            dth = inp["vdt"].astype(np.float64)[inp["tok"][b]] * m
            path = torch.tensor(np.concatenate([np.zeros((1, dx.shape[1])), np.cumsum(dx, 0)], 0))
            clock = torch.tensor(np.concatenate([[0.0], np.cumsum(dth)]))
            out = O.ews_layer(path, clock, torch.tensor(inp["A"], dtype=torch.float64), spec["N"], leaf=spec["leaf"],
                              series_q=spec["series_q"], reweighting_mode="displacement", readout="prefix")
            got = out[..., 1:].numpy()
            ref = fx["out"][b]
            assert np.max(np.abs(got - ref)) <= 1e-10 * max(1.0, float(np.max(np.abs(ref)))), name
