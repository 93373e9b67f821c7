"""Writes the golden fixtures ``tests/golden/<case>.npz`` from the REFERENCE's own code.

Test infrastructure, run once in the development container where the reference checkout exists:

    python tests/golden/make_golden.py --ref PATH_TO_REFERENCE_CHECKOUT [case ...]

The reference (alexandre-bloch/exponentially-weighted-signature) is JAX; jax, equinox and signax
cannot be installed on these machines. Its modules are imported unmodified (``refimport.py``) on the
numpy stand-ins of ``refshim/`` and evaluated in float64: the layer ``EWS`` / ``LogEWS`` of
ews/layer.py:43-302 / :440-556 with the case's options and ``combine="lean"`` (the same Chen
operator on precomputed flows, ews/core/kernels/combine.py:260-269); for the short cases the
associative-scan engine ``combine="assoc"`` (ews/core/chen_scan.py:172-214) is run too and must
agree to 1e-10. The lift is ``path @ B^T`` (ews/params.py:1181-1192).

Recorded per case and sample: the outputs of every readout (prefix rows at fixed indices), the loss
``<w, out>`` with the formula cotangent ``cases.weights``, and directional derivatives of that loss
along seeded directions of the knots, clock, generator and lift, by a fourth-order central
difference of the reference's forward (jax's autodiff is not available; the stencil's error is far
below the tests' tolerances). Inputs are not stored: ``cases.py`` regenerates them and the fixture
keeps their SHA-256 digests.
"""

from __future__ import annotations

import argparse
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

import cases  # noqa: E402

EPS = 1e-3
_REF = None


def _init(ref_root):
    global _REF
    import refimport

    _REF = refimport.import_reference(ref_root)


def _forward(name, b, readout, x, clock, A, lift, combine="lean"):
    """Reference output of one sample, float64."""
    spec = cases.CASES[name]
    layer_mod, params_mod = _REF
    cls = layer_mod.LogEWS if spec["layer"] == "LogEWS" else layer_mod.EWS
    A_arg = np.asarray(A, np.float64)
    if "jordan" in spec:  # the Jordan leaf reads its chains from the parametrisation's class
        A_arg = params_mod.AParamJordanRepeated(*cases.jordan_params(A_arg, spec["jordan"]))
    m = cls(A_arg, spec["depth"], dtype=np.float64, reweighting_mode=spec["mode"],
            combine=combine, **spec["kw"])
    lifted = np.asarray(x, np.float64) @ np.asarray(lift, np.float64).T
    return np.asarray(m(lifted, np.asarray(clock, np.float64), readout=readout), np.float64)


def _loss(name, b, readout, out):
    return float(np.sum(cases.weights(out.shape, salt=b) * out))


def _perturbed(name, b, d, s):
    spec = cases.CASES[name]
    inp = cases.case_inputs(name)
    x = inp["x"][b].astype(np.float64)
    clock = inp["clock"][b].astype(np.float64)
    A = inp["A"].astype(np.float64)
    lift = inp["lift"].astype(np.float64)
    if d is None:
        return x, clock, A, lift
    v = cases.directions(name)[d]
    if d == "x":
        vb = v[b]
        if spec["family"] == "c5":
            vb = np.concatenate([np.zeros((1, vb.shape[1])), np.cumsum(vb, 0)], 0)
        x = x + s * EPS * vb
    elif d == "clock":
        clock = clock + s * EPS * v[b]
    elif d == "A":
        A = A + s * EPS * v
    elif d == "lift":
        lift = lift + s * EPS * v
    return x, clock, A, lift


def _task(args):
    kind, name, b, readout, d, s = args
    x, clock, A, lift = _perturbed(name, b, d, s)
    if kind == "out":
        t0 = time.time()
        out = _forward(name, b, readout, x, clock, A, lift, "lean")
        extra = None
        if cases.CASES[name]["T"] <= 256:
            extra = float(np.max(np.abs(_forward(name, b, readout, x, clock, A, lift, "assoc") - out)))
        return args, out, extra, time.time() - t0
    out = _forward(name, b, readout, x, clock, A, lift, "lean")
    return args, _loss(name, b, readout, out), None, 0.0


def _tasks(name):
    spec = cases.CASES[name]
    out = []
    for b in range(spec["B"]):
        for r in spec["readouts"]:
            out.append(("out", name, b, r, None, 0))
        for r in spec["grads"]:
            for d in spec["dirs"]:
                for s in (-2, -1, 1, 2):
                    out.append(("dd", name, b, r, d, s))
    return out


def _write(name, results):
    spec = cases.CASES[name]
    inp = cases.case_inputs(name)
    fx = {f"sha_{k}": np.asarray(cases.sha(v)) for k, v in inp.items()}
    fx["rows"] = cases.prefix_rows(name)
    for r in spec["readouts"]:
        outs = [results[("out", name, b, r, None, 0)][0] for b in range(spec["B"])]
        if r == "prefix":
            fx["out_prefix"] = np.stack([o[fx["rows"]] for o in outs])
            fx["prefix_shape"] = np.asarray(outs[0].shape)
        else:
            fx[f"out_{r}"] = np.stack(outs)
        fx[f"loss_{r}"] = np.asarray([_loss(name, b, r, o) for b, o in enumerate(outs)])
        ex = [results[("out", name, b, r, None, 0)][1] for b in range(spec["B"])]
        if ex[0] is not None:
            # The associative engine agrees with "lean" except where its default terminal tree
            # (terminal_reduce="tree", ews/layer.py:217-220) takes one exponential per interval while
            # "lean" shares the uniform clock's flow: clock knots rounded to float32 are uniform only to
            # ~1e-8, so those two differ at that level. Recorded, and required below 1e-6 relative.
            fx[f"assoc_vs_lean_{r}"] = np.asarray(max(ex))
            limit = (1e-6 if r == "terminal" else 1e-10) * max(1.0, float(np.max(np.abs(np.stack(outs)))))
            assert max(ex) < limit, (name, r, ex)
    for r in spec["grads"]:
        for d in spec["dirs"]:
            dd = []
            for b in range(spec["B"]):
                g = {s: results[("dd", name, b, r, d, s)][0] for s in (-2, -1, 1, 2)}
                dd.append((8.0 * (g[1] - g[-1]) - (g[2] - g[-2])) / (12.0 * EPS))
            fx[f"dd_{r}_{d}"] = np.asarray(dd)
    np.savez_compressed(cases.fixture_path(name), **fx)
    print(f"wrote {cases.fixture_path(name)} ({os.path.getsize(cases.fixture_path(name)) // 1024} KiB)", flush=True)


def make(names, ref_root, procs):
    ctx = mp.get_context("spawn")
    t0 = time.time()
    with ctx.Pool(procs, initializer=_init, initargs=(ref_root,)) as pool:
        for name in names:
            results = {}
            for args, val, extra, dt in pool.imap_unordered(_task, _tasks(name)):
                results[args] = (val, extra)
                if args[0] == "out":
                    print(f"  {args[1]} b={args[2]} {args[3]}: {dt:.1f}s"
                          + (f" assoc-lean {extra:.2e}" if extra is not None else ""), flush=True)
            _write(name, results)
    print(f"done in {time.time() - t0:.0f}s")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("EWS_REFERENCE_ROOT"), required="EWS_REFERENCE_ROOT" not in os.environ)
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("names", nargs="*")
    args = ap.parse_args()
    names = args.names or list(cases.CASES)
    make(names, args.ref, args.procs)


if __name__ == "__main__":
    main()
