"""Writes the token-cached scan's golden fixtures from the REFERENCE's own code (test infrastructure).

    python tests/golden/make_token_golden.py --ref PATH_TO_REFERENCE_CHECKOUT

Runs the reference's unmodified ews/core/token_scan.py (build_token_cache + token_cached_prefix_scan,
ews/core/token_scan.py:55-118) on the numpy stand-ins of refshim/ in float64, per sample of each case in
token_cases.py, and records the prefixes (L, sum_k d^k), the loss <w, prefixes> and its directional
derivatives along seeded directions of the vocabulary displacements, the clock increments and A (fourth-order
central differences of the reference's forward).
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import token_cases as tc  # noqa: E402

EPS = 1e-3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("EWS_REFERENCE_ROOT"))
    args = ap.parse_args()
    import refimport

    refimport.import_reference(args.ref)
    import ews.core.token_scan as ts

    def forward(spec, inp, b, vdx, vdt, A):
        P, D = ts.build_token_cache(vdx, vdt, A, 20, spec["N"], "exact", "exact", spec["leaf"], spec["series_q"])
        return np.asarray(ts.token_cached_prefix_scan(inp["tok"][b], inp["mask"][b], P, D, spec["d"], spec["N"]))

    for name, spec in tc.CASES.items():
        inp = tc.case_inputs(name)
        dirs = tc.directions(name)
        base = dict(vdx=inp["vdx"].astype(np.float64), vdt=inp["vdt"].astype(np.float64), A=inp["A"].astype(np.float64))
        fx = {f"sha_{k}": np.asarray(tc.sha(v)) for k, v in inp.items()}
        outs, losses, dds = [], [], {k: [] for k in dirs}
        for b in range(spec["B"]):
            out = forward(spec, inp, b, base["vdx"], base["vdt"], base["A"])
            w = tc.weights(out.shape, salt=b)
            outs.append(out)
            losses.append(float(np.sum(w * out)))
            for k, v in dirs.items():
                vals = {}
                for s in (-2, -1, 1, 2):
                    pert = dict(base)
                    pert[k] = base[k] + s * EPS * v
                    vals[s] = float(np.sum(w * forward(spec, inp, b, pert["vdx"], pert["vdt"], pert["A"])))
                dds[k].append((8.0 * (vals[1] - vals[-1]) - (vals[2] - vals[-2])) / (12.0 * EPS))
        fx["out"] = np.stack(outs)
        fx["loss"] = np.asarray(losses)
        for k in dirs:
            fx[f"dd_{k}"] = np.asarray(dds[k])
        np.savez_compressed(tc.fixture_path(name), **fx)
        print(f"wrote {tc.fixture_path(name)}")


if __name__ == "__main__":
    main()
