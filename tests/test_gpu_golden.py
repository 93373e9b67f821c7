"""The CUDA engines against the REFERENCE's own outputs (tests/golden/, written by make_golden.py from the
reference's unmodified ews/layer.py and ews/core in float64), through the layer on the GPU.

Every golden case whose leaf and generator structure the engines implement runs here at its stored
size, including the full-length configurations (config 1 T = 4096, config 2 T = 17984, config 3
T = 2048, config 5 T = 8192). Tolerances (float32 engines against the float64 reference):

* outputs: global relative error max|a - b| / max|b| <= 1e-5 over the recorded rows of every readout,
  and the loss <w, out> over the whole output within 1e-5 relative to sum|w out|;
* gradients: for every recorded direction v (knots, clock, generator inside its structure, lift),
  |<grad, v> - reference directional derivative| <= 1e-5 sum|grad_i v_i|;
* bf16 increments (config 5's variant): the reference evaluated on the bf16-rounded increments, with
  the same 1e-5 (the rounding of the input is the variant's only difference).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import cases  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-5

# cases the engines do not run yet: (name -> reason); they stay pinned on the CPU oracle side
UNSUPPORTED = {}


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _jordan_matrix_param(A, chain):
    """An AParamJordanRepeated (so the layer sees the chains) that materialises the given matrix itself, so that
    the gradient is the full dL/dA the fixtures' directions are projected on."""
    from exponentially_weighted_signature_b200 import AParamJordanRepeated

    class JordanMatrix(AParamJordanRepeated):
        def forward(self):
            return self.matrix

    kind, size = chain
    K = A.shape[0] // size
    ap = JordanMatrix([size] * K, [kind] * K, [torch.zeros(1 if kind == "real" else 2)] * K)
    ap.matrix = torch.nn.Parameter(A.clone())
    return ap


def _model(name, inp):
    from exponentially_weighted_signature_b200 import EWS, LogEWS, AParamBlockDiag, AParamDiag, AParamGeneral

    spec = cases.CASES[name]
    A = torch.tensor(inp["A"], dtype=torch.float32)
    N = A.shape[0]
    if spec["a_struct"] == "jordan":
        Ap = _jordan_matrix_param(A, spec["jordan"])
    elif spec["a_struct"] == "diag":
        Ap = AParamDiag(torch.diagonal(A).clone())
    elif spec["a_struct"] == "block2":
        Ap = AParamBlockDiag([A[2 * k : 2 * k + 2, 2 * k : 2 * k + 2].clone() for k in range(N // 2)], (2,) * (N // 2))
    else:
        Ap = AParamGeneral(A.clone())
    cls = LogEWS if spec["layer"] == "LogEWS" else EWS
    return cls(Ap, spec["depth"], reweighting_mode=spec["mode"], **spec["kw"]).to(DEV)


def _a_grad(spec, model, N):
    ap = model.ewms.A_param if hasattr(model, "ewms") else model.A_param
    if spec["a_struct"] == "diag":
        return torch.diag(ap.values.grad).double().cpu().numpy()
    if spec["a_struct"] == "block2":
        return torch.block_diag(*[b.grad for b in ap.blocks]).double().cpu().numpy()
    return ap.matrix.grad.double().cpu().numpy()


def _run(name, readout, with_grad):
    spec = cases.CASES[name]
    fx, inp = cases.load_fixture(name)
    model = _model(name, inp)
    lift = torch.tensor(inp["lift"], device=DEV, requires_grad=with_grad)
    clock = torch.tensor(inp["clock"], device=DEV, requires_grad=with_grad and "clock" in spec["dirs"])
    if spec["family"] == "c5":
        x = torch.tensor(inp["increments"], device=DEV)
        if spec.get("bf16"):
            x = x.to(torch.bfloat16)
        x.requires_grad_(with_grad)
        out = model(x, clock, readout=readout, lift=lift, increments=True)
    else:
        x = torch.tensor(inp["x"], device=DEV, requires_grad=with_grad)
        out = model(x, clock, readout=readout, lift=lift)
    grads = None
    if with_grad:
        w = torch.tensor(np.stack([cases.weights(tuple(out.shape[1:]), salt=b) for b in range(spec["B"])]),
                         dtype=torch.float32, device=DEV)
        out.backward(w)
        grads = {"x": x.grad, "clock": clock.grad, "lift": lift.grad}
        grads = {k: (None if v is None else v.double().cpu().numpy()) for k, v in grads.items()}
        grads["A"] = _a_grad(spec, model, inp["A"].shape[0])
    torch.cuda.synchronize()
    return fx, out.detach().double().cpu().numpy(), grads


def _relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-300))


def _params():
    out = []
    for name, spec in cases.CASES.items():
        for r in spec["readouts"]:
            out.append(pytest.param(name, r, id=f"{name}-{r}"))
    return out


@pytest.mark.parametrize("name,readout", _params())
def test_engine_matches_reference(name, readout):
    _require_gpu()
    if name in UNSUPPORTED:
        pytest.skip(f"not on the engines: {UNSUPPORTED[name]}")
    spec = cases.CASES[name]
    with_grad = readout in spec["grads"]
    fx, out, grads = _run(name, readout, with_grad)
    assert np.isfinite(out).all()
    ref = fx[f"out_{readout}"]
    got = out[:, fx["rows"]] if readout == "prefix" else out
    assert _relerr(got, ref) <= TOL, (name, readout, _relerr(got, ref))
    for b in range(spec["B"]):
        w = cases.weights(out.shape[1:], salt=b)
        loss = float((w * out[b]).sum())
        assert abs(loss - fx[f"loss_{readout}"][b]) <= TOL * float(np.abs(w * out[b]).sum()), (name, b)
    if not with_grad:
        return
    dirs = cases.directions(name)
    for d in spec["dirs"]:
        g = grads[d]
        if d in ("x", "clock"):  # per-sample inputs: one directional derivative per sample
            for b in range(spec["B"]):
                proj = float((g[b] * dirs[d][b]).sum())
                mag = float(np.abs(g[b] * dirs[d][b]).sum())
                ref_dd = float(fx[f"dd_{readout}_{d}"][b])
                assert abs(proj - ref_dd) <= TOL * mag + 1e-12, (name, readout, d, b, proj, ref_dd, mag)
        else:  # shared parameters: the batch's loss is the sum of the samples' losses
            proj = float((g * dirs[d]).sum())
            mag = float(np.abs(g * dirs[d]).sum())
            ref_dd = float(np.sum(fx[f"dd_{readout}_{d}"]))
            assert abs(proj - ref_dd) <= TOL * mag + 1e-12, (name, readout, d, proj, ref_dd, mag)
