"""The token-cached scan (ews/core/token_scan.py:55-118) on the engines against the REFERENCE's own outputs:
tests/golden/token_*.npz were written by tests/golden/make_token_golden.py from the reference's unmodified
build_token_cache + token_cached_prefix_scan (float64, numpy stand-ins). Tolerances as for the other golden
tests: relative error <= 1e-5 for the prefixes, and for the loss's directional derivatives along the
vocabulary displacements, the clock increments and A, <= 1e-5 of sum|grad_i v_i|."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import token_cases as tc  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _load(name):
    fx = dict(np.load(tc.fixture_path(name), allow_pickle=False))
    inp = tc.case_inputs(name)
    for k, v in inp.items():
        assert str(fx[f"sha_{k}"]) == tc.sha(v), f"{name}: input {k} differs from the fixture's"
    return fx, inp


@pytest.mark.parametrize("name", list(tc.CASES))
def test_token_cached_prefix_matches_reference(name):
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from exponentially_weighted_signature_b200 import EWS, AParamBlockDiag, AParamDiag
    from exponentially_weighted_signature_b200.token_scan import token_cached_prefix

    spec = tc.CASES[name]
    fx, inp = _load(name)
    A = torch.tensor(inp["A"])
    d = spec["d"]
    if spec["a"] == "diag":
        Ap = AParamDiag(torch.diagonal(A).clone())
    else:
        Ap = AParamBlockDiag([A[2 * k : 2 * k + 2, 2 * k : 2 * k + 2].clone() for k in range(d // 2)], (2,) * (d // 2))
    layer = EWS(Ap, spec["N"], reweighting_mode="displacement", leaf=spec["leaf"], series_q=spec["series_q"]).cuda()
    vdx = torch.tensor(inp["vdx"], device="cuda", requires_grad=True)
    vdt = torch.tensor(inp["vdt"], device="cuda", requires_grad=True)
    tok = torch.tensor(inp["tok"], device="cuda")
    mask = torch.tensor(inp["mask"], device="cuda")
    out = token_cached_prefix(layer, tok, vdx, vdt, mask)
    ref = fx["out"]
    got = out.detach().double().cpu().numpy()
    assert got.shape == ref.shape
    assert float(np.max(np.abs(got - ref)) / np.max(np.abs(ref))) <= TOL
    dirs = tc.directions(name)
    for b in range(spec["B"]):
        w = torch.tensor(tc.weights(ref.shape[1:], salt=b), dtype=torch.float32, device="cuda")
        layer.zero_grad()
        vdx.grad = None
        vdt.grad = None
        loss = (out[b] * w).sum()
        loss.backward(retain_graph=True)
        if spec["a"] == "diag":
            gA = torch.diag(layer.A_param.values.grad).double().cpu().numpy()
        else:
            gA = torch.block_diag(*[blk.grad for blk in layer.A_param.blocks]).double().cpu().numpy()
        grads = {"vdx": vdx.grad.double().cpu().numpy(), "vdt": vdt.grad.double().cpu().numpy(), "A": gA}
        for k, v in dirs.items():
            proj = float((grads[k] * v).sum())
            mag = float(np.abs(grads[k] * v).sum())
            assert abs(proj - float(fx[f"dd_{k}"][b])) <= TOL * mag + 1e-12, (name, b, k, proj, float(fx[f"dd_{k}"][b]))
