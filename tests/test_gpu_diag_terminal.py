"""The diagonal engine's closed-form terminal readout (uniform clock): S1 = Q1 sum_t r_t,
S2 = diag(Q1) M diag(Q1) + Q2 G with r_t = exp(x (T-1-t)) dy_t, against the float64 oracle (the
reference's Chen recursion) and against the engine's own chunked scan (EWS_F_TERMINAL_SCAN).

Tolerances (written here): global relerr max|a-b| / max|b| <= 1e-5 for the forward and every gradient
against the oracle, with the forward also elementwise |out - ref| <= 1e-6 max(1, max|ref|) + 1e-5 |ref|
for paths up to 512 intervals; against the scan at config-5 length (T = 8192, N = 32, d_in = 16) the
same global 1e-5 for the forward and the gradients.
"""

import numpy as np
import pytest
import torch

from tests.conftest import relerr
from tests.test_gpu_diag import _assert_fwd, _case, _f32, _kernel, _oracle, _require_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("N,d_in,T", [(32, 16, 300), (16, 4, 512), (5, 3, 77), (8, None, 129)])
def test_forward_and_gradients_match_oracle(N, d_in, T):
    _require_gpu()
    path, clock, lam, lift = _case(3, T, N, d_in=d_in, seed=N + T)
    if d_in is None:
        lift = None
    ref, _ = _oracle(path, clock, lam, lift, "terminal")
    w = torch.tensor(np.random.default_rng(9).normal(size=ref.shape))
    _, gref = _oracle(path, clock, lam, lift, "terminal", w=w)
    out, gk = _kernel(path, clock, lam, lift, "terminal", w=w)
    _assert_fwd(out, ref)
    for name, a, b in zip(("path", "lambda", "lift"), gk, gref):
        if b is not None:
            e = relerr(a, b)
            assert e <= 1e-5, f"{name}: relerr {e:.2e}"


def test_fast_decay_and_large_steps():
    """Flows far from the identity (x down to -5 per step): the early intervals' weights underflow to 0."""
    _require_gpu()
    path, clock, lam, lift = _case(2, 200, 16, d_in=4, seed=3, lam_lo=-3.0, lam_hi=1.6, h=1.0)
    ref, _ = _oracle(path, clock, lam, lift, "terminal")
    out, _ = _kernel(path, clock, lam, lift, "terminal")
    _assert_fwd(out, ref)


def _scan_vs_closed(B, T, N, d_in, seed, bf16=False):
    from exponentially_weighted_signature_b200 import _lib, engine, series

    rng = np.random.default_rng(seed)
    inc = torch.tensor(rng.normal(size=(B, T, d_in)) / np.sqrt(T), dtype=torch.float32, device=DEV)
    if bf16:
        inc = inc.to(torch.bfloat16)
    lam = torch.tensor(np.exp(rng.uniform(-4, 0, N)), dtype=torch.float32, device=DEV)
    x = (-lam / T)[None].expand(B, N).contiguous()
    q1, q2 = series.diag_tables(x, 4)
    lift = torch.tensor(rng.normal(size=(N, d_in)) / np.sqrt(d_in), dtype=torch.float32, device=DEV)
    flags = _lib.EWS_F_UNIFORM | _lib.EWS_F_INCREMENTS | (_lib.EWS_F_BF16 if bf16 else 0)
    gw = torch.tensor(rng.normal(size=(B, 1 + N + N * N)), dtype=torch.float32, device=DEV)
    res = []
    for extra in (0, _lib.EWS_F_TERMINAL_SCAN):
        xs, q1s, q2s, ls = (t.detach().clone().requires_grad_(True) for t in (x, q1, q2, lift))
        ii = inc.detach().clone().float().requires_grad_(True) if not bf16 else inc
        out = engine.DiagScan.apply(ii, xs, q1s, q2s, ls, _lib.EWS_READOUT_TERMINAL, flags | extra, 0, True)
        (out * gw).sum().backward()
        torch.cuda.synchronize()
        grads = [xs.grad, q1s.grad, q2s.grad, ls.grad] + ([] if bf16 else [ii.grad])
        res.append([out.detach()] + [g.detach() for g in grads])
    return res


@pytest.mark.parametrize("bf16", [False, True])
def test_closed_form_equals_scan_at_config5_length(bf16):
    _require_gpu()
    closed, scan = _scan_vs_closed(6, 8192, 32, 16, seed=1, bf16=bf16)
    for name, a, b in zip(("out", "x", "q1", "q2", "lift", "increments"), closed, scan):
        e = relerr(a.double().cpu(), b.double().cpu())
        assert e <= 1e-5, f"{name}: relerr {e:.2e}"


def test_small_batch_splits_the_path():
    """B = 2 splits each path into many segments (combined in order in the finishing kernel)."""
    _require_gpu()
    closed, scan = _scan_vs_closed(2, 3000, 12, 5, seed=4)
    for name, a, b in zip(("out", "x", "q1", "q2", "lift", "increments"), closed, scan):
        e = relerr(a.double().cpu(), b.double().cpu())
        assert e <= 1e-5, f"{name}: relerr {e:.2e}"


def test_fused_log_epilogue_matches_the_unfused_one():
    """LogEWS's terminal log-signature from the closed-form kernels with the log / Lyndon epilogue fused
    (EWS_F_LOGSIG) against the same layer's EWS terminal followed by the tensor log and the Lyndon gather
    as separate device ops (ews/layer.py:488-498): forward and every gradient within relerr 1e-5."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from exponentially_weighted_signature_b200 import LogEWS, AParamDiag, logsig

    g = torch.Generator().manual_seed(3)
    B, T, N, d = 4, 300, 32, 16
    inc = (torch.randn(B, T, d, generator=g) / T**0.5).cuda().requires_grad_(True)
    lam = torch.exp(torch.rand(N, generator=g) * 4 - 4)
    lift = (torch.randn(N, d, generator=g) / 4).cuda().requires_grad_(True)
    clock = (torch.arange(T + 1, dtype=torch.float32) / T).expand(B, T + 1).contiguous().cuda()
    layer = LogEWS(AParamDiag(lam).cuda(), 2, reweighting_mode="displacement_uniform", leaf="series", series_q=6)
    assert layer.ewms.fused_logsig_applies(d)
    fused = layer(inc, clock, readout="terminal", lift=lift, increments=True)
    w = torch.randn(fused.shape, generator=g).cuda()
    gf = torch.autograd.grad((fused * w).sum(), [inc, lift, layer.ewms.A_param.values])
    flat = layer.ewms(inc, clock, readout="terminal", lift=lift, increments=True)
    levels = logsig.split_levels(flat[..., 1:], N, 2)
    ref = logsig.compress(logsig.tensor_log(levels), N)
    gr = torch.autograd.grad((ref * w).sum(), [inc, lift, layer.ewms.A_param.values])
    rel = lambda a, b: float((a - b).abs().max() / b.abs().max())  # noqa: E731
    assert rel(fused, ref) <= 1e-5
    for a, b in zip(gf, gr):
        assert rel(a, b) <= 1e-5
