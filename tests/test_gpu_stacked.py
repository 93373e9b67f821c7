"""A StackedEWS training step on the B200 engines against the same model with the CPU oracle's EWS.

The model mirrors the reference's block scaffold for config 4 (ews/block.py: pre-norm EWSBlocks with
the token-gated learned clock, diagonal generators, a Linear encoder and a per-position head). The twin
is a float64 CPU copy whose EWS layers are replaced by the oracle (ews/layer.py:154-265 restated in
oracle/ews_oracle.py) on the same parameters. Dropout is off.

Tolerance (written here): the loss and every parameter gradient within relative error
max|a-b|/max|b| <= 2e-5 (the EWS layer's own bound is 1e-5; the float32 scaffold around it, norms and
Linear layers, adds its rounding).
"""

import copy

import pytest
import torch
from torch import nn

from oracle import ews_oracle as O
from tests.conftest import relerr

pytestmark = pytest.mark.gpu


class _OracleEWS(nn.Module):
    def __init__(self, a_param, q):
        super().__init__()
        self.A_param = a_param
        self.q = q

    def forward(self, path, clock, readout="prefix", output_format="flat"):
        A = torch.diag(self.A_param.values)
        return O.ews_layer(path, clock, A, 2, leaf="series", series_q=self.q, reweighting_mode="displacement", readout=readout)


def _build(seed=0, blocks=2, H=16, m=4, T=24, B=2, q=6):
    from exponentially_weighted_signature_b200.block import StackedEWS

    torch.manual_seed(seed)
    model = StackedEWS(blocks, 5, H, 5, block_kwargs=dict(m=m, n=2, series_q=q, clock_norm_constant=float(T),
                                                          dropout_rate=0.0), seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    X = torch.randn(B, T, 5, generator=g)
    Y = torch.randn(B, T, 5, generator=g)
    return model, X, Y


def test_stacked_training_step_matches_oracle():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    model, X, Y = _build()
    twin = copy.deepcopy(model).double()
    for blk in twin.blocks:
        blk.ewms = _OracleEWS(blk.ewms.A_param, blk.ewms.series_q)
    model = model.cuda()
    loss = nn.functional.mse_loss(model(X.cuda()), Y.cuda())
    loss.backward()
    ref = nn.functional.mse_loss(twin(X.double()), Y.double())
    ref.backward()
    assert abs(float(loss) - float(ref)) <= 2e-5 * abs(float(ref))
    got = dict(model.named_parameters())
    for name, p in twin.named_parameters():
        assert p.grad is not None, name
        e = relerr(got[name].grad.double().cpu(), p.grad)
        assert e <= 2e-5, f"{name}: relerr {e:.2e}"


def test_stacked_adam_step_runs_and_lowers_the_loss():
    """A few Adam steps on a fixed batch: the full training step (forward, backward, optimizer) runs on
    the engines and the loss goes down."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    model, X, Y = _build(seed=3, blocks=2, H=32, m=8, T=64, B=4)
    model = model.cuda()
    X, Y = X.cuda(), Y.cuda()
    opt = torch.optim.Adam(model.parameters(), lr=3e-3)
    losses = []
    for _ in range(20):
        opt.zero_grad(set_to_none=True)
        loss = nn.functional.mse_loss(model(X), Y)
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("d,N,eps", [(16, 2, 1e-3), (4, 3, 1e-2), (7, 2, 0.5)])
def test_graded_norm_kernel_matches_torch(d, N, eps):
    """ews_graded_norm_fwd / _bwd (the block's level-0 drop, zero-row prepend and live-RMS graded norm in one
    pass each way, ews/block.py:282-306, ews/norms.py:47-135) against the same steps as torch ops in float64:
    relative error <= 1e-5 for the output, the input gradient and the gain gradients, including rows whose
    level is all zero (RMS 0: the output is 0 and the gradient g / eps)."""
    import numpy as np

    from exponentially_weighted_signature_b200.block import GradedRMSNorm

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    g = torch.Generator().manual_seed(d * 10 + N)
    B, L = 3, 37
    D = sum(d**k for k in range(1, N + 1))
    flat = torch.randn(B, L, 1 + D, generator=g) * torch.logspace(-3, 1, 1 + D)[None, None, :]
    flat[0, 5, 1 : 1 + d] = 0.0  # an all-zero level 1
    flat[1, 7, 1 + d :] = 0.0    # all-zero higher levels
    norm = GradedRMSNorm(d, N, eps=eps)
    with torch.no_grad():
        norm.gains.copy_(torch.linspace(0.5, 1.5, N))
    w = torch.randn(B, L + 1, D, generator=g)

    f64 = flat.double().requires_grad_(True)
    ref_norm = GradedRMSNorm(d, N, eps=eps).double()
    with torch.no_grad():
        ref_norm.gains.copy_(norm.gains.double())
    ref = ref_norm.from_prefix(f64)
    (ref * w.double()).sum().backward()

    norm = norm.cuda()
    fc = flat.cuda().requires_grad_(True)
    out = norm.from_prefix(fc)
    (out * w.cuda()).sum().backward()
    torch.cuda.synchronize()

    def rel(a, b):
        a, b = a.detach().double().cpu().numpy(), b.detach().double().cpu().numpy()
        return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-300))

    assert out.shape == (B, L + 1, D)
    assert float(out[:, 0].abs().max()) == 0.0
    assert rel(out, ref) <= 1e-5
    assert rel(fc.grad, f64.grad) <= 1e-5
    assert float(fc.grad[..., 0].abs().max()) == 0.0
    assert rel(norm.gains.grad, ref_norm.gains.grad) <= 1e-5


@pytest.mark.parametrize("B,L,H,s,c", [(3, 1441, 128, 1.0, 1440.0), (2, 3000, 21, 3.5, 7.0), (1, 2, 5, 1.0, 1.0)])
def test_gated_clock_kernel_matches_torch(B, L, H, s, c):
    """ews_gated_clock_fwd / _bwd (the block's token-gated clock, ews/clocks.py:409-466, one library pass each
    way) against the same steps as torch ops in float64: relative error <= 1e-5 for theta and for the
    gradients of the driver, the gate weights and the bias (the sequence spans several 1024-step tiles)."""
    import numpy as np

    from exponentially_weighted_signature_b200.block import TokenGatedClock

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    g = torch.Generator().manual_seed(B * 7 + L)
    clk = TokenGatedClock(H, init_bias=0.05, norm_constant=c, in_scale=s, generator=g)
    x = torch.cumsum(torch.randn(B, L, H, generator=g) * 0.3, 1)
    wt = torch.randn(B, L, generator=g)
    ref_clk = TokenGatedClock(H, init_bias=0.05, norm_constant=c, in_scale=s, generator=g).double()
    with torch.no_grad():
        ref_clk.w.copy_(clk.w.double())
        ref_clk.b.copy_(clk.b.double())
    x64 = x.double().requires_grad_(True)
    ref = ref_clk(x64)  # CPU tensors: the torch steps
    (ref * wt.double()).sum().backward()

    clk = clk.cuda()
    xc = x.cuda().requires_grad_(True)
    out = clk(xc)
    (out * wt.cuda()).sum().backward()
    torch.cuda.synchronize()

    def rel(a, b):
        a, b = a.detach().double().cpu().numpy(), b.detach().double().cpu().numpy()
        return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-300))

    assert out.shape == (B, L) and float(out[:, 0].abs().max()) == 0.0
    assert rel(out, ref) <= 1e-5
    assert rel(xc.grad, x64.grad) <= 1e-5
    assert rel(clk.w.grad, ref_clk.w.grad) <= 1e-5
    assert abs(float(clk.b.grad) - float(ref_clk.b.grad)) <= 1e-5 * max(1.0, abs(float(ref_clk.b.grad)))
