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
