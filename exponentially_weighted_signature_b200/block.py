"""The reference's residual block and stack around the EWS layer (ews/block.py, ews/norms.py,
ews/clocks.py), for the configuration the hot path's config 4 uses: the callers of the EWS call,
kept here so that a full training step runs on the B200 engines.

Built: ``EWSBlock`` with norm_placement="pre" (RMSNorm -> clock -> lift -> EWS prefix -> GradedRMSNorm
-> c_down -> dropout -> residual -> RMSNorm -> MLP channel stage -> dropout -> residual,
ews/block.py:376-424), path_mode="value", the "token_gated" clock on the block input
(ews/clocks.py:409-466), no appended clock, no basepoint; ``StackedEWS`` with a Linear encoder and a
per-position (seq2seq) head (ews/block.py:473-600). Other scaffold options raise NotImplementedError.
The EWS layer inside each block is this package's ``EWS`` (the diagonal engine's per-interval clock
mode for the "displacement" reweighting).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from .layer import EWS
from .params import AParamDiag, B


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight over the last axis (ews/norms.py:13-27)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = float(eps)
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + self.eps) * self.weight


class GradedRMSNorm(nn.Module):
    """Per-level live RMS normalisation of a level-0-free flat feature [lvl1 | ... | lvlN]
    (ews/norms.py:47-135, variant "live_rms"): g_k * block / (RMS_k + eps_k), exactly zero (value and
    gradient) for an all-zero level."""

    def __init__(self, d: int, N: int, eps: float = 1e-3):
        super().__init__()
        self.d, self.N = int(d), int(N)
        self.eps = [float(eps)] * self.N
        self.gains = nn.Parameter(torch.ones(self.N))
        self.slices = []
        start = 0
        for k in range(1, self.N + 1):
            self.slices.append((start, start + self.d**k))
            start += self.d**k

    def from_prefix(self, flat):
        """The norm of the block's mixer levels straight from the EWS prefix rows flat (B, L, 1 + D): level 0
        dropped, a zero row prepended (ews/block.py:282-306), then this norm. On CUDA one library pass each
        way (engine.GradedNorm); elsewhere the same steps as torch ops."""
        if flat.is_cuda:
            from .engine import GradedNorm

            return GradedNorm.apply(flat, self.gains, self.d, self.N, tuple(self.eps))
        levels = flat[..., 1:]
        return self(torch.cat([torch.zeros_like(levels[:, :1]), levels], 1))

    def forward(self, x):
        out = []
        for k, (s, e) in enumerate(self.slices):
            block = x[..., s:e]
            ms = (block * block).mean(-1, keepdim=True)
            safe = torch.where(ms > 0, ms, torch.ones_like(ms))
            rms = torch.where(ms > 0, torch.sqrt(safe), torch.zeros_like(ms))
            out.append(self.gains[k] * block / (rms + self.eps[k]))
        return torch.cat(out, -1)


class TokenGatedClock(nn.Module):
    """theta = [0, cumsum(relu(diff(driver * in_scale) @ w - b))] / norm_constant
    (ews/clocks.py:409-466, mode "token_gated", no mask)."""

    def __init__(self, dim: int, init_bias: float = 0.0, init_scale: Optional[float] = None,
                 norm_constant: float = 1.0, in_scale: float = 1.0, generator=None):
        super().__init__()
        gs = float(dim) ** -0.5 if init_scale is None else float(init_scale)
        self.w = nn.Parameter(gs * torch.randn(int(dim), generator=generator))
        self.b = nn.Parameter(torch.tensor(float(init_bias)))
        self.norm_constant = float(norm_constant)
        self.in_scale = float(in_scale)

    def forward(self, driver):
        if driver.is_cuda and driver.dim() == 3:  # one library pass each way (engine.GatedClock)
            from .engine import GatedClock

            return GatedClock.apply(driver, self.w, self.b, self.in_scale, self.norm_constant)
        dx = torch.diff(driver * self.in_scale, dim=-2)
        incr = F.relu(dx @ self.w - self.b)
        V = torch.cat([torch.zeros_like(incr[..., :1]), torch.cumsum(incr, -1)], -1)
        return V / self.norm_constant


class EWSBlock(nn.Module):
    """Pre-norm residual block around an EWS mixer (ews/block.py:36-470), batched (B, L, H)."""

    def __init__(self, hidden_dim: int, m: int = 8, n: int = 2, *, lam: Optional[torch.Tensor] = None,
                 series_q: int = 8, clock_norm_constant: float = 1.0, clock_init_bias: float = 0.0,
                 graded_eps: float = 1e-3, ff_mult: int = 4, dropout_rate: float = 0.01, norm_eps: float = 1e-6,
                 norm_placement: str = "pre", channel_stage: str = "mlp", path_mode: str = "value",
                 combine_chunk: int = 0, generator=None):
        super().__init__()
        if norm_placement != "pre" or channel_stage != "mlp" or path_mode != "value":
            raise NotImplementedError("this block mirrors norm_placement='pre', channel_stage='mlp', path_mode='value'")
        H = int(hidden_dim)
        self.hidden_dim, self.m, self.n = H, int(m), int(n)
        g = generator
        if lam is None:
            lam = torch.exp(torch.rand(self.m, generator=g) * 4.0 - 3.0)
        self.lift = B(torch.randn(self.m, H, generator=g) / math.sqrt(H), preserve_first_channel=False)
        self.ewms = EWS(AParamDiag(lam.to(torch.float32)), N=self.n, reweighting_mode="displacement",
                        leaf="series", series_q=series_q, combine="b200", combine_chunk=combine_chunk)
        D = sum(self.m**k for k in range(1, self.n + 1))
        self.D = D
        self.graded = GradedRMSNorm(self.m, self.n, eps=graded_eps)
        self.c_down = nn.Linear(D, H)
        self.norm1 = RMSNorm(H, eps=norm_eps)
        self.norm2 = RMSNorm(H, eps=norm_eps)
        self.ff1 = nn.Linear(H, ff_mult * H)
        self.ff2 = nn.Linear(ff_mult * H, H)
        self.drop = nn.Dropout(dropout_rate)
        self.clock = TokenGatedClock(H, init_bias=clock_init_bias, norm_constant=clock_norm_constant, generator=g)

    def mixer_levels(self, branch_in, theta):
        """EWS prefix of (theta, B(branch_in)), level 0 dropped and a zero row prepended
        (ews/block.py:282-306): (B, L, D)."""
        p = self.lift(branch_in)
        flat = self.ewms(p, theta, readout="prefix", output_format="flat")
        levels = flat[..., 1:]
        return torch.cat([torch.zeros_like(levels[:, :1]), levels], 1)

    def forward(self, x):
        theta = self.clock(x)  # the block-input driver
        branch_in = self.norm1(x)
        flat = self.ewms(self.lift(branch_in), theta, readout="prefix", output_format="flat")
        r = self.c_down(self.graded.from_prefix(flat))  # = c_down(graded(mixer_levels(branch_in, theta)))
        x = x + self.drop(r)
        mch = self.ff2(F.gelu(self.ff1(self.norm2(x))))
        return x + self.drop(mch)


class StackedEWS(nn.Module):
    """Linear encoder, ``num_blocks`` EWSBlocks and a per-position head (ews/block.py:473-600,
    tokens=False, head_mode="seq2seq")."""

    def __init__(self, num_blocks: int, data_dim: int, hidden_dim: int, label_dim: int, *,
                 block_kwargs: Optional[dict] = None, seed: int = 0):
        super().__init__()
        g = torch.Generator().manual_seed(int(seed))
        self.embedding = nn.Linear(data_dim, hidden_dim)
        kw = dict(block_kwargs or {})
        self.blocks = nn.ModuleList([EWSBlock(hidden_dim, generator=g, **kw) for _ in range(int(num_blocks))])
        self.head = nn.Linear(hidden_dim, label_dim)

    def hidden(self, X):
        h = self.embedding(X)
        for block in self.blocks:
            h = block(h)
        return h

    def forward(self, X):
        return self.head(self.hidden(X))
