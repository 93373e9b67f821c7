"""Generator parametrisations and the lift, mirroring the reference's classes (ews/params.py).

Only what the hot path needs: materialising A (``A_param()``), and the structure probes the engine
dispatch reads (``block_sizes_of`` / ``diag_values``), as in ews/core/kernels/combine.py:37-63.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F
from torch import nn


class AParamConstant(nn.Module):
    """A fixed (or learnable) dense matrix (ews/params.py:244-253)."""

    def __init__(self, matrix: torch.Tensor, learnable: bool = True):
        super().__init__()
        if learnable:
            self.matrix = nn.Parameter(torch.as_tensor(matrix))
        else:
            self.register_buffer("matrix", torch.as_tensor(matrix))
        self.dim = int(self.matrix.shape[0])

    def forward(self) -> torch.Tensor:
        return self.matrix


class AParamGeneral(AParamConstant):
    """Unconstrained dense generator (ews/params.py:268-277)."""


class AParamDiag(nn.Module):
    """Free diagonal generator A = diag(values): the reference's AParamBlockDiag with sizes (1,)*N
    (docs/params.md: "sizes 1 give a free diagonal")."""

    def __init__(self, values: torch.Tensor):
        super().__init__()
        self.values = nn.Parameter(torch.as_tensor(values))
        self.dim = int(self.values.shape[0])

    def diag_values(self) -> torch.Tensor:
        return self.values

    def forward(self) -> torch.Tensor:
        return torch.diag(self.values)


class AParamEFM(nn.Module):
    """Positive diagonal softplus(theta) or theta**2 (ews/params.py:280-301)."""

    def __init__(self, theta: torch.Tensor, positivity: str = "softplus"):
        super().__init__()
        if positivity not in ("softplus", "square"):
            raise ValueError(f"efm positivity must be one of ('softplus', 'square'), got {positivity!r}")
        self.theta = nn.Parameter(torch.as_tensor(theta))
        self.positivity = positivity
        self.dim = int(self.theta.shape[0])

    def diag_values(self) -> torch.Tensor:
        if self.positivity == "square":
            return self.theta**2
        return F.softplus(self.theta)

    def forward(self) -> torch.Tensor:
        return torch.diag(self.diag_values())


class AParamBlockDiag(nn.Module):
    """Block-diagonal generator from free blocks (ews/params.py:394-409)."""

    def __init__(self, blocks: Sequence[torch.Tensor], sizes: Sequence[int]):
        super().__init__()
        self.blocks = nn.ParameterList([nn.Parameter(torch.as_tensor(b)) for b in blocks])
        self.sizes = tuple(int(s) for s in sizes)
        self.dim = int(sum(self.sizes))

    def diag_values(self) -> torch.Tensor:
        if any(s != 1 for s in self.sizes):
            raise ValueError("diag_values needs blocks of size 1")
        return torch.stack([b.reshape(()) for b in self.blocks])

    def forward(self) -> torch.Tensor:
        return torch.block_diag(*self.blocks)


class AParamJordanRepeated(nn.Module):
    """Block-diagonal generator of Jordan blocks, one eigenvalue repeated down each block
    (ews/params.py:412-460): a real block of size n is lam = softplus(v) on the diagonal with ones
    directly above; a complex block of size 2k is R = [[a, -b], [b, a]] (a = softplus(v), b free) in
    every diagonal slot with the 2x2 identity above. ``block_params[j]`` holds (v,) for a real block
    and (v, b) for a complex one."""

    def __init__(self, block_sizes: Sequence[int], block_kinds: Sequence[str], block_params: Sequence[torch.Tensor]):
        super().__init__()
        self.block_sizes = tuple(int(x) for x in block_sizes)
        self.block_kinds = tuple(str(x) for x in block_kinds)
        for size, kind in zip(self.block_sizes, self.block_kinds):
            if kind not in ("real", "complex"):
                raise ValueError(f"Unknown Jordan block kind '{kind}'")
            if kind == "real" and size < 2:
                raise ValueError("a real Jordan block needs size >= 2 for the eigenvalue to repeat; "
                                 "size 1 is a plain diagonal entry")
            if kind == "complex" and (size % 2 != 0 or size < 4):
                raise ValueError(f"a complex Jordan block needs an even size >= 4, got {size}")
        self.block_params = nn.ParameterList([nn.Parameter(torch.as_tensor(p).reshape(-1)) for p in block_params])
        self.dim = int(sum(self.block_sizes))

    def forward(self) -> torch.Tensor:
        blocks = []
        for size, kind, p in zip(self.block_sizes, self.block_kinds, self.block_params):
            if kind == "real":
                lam = F.softplus(p[0])
                eye = torch.eye(size, dtype=p.dtype, device=p.device)
                blocks.append(lam * eye + torch.diag(torch.ones(size - 1, dtype=p.dtype, device=p.device), 1))
            else:
                k = size // 2
                a, b = F.softplus(p[0]), p[1]
                R = torch.stack([torch.stack([a, -b]), torch.stack([b, a])])
                shift = torch.diag(torch.ones(k - 1, dtype=p.dtype, device=p.device), 1)
                blocks.append(torch.kron(torch.eye(k, dtype=p.dtype, device=p.device), R)
                              + torch.kron(shift, torch.eye(2, dtype=p.dtype, device=p.device)))
        if not blocks:
            return torch.zeros((0, 0))
        return torch.block_diag(*blocks)


JORDAN_REAL_SIZES, JORDAN_COMPLEX_SIZES = (2, 3, 4), (4, 6, 8)


def jordan_chains_of(a_param) -> Optional[tuple]:
    """(kind, size) when A is an AParamJordanRepeated whose blocks all have one supported kind and size
    (real 2-4, complex 4 / 6 / 8), else None (ews/core/kernels/jordan_engine.py:29-43)."""
    if not isinstance(a_param, AParamJordanRepeated) or not a_param.block_sizes:
        return None
    sizes, kinds = set(a_param.block_sizes), set(a_param.block_kinds)
    if len(sizes) != 1 or len(kinds) != 1:
        return None
    kind, size = kinds.pop(), int(sizes.pop())
    if size not in (JORDAN_REAL_SIZES if kind == "real" else JORDAN_COMPLEX_SIZES):
        return None
    return kind, size


def block_sizes_of(a_param) -> Optional[tuple]:
    """Block structure of a parametrisation, decided from its class (ews/core/kernels/combine.py:37-58)."""
    if isinstance(a_param, AParamBlockDiag):
        return a_param.sizes
    if isinstance(a_param, AParamJordanRepeated):
        return a_param.block_sizes
    if isinstance(a_param, (AParamDiag, AParamEFM)):
        return (1,) * a_param.dim
    return None


def is_diagonal(a_param) -> bool:
    sizes = block_sizes_of(a_param)
    return sizes is not None and all(s == 1 for s in sizes)


class B(nn.Module):
    """Learnable linear lift path @ matrix^T, optionally keeping channel 0 (ews/params.py:1166-1192)."""

    def __init__(self, matrix: torch.Tensor, preserve_first_channel: bool = True):
        super().__init__()
        self.matrix = nn.Parameter(torch.as_tensor(matrix))
        self.preserve_first_channel = bool(preserve_first_channel)

    def full_matrix(self) -> torch.Tensor:
        """The lift as one (out, in) matrix: [[1, 0], [0, matrix]] when channel 0 is preserved."""
        if not self.preserve_first_channel:
            return self.matrix
        w, d = self.matrix.shape
        top = torch.zeros((1, d + 1), dtype=self.matrix.dtype, device=self.matrix.device)
        top[0, 0] = 1.0
        bottom = torch.cat([torch.zeros((w, 1), dtype=self.matrix.dtype, device=self.matrix.device), self.matrix], 1)
        return torch.cat([top, bottom], 0)

    def forward(self, path: torch.Tensor) -> torch.Tensor:
        if self.preserve_first_channel:
            if path.shape[-1] < 2:
                raise ValueError("preserve_first_channel=True requires path with at least 2 channels")
            return torch.cat([path[..., :1], path[..., 1:] @ self.matrix.T], dim=-1)
        return path @ self.matrix.T
