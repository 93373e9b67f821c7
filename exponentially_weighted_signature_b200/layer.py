"""The EWS layer on the B200 engines: same constructor and call as the reference's ews/layer.py.

``EWS(A, N, ...)`` keeps the reference's options, defaults and validation (ews/layer.py:82-152) and
its call ``layer(path, clock, return_terminal, output_format, readout, a_scale)`` (ews/layer.py:267-302),
with the flat output layout [1, level 1, ..., level N] (ews/core/output_format.py:12-30). Every
``combine`` kind selects the CUDA engines: the kinds are implementations of one scan with the same
result (ews/core/kernels/combine.py:1-14), so "assoc" (the default), "lean", "block_kernel",
"dense_kernel" and "b200" all run here; ``combine_chunk`` sets the engines' chunk length only with
``combine="b200"`` (the other kinds' chunk targets belong to the reference's Pallas kernels). A leaf or
generator structure the engines do not implement raises ``NotImplementedError``; there is no CPU
fallback.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from . import _lib, engine, logsig, series
from .params import AParamConstant, B, block_sizes_of, is_diagonal, jordan_chains_of

COMBINE_KINDS = ("assoc", "lean", "block_kernel", "dense_kernel", "b200")
LEAF_KINDS = ("van_loan", "series", "plane_closed", "block_series", "jordan_closed", "jordan_closed_tables")
JORDAN_LEAVES = ("jordan_closed", "jordan_closed_tables")
MODES = ("displacement", "displacement_uniform", "displacement_uniform_basepoint")

_DETERMINISTIC = False
# Extra EWS_F_* bits OR-ed into every engine call (failure-detection tests set EWS_F_TEST_WITHHOLD here).
_EXTRA_FLAGS = 0


def configure(deterministic: bool = False, check_status: bool = False) -> None:
    """``deterministic``: bit-reproducible engine results (the counterpart of the reference's XLA
    determinism switch, ews/determinism.py:32-106): chunks then wait for their neighbour's inclusive
    carry instead of folding in whatever aggregates are ready, which fixes the rounding of the carries.

    ``check_status``: synchronise after every engine call and raise ``EWSLookbackTimeout`` at once if a
    device-side wait ran out. By default the status is collected without synchronising and an error
    is raised by the next engine call on the device (or when a backward finishes)."""
    global _DETERMINISTIC
    _DETERMINISTIC = bool(deterministic)
    engine.CHECK_SYNC = bool(check_status)


def _det_flags() -> int:
    return (_lib.EWS_F_DETERMINISTIC if _DETERMINISTIC else 0) | _EXTRA_FLAGS


READOUTS = ("terminal", "prefix", "mean", "max")
VANLOAN_DEGREE = 8


def _normalize_expm_method(method: str) -> str:
    method = method.lower()
    if method in {"pade_lite", "pade-lite"}:
        return "pade"
    if method not in {"exact", "euler", "cayley", "pade"}:
        raise ValueError("expm method must be one of 'exact', 'euler', 'cayley', 'pade'")
    return method


class EWS(nn.Module):
    """Exponentially weighted signature layer on the B200 engines.

    Engine dispatch follows A's structure (ews/core/kernels/combine.py:37-63): a diagonal
    parametrisation runs the diagonal engine, 2x2 blocks at depth 3 the block engine, anything else at
    depth 2 the dense engine. Leaves: ``"series"`` at order ``series_q`` on every engine
    (``"block_series"`` is accepted for diagonal A, where both leaves agree to the series truncation);
    ``"van_loan"`` (the reference's default, M knots per interval, ews/core/van_loan.py:91-160) on the
    diagonal and dense engines; the closed-form leaves ``"plane_closed"`` and ``"jordan_closed"`` /
    ``"jordan_closed_tables"`` (an ``AParamJordanRepeated`` A with uniform chains) on the dense engine, as
    the series leaf's limit for the generator they read from A (uniform clock, ``||h A|| <= 0.5``).
    """

    def __init__(
        self,
        A,
        N: int,
        M: int = 20,
        dtype: torch.dtype = torch.float32,
        reweighting_mode: str = "displacement",
        terminal_reduce: str = "tree",
        van_loan_expm: str = "cayley",
        chen_expm: str = "exact",
        leaf: str = "van_loan",
        series_q: Optional[int] = None,
        combine: str = "assoc",
        combine_chunk: int = 1024,
        combine_tile: int = 4,
        jordan_flows: bool = False,
    ):
        super().__init__()
        self.A_param = A if isinstance(A, nn.Module) else AParamConstant(torch.as_tensor(A, dtype=dtype))
        self.d = int(self.A_param.dim)
        self.N = int(N)
        self.M = int(M)
        self.dtype = dtype
        if reweighting_mode not in MODES:
            raise ValueError(f"reweighting_mode must be one of {MODES}, got {reweighting_mode!r}")
        self.reweighting_mode = reweighting_mode
        if terminal_reduce not in {"tree", "assoc"}:
            raise ValueError("terminal_reduce must be 'tree' or 'assoc'")
        self.terminal_reduce = terminal_reduce
        self.van_loan_expm = _normalize_expm_method(van_loan_expm)
        self.chen_expm = _normalize_expm_method(chen_expm)
        if leaf not in LEAF_KINDS:
            raise ValueError(f"leaf must be one of {LEAF_KINDS}, got {leaf!r}")
        if leaf == "series" and series_q is None:
            raise ValueError("leaf='series' requires series_q (see ews.core.leaf.check_series_q)")
        if combine not in COMBINE_KINDS:
            raise ValueError(f"combine must be one of {COMBINE_KINDS}, got {combine!r}")
        if leaf == "block_series" and N == 2 and series_q is None:
            raise ValueError("leaf='block_series' at depth 2 requires series_q")
        if leaf == "plane_closed":
            if N > 2:
                raise NotImplementedError("leaf='plane_closed': closed-form local terms exist for depths 1 and 2")
            if self.d % 2:
                raise ValueError("leaf='plane_closed' needs an even dimension (2x2 planes)")
        self._jordan_chain = jordan_chains_of(self.A_param)
        if leaf in JORDAN_LEAVES:
            if self._jordan_chain is None:
                raise ValueError(
                    f"leaf={leaf!r} needs a jordan_repeated A with uniform chains (every block the same kind and size: "
                    "real 2-4 or complex 4, 6, 8); use leaf='series' or 'block_series' otherwise"
                )
            if N > 2:
                raise NotImplementedError(f"leaf={leaf!r}: closed-form local terms exist for depths 1 and 2")
        if leaf not in ("series", "block_series", "van_loan", "plane_closed") + JORDAN_LEAVES:
            raise NotImplementedError(
                f"leaf={leaf!r} is not built on the B200 engines; use leaf='series' (or 'van_loan' for a diagonal A)"
            )
        self.leaf = leaf
        self.series_q = None if series_q is None else int(series_q)
        self.combine = combine
        self.combine_chunk = int(combine_chunk)
        # the chunk length the engines get (0: the library's choice)
        self._chunk = self.combine_chunk if combine == "b200" else 0
        self.combine_tile = int(combine_tile)
        self.block_sizes = block_sizes_of(self.A_param)
        if leaf == "block_series" and self.block_sizes is None:
            raise ValueError("leaf='block_series' needs a block-diagonal A parametrisation")
        if jordan_flows and (combine != "block_kernel" or self._jordan_chain is None):
            raise ValueError("jordan_flows needs combine='block_kernel' and a jordan_repeated A with uniform chains")
        # The closed-form chain flows (ews/core/kernels/combine.py:143-190) and the engines' float64
        # exponential of -h A are the same matrices to float64 rounding, so the flag selects nothing else here.
        self.jordan_flows = bool(jordan_flows)
        sizes = self.block_sizes
        if self.N == 3:
            pairs = sizes is not None and (all(s == 2 for s in sizes) or all(s == 1 for s in sizes))
            if not (pairs and self.d % 2 == 0 and self.d <= 8):
                raise NotImplementedError("depth N=3 runs on the block engine: 2x2 (or 1x1) blocks, state dim even and <= 8")
            self.engine = "block"
        elif self.N == 2:
            # the plane leaf reads its own generator from A (per plane [[d, w], [-w, d]]): dense engine
            closed = leaf == "plane_closed" or leaf in JORDAN_LEAVES
            self.engine = "diag" if is_diagonal(self.A_param) and not closed else "dense"
        else:
            raise NotImplementedError("the B200 engines are built for depths N=2 and N=3")
        if leaf == "block_series" and self.N > 2:
            raise NotImplementedError("leaf='block_series': blockwise series local terms exist for depths 1 and 2")
        if leaf == "van_loan" and self.engine == "block":
            raise NotImplementedError(
                "leaf='van_loan' runs on the diagonal and dense engines (depth 2); use leaf='series' with "
                "series_q for depth 3"
            )
        # The Van Loan leaf with a per-interval clock (diagonal engine) and on the dense engine is the
        # series leaf's evaluation with the Van Loan leaf's coefficients, truncated at degree 8
        # (series.vanloan_poly_coeffs); under a uniform clock the diagonal engine takes its exact tables.
        if leaf == "van_loan":
            self._q = VANLOAN_DEGREE
        elif leaf == "plane_closed" or leaf in JORDAN_LEAVES:
            self._q = series.CLOSED_Q
        else:
            self._q = self.series_q

    @property
    def signature_dim(self) -> int:
        return sum(self.d**k for k in range(1, self.N + 1))

    # ------------------------------------------------------------------ the engine call

    def fused_logsig_applies(self, d_in: int) -> bool:
        """Whether the terminal log-signature can come out of the engine's closed-form terminal kernels
        (EWS_F_LOGSIG): diagonal engine, depth 2, uniform clock without a basepoint, d_in <= 32 and
        dim * d_in <= 1024."""
        return (self.engine == "diag" and self.N == 2 and self.reweighting_mode == "displacement_uniform"
                and self.d <= 32 and d_in <= 32 and self.d * d_in <= 1024)

    def _flat(self, path, clock, readout, a_scale=1.0, lift=None, increments=False, log_epilogue=False):
        """Batched flat EWS: path (B, L, d_in) knots [(B, L-1, d_in) increments], clock (B, L). With
        ``log_epilogue`` (terminal readout, ``fused_logsig_applies``) the compressed log-signature instead."""
        uniform = self.reweighting_mode != "displacement"
        basepoint = self.reweighting_mode == "displacement_uniform_basepoint"
        if self.engine == "dense":
            if not uniform:
                raise NotImplementedError("the dense engine is built for the uniform-clock reweighting modes")
            return self._flat_dense(path, clock, readout, a_scale, lift, increments, basepoint)
        if self.engine == "block":
            if basepoint:
                raise NotImplementedError("the block engine runs the displacement and displacement_uniform modes")
            return self._flat_block(path, clock, readout, a_scale, lift, increments)
        kernel_readout = _lib.EWS_READOUT_TERMINAL if readout == "terminal" else _lib.EWS_READOUT_PREFIX
        if not uniform:
            return self._flat_diag_clock(path, clock, kernel_readout, a_scale, lift, increments)
        lam = self.A_param.diag_values().to(torch.float32) * a_scale
        clock = clock.to(torch.float32)
        h = (clock[:, 2] - clock[:, 1]) if basepoint else (clock[:, 1] - clock[:, 0])
        x = -h[:, None] * lam[None, :]
        if self.leaf == "van_loan":
            q1, q2 = series.vanloan_diag_tables(lam, h, self.M, self.van_loan_expm)
            q1, q2 = q1.to(torch.float32), q2.to(torch.float32)
        else:
            q1, q2 = series.diag_tables(x, self.series_q)
        flags = _lib.EWS_F_UNIFORM | (_lib.EWS_F_BASEPOINT if basepoint else 0) | _det_flags()
        if log_epilogue:
            flags |= _lib.EWS_F_LOGSIG
        if increments:
            flags |= _lib.EWS_F_INCREMENTS
            if path.dtype == torch.bfloat16:
                flags |= _lib.EWS_F_BF16
            else:
                path = path.to(torch.float32)
        else:
            path = path.to(torch.float32)
        return engine.DiagScan.apply(path, x, q1, q2, lift, kernel_readout, flags, self._chunk, increments)

    def _flat_block(self, path, clock, readout, a_scale, lift, increments):
        """Depth 3 on 2x2 blocks: every interval has its own clock step (ews/core/chen_scan.py:155-168); a
        uniform clock is that with equal steps (the cached flow of displacement_uniform agrees with the
        per-interval one up to the rounding of the clock steps)."""
        if self._q > 8:
            raise NotImplementedError("the block engine evaluates series local terms up to series_q=8")
        A = self.A_param().to(torch.float32) * a_scale
        K = self.d // 2
        blocks = torch.stack([A[2 * k : 2 * k + 2, 2 * k : 2 * k + 2] for k in range(K)])
        kernel_readout = _lib.EWS_READOUT_TERMINAL if readout == "terminal" else _lib.EWS_READOUT_PREFIX
        flags = _det_flags()
        if increments:
            flags |= _lib.EWS_F_INCREMENTS
            if path.dtype == torch.bfloat16:
                flags |= _lib.EWS_F_BF16
            else:
                path = path.to(torch.float32)
        else:
            path = path.to(torch.float32)
        clock = clock.to(torch.float32)
        # terminal readout: the backward re-runs each chunk from the forward's saved chunk start
        # (ews/core/kernels/pallas_combine.py:1911-2027, block_terminal_vjp), no prefix stream
        return engine.BlockScan.apply(
            path, clock, blocks, lift, kernel_readout, flags, self._chunk, increments, self._q
        )

    def _flat_diag_clock(self, path, clock, kernel_readout, a_scale, lift, increments):
        """The "displacement" mode: every interval has its own clock step, flow and series tables
        (ews/core/chen_scan.py:155-168 with cached=False; ews/core/series_leaf.py:72-127 per interval)."""
        if self._q > 8:
            raise NotImplementedError("the per-interval diagonal engine evaluates series tables up to series_q=8")
        coef = None
        if self.leaf == "van_loan":
            k1, k2 = series.vanloan_poly_coeffs(self.M, self.van_loan_expm, VANLOAN_DEGREE)
            coef = list(k1) + list(k2.ravel())
        rates = -(self.A_param.diag_values().to(torch.float32) * a_scale)
        B = path.shape[0]
        rates = rates[None, :].expand(B, -1)
        flags = _det_flags()
        if increments:
            flags |= _lib.EWS_F_INCREMENTS
            if path.dtype == torch.bfloat16:
                flags |= _lib.EWS_F_BF16
            else:
                path = path.to(torch.float32)
        else:
            path = path.to(torch.float32)
        return engine.DiagScanClock.apply(
            path, clock.to(torch.float32), rates, lift, kernel_readout, flags, self._chunk, increments, self._q, coef
        )

    def _flat_dense(self, path, clock, readout, a_scale, lift, increments, basepoint):
        if basepoint:
            raise NotImplementedError("the dense engine runs the displacement_uniform mode")
        A = self.A_param().to(torch.float32) * a_scale
        clock = clock.to(torch.float32)
        h = clock[:, 1] - clock[:, 0]
        coeffs = None
        A_leaf = None
        if self.leaf == "van_loan":
            coeffs = series.vanloan_device_coeffs(self.M, self.van_loan_expm, VANLOAN_DEGREE, str(A.device))
        if self.leaf == "plane_closed":
            # The plane leaf's closed form (ews/core/kernels/plane_engine.py:134-155) is the series leaf's
            # limit; evaluated at order PLANE_Q it agrees to float32 rounding while ||h A_planes|| <= PLANE_X_MAX,
            # which a device-side check guards (the next call raises otherwise).
            A_leaf = series.plane_generator(A)
        elif self.leaf in JORDAN_LEAVES:
            # The Jordan leaf's closed forms (ews/core/kernels/jordan_engine.py:324-353) are the series leaf's
            # limit for the chain generator; the same order and range check as the plane leaf.
            A_leaf = series.jordan_generator(A, *self._jordan_chain)
        if A_leaf is not None:
            x = h.abs().max() * A_leaf.abs().sum(-1).max()
            engine.guard(x > series.CLOSED_X_MAX, A.device,
                         f"leaf={self.leaf!r} is evaluated as its series at order {series.CLOSED_Q}, exact to float32 "
                         f"for ||h A|| <= {series.CLOSED_X_MAX}; an earlier call on this device exceeded that range")
        M, F, G, H = series.dense_tables(A, h, self._q, lift, coeffs, A_leaf)
        flags = _lib.EWS_F_UNIFORM | _det_flags()
        if increments:
            flags |= _lib.EWS_F_INCREMENTS
            if path.dtype == torch.bfloat16:
                flags |= _lib.EWS_F_BF16
            else:
                path = path.to(torch.float32)
        else:
            path = path.to(torch.float32)
        # terminal readout: the backward re-runs windows of chunks from the forward's saved chunk starts
        # (ews/core/kernels/pallas_combine.py:1911-2027, block_terminal_vjp), no prefix stream
        kernel_readout = _lib.EWS_READOUT_TERMINAL if readout == "terminal" else _lib.EWS_READOUT_PREFIX
        return engine.DenseScan.apply(path, M, F, G, H, kernel_readout, flags, self._chunk, increments)

    def forward(
        self,
        path: torch.Tensor,
        clock: torch.Tensor,
        return_terminal: bool = True,
        output_format: str = "flat",
        readout: Optional[str] = None,
        a_scale=1.0,
        *,
        lift: Optional[torch.Tensor] = None,
        increments: bool = False,
    ):
        """path (L, d) or (B, L, d) knots, clock (L,) or (B, L) (ews/layer.py:267-302).

        Extensions for fused callers: ``lift`` (w, d) applies the lift B inside the kernel
        (ews/params.py:1181-1192); ``increments=True`` takes path as (B, L-1, d) increments (float32 or
        bfloat16) instead of knots."""
        if readout is None:
            readout = "terminal" if return_terminal else "prefix"
        if readout not in READOUTS:
            raise ValueError("readout must be 'terminal', 'prefix', 'mean', or 'max'")
        if output_format not in ("flat", "list"):
            raise ValueError("output_format must be 'flat' or 'list'")
        if output_format == "list" and readout in ("mean", "max"):
            raise ValueError(f"readout='{readout}' requires output_format='flat'")
        single = path.dim() == 2
        if single:
            if clock.dim() != 1 or clock.shape[0] != path.shape[0] + (1 if increments else 0):
                raise ValueError("clock must be 1D and aligned with path length")
            path, clock = path[None], clock[None]
        elif path.dim() == 3:
            if clock.dim() != 2:
                raise ValueError("clock must be 2D for batched paths")
        else:
            raise ValueError(f"Path must be 2D or 3D, got shape {tuple(path.shape)}")
        kernel_readout = "terminal" if readout == "terminal" else "prefix"
        flat = self._flat(path, clock, kernel_readout, a_scale, lift, increments)
        if readout == "mean":
            flat = flat.mean(dim=1)
        elif readout == "max":
            flat = flat.max(dim=1).values
        if output_format == "list":
            d = self.d
            out = logsig.split_levels(flat[..., 1:], d, self.N)
            lead = flat.shape[:-1]
            out = [lv.reshape(lead + (d,) * k) for k, lv in enumerate(out, start=1)]
            return [o[0] for o in out] if single else out
        return flat[0] if single else flat


class BToSignature(nn.Module):
    """Optional lift B + EWS (ews/layer.py:310-341); the lift runs inside the kernel."""

    def __init__(self, b: Optional[B], ewms: EWS):
        super().__init__()
        self.b = b
        self.ewms = ewms

    def forward(self, path, clock, return_terminal=True, output_format="flat", readout=None):
        lift = None if self.b is None else self.b.full_matrix()
        return self.ewms(path, clock, return_terminal=return_terminal, output_format=output_format, readout=readout, lift=lift)


class LogEWS(nn.Module):
    """log(EWS) in the Lyndon-word coordinates (ews/layer.py:440-556)."""

    def __init__(self, A, N: int, **kw):
        super().__init__()
        self.ewms = EWS(A, N, **kw)
        self.d = self.ewms.d
        self.N = self.ewms.N

    @property
    def log_signature_dim(self) -> int:
        return logsig.log_signature_dim(self.d, self.N)

    def forward(self, path, clock, return_terminal=True, output_format="flat", readout=None, *, lift=None, increments=False):
        if readout is None:
            readout = "terminal" if return_terminal else "prefix"
        if readout not in READOUTS:
            raise ValueError("readout must be 'terminal', 'prefix', 'mean', or 'max'")
        inner = "terminal" if readout == "terminal" else "prefix"
        d_in = path.shape[-1]
        if readout == "terminal" and output_format == "flat" and self.ewms.fused_logsig_applies(d_in):
            # the log / Lyndon epilogue fused into the engine's terminal kernels (EWS_F_LOGSIG)
            single = path.dim() == 2
            p3, c3 = (path[None], clock[None]) if single else (path, clock)
            if p3.dim() != 3 or c3.dim() != 2:
                raise ValueError("clock must be 2D for batched paths")
            feat = self.ewms._flat(p3, c3, "terminal", lift=lift, increments=increments, log_epilogue=True)
            return feat[0] if single else feat
        flat = self.ewms(path, clock, readout=inner, output_format="flat", lift=lift, increments=increments)
        levels = logsig.split_levels(flat[..., 1:], self.d, self.N)
        log_levels = logsig.tensor_log(levels)
        if output_format == "list":
            if readout in ("mean", "max"):
                raise ValueError(f"readout='{readout}' requires output_format='flat'")
            idx = logsig.flat_index_tensors(self.N, self.d, str(flat.device))
            return [lv[..., ix] for lv, ix in zip(log_levels, idx)]
        feat = logsig.compress(log_levels, self.d)
        if readout == "mean":
            return feat.mean(dim=-2)
        if readout == "max":
            return feat.max(dim=-2).values
        return feat
