"""torch.autograd bindings of the CUDA engines (through the C ABI in _lib).

Each engine is one autograd Function whose forward calls the library's *_fwd entry point and whose
backward calls *_bwd. The per-sample parameter tables (log-flows and series tables) are ordinary
differentiable torch tensors built from the generator and the clock, so their tiny maps back to the
generator parameters and the clock run through torch autograd; the kernels return the gradients of
the tables, of the input increments and of the lift.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_ptr(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "the EWS B200 engines run on CUDA tensors only (no CPU fallback); move the inputs to a GPU"
            )


# When set to a list, every library call appends (entry point, start event, end event, units) recorded on
# the launching stream: bench.py reads the kernels' device time from it.
PROFILE = None


class _timed:
    def __init__(self, name, device, units, launches=None):
        self.name, self.device, self.units, self.launches = name, device, units, launches

    def __enter__(self):
        if PROFILE is not None:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e1 = torch.cuda.Event(enable_timing=True)
            self.e0.record(torch.cuda.current_stream(self.device))
        return self

    def __exit__(self, *exc):
        if PROFILE is not None:
            self.e1.record(torch.cuda.current_stream(self.device))
            PROFILE.append((self.name, self.e0, self.e1, self.units, self.launches))
        return False


def _dense_launches(a):
    """(forward, backward) kernel launches of one dense call with these arguments."""
    f, b = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.load().ews_dense_launches(ctypes.byref(a), ctypes.byref(f), ctypes.byref(b)), "ews_dense_launches")
    return f.value, b.value


# ---------------------------------------------------------------------------------- device status
#
# Every library call leaves an error word at the start of its workspace (EWS_OK, or EWS_ERR_LOOKBACK_TIMEOUT
# when a bounded device wait ran out and the call's results are invalid). After each call the word is
# folded into a per-device sticky int on the GPU (ews_status_fold) and copied to pinned host memory
# asynchronously, so nothing waits on the GPU; the next call (and every backward on exit) reads the host
# copy and raises EWSLookbackTimeout if an earlier call failed. CHECK_SYNC makes each call synchronise
# and raise at once instead (``layer.configure(check_status=True)``).

CHECK_SYNC = False
# Polls before a device-side look-back wait gives up (0: the library's default, 2^21).
SPIN_LIMIT = 0
_STATUS = {}


def _status_slot(device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    slot = _STATUS.get(idx)
    if slot is None:
        sticky = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        host = torch.zeros(1, dtype=torch.int32).pin_memory()
        slot = _STATUS[idx] = (sticky, host)
    return slot


def raise_pending(device) -> None:
    """Raises (once) the first look-back timeout that an earlier call on ``device`` reported."""
    sticky, host = _status_slot(device)
    code = int(host[0])
    if code != _lib.EWS_OK:
        host.zero_()
        sticky.zero_()
        _lib.check(code, "an earlier EWS engine call on this device")
    raise_guard(device)


def reset_status(device=None) -> None:
    """Clears the pending status of ``device`` (all devices when None)."""
    for idx, (sticky, host) in list(_STATUS.items()):
        if device is None or idx == (device.index if device.index is not None else torch.cuda.current_device()):
            sticky.zero_()
            host.zero_()


def _fold_status(workspace: torch.Tensor, device) -> None:
    sticky, host = _status_slot(device)
    _lib.check(_lib.load().ews_status_fold(_ptr(workspace), _ptr(sticky), _stream_ptr(device)), "ews_status_fold")
    host.copy_(sticky, non_blocking=True)
    if CHECK_SYNC:
        torch.cuda.current_stream(device).synchronize()
        raise_pending(device)


# Range guards of leaves that the engines evaluate as truncated series (the plane leaf): the condition is
# computed on the device, folded into a per-device flag and copied to pinned host memory without a wait;
# the next engine call on the device raises. No host synchronisation in the call itself.
_GUARD = {}


def _guard_slot(device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    slot = _GUARD.get(idx)
    if slot is None:
        flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        host = torch.zeros(1, dtype=torch.int32).pin_memory()
        slot = _GUARD[idx] = [flag, host, ""]
    return slot


def guard(bad: torch.Tensor, device, message: str) -> None:
    """Records (without waiting) that an input violated a leaf's range (``bad``: a 0-dim bool tensor on the
    device); ``raise_guard`` raises ``message`` on the next call."""
    slot = _guard_slot(device)
    slot[0].copy_(torch.maximum(slot[0], bad.to(torch.int32).reshape(1)))
    slot[1].copy_(slot[0], non_blocking=True)
    slot[2] = message
    if CHECK_SYNC:
        torch.cuda.current_stream(device).synchronize()
        raise_guard(device)


def raise_guard(device) -> None:
    """Raises (once) the range violation that an earlier call on ``device`` recorded."""
    if not _GUARD:
        return
    slot = _guard_slot(device)
    if int(slot[1][0]) != 0:
        slot[0].zero_()
        slot[1].zero_()
        raise NotImplementedError(slot[2])


def _coef_buffer(coef):
    """Host buffer of a leaf's polynomial coefficients (9 + 81 floats) for ews_diag_args.leaf_coef, or None."""
    if coef is None:
        return None
    return (ctypes.c_float * len(coef))(*[float(v) for v in coef])


def increments_to_knots_grad(gdx: torch.Tensor) -> torch.Tensor:
    """Adjoint of dx_t = x_{t+1} - x_t: (B, T, d) -> (B, T+1, d)."""
    return F.pad(gdx, (0, 0, 1, 0)) - F.pad(gdx, (0, 0, 0, 1))


class DiagScan(torch.autograd.Function):
    """Diagonal engine, uniform clock: (path, x, Q1, Q2, lift) -> flat EWS (prefix or terminal)."""

    @staticmethod
    def forward(ctx, path, x, q1, q2, lift, readout, flags, chunk, increments):
        _require_cuda(path, x, q1, q2, lift)
        lib = _lib.load()
        B = path.shape[0]
        T = path.shape[1] if increments else path.shape[1] - 1
        d_in = path.shape[2]
        N = x.shape[-1]
        D = N + N * N
        dev = path.device
        path_c = path.contiguous()
        x_c, q1_c, q2_c = x.contiguous().float(), q1.contiguous().float(), q2.contiguous().float()
        lift_c = None if lift is None else lift.contiguous().float()
        if flags & _lib.EWS_F_LOGSIG:  # the fused log-signature epilogue: letters, then the Lyndon pairs
            out = torch.empty((B, N + N * (N - 1) // 2), device=dev, dtype=torch.float32)
        else:
            out = torch.empty((B, T, 1 + D) if readout == _lib.EWS_READOUT_PREFIX else (B, 1 + D), device=dev, dtype=torch.float32)
        a = _lib.DiagArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, 0, SPIN_LIMIT
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.check(lib.ews_diag_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)), "ews_diag_workspace_size")
        fwd_ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
        a.path, a.lift = _ptr(path_c), _ptr(lift_c)
        a.tab_x, a.tab_q1, a.tab_q2 = _ptr(x_c), _ptr(q1_c), _ptr(q2_c)
        a.out = _ptr(out)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fb.value
        raise_pending(dev)
        with _timed("ews_diag_fwd", dev, B * T):
            _lib.check(lib.ews_diag_fwd(ctypes.byref(a), _stream_ptr(dev)), "ews_diag_fwd")
        _fold_status(fwd_ws, dev)
        ctx.meta = (readout, flags, chunk, increments, B, T, d_in, N, bb.value, path.dtype)
        ctx.has_lift = lift is not None
        ctx.save_for_backward(path_c, x_c, q1_c, q2_c, lift_c if lift_c is not None else torch.empty(0, device=dev), out, fwd_ws)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        readout, flags, chunk, increments, B, T, d_in, N, bwd_bytes, path_dtype = ctx.meta
        path, x, q1, q2, lift, out, fwd_ws = ctx.saved_tensors
        lift = lift if ctx.has_lift else None
        lib = _lib.load()
        dev = path.device
        g = grad_out.contiguous().float()
        bwd_ws = torch.empty(bwd_bytes, dtype=torch.uint8, device=dev)
        gdx = torch.empty((B, T, d_in), device=dev, dtype=torch.float32)
        gx = torch.empty((B, N), device=dev, dtype=torch.float32)
        gq1 = torch.empty((B, N), device=dev, dtype=torch.float32)
        gq2 = torch.empty((B, N, N), device=dev, dtype=torch.float32)
        glift = torch.empty((N, d_in), device=dev, dtype=torch.float32) if lift is not None else None
        a = _lib.DiagArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, 0, SPIN_LIMIT
        a.path, a.lift = _ptr(path), _ptr(lift)
        a.tab_x, a.tab_q1, a.tab_q2 = _ptr(x), _ptr(q1), _ptr(q2)
        a.out, a.grad_out = _ptr(out), _ptr(g)
        a.grad_dx, a.grad_lift, a.grad_x, a.grad_q1, a.grad_q2 = _ptr(gdx), _ptr(glift), _ptr(gx), _ptr(gq1), _ptr(gq2)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fwd_ws.numel()
        a.bwd_ws, a.bwd_ws_bytes = _ptr(bwd_ws), bwd_bytes
        with _timed("ews_diag_bwd", dev, B * T):
            _lib.check(lib.ews_diag_bwd(ctypes.byref(a), _stream_ptr(dev)), "ews_diag_bwd")
        _fold_status(bwd_ws, dev)
        raise_pending(dev)
        gpath = gdx if increments else increments_to_knots_grad(gdx)
        return gpath.to(path_dtype), gx, gq1, gq2, glift, None, None, None, None


class Expm(torch.autograd.Function):
    """Batched float64 matrix exponential (B, n, n) on the device, n <= 64 (the adjoint: n <= 32). The
    forward and the VJP (the Frechet derivative L(X^T, G)) run in the library, so the dense engine's
    tables are built without a host round trip."""

    @staticmethod
    def forward(ctx, X):
        _require_cuda(X)
        if X.dtype != torch.float64:
            raise TypeError("Expm takes float64 matrices")
        Xc = X.contiguous()
        out = torch.empty_like(Xc)
        n = Xc.shape[-1]
        batch = Xc.numel() // (n * n) if n else 0
        with _timed("ews_expm", Xc.device, batch):
            _lib.check(_lib.load().ews_expm_batched(_ptr(Xc), _ptr(out), batch, n, _stream_ptr(Xc.device)), "ews_expm_batched")
        ctx.save_for_backward(Xc)
        return out

    @staticmethod
    def backward(ctx, G):
        (X,) = ctx.saved_tensors
        Gc = G.to(torch.float64).contiguous()
        out = torch.empty_like(X)
        n = X.shape[-1]
        batch = X.numel() // (n * n) if n else 0
        with _timed("ews_expm_adjoint", X.device, batch):
            _lib.check(
                _lib.load().ews_expm_adjoint_batched(_ptr(X), _ptr(Gc), _ptr(out), batch, n, _stream_ptr(X.device)),
                "ews_expm_adjoint_batched",
            )
        return out


class SeriesTables(torch.autograd.Function):
    """The dense engine's series-leaf tables in one library kernel per direction: (X = -h A (B, n, n)
    float64, lift W (n, d_in) float64 or None, coefficients c1 (q+1,), c2 (q+1, q+1) float64) ->
    F (B, n, d_in), G, H (B, q+1, n, d_in) float32, with P_a = X^a / a!, G_a = P_a W, F = sum_p c1_p G_p,
    H_a = sum_b c2_ab G_b (series.dense_leaf_tables in one pass); the VJP returns dX and dW."""

    @staticmethod
    def forward(ctx, X, W, c1, c2):
        _require_cuda(X)
        X = X.contiguous()
        B, n = X.shape[0], X.shape[-1]
        q = c1.shape[0] - 1
        Wc = None if W is None else W.to(torch.float64).contiguous()
        d = n if Wc is None else Wc.shape[-1]
        F = torch.empty((B, n, d), dtype=torch.float32, device=X.device)
        G = torch.empty((B, q + 1, n, d), dtype=torch.float32, device=X.device)
        H = torch.empty_like(G)
        c1c, c2c = c1.contiguous(), c2.contiguous()
        _lib.check(_lib.load().ews_series_tables(_ptr(X), None if Wc is None else _ptr(Wc), _ptr(c1c), _ptr(c2c), B, n,
                                                 d, q, _ptr(F), _ptr(G), _ptr(H), _stream_ptr(X.device)),
                   "ews_series_tables")
        ctx.save_for_backward(X, Wc, c1c, c2c)
        ctx.has_w = W is not None
        return F, G, H

    @staticmethod
    def backward(ctx, dF, dG, dH):
        X, Wc, c1, c2 = ctx.saved_tensors
        B, n = X.shape[0], X.shape[-1]
        q = c1.shape[0] - 1
        d = n if Wc is None else Wc.shape[-1]
        z = lambda t, shape: torch.zeros(shape, dtype=torch.float32, device=X.device) if t is None else t.float().contiguous()
        dF = z(dF, (B, n, d))
        dG = z(dG, (B, q + 1, n, d))
        dH = z(dH, (B, q + 1, n, d))
        dX = torch.empty_like(X)
        dW = torch.empty((B, n, d), dtype=torch.float64, device=X.device) if ctx.has_w else None
        _lib.check(_lib.load().ews_series_tables_adjoint(_ptr(X), None if Wc is None else _ptr(Wc), _ptr(c1), _ptr(c2), B, n,
                                                         d, q, _ptr(dF), _ptr(dG), _ptr(dH), _ptr(dX),
                                                         None if dW is None else _ptr(dW), _stream_ptr(X.device)),
                   "ews_series_tables_adjoint")
        return dX, (dW.sum(0) if dW is not None else None), None, None


class DenseLeaf(torch.autograd.Function):
    """Both per-sample tables of the dense engine for a uniform clock, one library launch each way:
    (A (n, n), h (B,), A_leaf (n, n) or None, W (n, d_in) or None, c1, c2 float64) -> D = I - expm(-h_b A)
    (B, n, n) and the series tables F, G, H of -h_b A_leaf (A unless given), all float32 (evaluated in
    float64). The VJP returns dA, dh, dA_leaf and dW, summed over samples in sample order on the device."""

    @staticmethod
    def forward(ctx, A, h, A_leaf, W, c1, c2):
        _require_cuda(A, h, A_leaf, W)
        A = A.to(torch.float32).contiguous()
        h = h.to(torch.float32).contiguous()
        Al = None if A_leaf is None else A_leaf.to(torch.float32).contiguous()
        Wc = None if W is None else W.to(torch.float32).contiguous()
        B, n = h.shape[0], A.shape[-1]
        d = n if Wc is None else Wc.shape[-1]
        q = c1.shape[0] - 1
        dev = A.device
        Dc = torch.empty((B, n, n), dtype=torch.float32, device=dev)
        F = torch.empty((B, n, d), dtype=torch.float32, device=dev)
        G = torch.empty((B, q + 1, n, d), dtype=torch.float32, device=dev)
        H = torch.empty_like(G)
        c1c, c2c = c1.contiguous(), c2.contiguous()
        with _timed("ews_dense_leaf", dev, B, 1):
            _lib.check(_lib.load().ews_dense_leaf(_ptr(A), _ptr(Al), _ptr(h), _ptr(Wc), _ptr(c1c), _ptr(c2c), B, n, d, q,
                                                  _ptr(Dc), _ptr(F), _ptr(G), _ptr(H), _stream_ptr(dev)),
                       "ews_dense_leaf")
        ctx.save_for_backward(A, h, Al, Wc, c1c, c2c)
        return Dc, F, G, H

    @staticmethod
    def backward(ctx, dDc, dF, dG, dH):
        A, h, Al, Wc, c1, c2 = ctx.saved_tensors
        B, n = h.shape[0], A.shape[-1]
        d = n if Wc is None else Wc.shape[-1]
        q = c1.shape[0] - 1
        dev = A.device
        f32 = lambda t: None if t is None else t.to(torch.float32).contiguous()
        dDc, dF, dG, dH = f32(dDc), f32(dF), f32(dG), f32(dH)
        lib = _lib.load()
        work = torch.empty(int(lib.ews_dense_leaf_work_size(B, n, d)) // 8, dtype=torch.float64, device=dev)
        dA = torch.empty((n, n), dtype=torch.float32, device=dev)
        dAl = torch.empty_like(dA) if Al is not None else None
        dh = torch.empty((B,), dtype=torch.float32, device=dev)
        dW = torch.empty((n, d), dtype=torch.float32, device=dev) if Wc is not None else None
        with _timed("ews_dense_leaf_adjoint", dev, B, 2):
            _lib.check(lib.ews_dense_leaf_adjoint(_ptr(A), _ptr(Al), _ptr(h), _ptr(Wc), _ptr(c1), _ptr(c2), B, n, d, q,
                                                  _ptr(dDc), _ptr(dF), _ptr(dG), _ptr(dH), _ptr(work),
                                                  work.numel() * 8, _ptr(dA), _ptr(dAl), _ptr(dh), _ptr(dW),
                                                  _stream_ptr(dev)),
                       "ews_dense_leaf_adjoint")
        need = ctx.needs_input_grad
        return (dA if need[0] else None, dh if need[1] else None, dAl if need[2] else None,
                dW if need[3] else None, None, None)


class GradedNorm(torch.autograd.Function):
    """The block's stream consumer in one library pass each way: EWS prefix rows flat (B, T, 1 + D) ->
    y (B, T + 1, D), level 0 dropped, a zero row prepended and every level normalised by its live RMS
    (ews/block.py:282-306, ews/norms.py:47-135, "live_rms"): y level k = g_k x_k / (RMS(x_k) + eps_k)."""

    @staticmethod
    def forward(ctx, flat, gains, d, levels, eps):
        _require_cuda(flat, gains)
        flat = flat.to(torch.float32).contiguous()
        g = gains.to(torch.float32).contiguous()
        B, T, W = flat.shape
        y = torch.empty((B, T + 1, W - 1), dtype=torch.float32, device=flat.device)
        ep = (ctypes.c_float * levels)(*[float(e) for e in eps])
        with _timed("ews_graded_norm_fwd", flat.device, B * T, 1):
            _lib.check(_lib.load().ews_graded_norm_fwd(_ptr(flat), _ptr(g), ep, B, T, d, levels, _ptr(y),
                                                        _stream_ptr(flat.device)), "ews_graded_norm_fwd")
        ctx.save_for_backward(flat, g)
        ctx.meta = (d, levels, tuple(float(e) for e in eps))
        return y

    @staticmethod
    def backward(ctx, dy):
        flat, g = ctx.saved_tensors
        d, levels, eps = ctx.meta
        B, T, _ = flat.shape
        lib = _lib.load()
        dyc = dy.to(torch.float32).contiguous()
        dflat = torch.empty_like(flat)
        dg = torch.empty((levels,), dtype=torch.float32, device=flat.device)
        work = torch.empty(max(1, int(lib.ews_graded_norm_work_size(B, T, d, levels)) // 4), dtype=torch.float32,
                           device=flat.device)
        ep = (ctypes.c_float * levels)(*eps)
        with _timed("ews_graded_norm_bwd", flat.device, B * T, 2):
            _lib.check(lib.ews_graded_norm_bwd(_ptr(flat), _ptr(g), ep, _ptr(dyc), B, T, d, levels, _ptr(dflat),
                                               _ptr(dg), _ptr(work), work.numel() * 4, _stream_ptr(flat.device)),
                       "ews_graded_norm_bwd")
        return dflat, dg, None, None, None


class GatedClock(torch.autograd.Function):
    """The block's token-gated clock in one library pass each way (ews/clocks.py:409-466, no mask):
    theta = [0, cumsum(relu(diff(in_scale x) @ w - b))] / norm_constant for x (B, L, H)."""

    @staticmethod
    def forward(ctx, x, w, b, in_scale, norm_constant):
        _require_cuda(x, w, b)
        xc = x.to(torch.float32).contiguous()
        wc, bc = w.to(torch.float32).contiguous(), b.to(torch.float32).reshape(1).contiguous()
        B, L, H = xc.shape
        theta = torch.empty((B, L), dtype=torch.float32, device=xc.device)
        with _timed("ews_gated_clock_fwd", xc.device, B * L, 2):
            _lib.check(_lib.load().ews_gated_clock_fwd(_ptr(xc), _ptr(wc), _ptr(bc), float(in_scale), float(norm_constant),
                                                        B, L, H, _ptr(theta), _stream_ptr(xc.device)),
                       "ews_gated_clock_fwd")
        ctx.save_for_backward(xc, wc, bc)
        ctx.consts = (float(in_scale), float(norm_constant))
        return theta

    @staticmethod
    def backward(ctx, dtheta):
        xc, wc, bc = ctx.saved_tensors
        s, c = ctx.consts
        B, L, H = xc.shape
        lib = _lib.load()
        dt = dtheta.to(torch.float32).contiguous()
        dx = torch.empty_like(xc)
        dw = torch.empty_like(wc)
        db = torch.empty((1,), dtype=torch.float32, device=xc.device)
        work = torch.empty(max(1, int(lib.ews_gated_clock_work_size(B, L, H)) // 4), dtype=torch.float32,
                           device=xc.device)
        with _timed("ews_gated_clock_bwd", xc.device, B * L, 4):
            _lib.check(lib.ews_gated_clock_bwd(_ptr(xc), _ptr(wc), _ptr(bc), s, c, _ptr(dt), B, L, H, _ptr(dx), _ptr(dw),
                                               _ptr(db), _ptr(work), work.numel() * 4, _stream_ptr(xc.device)),
                       "ews_gated_clock_bwd")
        return dx, dw, db.reshape(()), None, None


class DenseScan(torch.autograd.Function):
    """Dense engine, uniform clock: (path, D = I - M, F, G, H) -> flat EWS (prefix or terminal)."""

    @staticmethod
    def forward(ctx, path, M, F, G, H, readout, flags, chunk, increments):
        _require_cuda(path, M, F, G, H)
        lib = _lib.load()
        B = path.shape[0]
        T = path.shape[1] if increments else path.shape[1] - 1
        d_in = path.shape[2]
        N = M.shape[-1]
        QP = G.shape[1]
        D = N + N * N
        dev = path.device
        path_c = path.contiguous()
        tabs = [t.contiguous().float() for t in (M, F, G, H)]
        out = torch.empty((B, T, 1 + D) if readout == _lib.EWS_READOUT_PREFIX else (B, 1 + D), device=dev, dtype=torch.float32)
        a = _lib.DenseArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, QP - 1, SPIN_LIMIT
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.check(lib.ews_dense_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)), "ews_dense_workspace_size")
        fwd_ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
        a.path = _ptr(path_c)
        a.tab_d, a.tab_f, a.tab_g, a.tab_h = (_ptr(t) for t in tabs)
        a.out = _ptr(out)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fb.value
        raise_pending(dev)
        with _timed("ews_dense_fwd", dev, B * T, _dense_launches(a)[0] if PROFILE is not None else None):
            _lib.check(lib.ews_dense_fwd(ctypes.byref(a), _stream_ptr(dev)), "ews_dense_fwd")
        _fold_status(fwd_ws, dev)
        ctx.meta = (readout, flags, chunk, increments, B, T, d_in, N, QP, bb.value, path.dtype)
        ctx.save_for_backward(path_c, *tabs, out, fwd_ws)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        readout, flags, chunk, increments, B, T, d_in, N, QP, bwd_bytes, path_dtype = ctx.meta
        path, M, F, G, H, out, fwd_ws = ctx.saved_tensors
        lib = _lib.load()
        dev = path.device
        g = grad_out.contiguous().float()
        bwd_ws = torch.empty(bwd_bytes, dtype=torch.uint8, device=dev)
        gdx = torch.empty((B, T, d_in), device=dev, dtype=torch.float32)
        gM = torch.empty_like(M)
        gF = torch.empty_like(F)
        gG = torch.empty_like(G)
        gH = torch.empty_like(H)
        a = _lib.DenseArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, QP - 1, SPIN_LIMIT
        a.path = _ptr(path)
        a.tab_d, a.tab_f, a.tab_g, a.tab_h = (_ptr(t) for t in (M, F, G, H))
        a.out, a.grad_out, a.grad_dx = _ptr(out), _ptr(g), _ptr(gdx)
        a.grad_d, a.grad_f, a.grad_g, a.grad_h = (_ptr(t) for t in (gM, gF, gG, gH))
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fwd_ws.numel()
        a.bwd_ws, a.bwd_ws_bytes = _ptr(bwd_ws), bwd_bytes
        with _timed("ews_dense_bwd", dev, B * T, _dense_launches(a)[1] if PROFILE is not None else None):
            _lib.check(lib.ews_dense_bwd(ctypes.byref(a), _stream_ptr(dev)), "ews_dense_bwd")
        _fold_status(bwd_ws, dev)
        raise_pending(dev)
        gpath = gdx if increments else increments_to_knots_grad(gdx)
        return gpath.to(path_dtype), gM, gF, gG, gH, None, None, None, None


class DiagScanClock(torch.autograd.Function):
    """Diagonal engine, per-interval clock (the reference's "displacement" mode): (path, clock knots,
    rates r = -lambda, lift) -> flat EWS. Interval t uses x_t = (clock[t+1] - clock[t]) r with its own
    series tables, evaluated in the kernel; the backward returns the gradients of the path, the clock,
    the rates and the lift."""

    @staticmethod
    def forward(ctx, path, clock, rates, lift, readout, flags, chunk, increments, series_q, leaf_coef=None):
        _require_cuda(path, clock, rates, lift)
        lib = _lib.load()
        B = path.shape[0]
        T = path.shape[1] if increments else path.shape[1] - 1
        d_in = path.shape[2]
        N = rates.shape[-1]
        D = N + N * N
        dev = path.device
        path_c = path.contiguous()
        clock_c = clock.contiguous().float()
        rates_c = rates.contiguous().float()
        lift_c = None if lift is None else lift.contiguous().float()
        out = torch.empty((B, T, 1 + D) if readout == _lib.EWS_READOUT_PREFIX else (B, 1 + D), device=dev, dtype=torch.float32)
        a = _lib.DiagArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, series_q, SPIN_LIMIT
        coef_buf = _coef_buffer(leaf_coef)  # kept alive until the call returns
        a.leaf_coef = None if coef_buf is None else ctypes.cast(coef_buf, ctypes.c_void_p)
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.check(lib.ews_diag_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)), "ews_diag_workspace_size")
        fwd_ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
        a.path, a.clock, a.lift, a.tab_x = _ptr(path_c), _ptr(clock_c), _ptr(lift_c), _ptr(rates_c)
        a.out = _ptr(out)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fb.value
        raise_pending(dev)
        with _timed("ews_diag_fwd", dev, B * T):
            _lib.check(lib.ews_diag_fwd(ctypes.byref(a), _stream_ptr(dev)), "ews_diag_fwd")
        _fold_status(fwd_ws, dev)
        ctx.meta = (readout, flags, chunk, increments, series_q, B, T, d_in, N, bb.value, path.dtype, clock.dtype)
        ctx.leaf_coef = leaf_coef
        ctx.has_lift = lift is not None
        empty = torch.empty(0, device=dev)
        ctx.save_for_backward(path_c, clock_c, rates_c, lift_c if lift_c is not None else empty, out, fwd_ws)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        readout, flags, chunk, increments, series_q, B, T, d_in, N, bwd_bytes, path_dtype, clock_dtype = ctx.meta
        path, clock, rates, lift, out, fwd_ws = ctx.saved_tensors
        lift = lift if ctx.has_lift else None
        lib = _lib.load()
        dev = path.device
        g = grad_out.contiguous().float()
        bwd_ws = torch.empty(bwd_bytes, dtype=torch.uint8, device=dev)
        gdx = torch.empty((B, T, d_in), device=dev, dtype=torch.float32)
        gr = torch.empty((B, N), device=dev, dtype=torch.float32)
        gdt = torch.empty((B, T), device=dev, dtype=torch.float32)
        glift = torch.empty((N, d_in), device=dev, dtype=torch.float32) if lift is not None else None
        a = _lib.DiagArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 2
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, series_q, SPIN_LIMIT
        coef_buf = _coef_buffer(ctx.leaf_coef)
        a.leaf_coef = None if coef_buf is None else ctypes.cast(coef_buf, ctypes.c_void_p)
        a.path, a.clock, a.lift, a.tab_x = _ptr(path), _ptr(clock), _ptr(lift), _ptr(rates)
        a.out, a.grad_out = _ptr(out), _ptr(g)
        a.grad_dx, a.grad_lift, a.grad_x, a.grad_dtheta = _ptr(gdx), _ptr(glift), _ptr(gr), _ptr(gdt)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fwd_ws.numel()
        a.bwd_ws, a.bwd_ws_bytes = _ptr(bwd_ws), bwd_bytes
        with _timed("ews_diag_bwd", dev, B * T):
            _lib.check(lib.ews_diag_bwd(ctypes.byref(a), _stream_ptr(dev)), "ews_diag_bwd")
        _fold_status(bwd_ws, dev)
        raise_pending(dev)
        gpath = gdx if increments else increments_to_knots_grad(gdx)
        gclock = increments_to_knots_grad(gdt[..., None])[..., 0]
        return gpath.to(path_dtype), gclock.to(clock_dtype), gr, glift, None, None, None, None, None, None


class BlockScan(torch.autograd.Function):
    """Block engine (2x2 blocks, depth 3, per-interval clock): (path, clock knots, blocks (K, 2, 2), lift)
    -> flat EWS (prefix or terminal). The backward returns the gradients of the path, the clock, the
    blocks and the lift."""

    @staticmethod
    def forward(ctx, path, clock, blocks, lift, readout, flags, chunk, increments, series_q):
        _require_cuda(path, clock, blocks, lift)
        lib = _lib.load()
        B = path.shape[0]
        T = path.shape[1] if increments else path.shape[1] - 1
        d_in = path.shape[2]
        N = 2 * blocks.shape[0]
        D = N + N * N + N * N * N
        dev = path.device
        path_c = path.contiguous()
        clock_c = clock.contiguous().float()
        blocks_c = blocks.contiguous().float()
        lift_c = None if lift is None else lift.contiguous().float()
        out = torch.empty((B, T, 1 + D) if readout == _lib.EWS_READOUT_PREFIX else (B, 1 + D), device=dev, dtype=torch.float32)
        a = _lib.BlockArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 3
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, series_q, SPIN_LIMIT
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.check(lib.ews_block_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)), "ews_block_workspace_size")
        fwd_ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
        a.path, a.clock, a.blocks, a.lift = _ptr(path_c), _ptr(clock_c), _ptr(blocks_c), _ptr(lift_c)
        a.out = _ptr(out)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fb.value
        raise_pending(dev)
        with _timed("ews_block_fwd", dev, B * T):
            _lib.check(lib.ews_block_fwd(ctypes.byref(a), _stream_ptr(dev)), "ews_block_fwd")
        _fold_status(fwd_ws, dev)
        ctx.meta = (readout, flags, chunk, increments, series_q, B, T, d_in, N, bb.value, path.dtype, clock.dtype)
        ctx.has_lift = lift is not None
        empty = torch.empty(0, device=dev)
        ctx.save_for_backward(path_c, clock_c, blocks_c, lift_c if lift_c is not None else empty, out, fwd_ws)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        readout, flags, chunk, increments, series_q, B, T, d_in, N, bwd_bytes, path_dtype, clock_dtype = ctx.meta
        path, clock, blocks, lift, out, fwd_ws = ctx.saved_tensors
        lift = lift if ctx.has_lift else None
        lib = _lib.load()
        dev = path.device
        g = grad_out.contiguous().float()
        bwd_ws = torch.empty(bwd_bytes, dtype=torch.uint8, device=dev)
        gdx = torch.empty((B, T, d_in), device=dev, dtype=torch.float32)
        gdt = torch.empty((B, T), device=dev, dtype=torch.float32)
        gblk = torch.empty_like(blocks)
        glift = torch.empty((N, d_in), device=dev, dtype=torch.float32) if lift is not None else None
        a = _lib.BlockArgs()
        a.batch, a.steps, a.d_in, a.dim, a.depth = B, T, d_in, N, 3
        a.chunk, a.readout, a.flags, a.series_q, a.spin_limit = chunk, readout, flags, series_q, SPIN_LIMIT
        a.path, a.clock, a.blocks, a.lift = _ptr(path), _ptr(clock), _ptr(blocks), _ptr(lift)
        a.out, a.grad_out = _ptr(out), _ptr(g)
        a.grad_dx, a.grad_dtheta, a.grad_blocks, a.grad_lift = _ptr(gdx), _ptr(gdt), _ptr(gblk), _ptr(glift)
        a.fwd_ws, a.fwd_ws_bytes = _ptr(fwd_ws), fwd_ws.numel()
        a.bwd_ws, a.bwd_ws_bytes = _ptr(bwd_ws), bwd_bytes
        with _timed("ews_block_bwd", dev, B * T):
            _lib.check(lib.ews_block_bwd(ctypes.byref(a), _stream_ptr(dev)), "ews_block_bwd")
        _fold_status(bwd_ws, dev)
        raise_pending(dev)
        gpath = gdx if increments else increments_to_knots_grad(gdx)
        gclock = increments_to_knots_grad(gdt[..., None])[..., 0]
        return gpath.to(path_dtype), gclock.to(clock_dtype), gblk, glift, None, None, None, None, None
