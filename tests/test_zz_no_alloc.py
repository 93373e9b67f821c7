"""The allocation-free forward, ews_diag_fwd_noalloc, against the ordinary forward (collected last).

Callers that cannot allocate device memory for the library (a plugin host that passes only inputs and
outputs, a serving loop that forbids cudaMalloc because it can synchronise the device) use this entry
point; its look-back workspace is a fixed device array inside the library. The test drives both entry
points through the C ABI on the same inputs, twice in a row with different inputs (the array keeps the
previous call's contents), and compares them with the tolerance of tests/test_gpu_diag.py: global
relative error <= 1e-5 and elementwise |a - b| <= 1e-6 + 1e-5 |b|.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(lib, entry, B, T, N, d_in, seed, readout, use_ws):
    from exponentially_weighted_signature_b200 import _lib, series

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    path = torch.cumsum(torch.randn(B, T + 1, d_in, generator=g) / T**0.5, 1).to(dev)
    lift = (torch.randn(N, d_in, generator=g) / d_in**0.5).to(dev)
    lam = torch.exp(torch.rand(N, generator=g) * 4 - 3)
    x = (-(1.0 / T) * lam)[None].expand(B, N).contiguous().to(dev)
    q1, q2 = series.diag_tables(x, 6)
    q1, q2 = q1.contiguous(), q2.contiguous()
    W = 1 + N + N * N
    out = torch.full((B, T, W) if readout == 0 else (B, W), float("nan"), device=dev)
    a = _lib.DiagArgs()
    a.batch, a.steps, a.d_in, a.dim, a.depth, a.chunk = B, T, d_in, N, 2, 16
    a.readout, a.flags = readout, _lib.EWS_F_UNIFORM
    a.path, a.lift, a.tab_x, a.tab_q1, a.tab_q2, a.out = (
        ctypes.c_void_p(t.data_ptr()) for t in (path, lift, x, q1, q2, out)
    )
    ws = None
    if use_ws:
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        assert lib.ews_diag_workspace_size(ctypes.byref(a), ctypes.byref(fb), ctypes.byref(bb)) == 0
        ws = torch.empty(fb.value, dtype=torch.uint8, device=dev)
        a.fwd_ws, a.fwd_ws_bytes = ctypes.c_void_p(ws.data_ptr()), fb.value
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    rc = entry(ctypes.byref(a), stream)
    torch.cuda.synchronize()
    assert rc == 0
    if not use_ws:
        assert torch.cuda.memory_allocated() == before
    return out.double().cpu()


def test_noalloc_forward_matches_the_workspace_forward():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from exponentially_weighted_signature_b200 import _lib

    lib = _lib.load()
    for seed, (B, T, N, d_in, readout) in enumerate([(3, 200, 16, 4, 0), (5, 333, 32, 16, 1)]):
        ref = _run(lib, lib.ews_diag_fwd, B, T, N, d_in, seed, readout, True)
        got = _run(lib, lib.ews_diag_fwd_noalloc, B, T, N, d_in, seed, readout, False)
        assert torch.isfinite(got).all()
        err = (got - ref).abs()
        assert float(err.max() / ref.abs().max()) <= 1e-5
        assert bool((err <= 1e-6 + 1e-5 * ref.abs()).all())


def _noalloc_status(lib):
    from exponentially_weighted_signature_b200 import _lib

    st = ctypes.c_int(-1)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.ews_diag_fwd_noalloc_status(stream, ctypes.byref(st)) == _lib.EWS_OK
    return st.value


def test_noalloc_status_reports_a_timeout():
    """The no-alloc caller holds no workspace pointer, so ews_diag_fwd_noalloc_status reads the status
    word at the start of the library's array: clear after a good call, EWS_ERR_LOOKBACK_TIMEOUT after a
    call whose look-back waits ran out (EWS_F_TEST_WITHHOLD with a short spin limit), clear again after
    the next good call."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from exponentially_weighted_signature_b200 import _lib, series

    lib = _lib.load()
    dev = torch.device("cuda")
    B, T, N = 2, 256, 16
    path = torch.randn(B, T + 1, N, device=dev)
    x = torch.full((B, N), -1e-3, device=dev)
    q1, q2 = series.diag_tables(x, 4)
    q1, q2 = q1.contiguous(), q2.contiguous()
    out = torch.empty(B, T, 1 + N + N * N, device=dev)
    a = _lib.DiagArgs()
    a.batch, a.steps, a.d_in, a.dim, a.depth, a.chunk = B, T, N, N, 2, 8
    a.readout, a.flags = 0, _lib.EWS_F_UNIFORM
    a.path, a.tab_x, a.tab_q1, a.tab_q2, a.out = (ctypes.c_void_p(t.data_ptr()) for t in (path, x, q1, q2, out))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.ews_diag_fwd_noalloc(ctypes.byref(a), stream) == 0
    assert _noalloc_status(lib) == _lib.EWS_OK
    a.flags, a.spin_limit = _lib.EWS_F_UNIFORM | _lib.EWS_F_TEST_WITHHOLD, 2000
    assert lib.ews_diag_fwd_noalloc(ctypes.byref(a), stream) == 0
    assert _noalloc_status(lib) == _lib.EWS_ERR_LOOKBACK_TIMEOUT
    a.flags, a.spin_limit = _lib.EWS_F_UNIFORM, 0
    assert lib.ews_diag_fwd_noalloc(ctypes.byref(a), stream) == 0
    assert _noalloc_status(lib) == _lib.EWS_OK
    torch.cuda.synchronize()


def test_noalloc_rejects_oversized_problems():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from exponentially_weighted_signature_b200 import _lib

    lib = _lib.load()
    a = _lib.DiagArgs()
    a.batch, a.steps, a.d_in, a.dim, a.depth, a.chunk = 4096, 100000, 32, 32, 2, 8
    a.readout, a.flags = 0, _lib.EWS_F_UNIFORM
    a.path = a.out = a.tab_x = a.tab_q1 = a.tab_q2 = ctypes.c_void_p(16)
    fb = ctypes.c_size_t(0)
    assert lib.ews_diag_workspace_size(ctypes.byref(a), ctypes.byref(fb), None) == 0
    assert fb.value > _lib.EWS_NOALLOC_SCRATCH_BYTES
    assert lib.ews_diag_fwd_noalloc(ctypes.byref(a), None) == _lib.EWS_ERR_WORKSPACE
