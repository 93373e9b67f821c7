"""ctypes binding of libews_b200.so (the C ABI declared in include/ews_b200.h).

The library is loaded from the package directory. There is no CPU fallback: every entry point raises
when the library or a CUDA device is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libews_b200.so")

EWS_OK = 0
EWS_ERR_WORKSPACE = 3
EWS_ERR_LOOKBACK_TIMEOUT = 5
EWS_NOALLOC_SCRATCH_BYTES = 16 << 20

EWS_F_UNIFORM = 1
EWS_F_INCREMENTS = 2
EWS_F_BF16 = 4
EWS_F_BASEPOINT = 8
EWS_F_DETERMINISTIC = 16
EWS_F_TEST_WITHHOLD = 32
EWS_F_TERMINAL_SCAN = 64
EWS_F_LOGSIG = 128

EWS_READOUT_PREFIX = 0
EWS_READOUT_TERMINAL = 1

EXPORTED = (
    "ews_diag_workspace_size",
    "ews_diag_fwd",
    "ews_diag_bwd",
    "ews_diag_fwd_noalloc",
    "ews_diag_fwd_noalloc_status",
    "ews_dense_workspace_size",
    "ews_dense_launches",
    "ews_dense_fwd",
    "ews_dense_bwd",
    "ews_block_workspace_size",
    "ews_block_fwd",
    "ews_block_bwd",
    "ews_expm_batched",
    "ews_expm_adjoint_batched",
    "ews_series_tables",
    "ews_series_tables_adjoint",
    "ews_dense_leaf",
    "ews_dense_leaf_adjoint",
    "ews_dense_leaf_work_size",
    "ews_graded_norm_work_size",
    "ews_graded_norm_fwd",
    "ews_graded_norm_bwd",
    "ews_gated_clock_work_size",
    "ews_gated_clock_fwd",
    "ews_gated_clock_bwd",
    "ews_read_device_status",
    "ews_status_fold",
    "ews_error_string",
    "ews_version",
)

_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p


class DiagArgs(ctypes.Structure):
    """Mirror of ``ews_diag_args``."""

    _fields_ = [
        ("batch", _c_int),
        ("steps", _c_int),
        ("d_in", _c_int),
        ("dim", _c_int),
        ("depth", _c_int),
        ("chunk", _c_int),
        ("readout", _c_int),
        ("flags", ctypes.c_uint),
        ("series_q", _c_int),
        ("spin_limit", _c_int),
        ("path", _vp),
        ("clock", _vp),
        ("lift", _vp),
        ("tab_x", _vp),
        ("tab_q1", _vp),
        ("tab_q2", _vp),
        ("out", _vp),
        ("grad_out", _vp),
        ("grad_dx", _vp),
        ("grad_lift", _vp),
        ("grad_x", _vp),
        ("grad_q1", _vp),
        ("grad_q2", _vp),
        ("fwd_ws", _vp),
        ("fwd_ws_bytes", _c_size),
        ("bwd_ws", _vp),
        ("bwd_ws_bytes", _c_size),
        ("grad_dtheta", _vp),
        ("leaf_coef", _vp),
    ]


class BlockArgs(ctypes.Structure):
    """Mirror of ``ews_block_args``."""

    _fields_ = [
        ("batch", _c_int),
        ("steps", _c_int),
        ("d_in", _c_int),
        ("dim", _c_int),
        ("depth", _c_int),
        ("chunk", _c_int),
        ("readout", _c_int),
        ("flags", ctypes.c_uint),
        ("series_q", _c_int),
        ("spin_limit", _c_int),
        ("path", _vp),
        ("clock", _vp),
        ("blocks", _vp),
        ("lift", _vp),
        ("out", _vp),
        ("grad_out", _vp),
        ("grad_dx", _vp),
        ("grad_dtheta", _vp),
        ("grad_blocks", _vp),
        ("grad_lift", _vp),
        ("fwd_ws", _vp),
        ("fwd_ws_bytes", _c_size),
        ("bwd_ws", _vp),
        ("bwd_ws_bytes", _c_size),
    ]


class DenseArgs(ctypes.Structure):
    """Mirror of ``ews_dense_args``."""

    _fields_ = [
        ("batch", _c_int),
        ("steps", _c_int),
        ("d_in", _c_int),
        ("dim", _c_int),
        ("depth", _c_int),
        ("chunk", _c_int),
        ("readout", _c_int),
        ("flags", ctypes.c_uint),
        ("series_q", _c_int),
        ("spin_limit", _c_int),
        ("path", _vp),
        ("tab_d", _vp),
        ("tab_f", _vp),
        ("tab_g", _vp),
        ("tab_h", _vp),
        ("out", _vp),
        ("grad_out", _vp),
        ("grad_dx", _vp),
        ("grad_d", _vp),
        ("grad_f", _vp),
        ("grad_g", _vp),
        ("grad_h", _vp),
        ("fwd_ws", _vp),
        ("fwd_ws_bytes", _c_size),
        ("bwd_ws", _vp),
        ("bwd_ws_bytes", _c_size),
    ]


_lock = threading.Lock()
_lib = None


class EWSLibraryError(RuntimeError):
    pass


class EWSLookbackTimeout(EWSLibraryError):
    """A device-side wait for a neighbouring chunk ran out (EWS_ERR_LOOKBACK_TIMEOUT): the outputs and
    gradients of that call are invalid."""


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the library (once). Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise EWSLibraryError(
                f"{path} is missing: build it with `python -m exponentially_weighted_signature_b200.build` "
                "(this package has no CPU fallback)"
            )
        lib = ctypes.CDLL(path)
        for name in ("ews_diag_workspace_size",):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(DiagArgs), ctypes.POINTER(_c_size), ctypes.POINTER(_c_size)]
            fn.restype = _c_int
        for name in ("ews_diag_fwd", "ews_diag_bwd", "ews_diag_fwd_noalloc"):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(DiagArgs), _vp]
            fn.restype = _c_int
        lib.ews_dense_workspace_size.argtypes = [ctypes.POINTER(DenseArgs), ctypes.POINTER(_c_size), ctypes.POINTER(_c_size)]
        lib.ews_dense_workspace_size.restype = _c_int
        lib.ews_dense_launches.argtypes = [ctypes.POINTER(DenseArgs), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]
        lib.ews_dense_launches.restype = _c_int
        for name in ("ews_dense_fwd", "ews_dense_bwd"):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(DenseArgs), _vp]
            fn.restype = _c_int
        lib.ews_block_workspace_size.argtypes = [ctypes.POINTER(BlockArgs), ctypes.POINTER(_c_size), ctypes.POINTER(_c_size)]
        lib.ews_block_workspace_size.restype = _c_int
        for name in ("ews_block_fwd", "ews_block_bwd"):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(BlockArgs), _vp]
            fn.restype = _c_int
        lib.ews_expm_batched.argtypes = [_vp, _vp, _c_int, _c_int, _vp]
        lib.ews_expm_batched.restype = _c_int
        lib.ews_expm_adjoint_batched.argtypes = [_vp, _vp, _vp, _c_int, _c_int, _vp]
        lib.ews_expm_adjoint_batched.restype = _c_int
        lib.ews_series_tables.argtypes = [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp]
        lib.ews_series_tables.restype = _c_int
        lib.ews_series_tables_adjoint.argtypes = [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                                  _vp, _vp, _vp]
        lib.ews_series_tables_adjoint.restype = _c_int
        lib.ews_dense_leaf.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]
        lib.ews_dense_leaf.restype = _c_int
        lib.ews_dense_leaf_adjoint.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                               _vp, _vp, _c_size, _vp, _vp, _vp, _vp, _vp]
        lib.ews_dense_leaf_adjoint.restype = _c_int
        lib.ews_dense_leaf_work_size.argtypes = [_c_int, _c_int, _c_int]
        lib.ews_dense_leaf_work_size.restype = _c_size
        lib.ews_graded_norm_work_size.argtypes = [_c_int, _c_int, _c_int, _c_int]
        lib.ews_graded_norm_work_size.restype = _c_size
        lib.ews_graded_norm_fwd.argtypes = [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]
        lib.ews_graded_norm_fwd.restype = _c_int
        lib.ews_graded_norm_bwd.argtypes = [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_size,
                                            _vp]
        lib.ews_graded_norm_bwd.restype = _c_int
        _f = ctypes.c_float
        lib.ews_gated_clock_work_size.argtypes = [_c_int, _c_int, _c_int]
        lib.ews_gated_clock_work_size.restype = _c_size
        lib.ews_gated_clock_fwd.argtypes = [_vp, _vp, _vp, _f, _f, _c_int, _c_int, _c_int, _vp, _vp]
        lib.ews_gated_clock_fwd.restype = _c_int
        lib.ews_gated_clock_bwd.argtypes = [_vp, _vp, _vp, _f, _f, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp,
                                            _c_size, _vp]
        lib.ews_gated_clock_bwd.restype = _c_int
        lib.ews_read_device_status.argtypes = [_vp, _vp, ctypes.POINTER(_c_int)]
        lib.ews_read_device_status.restype = _c_int
        lib.ews_diag_fwd_noalloc_status.argtypes = [_vp, ctypes.POINTER(_c_int)]
        lib.ews_diag_fwd_noalloc_status.restype = _c_int
        lib.ews_status_fold.argtypes = [_vp, _vp, _vp]
        lib.ews_status_fold.restype = _c_int
        lib.ews_error_string.argtypes = [_c_int]
        lib.ews_error_string.restype = ctypes.c_char_p
        lib.ews_version.argtypes = []
        lib.ews_version.restype = _c_int
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != EWS_OK:
        msg = load().ews_error_string(rc).decode()
        if rc == EWS_ERR_LOOKBACK_TIMEOUT:
            raise EWSLookbackTimeout(f"{what}: {msg} (code {rc})")
        if rc == 1:
            raise ValueError(f"{what}: {msg} (code {rc})")
        if rc == 2:
            raise NotImplementedError(f"{what}: {msg} (code {rc})")
        raise EWSLibraryError(f"{what}: {msg} (code {rc})")


def read_device_status(workspace_ptr: int, stream_ptr: int) -> int:
    """Reads a workspace's device error word (synchronises the stream)."""
    st = _c_int(0)
    check(load().ews_read_device_status(_vp(workspace_ptr), _vp(stream_ptr), ctypes.byref(st)), "ews_read_device_status")
    return int(st.value)
