"""B200-native (sm_100a) engines for the exponentially weighted signature (EWS) hot path.

The EWS layer's local terms and its modified-Chen prefix / terminal scan, forward and custom-VJP
backward, as hand-written CUDA kernels behind the C ABI of include/ews_b200.h (libews_b200.so), with
the reference's layer API (alexandre-bloch/exponentially-weighted-signature, ews/layer.py) on top.
"""

from . import params, series
from .layer import COMBINE_KINDS, EWS, BToSignature, LogEWS, configure
from .logsig import log_level_sizes, log_signature_dim
from .params import AParamBlockDiag, AParamConstant, AParamDiag, AParamEFM, AParamGeneral, AParamJordanRepeated, B
from .series import check_series_q, series_error_bound, suggest_series_q

__all__ = [
    "COMBINE_KINDS",
    "EWS",
    "BToSignature",
    "LogEWS",
    "configure",
    "AParamBlockDiag",
    "AParamConstant",
    "AParamDiag",
    "AParamEFM",
    "AParamGeneral",
    "AParamJordanRepeated",
    "B",
    "check_series_q",
    "series_error_bound",
    "suggest_series_q",
    "log_level_sizes",
    "log_signature_dim",
    "params",
    "series",
]
