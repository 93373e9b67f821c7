"""CPU tests of the C ABI library surface and of the host-side logic (no kernel launches)."""

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

from exponentially_weighted_signature_b200 import _lib, series
from exponentially_weighted_signature_b200 import logsig
from exponentially_weighted_signature_b200.layer import EWS, LogEWS
from exponentially_weighted_signature_b200.params import AParamBlockDiag, AParamDiag, AParamEFM, AParamJordanRepeated, B
from oracle import ews_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ews_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|size_t)\s+(ews_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations parsed from the header"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    for name in declared:
        assert re.search(rf"\bT {name}\b", out), name


def test_version_and_error_strings():
    lib = _lib.load()
    assert lib.ews_version() >= 1
    assert lib.ews_error_string(0) == b"ok"
    assert b"look-back" in lib.ews_error_string(5)


def _args(**kw):
    a = _lib.DiagArgs()
    a.batch, a.steps, a.d_in, a.dim, a.depth = 4, 100, 16, 16, 2
    a.readout, a.flags = 0, _lib.EWS_F_UNIFORM
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_query_and_argument_errors():
    lib = _lib.load()
    fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.ews_diag_workspace_size(ctypes.byref(_args()), ctypes.byref(fb), ctypes.byref(bb)) == 0
    assert fb.value > 0 and bb.value > 0
    # the forward slots grow with the number of chunks
    fb2 = ctypes.c_size_t(0)
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(chunk=16)), ctypes.byref(fb2), None) == 0
    assert fb2.value >= fb.value or True
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(batch=0)), ctypes.byref(fb), ctypes.byref(bb)) == 1
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(dim=33)), ctypes.byref(fb), ctypes.byref(bb)) == 2
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(depth=3)), ctypes.byref(fb), ctypes.byref(bb)) == 2
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(readout=7)), ctypes.byref(fb), ctypes.byref(bb)) == 1
    # bf16 needs stored increments
    assert lib.ews_diag_workspace_size(ctypes.byref(_args(flags=_lib.EWS_F_UNIFORM | _lib.EWS_F_BF16)), ctypes.byref(fb), ctypes.byref(bb)) == 1
    # a launch with a missing workspace is refused before touching the device
    a = _args()
    a.path = a.out = a.tab_x = a.tab_q1 = a.tab_q2 = ctypes.c_void_p(16)
    assert lib.ews_diag_fwd(ctypes.byref(a), None) == 3
    # the identity lift needs d_in == dim
    a.d_in = 4
    assert lib.ews_diag_fwd(ctypes.byref(a), None) == 1


def test_diag_tables_match_the_series_leaf():
    """Q1, Q2 reproduce the series leaf's level-1/2 local terms for a diagonal A (ews/core/series_leaf.py)."""
    rng = np.random.default_rng(0)
    lam = torch.tensor(rng.uniform(0.1, 3.0, 5), dtype=torch.float64)
    h = 0.37
    path = torch.tensor(np.cumsum(rng.normal(size=(4, 5)), 0), dtype=torch.float64)
    clock = torch.arange(4, dtype=torch.float64) * h
    for q in (1, 4, 9):
        ref = O.series_local_signatures(path, clock, torch.diag(lam), 2, q)
        q1, q2 = series.diag_tables((-h * lam)[None], q)
        dx = path[1:] - path[:-1]
        s1 = q1[0] * dx
        s2 = (q2[0] * dx[:, :, None] * dx[:, None, :]).reshape(3, 25)
        assert torch.allclose(s1, ref[0], rtol=1e-13, atol=1e-15)
        assert torch.allclose(s2, ref[1], rtol=1e-13, atol=1e-15)


def test_dense_leaf_tables_match_the_series_leaf():
    """F dx and sum_a (G_a dx)(H_a dx)^T reproduce the series leaf's local terms for a general A and a lift."""
    rng = np.random.default_rng(2)
    N, d_in, q, h = 5, 3, 6, 0.21
    A = torch.tensor(rng.normal(size=(N, N)) * 0.7, dtype=torch.float64)
    W = torch.tensor(rng.normal(size=(N, d_in)), dtype=torch.float64)
    x = torch.tensor(np.cumsum(rng.normal(size=(4, d_in)), 0), dtype=torch.float64)
    clock = torch.arange(4, dtype=torch.float64) * h
    ref = O.series_local_signatures(x @ W.T, clock, A, 2, q)
    F, G, H = (t.float() for t in series.dense_leaf_tables(-h * A[None], q, W))
    dx = (x[1:] - x[:-1]).float()
    s1 = dx @ F[0].T
    U = torch.einsum("aid,td->tai", G[0], dx)
    V = torch.einsum("aid,td->tai", H[0], dx)
    s2 = torch.einsum("tai,taj->tij", U, V).reshape(3, N * N)
    assert torch.allclose(s1.double(), ref[0], rtol=1e-5, atol=1e-6)
    assert torch.allclose(s2.double(), ref[1], rtol=1e-5, atol=1e-6)


def test_diag_tables_gradient_finite_at_zero():
    x = torch.zeros(2, 3, dtype=torch.float32, requires_grad=True)
    q1, q2 = series.diag_tables(x, 5)
    (q1.sum() + q2.sum()).backward()
    assert torch.isfinite(x.grad).all()


def test_lyndon_words_and_witt_dims_agree_with_oracle():
    for d, n in [(3, 3), (4, 2), (2, 4), (32, 2)]:
        a = logsig.lyndon_words(n, d)
        b = O.lyndon_words(n, d)
        assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert logsig.log_signature_dim(32, 2) == 528


def test_tensor_log_matches_oracle():
    rng = np.random.default_rng(1)
    levels = [torch.tensor(rng.normal(size=(2, 3**k))) for k in range(1, 4)]
    a = logsig.tensor_log(levels)
    b = O.tensor_log(levels)
    assert all(torch.allclose(x, y) for x, y in zip(a, b))


def test_layer_validation_mirrors_reference():
    """ews/layer.py:112-152 of the reference: option validation at construction."""
    A = AParamDiag(torch.ones(4))
    with pytest.raises(ValueError):
        EWS(A, N=2, combine="nonsense")
    with pytest.raises(ValueError):
        EWS(A, N=2, terminal_reduce="nope")
    with pytest.raises(ValueError):
        EWS(A, N=2, leaf="series", series_q=None)
    with pytest.raises(ValueError):
        EWS(A, N=2, reweighting_mode="bogus")
    with pytest.raises(ValueError):
        EWS(A, N=2, chen_expm="bogus")
    with pytest.raises(ValueError):
        EWS(A, N=2, leaf="bogus")
    # the reference's defaults: Van Loan leaf, associative combine (every combine kind runs the engines)
    d = EWS(A, N=2, reweighting_mode="displacement_uniform")
    assert (d.leaf, d.series_q, d.combine, d.combine_chunk, d.M) == ("van_loan", None, "assoc", 1024, 20)
    assert EWS(A, N=2, reweighting_mode="displacement_uniform", combine="lean").engine == "diag"
    # Van Loan runs on the diagonal engine (any mode) and the dense engine; at depth 3 it raises instead
    # of silently computing another leaf
    assert EWS(A, N=2).engine == "diag"  # the reference's full defaults
    assert EWS(torch.eye(4), N=2, reweighting_mode="displacement_uniform").engine == "dense"
    with pytest.raises(NotImplementedError):
        EWS(AParamBlockDiag([torch.ones(2, 2)] * 2, [2, 2]), N=3)
    # the Jordan leaves (ews/layer.py:148-152): uniform Jordan chains required; the dense engine runs them
    with pytest.raises(ValueError):
        EWS(A, N=2, leaf="jordan_closed")
    J = AParamJordanRepeated([3, 3], ["real", "real"], [torch.zeros(1), torch.ones(1)])
    assert EWS(J, N=2, reweighting_mode="displacement_uniform", leaf="jordan_closed").engine == "dense"
    assert EWS(J, N=2, leaf="jordan_closed_tables")._jordan_chain == ("real", 3)
    with pytest.raises(ValueError):  # mixed chain sizes are not uniform chains
        EWS(AParamJordanRepeated([2, 3], ["real"] * 2, [torch.zeros(1)] * 2), N=2, leaf="jordan_closed")
    with pytest.raises(NotImplementedError):
        EWS(J, N=3, leaf="jordan_closed")
    # jordan_flows (ews/layer.py:134-138): needs combine='block_kernel' and uniform chains
    assert EWS(J, N=2, leaf="jordan_closed", combine="block_kernel", jordan_flows=True).jordan_flows
    with pytest.raises(ValueError):
        EWS(J, N=2, leaf="jordan_closed", jordan_flows=True)
    with pytest.raises(ValueError):
        EWS(A, N=2, combine="block_kernel", jordan_flows=True)
    with pytest.raises(ValueError):
        AParamJordanRepeated([2], ["complex"], [torch.zeros(2)])
    # the plane leaf (ews/core/leaf.py:116-136): depths 1-2, even dimension; the dense engine runs it
    assert EWS(A, N=2, reweighting_mode="displacement_uniform", leaf="plane_closed").engine == "dense"
    with pytest.raises(NotImplementedError):
        EWS(AParamBlockDiag([torch.ones(2, 2)] * 2, [2, 2]), N=3, leaf="plane_closed")
    with pytest.raises(ValueError):
        EWS(torch.eye(3), N=2, leaf="plane_closed")
    layer = EWS(AParamEFM(torch.zeros(3)), N=2, reweighting_mode="displacement_uniform")
    assert layer.engine == "diag" and layer.block_sizes == (1, 1, 1)
    assert EWS(AParamBlockDiag([torch.ones(1, 1)] * 3, [1, 1, 1]), N=2, leaf="series", series_q=4).engine == "diag"
    assert layer.signature_dim == 3 + 9
    assert LogEWS(A, N=2, reweighting_mode="displacement_uniform").log_signature_dim == 4 + 6


def test_readout_validation():
    layer = EWS(AParamDiag(torch.ones(4)), N=2, reweighting_mode="displacement_uniform")
    with pytest.raises(ValueError):
        layer(torch.zeros(5, 4), torch.zeros(5), readout="bogus")
    with pytest.raises(ValueError):
        layer(torch.zeros(5, 4), torch.zeros(5), readout="mean", output_format="list")
    with pytest.raises(ValueError):
        layer(torch.zeros(2, 5, 4), torch.zeros(5))
    with pytest.raises(ValueError):
        layer(torch.zeros(5, 4), torch.zeros(4))


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: the engine refuses host tensors."""
    layer = EWS(AParamDiag(torch.ones(4)), N=2, reweighting_mode="displacement_uniform")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        layer(torch.zeros(2, 5, 4), torch.arange(5.0).expand(2, 5))


def test_lift_full_matrix():
    m = torch.randn(3, 2)
    b = B(m, preserve_first_channel=True)
    x = torch.randn(7, 3)
    assert torch.allclose(b(x), x @ b.full_matrix().T)
    b2 = B(torch.randn(4, 3), preserve_first_channel=False)
    assert torch.allclose(b2(x), x @ b2.full_matrix().T)
