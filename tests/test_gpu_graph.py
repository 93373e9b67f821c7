"""The engines inside a captured CUDA graph: a forward + backward of the layer is captured once, then
replayed on new inputs copied into the captured buffers; every output and gradient must equal the eager
call's bit for bit (deterministic mode, so the look-back's rounding does not depend on timing).

This is how bench.py times the training step: the library never allocates and never waits on the host,
and every launch is stream-ordered, so the whole step can be captured.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


def _layer(kind, N):
    from exponentially_weighted_signature_b200 import EWS, LogEWS, AParamDiag, AParamGeneral, AParamBlockDiag

    rng = np.random.default_rng(0)
    if kind == "diag":
        A = AParamDiag(torch.tensor(np.exp(rng.uniform(-3, 1, N)), dtype=torch.float32))
        return EWS(A, N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=4, combine="b200", combine_chunk=16)
    if kind == "diag_clock":
        A = AParamDiag(torch.tensor(np.exp(rng.uniform(-3, 1, N)), dtype=torch.float32))
        return EWS(A, N=2, reweighting_mode="displacement", leaf="series", series_q=4, combine="b200", combine_chunk=16)
    if kind == "logews":
        A = AParamDiag(torch.tensor(np.exp(rng.uniform(-4, 0, N)), dtype=torch.float32))
        return LogEWS(A, N=2, reweighting_mode="displacement_uniform", leaf="series", series_q=4, combine="b200", combine_chunk=16)
    if kind == "dense":
        A = 0.5 * np.eye(N) - 0.1 * rng.normal(size=(N, N)) / np.sqrt(N)
        return EWS(AParamGeneral(torch.tensor(A, dtype=torch.float32)), N=2, reweighting_mode="displacement_uniform",
                   leaf="series", series_q=3, combine="b200", combine_chunk=16)
    blocks = [torch.tensor([[a, w], [-w, a]], dtype=torch.float32)
              for a, w in zip(rng.uniform(0.05, 1, N // 2), rng.uniform(0, np.pi, N // 2))]
    return EWS(AParamBlockDiag(blocks, (2,) * (N // 2)), N=3, reweighting_mode="displacement", leaf="series", series_q=4,
               combine="b200", combine_chunk=16)


def _inputs(seed, B, T, d, N):
    g = torch.Generator().manual_seed(seed)
    path = torch.cumsum(torch.randn(B, T + 1, d, generator=g) / T**0.5, 1)
    steps = torch.nn.functional.softplus(torch.randn(B, T, generator=g)) / T
    clock = torch.cat([torch.zeros(B, 1), torch.cumsum(steps, 1)], 1)
    lift = torch.randn(N, d, generator=g) / d**0.5
    return path, clock, lift


@pytest.mark.parametrize("kind,N", [("diag", 16), ("diag_clock", 8), ("logews", 8), ("dense", 32), ("block", 8)])
def test_graph_replay_matches_eager(kind, N):
    _require_gpu()
    from exponentially_weighted_signature_b200.layer import configure

    B, T, d = 3, 100, 4
    readout = "terminal" if kind == "logews" else "prefix"
    layer = _layer(kind, N).to(DEV)
    params = list(layer.parameters())
    configure(deterministic=True)
    try:
        path0, clock0, lift0 = _inputs(1, B, T, d, N)
        x = path0.to(DEV)
        c = clock0.to(DEV)
        lift = torch.nn.Parameter(lift0.to(DEV))
        params.append(lift)
        with torch.no_grad():
            shape = layer(x, c, readout=readout, lift=lift).shape
        w = torch.randn(shape, generator=torch.Generator().manual_seed(2)).to(DEV)

        def step():
            out = layer(x, c, readout=readout, lift=lift)
            (out * w).sum().backward()
            return out

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                for p in params:
                    p.grad = None
                step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for p in params:
            p.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out_static = step()

        # new inputs into the captured buffers, replay
        path1, clock1, _ = _inputs(7, B, T, d, N)
        x.copy_(path1.to(DEV))
        c.copy_(clock1.to(DEV))
        graph.replay()
        torch.cuda.synchronize()
        got = [out_static.clone()] + [p.grad.clone() for p in params]

        # the eager call on the same inputs
        saved = [p.grad for p in params]
        for p in params:
            p.grad = None
        out = step()
        torch.cuda.synchronize()
        ref = [out.detach()] + [p.grad for p in params]
        for p, s in zip(params, saved):
            p.grad = s
        for a, b in zip(got, ref):
            assert a.shape == b.shape
            assert torch.equal(a, b)
        del graph
    finally:
        configure(deterministic=False)
