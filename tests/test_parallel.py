"""Multi-process data parallelism on CPU (gloo, world size 2): batch sharding, the single gradient
allreduce, and detection of a rank that fails between steps.

The scan itself runs on the GPU engines; here the per-rank work is the float64 oracle on each rank's
shard, which is enough to check the host logic the GPU runs use (parallel.shard_range and
parallel.allreduce_gradients): the allreduced shard gradients must equal the full-batch gradients.
"""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from exponentially_weighted_signature_b200.parallel import allreduce_gradients, shard_range
from oracle import ews_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    g = torch.Generator().manual_seed(0)
    B, T, d, N = 5, 12, 3, 4
    path = torch.cumsum(torch.randn(B, T + 1, d, generator=g, dtype=torch.float64) / T**0.5, 1)
    clock = torch.linspace(0, 1, T + 1, dtype=torch.float64).expand(B, T + 1).contiguous()
    lam = torch.exp(torch.rand(N, generator=g, dtype=torch.float64) * 2 - 1)
    lift = torch.randn(N, d, generator=g, dtype=torch.float64) / d**0.5
    w = torch.randn(B, T, 1 + N + N * N, generator=g, dtype=torch.float64)
    return path, clock, lam, lift, w


def _grads(path, clock, lam, lift, w):
    L = lam.clone().requires_grad_(True)
    Bm = lift.clone().requires_grad_(True)
    out = O.ews_layer(O.lift(path, Bm), clock, torch.diag(L), 2, series_q=6, reweighting_mode="displacement_uniform")
    (out * w).sum().backward()
    return L, Bm


def _worker(rank, world, port, result_dir, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    status = "ok"
    try:
        path, clock, lam, lift, w = _problem()
        s0, s1 = shard_range(path.shape[0], rank, world)
        L, Bm = _grads(path[s0:s1], clock[s0:s1], lam, lift, w[s0:s1])
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 between steps")
        allreduce_gradients([L, Bm])
        torch.save({"lam": L.grad, "lift": Bm.grad}, os.path.join(result_dir, f"rank{rank}.pt"))
    except Exception as exc:  # recorded for the parent; rank 1's injected failure lands here too
        status = f"error: {type(exc).__name__}: {exc}"
        with open(os.path.join(result_dir, f"rank{rank}.err"), "w") as f:
            f.write(status + "\n" + traceback.format_exc())
    finally:
        if status == "ok":
            dist.destroy_process_group()


def test_shard_range_partitions_the_batch():
    for total in (1, 4, 7, 32, 1024):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_allreduced_shard_gradients_equal_full_batch(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), "ok"), nprocs=2, join=True, start_method="spawn")
    path, clock, lam, lift, w = _problem()
    L, Bm = _grads(path, clock, lam, lift, w)
    for rank in range(2):
        assert not (tmp_path / f"rank{rank}.err").exists(), (tmp_path / f"rank{rank}.err").read_text()
        got = torch.load(tmp_path / f"rank{rank}.pt")
        torch.testing.assert_close(got["lam"], L.grad, rtol=1e-12, atol=1e-12)
        torch.testing.assert_close(got["lift"], Bm.grad, rtol=1e-12, atol=1e-12)


def test_failed_rank_ends_the_collective_with_an_error(tmp_path):
    """Rank 1 raises before the allreduce (between steps, nothing in flight): rank 0's collective must
    end with an error within the process group's timeout instead of waiting for ever."""
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(2, port, str(tmp_path), "fail"), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank was still waiting after the failure"
    assert (tmp_path / "rank1.err").exists()
    assert (tmp_path / "rank0.err").exists(), "rank 0 did not see the failure"
    assert not (tmp_path / "rank0.pt").exists()
