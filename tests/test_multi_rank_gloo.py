"""Data-parallel host logic on CPU ranks (gloo, world size 2): sharding, the bias-gradient all-reduce, and a rank
that fails before the collective surfacing as an error on its peer (short process-group timeout)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from foreswe_gpu_optimization_b200.dp import allreduce_bias_grads, shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_covers_batch_exactly():
    for n in (0, 1, 7, 256, 257):
        for world in (1, 2, 3, 8):
            spans = [shard(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        from oracle import geo_attention as oga
        B, H, N, D = 4, 2, 12, 8
        g = torch.Generator().manual_seed(0)
        q, k, v, do = (torch.randn(B, H, N, D, generator=g, dtype=torch.float64) for _ in range(4))
        dmat = torch.rand(N, N, generator=g, dtype=torch.float64) * 100
        amat = torch.rand(N, N, generator=g, dtype=torch.float64) * 10
        params = [torch.tensor([0.4, 0.7], dtype=torch.float64, requires_grad=True),
                  torch.tensor([-0.2, 0.1], dtype=torch.float64, requires_grad=True),
                  torch.tensor([0.3, -0.5], dtype=torch.float64, requires_grad=True)]
        s0, s1 = shard(B, world, rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the all-reduce")
        o = oga.forward(q[s0:s1], k[s0:s1], v[s0:s1], dmat, amat, *params)
        o.backward(do[s0:s1])
        allreduce_bias_grads(params)
        full = [p.detach().clone().requires_grad_(True) for p in params]
        oga.forward(q, k, v, dmat, amat, *full).backward(do)
        out[rank] = all(torch.allclose(p.grad, f.grad, rtol=1e-12, atol=1e-14) for p, f in zip(params, full))
    except RuntimeError as e:
        out[rank] = "error: " + str(e)[:80]
    finally:
        dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(60)
            assert p.exitcode is not None, "a rank did not exit"
        return dict(out)


def test_sharded_bias_grads_allreduce_equals_full_batch():
    out = _run("ok")
    assert out == {0: True, 1: True}


def test_failed_rank_surfaces_as_error_on_peer():
    out = _run("fail")
    assert str(out[1]).startswith("error")
    assert str(out[0]).startswith("error")     # the peer's all-reduce ends with an error, not a hang


def _count_worker(rank, world, port, skew, out):
    """Each rank sizes a loop of collectives from its own (skewed) step-time estimate through `agreed_count`, then
    runs it: every iteration is an all-reduce, as every replay of the benchmark's captured step is."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        from foreswe_gpu_optimization_b200.dp import agreed_count
        est_ms = 0.775 * (1.0 + skew * rank)            # per-rank timings differ by a fraction of a percent
        local = int(300.0 / est_ms) + 1                  # what a rank would pick on its own
        n = agreed_count(est_ms, 0.3)
        one = torch.ones(1)
        issued = 0
        for _ in range(n):
            dist.all_reduce(one.clone())
            issued += 1
        counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(counts, torch.tensor([issued]))
        out[rank] = (local, n, [int(c.item()) for c in counts])
    except RuntimeError as e:
        out[rank] = "error: " + str(e)[:80]
    finally:
        dist.destroy_process_group()


def test_preroll_count_agreed_over_ranks_with_skewed_timings():
    """Four CPU ranks whose own estimates would give different loop lengths issue the same number of collectives
    once the count comes from `agreed_count` (the max estimate over the ranks)."""
    world = 4
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        procs = [ctx.Process(target=_count_worker, args=(r, world, port, 0.004, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode is not None, "a rank did not exit"
        res = dict(out)
    assert all(isinstance(res[r], tuple) for r in range(world)), res
    locals_ = {res[r][0] for r in range(world)}
    assert len(locals_) > 1, "the skew must make the ranks' own counts differ, or the test shows nothing"
    agreed = {res[r][1] for r in range(world)}
    assert len(agreed) == 1, res
    n = agreed.pop()
    assert n == min(locals_)          # sized from the slowest rank's estimate
    for r in range(world):
        assert res[r][2] == [n] * world, res[r]
