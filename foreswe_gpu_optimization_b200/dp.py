"""Data parallelism over issue dates for the geo-attention path (one process per GPU).

Issue dates (and weekly time steps) are independent attentions over the same station set, so the batch is split
contiguously across ranks with no exchange during forward or backward. The only collective is the sum of the
bias-parameter gradients (3 x n_params floats) once per step, which ``allreduce_bias_grads`` packs into one
buffer. The reference runs one process on one GPU (foreswe_bench/runtime.py:76-80); this module is new.
"""
import torch
import torch.distributed as dist


def shard(n_total, world, rank):
    """Contiguous [start, stop) of the issue dates owned by `rank` (sizes differ by at most one)."""
    if not (0 <= rank < world) or n_total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_bias_grads(params, group=None):
    """Sum the .grad of alpha, beta, gamma over all ranks in one all-reduce (in place)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return
    grads = [p.grad for p in params]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def agreed_count(est_ms, seconds, group=None, device=None):
    """The number of repetitions of a step estimated at `est_ms` that fill about `seconds`, identical on every rank.

    A loop whose body holds a collective must run the same number of times on every rank, or the ranks' collectives
    stop pairing up and the job waits until the process-group timeout. Per-rank timings differ slightly, so the
    count is taken from the MAX of the estimates over the ranks (one all-reduce) before any rank starts the loop."""
    est = float(est_ms)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        t = torch.tensor([est], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        est = float(t.item())
    return int(seconds * 1000.0 / max(est, 0.05)) + 1
