"""Attention fwd+bwd over issue dates that live in pinned host memory, with the host->device copies overlapped.

A training loop that keeps its batches on the host pays one PCIe copy of q, k, v and dO per step. Issue dates are
independent attentions, so the batch can be cut into slices along B: slice i+1 is copied on a side stream while
slice i runs forward and backward on the caller's stream (two device buffers per operand, reused in turn). The
bias-parameter gradients accumulate over the slices through autograd, exactly as for one call over the whole batch
(up to the order of the float32 additions of the per-slice sums).
"""
from __future__ import annotations

import torch

from .geo_attention_v2 import geo_attention

_STREAMS: dict = {}


def _copy_stream(device: torch.device) -> torch.cuda.Stream:
    s = _STREAMS.get(device)
    if s is None:
        s = _STREAMS[device] = torch.cuda.Stream(device)
    return s


class HostBatchPipeline:
    """Reusable device buffers and events for `step` on batches of a fixed shape [B, H, N, D]."""

    def __init__(self, shape, dtype, device, slices: int = 8):
        B = shape[0]
        if slices < 1 or slices > B:
            raise ValueError("slices must be in [1, B]")
        self.device = torch.device(device)
        self.bounds = [(B * i // slices, B * (i + 1) // slices) for i in range(slices)]
        rows = max(s1 - s0 for s0, s1 in self.bounds)
        self.bufs = [[torch.empty((rows,) + tuple(shape[1:]), dtype=dtype, device=self.device) for _ in range(4)]
                     for _ in range(2)]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]

    def step(self, hq, hk, hv, hdo, geometry, alpha, beta, gamma):
        """Forward and backward of every issue date of the pinned host tensors hq, hk, hv (and dO = hdo).

        Gradients of alpha, beta, gamma accumulate into their `.grad`; returns the number of slices run.
        """
        for h in (hq, hk, hv, hdo):
            if h.device.type != "cpu" or not h.is_pinned():
                raise ValueError("host inputs must be pinned CPU tensors")
        compute = torch.cuda.current_stream(self.device)
        side = _copy_stream(self.device)
        for i in range(2):
            self.free[i].record(compute)
        for i, (s0, s1) in enumerate(self.bounds):
            slot, n = i % 2, s1 - s0
            with torch.cuda.stream(side):
                side.wait_event(self.free[slot])          # the compute that last read this slot is done
                for dst, src in zip(self.bufs[slot], (hq, hk, hv, hdo)):
                    dst[:n].copy_(src[s0:s1], non_blocking=True)
                self.ready[slot].record(side)
            compute.wait_event(self.ready[slot])
            q, k, v, do = (t[:n] for t in self.bufs[slot])
            q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = geo_attention(q, k, v, geometry, alpha, beta, gamma)
            o.backward(do)
            self.free[slot].record(compute)
        return len(self.bounds)
