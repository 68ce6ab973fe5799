"""The geo-attention forward and backward as torch.library custom ops, for compiled and graph-captured steps.

`torch.compile` cannot trace the ctypes calls of FusedGeoAttentionV2 and breaks the graph there. Registered as
custom ops (`foreswe_geoattn::fwd`, `foreswe_geoattn::bwd`) the kernels are opaque nodes of the compiled graph: the
fake implementations give output shapes and strides, `register_autograd` connects the backward, and alpha/beta/gamma
reach the op as one differentiable concatenation, so their gradients flow through autograd. Same kernels and the
same results as FusedGeoAttentionV2 (the reference's call path keeps using that Function).
"""
from __future__ import annotations

import torch

from . import geo_attention_v2 as _gv2
from .geometry import StationGeometry


@torch.library.custom_op("foreswe_geoattn::fwd", mutates_args=(), device_types="cuda")
def geoattn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prior: torch.Tensor, abg: torch.Tensor,
                per_head: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(O, row statistics) for q, k, v [B, H, N, D]; abg = alpha, beta, gamma concatenated (fp32)."""
    return _gv2._forward(q, k, v, prior, abg.contiguous(), per_head)


@geoattn_fwd.register_fake
def _(q, k, v, prior, abg, per_head):
    B, H, N, _ = q.shape
    return torch.empty_like(q), q.new_empty((3 * B * H * N,), dtype=torch.float32)


@torch.library.custom_op("foreswe_geoattn::bwd", mutates_args=(), device_types="cuda")
def geoattn_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, do: torch.Tensor,
                prior: torch.Tensor, abg: torch.Tensor, stats: torch.Tensor,
                per_head: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dQ, dK, dV, d(alpha, beta, gamma)) for the forward's inputs, output and row statistics."""
    return _gv2._backward(q, k, v, o, do, prior, abg.contiguous(), stats, per_head)


@geoattn_bwd.register_fake
def _(q, k, v, o, do, prior, abg, stats, per_head):
    nabg = q.shape[1] if per_head else 1
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            q.new_empty((3 * nabg,), dtype=torch.float32))


def _setup_context(ctx, inputs, output):
    q, k, v, prior, abg, per_head = inputs
    o, stats = output
    ctx.save_for_backward(q, k, v, o, prior, abg, stats)
    ctx.per_head = per_head


def _backward(ctx, do, dstats):
    q, k, v, o, prior, abg, stats = ctx.saved_tensors
    dq, dk, dv, dabg = geoattn_bwd(q, k, v, o, do, prior, abg, stats, ctx.per_head)
    return dq, dk, dv, None, dabg.to(abg.dtype), None


geoattn_fwd.register_autograd(_backward, setup_context=_setup_context)


def geo_attention_op(q, k, v, prior, alpha, beta, gamma):
    """Drop-in for FusedGeoAttentionV2.apply(q, k, v, prior, alpha, beta, gamma) through the custom ops.

    alpha, beta, gamma: 1 or H entries each (per-head when H); `prior` from StationGeometry.prior or
    prior_from_dense for q's dtype."""
    H = q.shape[1]
    n = alpha.numel()
    if beta.numel() != n or gamma.numel() != n or n not in (1, H):
        raise ValueError("alpha, beta, gamma must all have 1 or H entries")
    per_head = int(n == H and H > 1)
    abg = torch.cat([alpha.reshape(-1), beta.reshape(-1), gamma.reshape(-1)]).to(device=q.device,
                                                                                 dtype=torch.float32)
    o, _ = geoattn_fwd(q, k, v, prior, abg, per_head)
    return o


def geo_attention_compiled(q, k, v, geometry: StationGeometry, alpha, beta, gamma, *, precision=None):
    """Coordinate form of geo_attention_op (the prior comes from `geometry`); `precision` as in geo_attention."""
    cd = _gv2._compute_dtype(q, precision, "reference")
    qc, kc, vc = (t if t.dtype == cd else t.to(cd) for t in (q, k, v))
    o = geo_attention_op(qc, kc, vc, geometry.prior(cd), alpha, beta, gamma)
    return o if o.dtype == q.dtype else o.to(q.dtype)
