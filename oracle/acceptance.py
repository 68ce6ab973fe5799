"""Seeded input regimes and acceptance rules for the attention path (TEST INFRASTRUCTURE ONLY).

Restates foreswe_bench/attn_check.py:
  * ``case_inputs``  (:20-45) -- six synthetic regimes drawn from one torch.Generator in the reference's order
    (q, k, v ~ N(0,1); dist ~ U(0,1500); ang ~ U(0,20); alpha, beta, gamma = 0.31, -0.21, 0.20), so the same seed
    gives bit-identical inputs to the reference's;
  * ``evaluate``     (:68-81) -- the 10x rule: for the output and every gradient, the candidate's max-abs error
    against the float64 oracle must be <= 10 x eager's max-abs error (same precision, same dO) + 1e-7*max|ref|;
  * ``err``          (:57-65) -- max-abs, rel-L2 and cosine against the reference.

The path's stated tolerances (rel-L2 vs the FP32 operator: 5e-4 for TF32, 8e-3 for BF16) are ``REL_L2_TOL``.
Eager's own error is computed here on the CPU: fp32 directly, TF32 with operands rounded to TF32
(``geo_attention.tf32_matmul``), which is the error model of cuBLAS TF32.
"""
import math

import torch

from . import geo_attention as ga

KEYS = ("output", "dQ", "dK", "dV", "dalpha", "dbeta", "dgamma")
FACTOR, FLOOR = 10.0, 1e-7
REL_L2_TOL = {"tf32": 5e-4, "bf16": 8e-3, "fp32": 5e-4}
CASES = ("random", "near_one_hot", "uniform", "moderate", "wide_signed", "large_alpha")


def case_inputs(name, B=1, H=4, N=128, D=192, seed=0):
    """CPU fp32 inputs [q, k, v, dist, ang, alpha, beta, gamma] for one of the six regimes."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, N, D, generator=g) for _ in range(3))
    dist = torch.rand(N, N, generator=g) * 1500
    ang = torch.rand(N, N, generator=g) * 20
    abg = [0.31, -0.21, 0.20]
    if name == "random":
        pass
    elif name == "near_one_hot":      # score std ~ 400: saturated rows
        q, k = q * 20, k * 20
    elif name == "uniform":           # Q = 0: P1 exactly uniform
        q = torch.zeros_like(q)
    elif name == "moderate":          # score std ~ 4
        q, k = q * 2, k * 2
    elif name == "wide_signed":       # scores spanning +-thousands with a large positive offset per row
        q, k = q * 12, k * 12
        q[..., 0] += 50.0
        k[..., 0] += 50.0
    elif name == "large_alpha":
        q, k = q * 8, k * 8
        abg = [3.0, -1.5, 2.5]
    else:
        raise ValueError(name)
    a, b, c = (torch.tensor([x]) for x in abg)
    return [q, k, v, dist, ang, a, b, c]


def grad_seed_do(shape, seed=1234):
    """dO drawn like attn_check.evaluate (:70-71)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g)


def err(a, ref):
    a64, r64 = a.double().cpu(), ref.double().cpu()
    rn = torch.linalg.vector_norm(r64).item()
    an = torch.linalg.vector_norm(a64).item()
    dot = float((a64 * r64).sum())
    return dict(max_abs=(a64 - r64).abs().max().item(),
                rel_l2=torch.linalg.vector_norm(a64 - r64).item() / rn if rn else math.nan,
                ref_norm=rn, ref_max_abs=r64.abs().max().item(),
                cosine=dot / (an * rn) if an and rn else math.nan)


def reference(inputs, do):
    """float64 oracle outputs and gradients."""
    return ga.grads(*inputs, do, dtype=torch.float64)


def eager(inputs, do, prec):
    """Eager operator's own result at the given precision ("fp32", "tf32" or "bf16": every matmul operand rounded to
    bf16, fp32 elsewhere, as under autocast), evaluated on the CPU."""
    mm = {"tf32": ga.tf32_matmul, "bf16": ga.bf16_matmul}.get(prec, torch.matmul)
    return ga.grads(*inputs, do, dtype=torch.float32, matmul=mm)


def evaluate(cand, inputs, do, prec="fp32", ref=None, eag=None):
    """Apply the 10x-eager rule to ``cand`` (a dict like grads()) and report rel-L2 per key."""
    ref = reference(inputs, do) if ref is None else ref
    eag = eager(inputs, do, prec) if eag is None else eag
    out = {}
    for k in KEYS:
        ec, ee = err(cand[k], ref[k]), err(eag[k], ref[k])
        bound = FACTOR * ee["max_abs"] + FLOOR * ec["ref_max_abs"]
        out[k] = dict(candidate=ec, eager=ee, bound=bound, passed=ec["max_abs"] <= bound,
                      ratio_to_eager=ec["max_abs"] / ee["max_abs"] if ee["max_abs"] else math.inf)
    return out
