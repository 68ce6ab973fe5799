"""Float32 model of the kernels' arithmetic (TEST INFRASTRUCTURE: used by tests only).

Restates in torch on the CPU the formulation that the sm_100a kernels (foreswe_gpu_optimization_b200/csrc/
geoattn_kernels.cuh) evaluate, with their rounding points, so that the numerics choices can be checked against the
float64 oracle without a GPU:

* scores in log2 units, t = acc * log2(e) / sqrt(d). Forward pass A keeps m = max t and l1 = sum 2^(t - m);
  P1 = 2^(t - m1) with m1 = m + log2 l1, the expression the backward kernels use to recompute P1;
* softmax #2 with the exact bound c = |alpha| + |beta| + |gamma| (P1, Dp, Ap lie in [0, 1]) instead of a running
  max: e = 2^(Z log2(e) - c log2(e)), pass B accumulates O += e V and l2 = sum e, O /= l2; the backward uses
  P2 = 2^(Z log2(e) - c2) with c2 = c log2(e) + log2 l2;
* backward from row records: delta2 = sum P2 dP, a = sum P2 dP P1, b = sum P2 P1, delta1 = alpha (a - delta2 b);
  dZ = P2 (dP - delta2), dS = P1 (alpha dZ - delta1); d(beta) = sum dZ Dp, d(gamma) = sum dZ Ap; d(alpha) is
  a - delta2 b per row (BF16 kernels) or sum dZ (P1 - b) from the explicit dZ (TF32 kernels, second row sweep);
* operands of each product. BF16 path: q, k, v, dO in bf16, the forward's e, P2 and dS rounded to bf16 for their
  MMAs, the prior stored as fp16 pairs, outputs rounded to bf16. TF32 path: QK^T and dO V^T as 3-term split
  products (hi hi + hi lo + lo hi of round-to-nearest TF32 planes), P V, dS K, P2^T dO and dS^T Q with 1-term
  round-to-nearest TF32 operands, the prior in fp32.

Accumulation is float32 in torch's CPU order (the tensor cores sum in another order; both are fp32 sums), and exp2 /
log2 are torch's (the kernels use the hardware approximations, a few fp32 ulps apart).
"""
import math

import torch

from oracle.geo_attention import round_tf32

LOG2E = 1.4426950408889634


def _bf16(x):
    return x.to(torch.bfloat16).float()


def _split(x):
    hi = round_tf32(x)
    return hi, round_tf32(x - hi)


def matmul(a, b, kind):
    """a @ b in fp32 with the kernels' operand rounding: "bf16", "tf32" (1 term) or "tf32x3" (3-term split)."""
    a, b = a.float(), b.float()
    if kind == "bf16":
        return _bf16(a) @ _bf16(b)
    if kind == "tf32":
        return round_tf32(a) @ round_tf32(b)
    if kind == "tf32x3":
        ah, al = _split(a)
        bh, bl = _split(b)
        return ah @ bh + (ah @ bl + al @ bh)
    raise ValueError(kind)


def _per_head(x, H):
    x = x.reshape(-1).float()
    return x.reshape(1, -1, 1, 1) if x.numel() == H else x.reshape(1, 1, 1, 1)


def grads(q, k, v, dist, ang, alpha, beta, gamma, do, path, score_terms=3, dp_terms=None, prior_fp16=None,
          dalpha_form=None, row_sums="tiles", fwd_p1="exact"):
    """Output and gradients (dict keyed like the oracle's grads) of the kernels' formulation on the CPU.

    path: "bf16" or "tf32". score_terms: TF32 terms of QK^T and (unless dp_terms says otherwise) dO V^T, 3 as in
    the kernels or 1 (a cheaper variant, for comparison).
    prior_fp16: store the prior as fp16 (default: the path's choice, True for bf16). dalpha_form: "a-d2b" or
    "dz" (default: the path's choice). row_sums: "tiles" (the kernels: delta2 and a from the recomputed tiles) or
    "output" (a variant without the BF16 row pass's sweep: delta2 = rowsum(dO O) from the stored output and
    a = rowsum(dO O') with O' = (P2 P1) V accumulated by the forward, both stored in the output dtype).
    fwd_p1: "exact" (the forward recomputes P1 = 2^(t - m1) from a second score pass) or "fp16_chunks" (a single
    score pass: 2^(t - m_c) against the running row max m_c after each 128-key chunk, kept as fp16 until pass B
    scales it by 2^(m_c - m1)); the backward recomputes P1 from the scores either way."""
    bf = path == "bf16"
    prior_fp16 = bf if prior_fp16 is None else prior_fp16
    dalpha_form = ("a-d2b" if bf else "dz") if dalpha_form is None else dalpha_form
    score_kind = "bf16" if bf else ("tf32x3" if score_terms == 3 else "tf32")
    dp_terms = score_terms if dp_terms is None else dp_terms
    dp_kind = "bf16" if bf else ("tf32x3" if dp_terms == 3 else "tf32")
    prod_kind = "bf16" if bf else "tf32"
    q, k, v, do = (_bf16(t) if bf else t.float() for t in (q, k, v, do))
    H, D = q.shape[1], q.shape[-1]
    a, b, g = (_per_head(t, H) for t in (alpha, beta, gamma))
    dp = (1.0 / (1.0 + dist.double())).float()
    ap = (1.0 / (1.0 + ang.double())).float()
    if prior_fp16:
        dp, ap = dp.half().float(), ap.half().float()
    sc = LOG2E / math.sqrt(D)
    inv_sqrt_d = 1.0 / math.sqrt(D)
    c = a.abs() + b.abs() + g.abs()

    # forward
    acc = matmul(q, k.transpose(-1, -2), score_kind)
    t = acc * sc
    m = t.amax(-1, keepdim=True)
    l1 = torch.exp2(t - m).sum(-1, keepdim=True)
    m1 = m + torch.log2(l1)
    p1 = torch.exp2(t - m1)
    zl = (a * p1 + b * dp + g * ap) * LOG2E
    if fwd_p1 == "fp16_chunks":
        p1f = torch.empty_like(t)
        run = torch.full_like(m, -math.inf)
        for c0 in range(0, t.shape[-1], 128):
            blk = t[..., c0:c0 + 128]
            run = torch.maximum(run, blk.amax(-1, keepdim=True))
            p1f[..., c0:c0 + 128] = torch.exp2(blk - run).half().float() * torch.exp2(run - m1)
        zl_f = (a * p1f + b * dp + g * ap) * LOG2E
    else:
        zl_f = zl
    e = torch.exp2(zl_f - c * LOG2E)
    l2 = e.sum(-1, keepdim=True)
    o = matmul(e, v, prod_kind) / l2
    c2 = c * LOG2E + torch.log2(l2)

    # backward (P1, P2 recomputed from the row statistics)
    p2 = torch.exp2(zl - c2)
    dpm = matmul(do, v.transpose(-1, -2), dp_kind)
    if row_sums == "tiles":
        delta2 = (p2 * dpm).sum(-1, keepdim=True)
        ra = (p2 * dpm * p1).sum(-1, keepdim=True)
    else:
        store = _bf16 if bf else (lambda x: x)
        delta2 = (do * store(o)).sum(-1, keepdim=True)
        ra = (do * store(matmul(p2 * p1, v, prod_kind))).sum(-1, keepdim=True)
    rb = (p2 * p1).sum(-1, keepdim=True)
    delta1 = a * (ra - delta2 * rb)
    dz = p2 * (dpm - delta2)
    ds = p1 * (a * dz - delta1)
    dv = matmul(p2.transpose(-1, -2), do, prod_kind)
    dk = matmul(ds.transpose(-1, -2), q, prod_kind) * inv_sqrt_d
    dq = matmul(ds, k, prod_kind) * inv_sqrt_d
    if dalpha_form == "a-d2b":
        dal_rows = ra - delta2 * rb
    else:
        dal_rows = (dz * (p1 - rb)).sum(-1, keepdim=True)
    red = (0, 2, 3) if a.shape[1] == H and H > 1 else (0, 1, 2, 3)
    dal = dal_rows.double().sum(red)
    dbe = (dz * dp).double().sum(red)
    dga = (dz * ap).double().sum(red)
    out = dict(output=o, dQ=dq, dK=dk, dV=dv)
    if bf:
        out = {key: _bf16(val) for key, val in out.items()}
    out.update(dalpha=dal.float().reshape(alpha.shape), dbeta=dbe.float().reshape(beta.shape),
               dgamma=dga.float().reshape(gamma.shape))
    return out
