"""Geo-biased station attention oracle (torch on the CPU, float64 by default).

Operator (fore_swe/custom_encoder_model.py:25-39; identical to foreswe_bench/geo_attention.py:311-319):

    S  = Q K^T / sqrt(d)                 (custom_encoder_model.py:26)
    P1 = softmax(S)                      (:30)
    Dp = 1 / (1 + dist),  Ap = 1 / (1 + ang)        (:32-33)
    Z  = alpha*P1 + beta*Dp + gamma*Ap   (:35)
    P2 = softmax(Z)                      (:36)
    O  = P2 V                            (:38)

alpha, beta, gamma are per-layer scalars in the reference (custom_encoder_model.py:16-18, shape [1]). This
oracle also accepts per-head vectors of shape [H] (broadcast over [B, H, N, N]); with all H entries equal it
is the reference operator, and the per-head gradient summed over h is the reference's scalar gradient.

Gradients (the math written out in benchmarks/attention_backward_debug.py:28-47):

    dV = P2^T dO;  dP2 = dO V^T;  delta2 = rowsum(P2*dP2);  dZ = P2*(dP2 - delta2)
    dalpha = sum(dZ*P1);  dbeta = sum(dZ*Dp);  dgamma = sum(dZ*Ap)
    delta1 = alpha*rowsum(dZ*P1);  dS = P1*(alpha*dZ - delta1)
    dQ = dS K / sqrt(d);  dK = dS^T Q / sqrt(d)

``grads`` uses torch autograd on ``forward`` (what the reference's tests do, foreswe_bench/attn_check.py:48-54);
``analytic_grads`` evaluates the formulas above and is checked against autograd in the tests.

TEST INFRASTRUCTURE: used by tests and the CPU baseline only.
"""
import math

import torch


def _per_head(x, H):
    """[1] or [H] parameter -> broadcastable [1, H, 1, 1] (or [1, 1, 1, 1])."""
    x = x.reshape(-1)
    if x.numel() not in (1, H):
        raise ValueError("bias parameter must have 1 or H entries")
    return x.reshape(1, -1, 1, 1)


def prior(dist, ang):
    """Dp = 1/(1+dist), Ap = 1/(1+ang) in the dtype of the inputs (custom_encoder_model.py:32-33)."""
    return 1 / (1 + dist), 1 / (1 + ang)


def forward(q, k, v, dist, ang, alpha, beta, gamma, matmul=torch.matmul):
    """O = softmax(alpha*softmax(QK^T/sqrt d) + beta/(1+dist) + gamma/(1+ang)) V, in the inputs' dtype.

    ``matmul`` lets the acceptance rule evaluate "eager TF32" with emulated TF32 operand rounding."""
    H = q.shape[1]
    s = matmul(q, k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    p1 = torch.softmax(s, dim=-1)
    dp, ap = prior(dist, ang)
    z = _per_head(alpha, H) * p1 + _per_head(beta, H) * dp + _per_head(gamma, H) * ap
    p2 = torch.softmax(z, dim=-1)
    return matmul(p2, v)


def grads(q, k, v, dist, ang, alpha, beta, gamma, do, dtype=torch.float64, matmul=torch.matmul):
    """Output and gradients of forward() by autograd: dict(output, dQ, dK, dV, dalpha, dbeta, dgamma)."""
    x = [t.detach().to(dtype).requires_grad_(i in (0, 1, 2, 5, 6, 7))
         for i, t in enumerate((q, k, v, dist, ang, alpha, beta, gamma))]
    o = forward(*x, matmul=matmul)
    o.backward(do.to(dtype))
    return dict(output=o.detach(), dQ=x[0].grad, dK=x[1].grad, dV=x[2].grad,
                dalpha=x[5].grad, dbeta=x[6].grad, dgamma=x[7].grad)


def analytic_grads(q, k, v, dist, ang, alpha, beta, gamma, do, dtype=torch.float64):
    """The same quantities from the closed-form backward (no autograd)."""
    q, k, v, dist, ang, alpha, beta, gamma, do = (t.detach().to(dtype) for t in
                                                  (q, k, v, dist, ang, alpha, beta, gamma, do))
    H, D = q.shape[1], q.shape[-1]
    a, b, g = (_per_head(t, H) for t in (alpha, beta, gamma))
    s = q @ k.transpose(-2, -1) / math.sqrt(D)
    p1 = torch.softmax(s, dim=-1)
    dp, ap = prior(dist, ang)
    p2 = torch.softmax(a * p1 + b * dp + g * ap, dim=-1)
    o = p2 @ v
    dv = p2.transpose(-2, -1) @ do
    dp2 = do @ v.transpose(-2, -1)
    delta2 = (p2 * dp2).sum(-1, keepdim=True)
    dz = p2 * (dp2 - delta2)
    red = (0, 2, 3) if alpha.numel() == H and H > 1 else (0, 1, 2, 3)
    dalpha = (dz * p1).sum(red).reshape(alpha.shape)
    dbeta = (dz * dp).sum(red).reshape(beta.shape)
    dgamma = (dz * ap).sum(red).reshape(gamma.shape)
    delta1 = a * (dz * p1).sum(-1, keepdim=True)
    ds = p1 * (a * dz - delta1)
    dq = ds @ k / math.sqrt(D)
    dk = ds.transpose(-2, -1) @ q / math.sqrt(D)
    return dict(output=o, dQ=dq, dK=dk, dV=dv, dalpha=dalpha, dbeta=dbeta, dgamma=dgamma)


def round_tf32(x):
    """fp32 -> TF32 (10-bit mantissa) round-to-nearest, ties away from zero, as a TF32 tensor-core operand
    conversion does (the reference's _rn_tf32, foreswe_bench/geo_attention_v2.py:38-43)."""
    i = x.float().contiguous().view(torch.int32)
    return ((i + 0x1000) & -8192).view(torch.float32)


class _TF32MatMul(torch.autograd.Function):
    """Matmul whose forward and backward products all take TF32-rounded operands (eager TF32 under cuBLAS)."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return (round_tf32(a).double() @ round_tf32(b).double()).to(a.dtype)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = (round_tf32(g).double() @ round_tf32(b).double().transpose(-2, -1)).to(a.dtype)
        gb = (round_tf32(a).double().transpose(-2, -1) @ round_tf32(g).double()).to(b.dtype)
        return ga, gb


def tf32_matmul(a, b):
    """Matmul with TF32-rounded operands and a wide accumulator: the error model of eager TF32."""
    return _TF32MatMul.apply(a, b)


def round_bf16(x):
    """fp32 -> bf16 round-to-nearest-even, back in fp32 (a bf16 tensor-core operand under autocast)."""
    return x.float().to(torch.bfloat16).float()


class _BF16MatMul(torch.autograd.Function):
    """Matmul whose forward and backward products all take bf16-rounded operands with a wide accumulator: the error
    model of eager PyTorch under bf16 autocast (cuBLAS bf16 GEMMs, fp32 accumulation)."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return (round_bf16(a).double() @ round_bf16(b).double()).to(a.dtype)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = (round_bf16(g).double() @ round_bf16(b).double().transpose(-2, -1)).to(a.dtype)
        gb = (round_bf16(a).double().transpose(-2, -1) @ round_bf16(g).double()).to(b.dtype)
        return ga, gb


def bf16_matmul(a, b):
    """Matmul with bf16-rounded operands and a wide accumulator: the error model of eager bf16 autocast."""
    return _BF16MatMul.apply(a, b)
