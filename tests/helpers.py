"""Shared helpers for the parity tests: seeded inputs in the configurations' distributions and error metrics."""
import math

import numpy as np
import torch
import torch.nn as nn

from oracle import geometry as ogeo

TOL = {torch.bfloat16: 8e-3, torch.float32: 5e-4}   # rel-L2 vs the FP32 operator (the path's stated tolerances)
KEYS = ("output", "dQ", "dK", "dV", "dalpha", "dbeta", "dgamma")


def stations(n, seed):
    """lat ~ U(35,49) deg, lon ~ U(-124,-104) deg, elevation ~ U(500,3500) m (converted to feet)."""
    rng = np.random.default_rng(seed)
    lat = rng.uniform(35.0, 49.0, n)
    lon = rng.uniform(-124.0, -104.0, n)
    elev_ft = ogeo.metres_to_feet(rng.uniform(500.0, 3500.0, n))
    return lat, lon, elev_ft


def attn_inputs(B, H, N, D, seed=0, qscale=1.0, per_head=True, dtype=torch.float32):
    """q, k, v ~ N(0,1) * D^-0.25 (q optionally scaled); alpha_h ~ U(0.1,1), beta_h, gamma_h ~ N(0, 0.5)."""
    g = torch.Generator().manual_seed(seed)
    s = D ** -0.25
    q, k, v = (torch.randn(B, H, N, D, generator=g) * s for _ in range(3))
    q = q * qscale
    nh = H if per_head else 1
    a = torch.rand(nh, generator=g) * 0.9 + 0.1
    b = torch.randn(nh, generator=g) * 0.5
    c = torch.randn(nh, generator=g) * 0.5
    do = torch.randn(B, H, N, D, generator=g)
    q, k, v, do = (t.to(dtype) for t in (q, k, v, do))
    return q, k, v, a, b, c, do


def dense_geometry(lat, lon, elev_ft):
    d, a = ogeo.distance_and_angularity(lat, lon, elev_ft)
    return torch.from_numpy(d).float(), torch.from_numpy(a).float()


def rel_l2(x, ref):
    x, ref = x.double().cpu(), ref.double().cpu()
    n = torch.linalg.vector_norm(ref).item()
    return torch.linalg.vector_norm(x - ref).item() / n if n else torch.linalg.vector_norm(x).item()


def run_device(fn, q, k, v, a, b, c, do, **kw):
    """Forward + backward of a device op; returns dict of CPU results keyed like KEYS."""
    dev = torch.device("cuda")
    x = [t.to(dev).detach().requires_grad_(True) for t in (q, k, v, a, b, c)]
    o = fn(x[0], x[1], x[2], *x[3:], **kw)
    o.backward(do.to(dev))
    torch.cuda.synchronize()
    return dict(output=o.detach().cpu(), dQ=x[0].grad.cpu(), dK=x[1].grad.cpu(), dV=x[2].grad.cpu(),
                dalpha=x[3].grad.cpu(), dbeta=x[4].grad.cpu(), dgamma=x[5].grad.cpu())


class MHA(nn.Module):
    """Minimal module with the reference's attention call site (custom_encoder_model.py:7-58): W_q/W_k/W_v
    projections, split_heads views, the attention core, combine_heads, W_o."""

    def __init__(self, d_model, heads):
        super().__init__()
        self.d_model, self.num_heads, self.d_k = d_model, heads, d_model // heads
        self.alpha, self.beta, self.gamma = (nn.Parameter(torch.tensor([x])) for x in (0.7, 0.4, -0.3))
        self.W_q, self.W_k, self.W_v, self.W_o = (nn.Linear(d_model, d_model) for _ in range(4))

    def scaled_dot_product_attention(self, Q, K, V, distances, angularities, mask=None):
        s = torch.softmax(torch.matmul(Q, K.transpose(-2, -1)) / math.sqrt(self.d_k), dim=-1)
        z = self.alpha * s + self.beta / (1 + distances) + self.gamma / (1 + angularities)
        return torch.matmul(torch.softmax(z, dim=-1), V)

    def split_heads(self, x):
        B, N, _ = x.size()
        return x.view(B, N, self.num_heads, self.d_k).transpose(1, 2)

    def combine_heads(self, x):
        B, _, N, _ = x.size()
        return x.transpose(1, 2).contiguous().view(B, N, self.d_model)

    def forward(self, x, distances, angularities):
        Q, K, V = (self.split_heads(w(x)) for w in (self.W_q, self.W_k, self.W_v))
        return self.W_o(self.combine_heads(self.scaled_dot_product_attention(Q, K, V, distances, angularities)))


class Encoder(nn.Module):
    def __init__(self, d_model, heads, layers):
        super().__init__()
        self.encoder_layers = nn.ModuleList(nn.Module() for _ in range(layers))
        for layer in self.encoder_layers:
            layer.self_attn = MHA(d_model, heads)

    def forward(self, x, d, a):
        for layer in self.encoder_layers:
            x = x + layer.self_attn(x, d, a)
        return x
