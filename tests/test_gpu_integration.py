"""Step-level integration on the GPU: the custom ops under torch.library.opcheck and torch.compile, and the model
call site (split_heads views in, combine_heads out) through patch_model."""
import math

import pytest
import torch
import torch.nn as nn

from helpers import attn_inputs, rel_l2, stations

pytestmark = pytest.mark.gpu


def test_custom_op_opcheck():
    import foreswe_gpu_optimization_b200 as g
    B, H, N, D = 1, 2, 128, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=3, dtype=torch.bfloat16)
    geom = g.StationGeometry(*stations(N, 4), device="cuda")
    prior = geom.prior(torch.bfloat16)
    abg = torch.cat([a, b, c]).cuda().requires_grad_(True)
    args = (q.cuda().requires_grad_(True), k.cuda().requires_grad_(True), v.cuda().requires_grad_(True), prior, abg, 1)
    torch.library.opcheck(torch.ops.foreswe_geoattn.fwd.default, args,
                          test_utils=("test_schema", "test_faketensor", "test_autograd_registration"))


def test_compiled_fullgraph_matches_eager():
    import foreswe_gpu_optimization_b200 as g
    B, H, N, D = 2, 4, 256, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=8, dtype=torch.bfloat16)
    geom = g.StationGeometry(*stations(N, 9), device="cuda")

    def step(q, k, v, a, b, c):
        o = g.geo_attention_compiled(q, k, v, geom, a, b, c)
        return (o.float() * do.cuda().float()).sum()

    def run(fn):
        x = [t.cuda().requires_grad_(True) for t in (q, k, v, a, b, c)]
        loss = fn(*x)
        loss.backward()
        return [loss.detach()] + [t.grad for t in x]

    eager = run(step)
    compiled = run(torch.compile(step, backend="aot_eager", fullgraph=True))
    for e, c_ in zip(eager, compiled):
        assert torch.equal(e, c_)
    # and the custom-op path gives the autograd Function's results
    ref = [t.cuda().requires_grad_(True) for t in (q, k, v, a, b, c)]
    (g.geo_attention(*ref[:3], geom, *ref[3:]).float() * do.cuda().float()).sum().backward()
    for r, c_ in zip(ref, compiled[1:]):
        assert torch.equal(r.grad, c_)


class _MHA(nn.Module):
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


class _Encoder(nn.Module):
    def __init__(self, d_model, heads, layers):
        super().__init__()
        self.encoder_layers = nn.ModuleList(nn.Module() for _ in range(layers))
        for layer in self.encoder_layers:
            layer.self_attn = _MHA(d_model, heads)

    def forward(self, x, d, a):
        for layer in self.encoder_layers:
            x = x + layer.self_attn(x, d, a)
        return x


@pytest.mark.parametrize("autocast", [False, True], ids=["fp32-tf32", "bf16-autocast"])
def test_patch_model_call_site(autocast):
    """The patched encoder matches the unpatched one: tightly in fp32 (the op's TF32 path), loosely under bf16
    autocast (bf16 projections in two layers dominate the difference there)."""
    import foreswe_gpu_optimization_b200 as g
    torch.manual_seed(0)
    B, N, H, D = 2, 192, 4, 64
    model = _Encoder(H * D, H, 2).cuda()
    lat, lon, el = stations(N, 12)
    geom = g.StationGeometry(lat, lon, el, device="cuda")
    dist, ang = geom.distance_and_angularity()
    x = torch.randn(B, N, H * D, device="cuda") * 0.5
    ref_model = _Encoder(H * D, H, 2).cuda()
    ref_model.load_state_dict(model.state_dict())
    y_ref = ref_model(x, dist, ang)                      # fp32 eager (the production method)
    y_ref.square().sum().backward()
    g.patch_model(model, geometry=geom)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        y = model(x, dist, ang)
    y.float().square().sum().backward()
    tol_o, tol_g = (2e-2, 0.15) if autocast else (2e-3, 5e-3)
    assert rel_l2(y.float(), y_ref) < tol_o
    for (n, p), (_, pr) in zip(model.named_parameters(), ref_model.named_parameters()):
        assert torch.isfinite(p.grad).all(), n
        if n.endswith("W_k.bias"):
            # adds q.b_k to every score of a row: softmax is shift-invariant, the exact gradient is zero and both
            # sides hold only rounding noise
            continue
        assert rel_l2(p.grad, pr.grad) < tol_g, n
    g.patch_model(model, "eager")                         # restores the module's own method
    assert "scaled_dot_product_attention" not in model.encoder_layers[0].self_attn.__dict__
