"""Step-level integration on the GPU: the custom ops under torch.library.opcheck and torch.compile, and the model
call site (split_heads views in, combine_heads out) through patch_model."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from helpers import MHA, Encoder, attn_inputs, rel_l2, stations

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


@pytest.mark.parametrize("autocast", [False, True], ids=["fp32-tf32", "bf16-autocast"])
def test_patch_model_call_site(autocast):
    """The patched encoder matches the unpatched one: tightly in fp32 (the op's TF32 path), loosely under bf16
    autocast (bf16 projections in two layers dominate the difference there)."""
    import foreswe_gpu_optimization_b200 as g
    torch.manual_seed(0)
    B, N, H, D = 2, 192, 4, 64
    model = Encoder(H * D, H, 2).cuda()
    lat, lon, el = stations(N, 12)
    geom = g.StationGeometry(lat, lon, el, device="cuda")
    dist, ang = geom.distance_and_angularity()
    x = torch.randn(B, N, H * D, device="cuda") * 0.5
    ref_model = Encoder(H * D, H, 2).cuda()
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


def test_compiled_inductor_fullgraph_matches_eager():
    """torch.compile with the default (Inductor) backend and fullgraph=True around the custom op: Inductor generates
    the surrounding elementwise and reduction kernels, the op stays opaque, and q, k, v, alpha, beta, gamma get the
    eager gradients bitwise (the loss, reduced by Inductor's own kernel, agrees to rounding)."""
    import foreswe_gpu_optimization_b200 as g
    B, H, N, D = 2, 4, 256, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=18, dtype=torch.bfloat16)
    geom = g.StationGeometry(*stations(N, 19), device="cuda")
    dd = do.cuda().float()

    def step(q, k, v, a, b, c):
        o = g.geo_attention_compiled(q, k, v, geom, a, b, c)
        return (o.float() * dd).sum()

    def run(fn):
        x = [t.cuda().requires_grad_(True) for t in (q, k, v, a, b, c)]
        loss = fn(*x)
        loss.backward()
        return loss.detach(), [t.grad for t in x]

    le, ge = run(step)
    torch._dynamo.reset()
    lc, gc = run(torch.compile(step, fullgraph=True))
    torch.testing.assert_close(lc, le, rtol=1e-5, atol=1e-5)
    for name, x, y in zip(("dq", "dk", "dv", "dalpha", "dbeta", "dgamma"), ge, gc):
        assert torch.equal(x, y), name


def test_whole_training_step_captured_as_one_graph():
    """The reference's G3 step (foreswe_bench/graphs.py:213-310): forward, MSE loss, backward and fused AdamW
    (capturable) of a patched two-layer encoder captured as ONE CUDA graph, warm-up effects on the weights and the
    optimizer state undone before capture. Replayed on three fresh batches it gives the losses and final weights of
    the same three steps run eagerly, bitwise."""
    import foreswe_gpu_optimization_b200 as g
    B, N, H, D = 2, 128, 4, 64
    geom = g.StationGeometry(*stations(N, 23), device="cuda")
    dist, ang = geom.distance_and_angularity()
    gen = torch.Generator().manual_seed(5)
    batches = [(torch.randn(B, N, H * D, generator=gen).cuda() * 0.5, torch.rand(B, N, H * D, generator=gen).cuda())
               for _ in range(3)]

    def make():
        torch.manual_seed(0)
        m = Encoder(H * D, H, 2).cuda()
        g.patch_model(m, geometry=geom)
        opt = torch.optim.AdamW(m.parameters(), lr=1e-3, weight_decay=1e-4, fused=True, capturable=True)
        return m, opt

    def body(m, opt, x, t):
        loss = torch.nn.functional.mse_loss(m(x, dist, ang), t)
        loss.backward()
        opt.step()
        return loss

    m_e, opt_e = make()
    losses_e = []
    for x, t in batches:
        opt_e.zero_grad(set_to_none=True)
        losses_e.append(body(m_e, opt_e, x, t).detach().clone())

    m_g, opt_g = make()
    sx, st = torch.zeros_like(batches[0][0]), torch.zeros_like(batches[0][1])
    sx.copy_(batches[0][0])
    st.copy_(batches[0][1])
    snap = [p.detach().clone() for p in m_g.parameters()]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            opt_g.zero_grad(set_to_none=True)
            body(m_g, opt_g, sx, st)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.no_grad():                      # pristine weights and a fresh optimizer state, same storage
        for p, s in zip(m_g.parameters(), snap):
            p.copy_(s)
        for state in opt_g.state.values():
            state["exp_avg"].zero_()
            state["exp_avg_sq"].zero_()
            state["step"].zero_()
    opt_g.zero_grad(set_to_none=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_loss = body(m_g, opt_g, sx, st)
    losses_g = []
    for x, t in batches:
        sx.copy_(x)
        st.copy_(t)
        graph.replay()
        losses_g.append(static_loss.detach().clone())
    torch.cuda.synchronize()
    for i, (le, lg) in enumerate(zip(losses_e, losses_g)):
        assert torch.equal(le, lg), (i, le.item(), lg.item())
    for (n, pe), pg in zip(m_e.named_parameters(), m_g.parameters()):
        assert torch.equal(pe, pg), n
    del graph


def test_patched_call_site_matches_reference_class_fixture():
    """The reference's own MultiHeadAttention, run in float64 by tests/golden/make_golden.py, against the mirror of
    its call site with the reference's weights, patched onto the kernels (fp32 storage: the TF32 path; the
    projections in fp32): output, input gradient and every parameter gradient within the TF32 tolerance."""
    import foreswe_gpu_optimization_b200 as g
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mha_reference.npz"))
    heads, d_model = int(z["heads"]), z["x"].shape[-1]
    holder = nn.Module()
    holder.encoder_layers = nn.ModuleList([nn.Module()])
    att = MHA(d_model, heads).cuda()
    att.load_state_dict({k[len("param."):]: torch.from_numpy(z[k]).float() for k in z.files if k.startswith("param.")})
    holder.encoder_layers[0].self_attn = att
    g.patch_model(holder)
    x = torch.from_numpy(z["x"]).float().cuda().requires_grad_(True)
    dist, ang = torch.from_numpy(z["dist"]).float().cuda(), torch.from_numpy(z["ang"]).float().cuda()
    out = att(x, dist, ang)
    (out * torch.from_numpy(z["gout"]).float().cuda()).sum().backward()
    assert rel_l2(out.detach(), torch.from_numpy(z["out"])) <= 5e-4
    assert rel_l2(x.grad, torch.from_numpy(z["grad_x"])) <= 5e-4
    for name, p in att.named_parameters():
        ref = torch.from_numpy(z["grad." + name])
        if name == "W_k.bias":
            # adds q.b_k to every score of a row: softmax is shift-invariant, so the exact gradient is zero (the
            # fixture holds 3e-18) and both sides hold rounding noise, judged against the weight gradient's scale
            e = p.grad.double().abs().max().item() / torch.from_numpy(z["grad.W_k.weight"]).norm().item()
        else:
            e = rel_l2(p.grad, ref)
        assert e <= 5e-4, (name, e)
