"""Parity of the B200 kernels (through libgeoattn's C ABI) with the float64 oracle on seeded inputs.

Tolerances (rel-L2 against the FP32 operator): TF32 path 5e-4, BF16 path 8e-3, for the output and every gradient;
saturated inputs must stay finite. The oracle is evaluated on exactly the values the kernels see (bf16 inputs are
compared with the oracle on the same bf16 values).
"""
import glob
import os

import numpy as np
import pytest
import torch

from helpers import KEYS, TOL, attn_inputs, dense_geometry, rel_l2, run_device, stations
from oracle import acceptance
from oracle import geo_attention as oga

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ops():
    import foreswe_gpu_optimization_b200 as g
    return g


def _oracle(q, k, v, dist, ang, a, b, c, do):
    return oga.grads(q.double(), k.double(), v.double(), dist.double(), ang.double(), a, b, c, do.double())


def _check(res, ref, tol, label):
    bad = {}
    for key in KEYS:
        assert torch.isfinite(res[key].float()).all(), (label, key, "non-finite")
        e = rel_l2(res[key], ref[key])
        if not e <= tol:
            bad[key] = e
    assert not bad, "%s: rel-L2 above %.1e: %s" % (label, tol, bad)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "tf32"])
@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "saturated_x30"])
def test_c2_shape_coordinate_geometry(ops, dtype, qscale):
    """N = 512 stations, D = 64, per-head parameters, prior from coordinates (the coordinate call form)."""
    B, H, N, D = 2, 4, 512, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=1, qscale=qscale, dtype=dtype)
    lat, lon, el = stations(N, seed=2)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    dist, ang = dense_geometry(lat, lon, el)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[dtype], "C2 %s x%g" % (dtype, qscale))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "tf32"])
@pytest.mark.parametrize("N,D", [(1, 64), (33, 48), (100, 64), (129, 8), (200, 64), (300, 24), (70, 30)])
def test_ragged_shapes_dense_prior(ops, dtype, N, D):
    """N not a multiple of the tiles, D below the 64-wide tile (D = 30: fp32 operands split element by element, the
    others with 16-byte accesses); reference call with dense dist/ang."""
    B, H = 1, 3
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=N + D, qscale=3.0, per_head=False, dtype=dtype)
    g = torch.Generator().manual_seed(N)
    dist = torch.rand(N, N, generator=g) * 1500
    ang = torch.rand(N, N, generator=g) * 20
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[dtype], "N=%d D=%d" % (N, D))


@pytest.mark.parametrize("D", [128, 192, 96, 160])
def test_bf16_wide_heads(ops, D):
    """bf16 head dims up to the production d_k = 192 (3 x 1024 / 16)."""
    B, H, N = 1, 2, 384
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=D, qscale=2.0, dtype=torch.bfloat16)
    lat, lon, el = stations(N, seed=D)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    dist, ang = dense_geometry(lat, lon, el)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[torch.bfloat16], "D=%d" % D)


@pytest.mark.parametrize("precision,dtype", [("bf16", torch.float32), ("tf32", torch.bfloat16)])
def test_precision_override(ops, precision, dtype):
    """precision='bf16' runs fp32 inputs through the BF16 kernels, precision='tf32' bf16 inputs through the TF32
    kernels; output and gradients come back in the inputs' dtype, within the BF16 tolerance of the oracle evaluated
    on the values the kernels saw (inputs and dO rounded to bf16 where the kernels or the output are bf16)."""
    B, H, N, D = 2, 4, 200, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=21, qscale=2.0, dtype=dtype)
    lat, lon, el = stations(N, seed=22)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:], precision=precision),
                     q, k, v, a, b, c, do)
    for key in ("output", "dQ", "dK", "dV"):
        assert res[key].dtype == dtype, (key, res[key].dtype)
    qr, kr, vr, dor = (t.to(torch.bfloat16).float() for t in (q, k, v, do))
    dist, ang = dense_geometry(lat, lon, el)
    _check(res, _oracle(qr, kr, vr, dist, ang, a, b, c, dor), TOL[torch.bfloat16], "precision=%s" % precision)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "tf32"])
@pytest.mark.parametrize("shape", [(0, 2, 64, 64), (2, 0, 64, 64), (1, 2, 0, 64)], ids=["B0", "H0", "N0"])
def test_empty_inputs(ops, dtype, shape):
    """An empty batch, head set or station set returns empty outputs and gradients and zero bias gradients, as the
    eager operator does, without launching."""
    B, H, N, D = shape
    x = [torch.randn(B, H, N, D, device="cuda").to(dtype).requires_grad_(True) for _ in range(3)]
    p = [torch.tensor([v], device="cuda", requires_grad=True) for v in (0.5, -0.2, 0.3)]
    dist = torch.zeros(N, N, device="cuda")
    o = ops.fused_geo_attention_v2(*x, dist, dist, *p)
    assert o.shape == (B, H, N, D) and o.dtype == dtype
    o.sum().backward()
    for t in x:
        assert t.grad.shape == t.shape
    for t in p:
        assert t.grad is not None and t.grad.item() == 0.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "tf32"])
def test_many_chunks_per_row(ops, dtype):
    """N = 1500 stations (24 bf16 / 47 fp32 key chunks per row, 12 row blocks, ragged last chunk and block)."""
    B, H, N, D = 1, 2, 1500, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=31, qscale=2.0, dtype=dtype)
    lat, lon, el = stations(N, seed=32)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    dist, ang = dense_geometry(lat, lon, el)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[dtype], "N=1500 %s" % dtype)


def test_tf32_pooled_tiles_per_cta_repeat_bitwise(ops):
    """fp32 at head dim 64 hands each tile's A operand (Q, Q/dO, K/V) from a shared-memory landing pool to tensor
    memory and reuses the pool for the chunk rings. 384 tiles on 148 persistent CTAs (2-3 tiles each) with an odd
    chunk count (N = 330: 11 key chunks, padded to whole pairs in the forward) exercise the hand-over between tiles:
    repeated runs agree bitwise and match the oracle. (A pool released before its tensor-memory copies had read it
    showed here as dK differing between runs in about one run of three.)"""
    B, H, N, D = 16, 8, 330, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=41, qscale=3.0, dtype=torch.float32)
    lat, lon, el = stations(N, seed=42)
    geom = ops.StationGeometry(lat, lon, el)
    fn = lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:])  # noqa: E731
    r1 = run_device(fn, q, k, v, a, b, c, do)
    for _ in range(5):
        r2 = run_device(fn, q, k, v, a, b, c, do)
        for key in KEYS:
            assert torch.equal(r1[key], r2[key]), key
    dist, ang = dense_geometry(lat, lon, el)
    _check(r1, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[torch.float32], "pooled tf32 N=330")


@pytest.mark.parametrize("D", [128, 192, 96, 160])
def test_tf32_wide_heads(ops, D):
    """fp32 head dims above 64 (Q/K and dO/V streamed through the score MMAs in 32-wide head-dim chunks), up to the
    production d_k = 192, per-head parameters, coordinate prior, N not a multiple of the tiles."""
    B, H, N = 1, 2, 300
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=D + 1, qscale=2.0, dtype=torch.float32)
    lat, lon, el = stations(N, seed=D)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    dist, ang = dense_geometry(lat, lon, el)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[torch.float32], "tf32 D=%d" % D)


def _regime(ops, case, B, H, N, D):
    inp = acceptance.case_inputs(case, B=B, H=H, N=N, D=D, seed=0)
    do = acceptance.grad_seed_do(inp[0].shape)
    q, k, v, dist, ang, a, b, c = inp
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    for key in KEYS:
        assert torch.isfinite(res[key]).all(), (case, key)
    ev = acceptance.evaluate(res, inp, do, "tf32", ref=acceptance.reference(inp, do))
    bad = {k: (r["candidate"]["max_abs"], r["bound"]) for k, r in ev.items() if not r["passed"]}
    assert not bad, "%s %s: above 10x eager TF32: %s" % (case, (B, H, N, D), bad)


@pytest.mark.parametrize("case", acceptance.CASES)
def test_reference_regimes_tf32_d192(ops, case):
    """The reference's acceptance test (tests/test_gpu_geo_attention_v2.py:32-50): its six synthetic regimes at its
    own shape (1, 2, 100, 192), fp32 storage, within 10x eager TF32's max-abs error of the float64 operator."""
    _regime(ops, case, 1, 2, 100, 192)


def test_reference_regime_tf32_full_d192(ops):
    """The reference's full-size acceptance shape (1, 16, 512, 192) in its hardest regime (score std ~ 400)."""
    _regime(ops, "near_one_hot", 1, 16, 512, 192)


def test_tf32_wide_repeat_bitwise(ops):
    """The streamed fp32 path is deterministic: two runs give bitwise-equal outputs and gradients."""
    B, H, N, D = 2, 2, 260, 192
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=9, qscale=3.0, dtype=torch.float32)
    lat, lon, el = stations(N, seed=9)
    geom = ops.StationGeometry(lat, lon, el)
    fn = lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:])  # noqa: E731
    r1 = run_device(fn, q, k, v, a, b, c, do)
    r2 = run_device(fn, q, k, v, a, b, c, do)
    for key in KEYS:
        assert torch.equal(r1[key], r2[key]), key


@pytest.mark.parametrize("case", acceptance.CASES)
def test_reference_regimes_tf32(ops, case):
    """The reference's six synthetic regimes (foreswe_bench/attn_check.py:20-45) at D = 64 on the TF32 path:
    within the TF32 tolerance of the oracle, finite, and within 10x eager TF32's max-abs error."""
    inp = acceptance.case_inputs(case, B=1, H=2, N=128, D=64, seed=0)
    do = acceptance.grad_seed_do(inp[0].shape)
    q, k, v, dist, ang, a, b, c = inp
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    ref = acceptance.reference(inp, do)
    for key in KEYS:
        assert torch.isfinite(res[key]).all(), (case, key)
    ev = acceptance.evaluate(res, inp, do, "tf32", ref=ref)
    bad = {k: (r["candidate"]["max_abs"], r["bound"]) for k, r in ev.items() if not r["passed"]}
    assert not bad, "%s: above 10x eager TF32: %s" % (case, bad)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_reference_golden_vectors_tf32(ops, path):
    """Golden vectors produced by the reference's eager operator (float64 autograd) through the TF32 path: each
    quantity within the TF32 rel-L2 tolerance of the golden value, or -- where the golden value itself is
    vanishingly small (saturated rows: dQ ~ 1e-29 in near_one_hot) -- within the reference's own acceptance rule,
    10x eager TF32's max-abs error (foreswe_bench/attn_check.py:68-81)."""
    z = np.load(path)
    q, k, v, dist, ang = (torch.from_numpy(z[n]).float() for n in ("q", "k", "v", "dist", "ang"))
    a, b, c = (torch.from_numpy(z[n]).float().reshape(-1) for n in ("alpha", "beta", "gamma"))
    do = torch.from_numpy(z["do"]).float()
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    gold = {key: torch.from_numpy(z[key]).reshape(res[key].shape) for key in KEYS}
    inp = [q, k, v, dist, ang, a, b, c]
    ev = acceptance.evaluate(res, inp, do, "tf32", ref=gold)
    for key in KEYS:
        e = rel_l2(res[key], gold[key])
        assert torch.isfinite(res[key]).all(), key
        assert e <= 5e-4 or ev[key]["passed"], (key, e, ev[key]["candidate"]["max_abs"], ev[key]["bound"])


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 64), (torch.float32, 64), (torch.float32, 192)],
                         ids=["bf16-d64", "tf32-d64", "tf32-d192"])
def test_split_heads_strided_views(ops, dtype, D):
    """Q/K/V as the transposed split_heads views of [B, N, H*D] (custom_encoder_model.py:41-43); gradients keep
    the input strides."""
    B, N, H = 2, 160, 4
    g = torch.Generator().manual_seed(5)
    base = [torch.randn(B, N, H * D, generator=g).cuda().to(dtype) * 0.4 for _ in range(3)]
    views = [t.view(B, N, H, D).transpose(1, 2).detach().requires_grad_(True) for t in base]
    a, b, c = (torch.tensor([x], device="cuda", requires_grad=True) for x in (0.5, -0.3, 0.2))
    dist = torch.rand(N, N, generator=g).cuda() * 900
    ang = torch.rand(N, N, generator=g).cuda() * 12
    o = ops.fused_geo_attention_v2(*views, dist, ang, a, b, c)
    do = torch.randn(o.shape, generator=g).cuda().to(dtype)
    o.backward(do)
    for x in views:
        assert x.grad.stride() == x.stride()
    # O has q's layout, so the call site's combine_heads (transpose(1, 2).contiguous()) copies nothing
    assert o.stride() == views[0].stride() and o.transpose(1, 2).is_contiguous()
    ref = oga.grads(*(t.detach().double().cpu() for t in views), dist.cpu().double(), ang.cpu().double(),
                    a.detach().cpu(), b.detach().cpu(), c.detach().cpu(), do.double().cpu())
    res = dict(output=o.detach().cpu(), dQ=views[0].grad.cpu(), dK=views[1].grad.cpu(), dV=views[2].grad.cpu(),
               dalpha=a.grad.cpu(), dbeta=b.grad.cpu(), dgamma=c.grad.cpu())
    _check(res, ref, TOL[dtype], "strided %s D=%d" % (dtype, D))


def test_device_geometry_matches_oracle(ops):
    """Device float64 haversine / Kahan angle, rounded to fp32, equal the oracle's within an ulp."""
    z = np.load(os.path.join(GOLD, "geometry.npz"))
    geom = ops.StationGeometry(z["lat"], z["lon"], z["elev_ft"])
    dist, ang = geom.distance_and_angularity()
    np.testing.assert_allclose(dist.cpu().numpy(), z["dist_km"].astype(np.float32), rtol=2.5e-7, atol=1e-6)
    np.testing.assert_allclose(ang.cpu().numpy(), z["ang_deg"].astype(np.float32), rtol=2.5e-7, atol=1e-6)
    lat, lon, el = stations(300, seed=9)
    d2, a2 = ops.StationGeometry(lat, lon, el).distance_and_angularity()
    rd, ra = dense_geometry(lat, lon, el)
    torch.testing.assert_close(d2.cpu(), rd, rtol=2.5e-7, atol=1e-6)
    torch.testing.assert_close(a2.cpu(), ra, rtol=2.5e-7, atol=1e-6)


def test_coordinate_and_dense_priors_agree(ops):
    """geo_attention(geometry) and fused_geo_attention_v2(dist, ang) give identical results."""
    B, H, N, D = 1, 2, 200, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=3, dtype=torch.float32)
    lat, lon, el = stations(N, seed=4)
    geom = ops.StationGeometry(lat, lon, el)
    dist, ang = geom.distance_and_angularity()
    r1 = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    r2 = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist, ang, *x[3:]), q, k, v, a, b, c, do)
    for key in KEYS:
        assert torch.equal(r1[key], r2[key]), key


@pytest.mark.parametrize("D", [64, 128, 160, 192])
def test_bf16_repeat_bitwise_every_head_dim(ops, D):
    """Every bf16 tile configuration (single- and double-buffered rings) gives bitwise identical results on
    repeated launches: a buffer handed back to its producer too early shows up as run-to-run differences."""
    B, H, N = 2, 2, 384
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=40 + D, qscale=2.0, dtype=torch.bfloat16)
    geom = ops.StationGeometry(*stations(N, seed=D))
    fn = lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:])
    r0 = run_device(fn, q, k, v, a, b, c, do)
    for _ in range(3):
        r = run_device(fn, q, k, v, a, b, c, do)
        for key in KEYS:
            assert torch.equal(r0[key], r[key]), (D, key)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "tf32"])
def test_deterministic_and_graph_replay_bitwise(ops, dtype):
    """Two direct launches agree bitwise, and a CUDA-graph capture of fwd+bwd replays bitwise equal to direct
    launches for fresh inputs (tests/test_gpu_geo_attention_v2.py:85-114 in the reference)."""
    B, H, N, D = 1, 2, 256, 64
    lat, lon, el = stations(N, seed=11)
    geom = ops.StationGeometry(lat, lon, el)
    fn = lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:])
    ins = [attn_inputs(B, H, N, D, seed=s, qscale=4.0, dtype=dtype) for s in (21, 22)]
    r1 = run_device(fn, *ins[0])
    r2 = run_device(fn, *ins[0])
    for key in KEYS:
        assert torch.equal(r1[key], r2[key]), key
    dev = torch.device("cuda")
    static = [t.to(dev).detach().clone().requires_grad_(True) for t in ins[0][:6]]
    do = ins[0][6].to(dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            for t in static:
                t.grad = None
            fn(*static).backward(do)
    torch.cuda.current_stream().wait_stream(s)
    for t in static:
        t.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn(*static)
        out.backward(do)
    for inp in ins:
        with torch.no_grad():
            for t, src in zip(static, inp[:6]):
                t.copy_(src.to(dev))
            do.copy_(inp[6].to(dev))
        graph.replay()
        ref = run_device(fn, *inp)
        assert torch.equal(out.detach().cpu(), ref["output"])
        for i, key in zip(range(6), ("dQ", "dK", "dV", "dalpha", "dbeta", "dgamma")):
            assert torch.equal(static[i].grad.cpu(), ref[key]), key


def test_status_word_clean_and_errors_raise(ops):
    """No bounded wait expires on a normal launch; unsupported shapes raise through geoattn_error_string."""
    from foreswe_gpu_optimization_b200 import _lib
    import ctypes
    B, H, N, D = 1, 1, 64, 64
    sh = _lib.Shape(B, H, N, D, _lib.DTYPE_FP32, 0)
    L = _lib.lib()
    ws = torch.zeros(L.geoattn_fwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device="cuda")
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, per_head=False)
    dist = torch.rand(N, N).cuda() * 100
    ang = torch.rand(N, N).cuda() * 5
    prior = ops.prior_from_dense(dist, ang, torch.float32)
    abg = torch.cat([a, b, c]).cuda()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.empty_like(qd)
    stats = torch.empty(3 * N, device="cuda")
    args = _lib.FwdArgs(sh, _lib.tensor_arg(qd), _lib.tensor_arg(kd), _lib.tensor_arg(vd),
                        ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                        ctypes.c_void_p(o.data_ptr()), _lib.c_ll4(*o.stride()), ctypes.c_void_p(stats.data_ptr()),
                        ctypes.c_void_p(ws.data_ptr()))
    _lib.check(L.geoattn_fwd(ctypes.byref(args), None))
    from foreswe_gpu_optimization_b200.geo_attention_v2 import read_status
    assert read_status(ws) == 0
    with pytest.raises(_lib.GeoAttnError):
        x = torch.randn(1, 1, 16, 200, device="cuda")  # head_dim above 192
        ops.fused_geo_attention_v2(x, x, x, dist[:16, :16], ang[:16, :16], a.cuda(), b.cuda(), c.cuda())
    # a host pointer where the library expects device memory is rejected before any launch
    bad = _lib.FwdArgs(sh, _lib.tensor_arg(qd), _lib.tensor_arg(kd), _lib.tensor_arg(vd),
                       ctypes.c_void_p(torch.cat([a, b, c]).data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                       ctypes.c_void_p(o.data_ptr()), _lib.c_ll4(*o.stride()), ctypes.c_void_p(stats.data_ptr()),
                       ctypes.c_void_p(ws.data_ptr()))
    assert L.geoattn_fwd(ctypes.byref(bad), None) == 1


def test_inputs_on_another_device_rejected(ops):
    """k on the host while q is on the GPU raises before any launch (the kernels would dereference it on q's
    device)."""
    q = torch.randn(1, 2, 64, 64, device="cuda")
    d = torch.zeros(64, 64, device="cuda")
    a = torch.ones(1, device="cuda")
    with pytest.raises(ValueError, match="k lives on cpu"):
        ops.fused_geo_attention_v2(q, q.cpu(), q, d, d, a, a, a)


def test_host_bias_parameters_get_host_gradients(ops):
    """alpha, beta, gamma kept on the host (q, k, v on the GPU) get their gradients on the host, equal to the
    gradients of the same parameters on the GPU."""
    B, H, N, D = 1, 2, 96, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=21, per_head=True)
    dist, ang = dense_geometry(*stations(N, 22))
    dist, ang = dist.cuda(), ang.cuda()
    grads = {}
    for where in ("cpu", "cuda"):
        x = [t.cuda().requires_grad_(True) for t in (q, k, v)]
        p = [t.detach().to(where).requires_grad_(True) for t in (a, b, c)]  # fresh leaves on each device
        o = ops.fused_geo_attention_v2(*x, dist, ang, *p)
        o.backward(do.cuda())
        assert all(t.grad.device.type == where for t in p)
        grads[where] = [t.grad.cpu() for t in p]
    for g_host, g_dev in zip(grads["cpu"], grads["cuda"]):
        assert torch.equal(g_host, g_dev)


def test_bounded_wait_expires_into_the_status_word(ops):
    """A wait that nothing completes gives up after its limit (about 2 s): the kernel records the timeout in the
    status word and returns, and the context keeps working (an attention call right after matches the oracle)."""
    import ctypes
    import time
    from foreswe_gpu_optimization_b200 import _lib
    L = _lib.lib()
    word = torch.full((4,), -1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.geoattn_wait_selftest(None, stream) == 1                                   # no word: rejected
    assert L.geoattn_wait_selftest(ctypes.c_void_p(word.data_ptr() + 2), stream) == 1   # misaligned: rejected
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(L.geoattn_wait_selftest(ctypes.c_void_p(word.data_ptr()), stream))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert word[0].item() == 1, "the expired wait records status 1"
    assert 1.5 < waited < 60, waited
    B, H, N, D = 1, 2, 96, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=31)
    dist, ang = dense_geometry(*stations(N, 32))
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    _check(res, _oracle(q, k, v, dist, ang, a, b, c, do), TOL[torch.float32], "after an expired wait")


def _rel_dev(x, ref):
    """rel-L2 of x against ref, in float64 on the device (full-size tensors stay off the host)."""
    x, ref = x.double(), ref.double()
    return ((x - ref).norm() / ref.norm()).item()


@pytest.mark.parametrize("dtype,B,H,D", [(torch.bfloat16, 256, 16, 128), (torch.float32, 32, 8, 64)],
                         ids=["bf16-256x16x512x128", "tf32-32x8x512x64"])
def test_full_size_step_properties(ops, dtype, B, H, D):
    """Full-size workloads -- the benchmarked one (256 issue dates x 16 heads x 512 stations x D = 128, bf16; ~110
    tiles per persistent CTA) and the TF32 one (32 x 8 x 512 x 64; ~7 tiles per CTA) -- with per-head parameters
    and the coordinate prior, checked through properties that hold at any size:
      * O is linear in V and the backward is linear in dO; doubling scales every intermediate exactly in binary
        floating point (TF32 hi/lo splits included), so O(2V) = 2 O(V) and grads(2 dO) = 2 grads(dO) (rel-L2 1e-4);
      * P2's rows sum to one, so sum_k dV[k] = sum_q dO[q] (rel-L2 2e-3; rounding of P2 and dV, ~1e-4 expected);
      * dS's rows sum to zero (softmax backward), so sum_k dK[k] = 0 (2e-3 of sum_k |dK[k]|; ~1e-4 expected);
      * a repeated backward is bitwise equal (every CTA runs several tiles, so a buffer handed back too early between
        tiles shows up here)."""
    N = 512
    g = torch.Generator(device="cuda").manual_seed(40)
    s = D ** -0.25
    q, k, v = (torch.randn(B, H, N, D, device="cuda", generator=g).mul_(s).to(dtype).requires_grad_(True)
               for _ in range(3))
    do = torch.randn(B, H, N, D, device="cuda", generator=g).to(dtype)
    a = (torch.rand(H, device="cuda", generator=g) * 0.9 + 0.1).requires_grad_(True)
    b = (torch.randn(H, device="cuda", generator=g) * 0.5).requires_grad_(True)
    c = (torch.randn(H, device="cuda", generator=g) * 0.5).requires_grad_(True)
    geom = ops.StationGeometry(*stations(N, 41))
    o = ops.geo_attention(q, k, v, geom, a, b, c)
    assert torch.isfinite(o.float()).all()
    with torch.no_grad():
        o2v = ops.geo_attention(q, k, v * 2, geom, a, b, c)
    assert _rel_dev(o2v, 2 * o.detach()) <= 1e-4
    del o2v
    ins = (q, k, v, a, b, c)
    g1 = torch.autograd.grad(o, ins, do, retain_graph=True)
    g1b = torch.autograd.grad(o, ins, do, retain_graph=True)
    for name, x, y in zip(("dq", "dk", "dv", "dalpha", "dbeta", "dgamma"), g1, g1b):
        assert torch.equal(x, y), name
    del g1b
    g2 = torch.autograd.grad(o, ins, do * 2)
    for name, x, y in zip(("dq", "dk", "dv", "dalpha", "dbeta", "dgamma"), g1, g2):
        assert torch.isfinite(x.float()).all(), name
        assert _rel_dev(y, 2 * x) <= 1e-4, name
    del g2
    dk, dv = g1[1].double(), g1[2].double()
    assert _rel_dev(dv.sum(dim=2), do.double().sum(dim=2)) <= 2e-3
    assert (dk.sum(dim=2).norm() / dk.abs().sum(dim=2).norm()).item() <= 2e-3


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_reference_golden_vectors_bf16(ops, path):
    """The reference-generated golden inputs through the BF16 path. The kernels see the inputs and dO rounded to
    bf16, so they are judged against the float64 oracle on those values (the fixture's outputs pin the oracle on the
    unrounded inputs, tests/test_oracle_golden.py): each quantity within the BF16 rel-L2 tolerance, or -- where the
    oracle's value vanishes (uniform: Q = 0 makes the true d(alpha) zero) -- within 10x the max-abs error of eager
    bf16 (every matmul operand rounded to bf16, as under autocast), the reference's own acceptance rule."""
    z = np.load(path)
    rb = lambda t: torch.from_numpy(t).float().to(torch.bfloat16)  # noqa: E731
    q, k, v, do = (rb(z[n]) for n in ("q", "k", "v", "do"))
    dist, ang = (torch.from_numpy(z[n]).float() for n in ("dist", "ang"))
    a, b, c = (torch.from_numpy(z[n]).float().reshape(-1) for n in ("alpha", "beta", "gamma"))
    res = run_device(lambda *x: ops.fused_geo_attention_v2(x[0], x[1], x[2], dist.cuda(), ang.cuda(), *x[3:]),
                     q, k, v, a, b, c, do)
    inp = [q.float(), k.float(), v.float(), dist, ang, a, b, c]
    ref = acceptance.reference(inp, do.float())
    ev = acceptance.evaluate(res, inp, do.float(), "bf16", ref=ref)
    for key in KEYS:
        assert torch.isfinite(res[key].float()).all(), key
        e = rel_l2(res[key], ref[key].reshape(res[key].shape))
        assert e <= TOL[torch.bfloat16] or ev[key]["passed"], (key, e, ev[key]["candidate"]["max_abs"],
                                                               ev[key]["bound"])


@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "saturated_x30"])
def test_full_c2_tf32_every_head_against_oracle(ops, qscale):
    """The full TF32 configuration, 32 issue dates x 8 heads x 512 stations x D = 64 (~7 tiles per persistent CTA),
    plain and with logits x30: all 256 heads and the bias gradients against the float64 oracle (evaluated on the CPU
    four issue dates at a time, bias gradients summed over the slices) within the TF32 tolerance."""
    B, H, N, D = 32, 8, 512, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=50, qscale=qscale, dtype=torch.float32)
    lat, lon, el = stations(N, seed=51)
    geom = ops.StationGeometry(lat, lon, el)
    res = run_device(lambda *x: ops.geo_attention(x[0], x[1], x[2], geom, *x[3:]), q, k, v, a, b, c, do)
    dist, ang = dense_geometry(lat, lon, el)
    parts = [_oracle(q[s:s + 4], k[s:s + 4], v[s:s + 4], dist, ang, a, b, c, do[s:s + 4]) for s in range(0, B, 4)]
    ref = {key: torch.cat([p[key] for p in parts]) for key in ("output", "dQ", "dK", "dV")}
    for key in ("dalpha", "dbeta", "dgamma"):
        ref[key] = sum(p[key] for p in parts)
    _check(res, ref, TOL[torch.float32], "full C2 x%g" % qscale)


@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "saturated_x30"])
def test_full_size_tf32_d192_sampled_heads_against_oracle(ops, qscale):
    """The production head dim in TF32 at 32 issue dates x 16 heads x 512 stations (13.8 tiles per persistent CTA in
    every kernel; the dS-scratch backward with the transposing dQ GEMM and d(alpha) from the key pass): sampled heads
    -- first, middle and last issue dates and heads -- against the float64 oracle within the TF32 tolerance."""
    B, H, N, D = 32, 16, 512, 192
    g = torch.Generator(device="cuda").manual_seed(71)
    s = D ** -0.25
    q = torch.randn(B, H, N, D, device="cuda", generator=g).mul_(s * qscale)
    k, v = (torch.randn(B, H, N, D, device="cuda", generator=g).mul_(s) for _ in range(2))
    do = torch.randn(B, H, N, D, device="cuda", generator=g)
    pa = torch.rand(H, device="cuda", generator=g) * 0.9 + 0.1
    pb, pc = (torch.randn(H, device="cuda", generator=g) * 0.5 for _ in range(2))
    lat, lon, el = stations(N, seed=72)
    geom = ops.StationGeometry(lat, lon, el)
    x = [t.detach().requires_grad_(True) for t in (q, k, v)]
    o = ops.geo_attention(x[0], x[1], x[2], geom, pa, pb, pc)
    o.backward(do)
    torch.cuda.synchronize()
    dist, ang = dense_geometry(lat, lon, el)
    for bi in (0, 13, B - 1):
        for hi in (0, 9, H - 1):
            sl = (slice(bi, bi + 1), slice(hi, hi + 1))
            ref = _oracle(q[sl].cpu(), k[sl].cpu(), v[sl].cpu(), dist, ang, pa[hi:hi + 1].cpu(), pb[hi:hi + 1].cpu(),
                          pc[hi:hi + 1].cpu(), do[sl].cpu())
            got = dict(output=o.detach()[sl], dQ=x[0].grad[sl], dK=x[1].grad[sl], dV=x[2].grad[sl])
            for key, val in got.items():
                assert torch.isfinite(val).all(), (bi, hi, key)
                e = rel_l2(val, ref[key])
                assert e <= TOL[torch.float32], (bi, hi, key, e)


@pytest.mark.parametrize("B,H,D", [(256, 16, 128), (384, 16, 64)], ids=["c5-256x16x512x128", "c3-384x16x512x64"])
def test_full_size_bf16_sampled_heads_against_oracle(ops, B, H, D):
    """The benchmarked configuration (256 issue dates x 16 heads x 512 stations x D = 128, bf16; ~110 tiles per
    persistent CTA) and the temporal-batched one (384 x 16 x 512 x 64): one full-size fwd+bwd on the device, then
    the output and dQ, dK, dV of sampled heads -- the first and last issue dates and one in the middle of the
    persistent tile order, first, middle and last heads -- against the float64 oracle on the same bf16 values, within
    the BF16 tolerance. A wrong (b, h) offset or a tile handed between CTAs wrongly shows up in these heads."""
    N = 512
    g = torch.Generator(device="cuda").manual_seed(60 + D)
    s = D ** -0.25
    q, k, v = (torch.randn(B, H, N, D, device="cuda", generator=g).mul_(s).to(torch.bfloat16) for _ in range(3))
    do = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
    pa = torch.rand(H, device="cuda", generator=g) * 0.9 + 0.1
    pb, pc = (torch.randn(H, device="cuda", generator=g) * 0.5 for _ in range(2))
    lat, lon, el = stations(N, seed=61)
    geom = ops.StationGeometry(lat, lon, el)
    x = [t.detach().requires_grad_(True) for t in (q, k, v)]
    o = ops.geo_attention(x[0], x[1], x[2], geom, pa, pb, pc)
    o.backward(do)
    torch.cuda.synchronize()
    dist, ang = dense_geometry(lat, lon, el)
    for bi in (0, 97, B - 1):
        for hi in (0, 7, H - 1):
            sl = (slice(bi, bi + 1), slice(hi, hi + 1))
            ref = _oracle(q[sl].cpu().float(), k[sl].cpu().float(), v[sl].cpu().float(), dist, ang,
                          pa[hi:hi + 1].cpu(), pb[hi:hi + 1].cpu(), pc[hi:hi + 1].cpu(), do[sl].cpu().float())
            got = dict(output=o.detach()[sl], dQ=x[0].grad[sl], dK=x[1].grad[sl], dV=x[2].grad[sl])
            for key, val in got.items():
                assert torch.isfinite(val.float()).all(), (bi, hi, key)
                e = rel_l2(val, ref[key])
                assert e <= TOL[torch.bfloat16], (bi, hi, key, e)
