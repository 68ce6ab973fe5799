"""geoattn_bwd_noalloc: the backward for callers that cannot allocate device memory.

Plugin/custom-op hosts that own every device buffer (and code with a fixed memory plan) cannot hand the backward a
workspace; geoattn_bwd_noalloc takes its scratch from a static device array inside the library instead. This test
calls it through the C ABI twice in a row, on different inputs, and checks each result against geoattn_bwd (the
entry point that takes a caller-allocated workspace) and against the float64 oracle, within the BF16 tolerance used
by the other parity tests, at head dims 64, 128 and 192 (each a different tile configuration of the row pass's
second sweep, which only this entry point runs in bf16).
It lives in its own file, collected last, and passes alone in a fresh process as well as after the other tests.
"""
import ctypes

import pytest
import torch

from helpers import attn_inputs, rel_l2, stations

pytestmark = pytest.mark.gpu
TOL = 8e-3


@pytest.fixture(scope="module")
def L():
    from foreswe_gpu_optimization_b200 import _lib, build
    build.build()
    return _lib.lib()


def _forward(L, q, k, v, abg, prior, per_head):
    from foreswe_gpu_optimization_b200 import _lib
    B, H, N, D = q.shape
    sh = _lib.Shape(B, H, N, D, _lib.DTYPE_BF16, per_head)
    o = torch.empty_like(q)
    stats = torch.empty(L.geoattn_stats_bytes(ctypes.byref(sh)) // 4, dtype=torch.float32, device=q.device)
    ws = torch.empty(L.geoattn_fwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=q.device)
    args = _lib.FwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v),
                        ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                        ctypes.c_void_p(o.data_ptr()), _lib.c_ll4(*o.stride()), ctypes.c_void_p(stats.data_ptr()),
                        ctypes.c_void_p(ws.data_ptr()))
    _lib.check(L.geoattn_fwd(ctypes.byref(args), None))
    return sh, o, stats


def _backward(L, entry, sh, q, k, v, o, do, abg, prior, stats, nabg):
    from foreswe_gpu_optimization_b200 import _lib
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dabg = torch.empty(3 * nabg, dtype=torch.float32, device=q.device)
    ws = None
    if entry == "geoattn_bwd":
        ws = torch.empty(L.geoattn_bwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=q.device)
    args = _lib.BwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v), _lib.tensor_arg(o),
                        _lib.tensor_arg(do), ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                        ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(dq.data_ptr()), _lib.c_ll4(*dq.stride()),
                        ctypes.c_void_p(dk.data_ptr()), _lib.c_ll4(*dk.stride()), ctypes.c_void_p(dv.data_ptr()),
                        _lib.c_ll4(*dv.stride()), ctypes.c_void_p(dabg.data_ptr()),
                        ctypes.c_void_p(ws.data_ptr() if ws is not None else None))
    _lib.check(getattr(L, entry)(ctypes.byref(args), None))
    torch.cuda.synchronize()
    return dict(dQ=dq.cpu(), dK=dk.cpu(), dV=dv.cpu(), dabg=dabg.cpu())


def _oracle(q, k, v, lat, lon, el, a, b, c, do):
    from helpers import dense_geometry
    from oracle import geo_attention as oga
    dist, ang = dense_geometry(lat, lon, el)
    return oga.grads(*(t.cpu().double() for t in (q, k, v)), dist.double(), ang.double(), a, b, c, do.cpu().double())


@pytest.mark.parametrize("per_head", [1, 0], ids=["per_head", "scalar"])
@pytest.mark.parametrize("N,D", [(512, 64), (260, 64), (260, 128), (260, 192)])
def test_noalloc_backward_matches_workspace_backward_twice(L, N, D, per_head):
    """Two calls in a row (the static scratch keeps the previous call's contents) at every bf16 head-dim tile
    configuration, a ragged station count and scalar or per-head parameters: each call's gradients are within the
    BF16 tolerance of geoattn_bwd's and of the float64 oracle's, and the status word of the static scratch reads 0."""
    from foreswe_gpu_optimization_b200 import StationGeometry
    from foreswe_gpu_optimization_b200.geo_attention_v2 import read_status
    B, H = 2, 3
    lat, lon, el = stations(N, seed=31 + D)
    geom = StationGeometry(lat, lon, el)
    prior = geom.prior(torch.bfloat16)
    for seed in (41, 42):
        q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=seed + D, qscale=3.0, per_head=bool(per_head),
                                           dtype=torch.bfloat16)
        q, k, v, do = (t.cuda() for t in (q, k, v, do))
        nabg = a.numel()
        abg = torch.cat([a, b, c]).cuda()
        sh, o, stats = _forward(L, q, k, v, abg, prior, per_head=per_head)
        ref = _backward(L, "geoattn_bwd", sh, q, k, v, o, do, abg, prior, stats, nabg)
        got = _backward(L, "geoattn_bwd_noalloc", sh, q, k, v, o, do, abg, prior, stats, nabg)
        assert read_status(None) == 0
        for key in ref:
            assert torch.isfinite(got[key].float()).all(), key
            assert rel_l2(got[key], ref[key]) <= TOL, (seed, key, rel_l2(got[key], ref[key]))
        gold = _oracle(q, k, v, lat, lon, el, a, b, c, do)
        # a shared (scalar) parameter's gradient is a sum over the heads that can cancel (one draw here sums per-head
        # terms of ~0.5 to -0.003): it is judged against the magnitude of the per-head terms, from the oracle with
        # the parameter repeated per head
        scale = {}
        if nabg == 1:
            ph = _oracle(q, k, v, lat, lon, el, a.repeat(H), b.repeat(H), c.repeat(H), do)
            scale = {key: ph[key].abs().sum().item() for key in ("dalpha", "dbeta", "dgamma")}
        dabg = got["dabg"].view(3, nabg)
        mine = dict(dQ=got["dQ"], dK=got["dK"], dV=got["dV"], dalpha=dabg[0], dbeta=dabg[1], dgamma=dabg[2])
        for key, val in mine.items():
            ref_v = gold[key].reshape(val.shape)
            e = rel_l2(val, ref_v)
            if key in scale:
                e = (val.double() - ref_v.double()).abs().max().item() / max(scale[key], ref_v.abs().max().item())
            assert e <= TOL, (seed, key, e)


def test_noalloc_rejects_sizes_beyond_its_buffer(L):
    from foreswe_gpu_optimization_b200 import _lib
    args = _lib.BwdArgs()
    args.shape = _lib.Shape(256, 16, 512, 128, _lib.DTYPE_BF16, 1)      # ~34 MB of row records > 16 MiB
    assert L.geoattn_bwd_noalloc(ctypes.byref(args), None) == 7
    args.shape = _lib.Shape(1, 1, 64, 64, _lib.DTYPE_FP32, 0)
    assert L.geoattn_bwd_noalloc(ctypes.byref(args), None) == 2
    assert b"16 MiB" in L.geoattn_error_string(7)
