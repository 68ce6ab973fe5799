"""Outputs that a TMA store cannot write (row stride not a multiple of 16 bytes) leave the kernels by row stores:
same values, bit for bit, as through the TMA-store epilogues. Called through the C ABI, as a caller with its own
output buffers would."""
import ctypes

import pytest
import torch

from helpers import attn_inputs, stations

pytestmark = pytest.mark.gpu


def _strided_like(t, pad):
    """A [B, H, N, D] view of a buffer whose rows are D + pad elements apart."""
    B, H, N, D = t.shape
    return torch.zeros(B, H, N, D + pad, dtype=t.dtype, device=t.device)[..., :D]


@pytest.mark.parametrize("D", [64, 128])
def test_row_store_fallback_bitwise(D):
    import foreswe_gpu_optimization_b200 as g
    from foreswe_gpu_optimization_b200 import _lib
    L = _lib.lib()
    B, H, N = 2, 2, 200
    q, k, v, a, b, c, do = (t.cuda() for t in attn_inputs(B, H, N, D, seed=D, qscale=2.0, dtype=torch.bfloat16))
    geom = g.StationGeometry(*stations(N, D), device="cuda")
    prior = geom.prior(torch.bfloat16)
    abg = torch.cat([a, b, c]).float().contiguous()
    sh = _lib.Shape(B, H, N, D, _lib.DTYPE_BF16, 1)

    def run(pad):
        o = _strided_like(q, pad) if pad else torch.empty_like(q)
        stats = torch.empty(L.geoattn_stats_bytes(ctypes.byref(sh)) // 4, dtype=torch.float32, device="cuda")
        ws = torch.empty(L.geoattn_fwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device="cuda")
        fa = _lib.FwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v),
                          ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                          ctypes.c_void_p(o.data_ptr()), _lib.c_ll4(*o.stride()), ctypes.c_void_p(stats.data_ptr()),
                          ctypes.c_void_p(ws.data_ptr()))
        _lib.check(L.geoattn_fwd(ctypes.byref(fa), None))
        grads = [(_strided_like(q, pad) if pad else torch.empty_like(q)) for _ in range(3)]
        dabg = torch.empty(3 * H, dtype=torch.float32, device="cuda")
        wsb = torch.empty(L.geoattn_bwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device="cuda")
        ba = _lib.BwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v), _lib.tensor_arg(o),
                          _lib.tensor_arg(do), ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                          ctypes.c_void_p(stats.data_ptr()),
                          *sum(([ctypes.c_void_p(t.data_ptr()), _lib.c_ll4(*t.stride())] for t in grads), []),
                          ctypes.c_void_p(dabg.data_ptr()), ctypes.c_void_p(wsb.data_ptr()))
        _lib.check(L.geoattn_bwd(ctypes.byref(ba), None))
        torch.cuda.synchronize()
        return [o.contiguous()] + [t.contiguous() for t in grads] + [dabg]

    tma = run(0)       # contiguous outputs: TMA-store epilogues
    rows = run(1)      # row stride D + 1 elements: not TMA-compatible, row stores
    for name, x, y in zip(("O", "dQ", "dK", "dV", "dabg"), tma, rows):
        assert torch.equal(x, y), name
