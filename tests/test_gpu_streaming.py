"""HostBatchPipeline: fwd+bwd over pinned host batches in slices, copies overlapped with compute."""
import pytest
import torch

from helpers import attn_inputs, stations

pytestmark = pytest.mark.gpu


def test_sliced_host_step_matches_one_call():
    import foreswe_gpu_optimization_b200 as g
    B, H, N, D = 7, 4, 256, 64
    q, k, v, a, b, c, do = attn_inputs(B, H, N, D, seed=5, dtype=torch.bfloat16)
    dev = torch.device("cuda")
    geom = g.StationGeometry(*stations(N, 3), device=dev)

    ref = [t.to(dev).requires_grad_(True) for t in (a, b, c)]
    x = [t.to(dev).requires_grad_(True) for t in (q, k, v)]
    g.geo_attention(*x, geom, *ref).backward(do.to(dev))

    got = [t.to(dev).requires_grad_(True) for t in (a, b, c)]
    pipe = g.HostBatchPipeline(q.shape, q.dtype, dev, slices=3)   # uneven slices: 2, 2, 3 issue dates
    host = [t.pin_memory() for t in (q, k, v, do)]
    for _ in range(2):                                             # buffers reused across steps
        for t in got:
            t.grad = None
        assert pipe.step(*host, geom, *got) == 3
    torch.cuda.synchronize()
    for r, o in zip(ref, got):
        assert torch.allclose(o.grad, r.grad, rtol=1e-5, atol=1e-6), (o.grad, r.grad)
    with pytest.raises(ValueError):
        pipe.step(q, k, v, do, geom, *got)                         # pageable host memory is refused
