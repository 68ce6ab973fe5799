"""The torch.library registration of the geo-attention ops: fake (meta) implementations, no GPU needed."""
import torch

import foreswe_gpu_optimization_b200 as g  # noqa: F401  (registers foreswe_geoattn::fwd / ::bwd)


def test_fake_shapes_and_layouts():
    B, N, H, D = 2, 96, 4, 32
    # split_heads view of a [B, N, H*D] projection: O must come back in the same layout
    q = torch.empty(B, N, H * D, device="meta", dtype=torch.bfloat16).view(B, N, H, D).transpose(1, 2)
    prior = torch.empty(2 * 128 * 128, device="meta", dtype=torch.int32)
    for per_head, nabg in ((1, H), (0, 1)):
        abg = torch.empty(3 * nabg, device="meta")
        o, stats = torch.ops.foreswe_geoattn.fwd(q, q, q, prior, abg, per_head)
        assert o.shape == q.shape and o.dtype == q.dtype and o.stride() == q.stride()
        assert stats.shape == (3 * B * H * N,) and stats.dtype == torch.float32
        dq, dk, dv, dabg = torch.ops.foreswe_geoattn.bwd(q, q, q, o, o, prior, abg, stats, per_head)
        assert dq.shape == dk.shape == dv.shape == q.shape and dq.stride() == q.stride()
        assert dabg.shape == (3 * nabg,) and dabg.dtype == torch.float32


def test_schema_registered():
    assert "per_head" in str(torch.ops.foreswe_geoattn.fwd.default._schema)
    assert "stats" in str(torch.ops.foreswe_geoattn.bwd.default._schema)
