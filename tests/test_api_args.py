"""Argument checks of the Python surface that need no GPU: precision / mode selection is validated before any
device work."""
import pytest
import torch

import foreswe_gpu_optimization_b200 as g
from foreswe_gpu_optimization_b200 import geo_attention_v2 as gv2


def _cpu_inputs():
    q = torch.zeros(1, 2, 8, 16)
    d = torch.zeros(8, 8)
    a = torch.ones(1)
    return q, d, a


def test_unknown_mode_and_precision_rejected():
    q, d, a = _cpu_inputs()
    with pytest.raises(NotImplementedError, match="mode"):
        g.fused_geo_attention_v2(q, q, q, d, d, a, a, a, mode="additive")
    with pytest.raises(ValueError, match="precision"):
        g.fused_geo_attention_v2(q, q, q, d, d, a, a, a, precision="fp16")


def test_compute_dtype_selection():
    q32, qbf = torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8, dtype=torch.bfloat16)
    assert gv2._compute_dtype(q32, "auto", "reference") == torch.float32
    assert gv2._compute_dtype(qbf, None, "reference") == torch.bfloat16
    assert gv2._compute_dtype(q32, "bf16", "reference") == torch.bfloat16
    assert gv2._compute_dtype(qbf, "tf32", "reference") == torch.float32
    with pytest.raises(TypeError):
        gv2._compute_dtype(q32.half(), "auto", "reference")


def test_patch_model_validates_before_patching():
    class Att(torch.nn.Module):
        pass

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.encoder_layers = torch.nn.ModuleList([torch.nn.Module()])
            self.encoder_layers[0].self_attn = Att()

    m = Model()
    with pytest.raises(ValueError):
        g.patch_model(m, precision="int8")
    with pytest.raises(NotImplementedError):
        g.patch_model(m, mode="additive")
    assert "scaled_dot_product_attention" not in m.encoder_layers[0].self_attn.__dict__
    g.patch_model(m, precision="bf16")
    assert callable(m.encoder_layers[0].self_attn.__dict__["scaled_dot_product_attention"])


def test_dense_prior_arguments_checked_before_any_launch():
    """dist / ang must be [N, N] on one CUDA device (the reference's kernels read them with two strides)."""
    with pytest.raises(ValueError, match=r"\[N, N\]"):
        g.prior_from_dense(torch.zeros(1, 8, 8), torch.zeros(1, 8, 8), torch.float32)
    with pytest.raises(ValueError, match="CUDA"):
        g.prior_from_dense(torch.zeros(8, 8), torch.zeros(8, 8), torch.float32)


def test_tensors_on_other_devices_rejected():
    """Every tensor a launch reads or writes must live on q's device; the check names the first one that does not."""
    q = torch.zeros(1, 1, 4, 8)
    gv2._same_device(q, k=torch.zeros(1, 1, 4, 8), abg=torch.zeros(3))
    with pytest.raises(ValueError, match="abg lives on meta"):
        gv2._same_device(q, k=torch.zeros(1, 1, 4, 8), abg=torch.zeros(3, device="meta"))
