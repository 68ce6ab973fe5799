"""The call site the drop-in replaces: the reference's own MultiHeadAttention (fore_swe/custom_encoder_model.py:7-58).

* The fixture tests/golden/mha_reference.npz holds the reference class's parameters, inputs, output and gradients
  (float64), written by tests/golden/make_golden.py from the class's source. The test suite's mirror of that call
  site (helpers.MHA: W_q/W_k/W_v, split_heads views, the attention core, combine_heads, W_o) reproduces them here,
  so a GPU test that patches the mirror checks the kernels against the reference class's own numbers.
* With the reference checkout named by the REFERENCE_ROOT environment variable, patch_model is applied to an instance of the reference class itself, with the attention core routed to the float64
  oracle, and must leave its output unchanged -- the method swap, the argument order (Q, K, V, distances,
  angularities, mask=None) and the bias parameters read from the module are those of the reference's call.
"""
import importlib.util
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from helpers import MHA

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mha_reference.npz")
REF_ROOT = os.environ.get("REFERENCE_ROOT", "")
REF_SRC = os.path.join(REF_ROOT, "fore_swe", "custom_encoder_model.py") if REF_ROOT else ""


def _mirror_from_fixture(z, dtype=torch.float64, device="cpu"):
    heads = int(z["heads"])
    d_model = z["x"].shape[-1]
    m = MHA(d_model, heads).to(device=device, dtype=dtype)
    state = {k[len("param."):]: torch.from_numpy(z[k]) for k in z.files if k.startswith("param.")}
    m.load_state_dict(state)
    return m


def test_mirror_reproduces_reference_class_fixture():
    z = np.load(GOLD)
    m = _mirror_from_fixture(z)
    x = torch.from_numpy(z["x"]).requires_grad_(True)
    dist, ang = torch.from_numpy(z["dist"]), torch.from_numpy(z["ang"])
    out = m(x, dist, ang)
    (out * torch.from_numpy(z["gout"])).sum().backward()
    np.testing.assert_allclose(out.detach().numpy(), z["out"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(x.grad.numpy(), z["grad_x"], rtol=1e-10, atol=1e-12)
    for name, p in m.named_parameters():
        np.testing.assert_allclose(p.grad.numpy(), z["grad." + name], rtol=1e-10, atol=1e-12, err_msg=name)


@pytest.mark.skipif(not (REF_SRC and os.path.exists(REF_SRC)), reason="REFERENCE_ROOT (reference checkout) not set")
def test_patch_model_on_the_reference_class(monkeypatch):
    from foreswe_gpu_optimization_b200 import geo_attention_v2 as gv2
    from oracle import geo_attention as oga
    spec = importlib.util.spec_from_file_location("ref_custom_encoder_model", REF_SRC)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    z = np.load(GOLD)
    torch.manual_seed(0)
    holder = nn.Module()
    holder.encoder_layers = nn.ModuleList([nn.Module()])
    att = mod.MultiHeadAttention(int(z["x"].shape[-1]), int(z["heads"])).double()
    att.load_state_dict({k[len("param."):]: torch.from_numpy(z[k]) for k in z.files if k.startswith("param.")})
    holder.encoder_layers[0].self_attn = att
    x = torch.from_numpy(z["x"])
    dist, ang = torch.from_numpy(z["dist"]), torch.from_numpy(z["ang"])
    ref = att(x, x, x, dist, ang)
    np.testing.assert_allclose(ref.detach().numpy(), z["out"], rtol=1e-12, atol=1e-12)

    calls = []

    def core_on_oracle(q, k, v, d, a, alpha, beta, gamma, *, precision=None, mode="reference"):
        calls.append((q.shape, alpha is att.alpha, beta is att.beta, gamma is att.gamma, d is dist, a is ang))
        return oga.forward(q, k, v, d, a, alpha, beta, gamma)

    monkeypatch.setattr(gv2, "fused_geo_attention_v2", core_on_oracle)
    gv2.patch_model(holder)
    out = att(x, x, x, dist, ang)
    assert calls == [((2, int(z["heads"]), x.shape[1], x.shape[2] // int(z["heads"])), True, True, True, True, True)]
    np.testing.assert_allclose(out.detach().numpy(), z["out"], rtol=1e-12, atol=1e-12)
    with pytest.raises(AssertionError, match="mask"):
        att.scaled_dot_product_attention(x, x, x, dist, ang, mask=torch.ones(1))
    gv2.patch_model(holder, "eager")
    assert "scaled_dot_product_attention" not in att.__dict__
