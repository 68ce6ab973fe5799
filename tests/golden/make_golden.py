"""Generate the golden vectors that pin the oracle, by running the REFERENCE's own code.

Run once in a container that has the reference checkout (read-only) at REF_ROOT:

    python tests/golden/make_golden.py REF_ROOT      (REF_ROOT: the reference checkout, required)

It writes tests/golden/*.npz. What each file holds and which reference code produced it:

* attn_<case>.npz   foreswe_bench.attn_check.case_inputs(..., device="cpu") draws the inputs (the reference's
                    own seeded generator); foreswe_bench.geo_attention.eager_geo_attention with torch autograd in
                    float64 gives output, dQ, dK, dV, dalpha, dbeta, dgamma for a fixed dO.
* attn_moderate_d192.npz  one "moderate" instance at the reference's default head dim D = 192.
* attn_perhead.npz  the same operator with per-head alpha/beta/gamma of shape [1, H, 1, 1] (reference broadcasting).
* attn_stations.npz real station geometry (below) as dist/ang, cast to fp32 as foreswe_bench/data.py:58-59 does.
* geometry.npz      the first 48 stations of data/snotel_location_info_2.csv (lat, lon, elevation in feet) and
                    DataLoader.getHaversineDistance / getAlgularityOfLocations (fore_swe/extended_dl_forecasting.py
                    :305-344, executed from source with ast because the module imports sentence-transformers).
* kahan.npz         fore_swe/extended_dl_forecasting.py:20-30 pairwise_vector_angle on seeded vectors.
* regression_ref_norms.json  the float64 reference norms of the output and of every gradient that the reference
                    recorded for its six regimes at case_inputs' default shape (1, 4, 128, 192) with attn_check's
                    dO (engineering_audit/optimization/fused_attention/benchmark_results/final/regression_table.csv,
                    column ref_norm; the same for every preset and precision).
"""
import ast
import contextlib
import csv
import io
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if len(sys.argv) != 2 or not os.path.isdir(sys.argv[1]):
    sys.exit("usage: python make_golden.py <path of the reference checkout>")
REF = os.path.abspath(sys.argv[1])
sys.path.insert(0, REF)

from foreswe_bench.attn_check import case_inputs  # noqa: E402
from foreswe_bench.geo_attention import eager_geo_attention  # noqa: E402

DL_SRC = os.path.join(REF, "fore_swe", "extended_dl_forecasting.py")


def _exec_functions(names, cls=None):
    """Exec selected top-level functions (or methods of class ``cls``) from the reference's DataLoader module."""
    with open(DL_SRC) as f:
        tree = ast.parse(f.read())
    body = tree.body
    if cls is not None:
        body = [n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls][0].body
    fns = [n for n in body if isinstance(n, ast.FunctionDef) and n.name in names]
    from sklearn.metrics.pairwise import haversine_distances
    ns = {"np": np, "haversine_distances": haversine_distances}
    exec(compile(ast.Module(body=fns, type_ignores=[]), DL_SRC, "exec"), ns)
    return ns


def ref_grads(inputs, do):
    x = [t.detach().double().requires_grad_(i in (0, 1, 2, 5, 6, 7)) for i, t in enumerate(inputs)]
    o = eager_geo_attention(*x)
    o.backward(do.double())
    return dict(output=o.detach(), dQ=x[0].grad, dK=x[1].grad, dV=x[2].grad,
                dalpha=x[5].grad, dbeta=x[6].grad, dgamma=x[7].grad)


def save_attn(name, inputs, do):
    r = ref_grads(inputs, do)
    q, k, v, dist, ang, a, b, c = inputs
    np.savez_compressed(os.path.join(HERE, name + ".npz"),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), dist=dist.numpy(), ang=ang.numpy(),
                        alpha=a.numpy(), beta=b.numpy(), gamma=c.numpy(), do=do.numpy(),
                        **{key: val.numpy() for key, val in r.items()})


def save_regression_norms():
    path = os.path.join(REF, "engineering_audit", "optimization", "fused_attention", "benchmark_results", "final",
                        "regression_table.csv")
    norms = {}
    with open(path) as f:
        for row in csv.DictReader(f):
            seen = norms.setdefault(row["case"], {}).setdefault(row["quantity"], float(row["ref_norm"]))
            assert seen == float(row["ref_norm"]), row  # one reference per (case, quantity)
    with open(os.path.join(HERE, "regression_ref_norms.json"), "w") as f:
        json.dump({"shape": [1, 4, 128, 192], "source": os.path.relpath(path, REF), "ref_norm": norms}, f, indent=1)


def save_reference_mha():
    """The reference's own MultiHeadAttention (fore_swe/custom_encoder_model.py:7-58), imported from its source file,
    run forward and backward in float64 on seeded inputs: its parameters, inputs, output and every gradient, so a GPU
    test can check that the patched call site reproduces the reference class's numbers."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_custom_encoder_model",
                                                  os.path.join(REF, "fore_swe", "custom_encoder_model.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    torch.manual_seed(2024)
    B, N, d_model, heads = 2, 48, 64, 4
    mha = mod.MultiHeadAttention(d_model, heads).double()
    with torch.no_grad():                      # bias parameters in the trained model's range
        mha.alpha.fill_(0.8)
        mha.beta.fill_(0.3)
        mha.gamma.fill_(-0.4)
    g = torch.Generator().manual_seed(2025)
    x = (torch.randn(B, N, d_model, generator=g, dtype=torch.float64) * 0.5).requires_grad_(True)
    dist = torch.rand(N, N, generator=g, dtype=torch.float64) * 1500
    dist = (dist + dist.T) / 2
    dist.fill_diagonal_(0)
    ang = torch.rand(N, N, generator=g, dtype=torch.float64) * 20
    ang = (ang + ang.T) / 2
    ang.fill_diagonal_(0)
    gout = torch.randn(B, N, d_model, generator=g, dtype=torch.float64)
    out = mha(x, x, x, dist, ang)
    (out * gout).sum().backward()
    arrays = {"x": x.detach().numpy(), "dist": dist.numpy(), "ang": ang.numpy(), "gout": gout.numpy(),
              "out": out.detach().numpy(), "grad_x": x.grad.numpy(), "heads": np.array(heads)}
    for name, prm in mha.named_parameters():
        arrays["param." + name] = prm.detach().numpy()
        arrays["grad." + name] = prm.grad.numpy()
    np.savez_compressed(os.path.join(HERE, "mha_reference.npz"), **arrays)


def main():
    torch.manual_seed(0)
    cases = [("random", 1, 2, 32, 16, 0), ("near_one_hot", 1, 2, 33, 16, 1), ("uniform", 1, 1, 16, 8, 2),
             ("moderate", 1, 2, 65, 48, 3), ("wide_signed", 1, 2, 24, 12, 4), ("large_alpha", 2, 1, 20, 8, 5)]
    for case, B, H, N, D, seed in cases:
        inp = case_inputs(case, B=B, H=H, N=N, D=D, seed=seed, device="cpu")
        g = torch.Generator().manual_seed(1234 + seed)
        save_attn("attn_" + case, inp, torch.randn(inp[0].shape, generator=g))

    # the reference's default head dim (case_inputs' D = 192), one small instance
    inp = case_inputs("moderate", B=1, H=1, N=40, D=192, seed=8, device="cpu")
    g = torch.Generator().manual_seed(1242)
    save_attn("attn_moderate_d192", inp, torch.randn(inp[0].shape, generator=g))

    # per-head bias parameters, broadcast by the reference operator itself
    inp = case_inputs("moderate", B=2, H=3, N=17, D=8, seed=7, device="cpu")
    g = torch.Generator().manual_seed(77)
    a = (torch.rand(3, generator=g) * 0.9 + 0.1).reshape(1, 3, 1, 1)
    b = (torch.randn(3, generator=g) * 0.5).reshape(1, 3, 1, 1)
    c = (torch.randn(3, generator=g) * 0.5).reshape(1, 3, 1, 1)
    save_attn("attn_perhead", inp[:5] + [a, b, c], torch.randn(inp[0].shape, generator=g))

    # real station geometry through the reference's DataLoader methods
    import pandas as pd
    info = pd.read_csv(os.path.join(REF, "data", "snotel_location_info_2.csv"))
    locs = info.loc[:47, ["Station Name", "Elevation", "Latitude", "Longitude"]]
    ns = _exec_functions({"getHaversineDistance", "getAlgularityOfLocations"}, cls="DataLoader")
    ns.update(_exec_functions({"pairwise_vector_angle"}))
    # the methods refer to pairwise_vector_angle as a module global
    ns["getAlgularityOfLocations"].__globals__["pairwise_vector_angle"] = ns["pairwise_vector_angle"]
    with contextlib.redirect_stdout(io.StringIO()):  # the methods print their matrices
        dist = ns["getHaversineDistance"](None, locs)
        ang = ns["getAlgularityOfLocations"](None, locs)
    np.savez_compressed(os.path.join(HERE, "geometry.npz"), lat=locs["Latitude"].to_numpy(np.float64),
                        lon=locs["Longitude"].to_numpy(np.float64), elev_ft=locs["Elevation"].to_numpy(np.float64),
                        dist_km=dist, ang_deg=ang)

    g = torch.Generator().manual_seed(11)
    B, H, N, D = 1, 2, 48, 16
    q, k, v = (torch.randn(B, H, N, D, generator=g) * 2 for _ in range(3))
    abg = [torch.tensor([x]) for x in (0.6, 0.4, -0.3)]
    save_attn("attn_stations", [q, k, v, torch.from_numpy(dist).float(), torch.from_numpy(ang).float()] + abg,
              torch.randn(B, H, N, D, generator=g))

    rng = np.random.default_rng(0)
    vec = rng.normal(size=(40, 3)) * 6371.0
    vec[1] = vec[0] * 3.0                                  # parallel pair -> exactly 0
    vec[2] = -vec[0]                                       # antiparallel pair -> pi
    np.savez_compressed(os.path.join(HERE, "kahan.npz"), vectors=vec, angle=ns["pairwise_vector_angle"](vec))
    save_regression_norms()
    save_reference_mha()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
