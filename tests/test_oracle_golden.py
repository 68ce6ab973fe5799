"""The oracle against golden vectors produced by the reference's own code (tests/golden/make_golden.py)."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import acceptance, geo_attention as ga, geometry

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATTN = sorted(glob.glob(os.path.join(GOLD, "attn_*.npz")))
KEYS = ("output", "dQ", "dK", "dV", "dalpha", "dbeta", "dgamma")


def load(path):
    z = np.load(path)
    inp = [torch.from_numpy(z[n]) for n in ("q", "k", "v", "dist", "ang", "alpha", "beta", "gamma")]
    return inp, torch.from_numpy(z["do"]), {k: torch.from_numpy(z[k]) for k in KEYS}


@pytest.mark.parametrize("path", ATTN, ids=[os.path.basename(p)[5:-4] for p in ATTN])
def test_autograd_oracle_matches_reference(path):
    inp, do, gold = load(path)
    r = ga.grads(*inp, do)
    for k in KEYS:
        assert r[k].shape == gold[k].shape, k
        torch.testing.assert_close(r[k], gold[k], rtol=1e-12, atol=1e-14 * max(1.0, gold[k].abs().max().item()))


@pytest.mark.parametrize("path", ATTN, ids=[os.path.basename(p)[5:-4] for p in ATTN])
def test_analytic_backward_matches_reference(path):
    inp, do, gold = load(path)
    r = ga.analytic_grads(*inp, do)
    for k in KEYS:
        scale = max(1.0, gold[k].abs().max().item())
        torch.testing.assert_close(r[k].reshape(gold[k].shape), gold[k], rtol=1e-9, atol=1e-11 * scale)


def test_case_inputs_reproduce_reference_draws():
    """The restated seeded generator gives the reference's inputs bit for bit."""
    z = np.load(os.path.join(GOLD, "attn_moderate.npz"))
    inp = acceptance.case_inputs("moderate", B=1, H=2, N=65, D=48, seed=3)
    for n, t in zip(("q", "k", "v", "dist", "ang", "alpha", "beta", "gamma"), inp):
        assert np.array_equal(t.numpy(), z[n]), n


def test_geometry_matches_reference_dataloader():
    z = np.load(os.path.join(GOLD, "geometry.npz"))
    d, a = geometry.distance_and_angularity(z["lat"], z["lon"], z["elev_ft"])
    np.testing.assert_allclose(d, z["dist_km"], rtol=1e-14, atol=1e-9)
    np.testing.assert_array_equal(a, z["ang_deg"])


def test_kahan_angle_matches_reference():
    z = np.load(os.path.join(GOLD, "kahan.npz"))
    a = geometry.pairwise_vector_angle(z["vectors"])
    np.testing.assert_array_equal(a, z["angle"])
    assert a[0, 1] < 1e-15 and abs(a[0, 2] - np.pi) < 1e-15
    same = geometry.pairwise_vector_angle(np.array([[1.0, 2.0, 3.0], [1.0, 2.0, 3.0]]))
    assert np.all(same == 0.0)


def test_haversine_matches_sklearn():
    from sklearn.metrics.pairwise import haversine_distances
    rng = np.random.default_rng(5)
    lat, lon = rng.uniform(35, 49, 64), rng.uniform(-124, -104, 64)
    ref = haversine_distances(np.deg2rad(np.stack([lat, lon], 1))) * 6371
    np.testing.assert_allclose(geometry.haversine_km(lat, lon), ref, rtol=1e-13, atol=1e-9)


def test_haversine_known_answers():
    """A quarter meridian and antipodes on the 6371 km sphere."""
    d = geometry.haversine_km(np.array([0.0, 90.0, 0.0]), np.array([0.0, 0.0, 180.0]))
    assert d[0, 1] == pytest.approx(np.pi / 2 * 6371, rel=1e-15)
    assert d[0, 2] == pytest.approx(np.pi * 6371, rel=1e-15)
    assert np.all(np.diag(d) == 0)


def test_oracle_gradcheck_float64():
    """Finite-difference check of the oracle (benchmarks/attention_study.py:57-64 uses [1,2,8,16], seed 11)."""
    g = torch.Generator().manual_seed(11)
    x = [torch.randn(1, 2, 8, 16, generator=g, dtype=torch.float64, requires_grad=True) for _ in range(3)]
    dist = torch.rand(8, 8, generator=g, dtype=torch.float64) * 1500
    ang = torch.rand(8, 8, generator=g, dtype=torch.float64) * 20
    abg = [((torch.rand(1, generator=g, dtype=torch.float64) - 0.5) * 2).requires_grad_() for _ in range(3)]
    assert torch.autograd.gradcheck(ga.forward, (*x, dist, ang, *abg), eps=1e-6, atol=1e-8, rtol=1e-6)


def test_perhead_equal_values_reduce_to_scalar():
    inp = acceptance.case_inputs("moderate", B=1, H=3, N=12, D=8, seed=9)
    do = acceptance.grad_seed_do(inp[0].shape)
    r1 = ga.grads(*inp, do)
    per = inp[:5] + [t.repeat(3) for t in inp[5:]]
    r3 = ga.grads(*per, do)
    for k in ("output", "dQ", "dK", "dV"):
        torch.testing.assert_close(r1[k], r3[k])
    for k in ("dalpha", "dbeta", "dgamma"):
        torch.testing.assert_close(r1[k], r3[k].sum().reshape(1))


def test_acceptance_rule_flags_planted_error():
    """A mistake planted in the oracle's output must fail the 10x rule (the rule is not vacuous)."""
    inp = acceptance.case_inputs("random", B=1, H=2, N=16, D=8, seed=0)
    do = acceptance.grad_seed_do(inp[0].shape)
    good = ga.grads(*inp, do, dtype=torch.float32)
    res = acceptance.evaluate(good, inp, do, "fp32")
    assert all(r["passed"] for r in res.values())
    bad = dict(good)
    bad["dQ"] = good["dQ"].clone()
    bad["dQ"][0, 0, 0, 0] += 1e-3
    assert not acceptance.evaluate(bad, inp, do, "fp32")["dQ"]["passed"]


def test_eager_tf32_error_model_is_differentiable_and_lossier():
    inp = acceptance.case_inputs("moderate", B=1, H=2, N=24, D=16, seed=1)
    do = acceptance.grad_seed_do(inp[0].shape)
    ref = acceptance.reference(inp, do)
    e32, etf = acceptance.eager(inp, do, "fp32"), acceptance.eager(inp, do, "tf32")
    for k in ("output", "dQ", "dK", "dV"):
        assert acceptance.err(etf[k], ref[k])["max_abs"] > acceptance.err(e32[k], ref[k])["max_abs"]


@pytest.mark.parametrize("case", acceptance.CASES)
def test_oracle_reproduces_the_reference_recorded_norms(case):
    """The reference's recorded accuracy table holds the float64 reference's norm of the output and of every
    gradient for its six regimes at case_inputs' default shape with attn_check's dO; the oracle's draws and
    operator reproduce them (to ~1e-15 relative; a norm that is rounding noise around a true zero, d(alpha) of the
    `uniform` regime, only to that noise level)."""
    import json
    with open(os.path.join(GOLD, "regression_ref_norms.json")) as f:
        gold = json.load(f)
    B, H, N, D = gold["shape"]
    x = acceptance.case_inputs(case, B=B, H=H, N=N, D=D)
    ref = acceptance.reference(x, acceptance.grad_seed_do(x[0].shape))
    for key in KEYS:
        want = gold["ref_norm"][case][key]
        got = torch.linalg.vector_norm(ref[key].double()).item()
        if want > 1e-12:
            assert abs(got - want) <= 1e-12 * want, (key, got, want)
        else:
            assert got <= 1e-15, (key, got, want)
