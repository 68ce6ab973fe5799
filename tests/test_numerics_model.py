"""The kernels' numerics choices, checked on the CPU through a float32 model of their arithmetic.

tests/numerics_model.py restates the formulation the kernels evaluate (log2-domain softmaxes, the exact bound of the
second softmax, the row-record backward) with the kernels' rounding points. Against the float64 oracle:

* the model meets the path's tolerances (rel-L2 8e-3 BF16, 5e-4 TF32) on the benchmark's input distribution, plain
  and with x30 logits, at head dims 64 and 192, and the reference's 10x-eager rule in its six regimes at D = 192;
* one TF32 term for the score-shaped products (QK^T, dO V^T) breaks the 5e-4 bound at x30 logits, and one term for
  dO V^T alone breaks it for the bias-parameter gradients; three terms hold it -- why the kernels issue three;
* the BF16 backward's row sums (delta2, a) come from the recomputed tiles, not from the stored output;
* storing the prior as fp16 pairs (BF16 path) leaves O, dQ, dK, dV where they were and costs d(gamma) ~3e-4;
* d(alpha) from the explicit dZ, sum dZ (P1 - b), as the TF32 row pass computes it, is orders of magnitude closer
  than a - delta2 b where the true d(alpha) is ~0 (the reference's `uniform` regime, Q = 0).
"""
import pytest
import torch

import numerics_model as nm
from helpers import KEYS, TOL, attn_inputs, dense_geometry, rel_l2, stations
from oracle import acceptance
from oracle import geo_attention as oga


def _rels(res, ref):
    return {key: rel_l2(res[key], ref[key]) for key in KEYS}


def _plain_inputs(D, qscale, bf16):
    q, k, v, a, b, c, do = attn_inputs(1, 4, 256, D, seed=1, qscale=qscale)
    if bf16:  # the oracle sees exactly the bf16 values the kernels read
        q, k, v, do = (t.to(torch.bfloat16).float() for t in (q, k, v, do))
    dist, ang = dense_geometry(*stations(256, 2))
    return (q, k, v, dist, ang, a, b, c, do)


@pytest.mark.parametrize("path", ["bf16", "tf32"])
@pytest.mark.parametrize("D", [64, 192])
@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "x30"])
def test_model_meets_the_path_tolerances(path, D, qscale):
    x = _plain_inputs(D, qscale, path == "bf16")
    rels = _rels(nm.grads(*x, path=path), oga.grads(*x))
    tol = TOL[torch.bfloat16 if path == "bf16" else torch.float32]
    assert all(e <= tol for e in rels.values()), rels


@pytest.mark.parametrize("case", acceptance.CASES)
def test_tf32_model_passes_the_reference_rule_at_d192(case):
    """The reference's acceptance rule (max-abs error within 10x eager TF32's, foreswe_bench/attn_check.py:68-81)
    at its own acceptance shape (1, 2, 100, 192)."""
    x = acceptance.case_inputs(case, B=1, H=2, N=100, D=192)
    do = acceptance.grad_seed_do(x[0].shape)
    ev = acceptance.evaluate(nm.grads(*x, do, path="tf32"), x, do, "tf32")
    assert all(r["passed"] for r in ev.values()), {key: r["ratio_to_eager"] for key, r in ev.items()}


@pytest.mark.parametrize("D", [64, 192])
def test_one_tf32_term_for_the_scores_fails_at_x30_logits(D):
    x = _plain_inputs(D, 30.0, False)
    ref = oga.grads(*x)
    one = _rels(nm.grads(*x, path="tf32", score_terms=1), ref)
    three = _rels(nm.grads(*x, path="tf32", score_terms=3), ref)
    assert max(one["dQ"], one["dK"]) > TOL[torch.float32], one
    assert max(three.values()) <= TOL[torch.float32], three


@pytest.mark.parametrize("case", ["random", "moderate", "large_alpha"])
def test_one_tf32_term_for_dO_Vt_breaks_the_bias_gradients(case):
    """With QK^T in three terms but dO V^T in one, d(alpha), d(beta), d(gamma) (sums of dZ over N^2 elements, dZ
    being a difference of dP and its row mean) leave the 5e-4 bound; three terms keep them far inside."""
    x = acceptance.case_inputs(case, B=1, H=2, N=100, D=192)
    do = acceptance.grad_seed_do(x[0].shape)
    ref = oga.grads(*x, do)
    one = _rels(nm.grads(*x, do, path="tf32", dp_terms=1), ref)
    three = _rels(nm.grads(*x, do, path="tf32"), ref)
    bias = ("dalpha", "dbeta", "dgamma")
    assert max(one[key] for key in bias) > TOL[torch.float32], one
    assert max(three[key] for key in bias) <= 0.2 * TOL[torch.float32], three


@pytest.mark.parametrize("case", ["near_one_hot", "wide_signed", "large_alpha"])
def test_bf16_row_sums_come_from_the_tiles(case):
    """delta1 = alpha (a - delta2 b) is a difference of nearly equal sums in saturated rows, so a, delta2 and b must
    come from the same bf16-rounded tiles as dZ: taken from the stored output instead (delta2 = dO . O,
    a = dO . O'), the variant that would drop the BF16 row pass's sweep leaves dQ and dK off by several 1e-2."""
    x = acceptance.case_inputs(case, B=1, H=2, N=100, D=192)
    do = acceptance.grad_seed_do(x[0].shape)
    x = [t.to(torch.bfloat16).float() if i < 3 else t for i, t in enumerate(x)]
    do = do.to(torch.bfloat16).float()
    ref = oga.grads(*x, do)
    tiles = _rels(nm.grads(*x, do, path="bf16"), ref)
    output = _rels(nm.grads(*x, do, path="bf16", row_sums="output"), ref)
    assert max(tiles.values()) <= TOL[torch.bfloat16], tiles
    assert min(output["dQ"], output["dK"]) > 2 * TOL[torch.bfloat16], output


def test_fp16_prior_pairs_cost_little():
    x = _plain_inputs(64, 1.0, True)
    ref = oga.grads(*x)
    r16 = _rels(nm.grads(*x, path="bf16", prior_fp16=True), ref)
    r32 = _rels(nm.grads(*x, path="bf16", prior_fp16=False), ref)
    for key in ("output", "dQ", "dK", "dV"):
        assert abs(r16[key] - r32[key]) <= 0.05 * r32[key], (key, r16[key], r32[key])
    assert r16["dgamma"] <= 1e-3 and r16["dbeta"] <= 1e-3, r16


def test_dalpha_from_explicit_dz_where_it_vanishes():
    """Q = 0: P1 is uniform and the true d(alpha) is ~0. The recomputed P2 rows sum to 1 + eps, so a - delta2 b
    carries a bias of order eps * delta2; sum dZ (P1 - b) cancels it."""
    x = acceptance.case_inputs("uniform", B=1, H=2, N=100, D=192)
    do = acceptance.grad_seed_do(x[0].shape)
    ref, eag = acceptance.reference(x, do), acceptance.eager(x, do, "tf32")
    err = {}
    for form in ("dz", "a-d2b"):
        ev = acceptance.evaluate(nm.grads(*x, do, path="tf32", dalpha_form=form), x, do, "tf32", ref=ref, eag=eag)
        err[form] = ev["dalpha"]["candidate"]["max_abs"]
        bound = ev["dalpha"]["bound"]
    assert err["dz"] <= 1e-3 * bound, (err, bound)
    assert err["dz"] * 100 <= err["a-d2b"], err


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "x30"])
def test_single_score_pass_forward_with_fp16_p1(D, qscale):
    """A BF16 forward with one score pass (2^(t - m_c) kept as fp16 per 128-key chunk, scaled in pass B) meets the
    BF16 tolerance and moves the errors by a few per cent of the two-pass forward's; the reference's regimes too."""
    x = _plain_inputs(D, qscale, True)
    ref = oga.grads(*x)
    one = _rels(nm.grads(*x, path="bf16", fwd_p1="fp16_chunks"), ref)
    two = _rels(nm.grads(*x, path="bf16"), ref)
    assert all(e <= TOL[torch.bfloat16] for e in one.values()), one
    for key in KEYS:
        assert one[key] <= 1.1 * two[key] + 1e-5, (key, one[key], two[key])


@pytest.mark.parametrize("case", acceptance.CASES)
def test_single_score_pass_forward_reference_regimes(case):
    q, k, v, dist, ang, a, b, c = acceptance.case_inputs(case, B=1, H=2, N=300, D=128)
    do = acceptance.grad_seed_do(q.shape)
    q, k, v, do = (t.to(torch.bfloat16).float() for t in (q, k, v, do))
    x = (q, k, v, dist, ang, a, b, c)
    ref = oga.grads(*x, do)
    one = _rels(nm.grads(*x, do, path="bf16", fwd_p1="fp16_chunks"), ref)
    two = _rels(nm.grads(*x, do, path="bf16"), ref)
    for key in KEYS:
        assert one[key] <= 1.1 * two[key] + 1e-5, (case, key, one[key], two[key])


@pytest.mark.parametrize("qscale", [1.0, 30.0], ids=["plain", "x30"])
def test_single_score_pass_forward_tf32_d64(qscale):
    """The TF32 forward at head dim 64 keeps the same fp16 values: within the TF32 tolerance and within 10 % of the
    two-pass forward's error (its P enters P.V as a TF32 operand, 11 bits like fp16)."""
    x = _plain_inputs(64, qscale, False)
    ref = oga.grads(*x)
    one = _rels(nm.grads(*x, path="tf32", fwd_p1="fp16_chunks"), ref)
    two = _rels(nm.grads(*x, path="tf32"), ref)
    assert all(e <= TOL[torch.float32] for e in one.values()), one
    for key in KEYS:
        assert one[key] <= 1.1 * two[key] + 1e-6, (key, one[key], two[key])


@pytest.mark.parametrize("case", acceptance.CASES)
def test_single_score_pass_forward_tf32_reference_rule(case):
    """The reference's 10x-eager rule (foreswe_bench/attn_check.py:68-81) at head dim 64 with the fp16 values."""
    x = acceptance.case_inputs(case, B=1, H=2, N=100, D=64)
    do = acceptance.grad_seed_do(x[0].shape)
    ev = acceptance.evaluate(nm.grads(*x, do, path="tf32", fwd_p1="fp16_chunks"), x, do, "tf32")
    assert all(r["passed"] for r in ev.values()), {key: r["ratio_to_eager"] for key, r in ev.items()}

