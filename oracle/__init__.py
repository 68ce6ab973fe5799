"""CPU oracle for the geo-biased station attention path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, the reference's algorithm for the hot path:

* ``oracle.geometry``      -- station geometry (haversine km, Kahan 2*atan2 angle in degrees)
                              following fore_swe/extended_dl_forecasting.py:20-30 and :305-352;
* ``oracle.geo_attention`` -- the two-softmax geo-biased attention operator and its gradients
                              following fore_swe/custom_encoder_model.py:25-39 and
                              foreswe_bench/geo_attention.py:311-319;
* ``oracle.acceptance``    -- the reference's seeded input regimes and its 10x-eager acceptance rule
                              following foreswe_bench/attn_check.py:16-81.

Parity is pinned: tests/test_oracle_golden.py checks every function here against golden vectors that
tests/golden/make_golden.py produced by running the reference's own code (eager_geo_attention with
autograd in float64, pairwise_vector_angle, the DataLoader geometry methods and sklearn's haversine).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import this package, and only
as the checker or the timed CPU baseline. The product path (foreswe_gpu_optimization_b200) never imports it.
"""
