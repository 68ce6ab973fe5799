"""B200-native (sm_100a) fused geo-biased station attention for ForeSWE.

Drop-in for foreswe_bench/geo_attention_v2.py (same call surface) backed by libgeoattn.so: hand-written
tcgen05/TMA kernels with fp32 accumulators in tensor memory, forward and backward, bf16 and TF32.
"""
from .geo_attention_v2 import (CFG, PRESETS, FusedGeoAttentionV2, fused_geo_attention_v2, geo_attention,
                               patch_model, use_preset)
from .geometry import StationGeometry, prior_from_dense
from .streaming import HostBatchPipeline
from .custom_op import geo_attention_compiled, geo_attention_op

__all__ = ["CFG", "PRESETS", "FusedGeoAttentionV2", "fused_geo_attention_v2", "geo_attention", "patch_model",
           "use_preset", "StationGeometry", "prior_from_dense", "HostBatchPipeline", "geo_attention_op",
           "geo_attention_compiled"]
