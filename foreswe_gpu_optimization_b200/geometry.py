"""Station geometry on the device: the geo prior from per-station coordinates.

Replaces the reference's bias construction (fore_swe/extended_dl_forecasting.py:305-352), which builds float64
[N, N] distance/angle matrices on the host once per run and copies fp32 slices to the GPU every step
(foreswe_bench/data.py:58-59). Here the coordinates live on the device ([N] float64 each) and one kernel evaluates,
per station pair and in float64, the 6371 km haversine and Kahan's 2*atan2 angle between the reference's station
vectors (including its [x, y, x] component order and its km + feet*0.3048 radius), rounds both to fp32 as the
reference's fp32 copies are, and writes the prior table Dp = 1/(1+dist), Ap = 1/(1+ang) consumed by the attention
kernels. The table is 2 x N_pad^2 pairs (fp16 pairs for bf16 inputs, fp32 pairs for fp32 inputs; 2 MiB at N = 512,
resident in L2), built once per geometry and reused by every layer, head and step.
"""
import ctypes

import torch

from . import _lib


def _shape(n, dtype, batch=1, heads=1, head_dim=64, per_head=0):
    return _lib.Shape(batch, heads, n, head_dim, _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_FP32,
                      per_head)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def prior_from_dense(dist, ang, dtype):
    """Prior table from dense [N, N] distance (km) / angle (deg) matrices, the reference's call signature."""
    n = dist.shape[-1]
    if dist.shape != (n, n) or ang.shape != (n, n):
        raise ValueError("dist and ang must be [N, N], got %s and %s" % (tuple(dist.shape), tuple(ang.shape)))
    if not dist.is_cuda or ang.device != dist.device:
        raise ValueError("dist and ang must be on one CUDA device, got %s and %s" % (dist.device, ang.device))
    dist = dist.detach().float().contiguous()
    ang = ang.detach().float().contiguous()
    sh = _shape(n, dtype)
    L = _lib.lib()
    with torch.cuda.device(dist.device):  # the library launches on the current device's stream
        prior = torch.empty(L.geoattn_prior_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=dist.device)
        _lib.check(L.geoattn_prior_from_dense(ctypes.byref(sh), ctypes.c_void_p(dist.data_ptr()), n,
                                              ctypes.c_void_p(ang.data_ptr()), n, ctypes.c_void_p(prior.data_ptr()),
                                              _stream()))
    return prior


class StationGeometry:
    """Per-station coordinates resident on one device, with the prior tables built on demand (cached per dtype).

    lat_deg, lon_deg: degrees; elev_ft: elevation in feet (the reference's unit; use ``from_metres`` for metres).
    """

    def __init__(self, lat_deg, lon_deg, elev_ft, device="cuda"):
        self.lat = torch.as_tensor(lat_deg, dtype=torch.float64).to(device).contiguous()
        self.lon = torch.as_tensor(lon_deg, dtype=torch.float64).to(device).contiguous()
        self.elev_ft = torch.as_tensor(elev_ft, dtype=torch.float64).to(device).contiguous()
        if not (self.lat.shape == self.lon.shape == self.elev_ft.shape and self.lat.dim() == 1):
            raise ValueError("lat, lon, elev must be 1-D tensors of equal length")
        self.n = self.lat.numel()
        self._prior = {}

    @classmethod
    def from_metres(cls, lat_deg, lon_deg, elev_m, device="cuda"):
        return cls(lat_deg, lon_deg, torch.as_tensor(elev_m, dtype=torch.float64) / 0.3048, device)

    @property
    def device(self):
        return self.lat.device

    def prior(self, dtype):
        key = torch.bfloat16 if dtype == torch.bfloat16 else torch.float32
        if key not in self._prior:
            sh = _shape(self.n, key)
            L = _lib.lib()
            with torch.cuda.device(self.device):
                t = torch.empty(L.geoattn_prior_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=self.device)
                _lib.check(L.geoattn_prior_from_coords(ctypes.byref(sh), ctypes.c_void_p(self.lat.data_ptr()),
                                                       ctypes.c_void_p(self.lon.data_ptr()),
                                                       ctypes.c_void_p(self.elev_ft.data_ptr()),
                                                       ctypes.c_void_p(t.data_ptr()), None, None, _stream()))
            self._prior[key] = t
        return self._prior[key]

    def distance_and_angularity(self):
        """fp32 [N, N] (distance_km, angle_deg) on the device -- DataLoader.getDistanceAndAngularity's outputs,
        for callers that keep the reference's (distances, angularities) arguments."""
        sh = _shape(self.n, torch.float32)
        dist = torch.empty(self.n, self.n, dtype=torch.float32, device=self.device)
        ang = torch.empty_like(dist)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().geoattn_prior_from_coords(
                ctypes.byref(sh), ctypes.c_void_p(self.lat.data_ptr()), ctypes.c_void_p(self.lon.data_ptr()),
                ctypes.c_void_p(self.elev_ft.data_ptr()), None, ctypes.c_void_p(dist.data_ptr()),
                ctypes.c_void_p(ang.data_ptr()), _stream()))
        return dist, ang
