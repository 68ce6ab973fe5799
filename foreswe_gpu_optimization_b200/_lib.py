"""ctypes binding of libgeoattn.so (the C ABI declared in include/geoattn.h).

The library is built in-tree by ``foreswe_gpu_optimization_b200.build.build()``. Loading fails loudly: there is no
CPU or eager fallback for the hot path.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgeoattn.so")
ABI_VERSION = 2  # GEOATTN_VERSION of include/geoattn.h that these ctypes structures mirror

GEOATTN_OK = 0
DTYPE_BF16, DTYPE_FP32 = 0, 1

EXPORTED = ("geoattn_version", "geoattn_error_string", "geoattn_prior_bytes", "geoattn_prior_from_dense",
            "geoattn_prior_from_coords", "geoattn_stats_bytes", "geoattn_fwd_workspace_bytes",
            "geoattn_bwd_workspace_bytes", "geoattn_fwd", "geoattn_bwd", "geoattn_bwd_noalloc",
            "geoattn_read_status", "geoattn_wait_selftest")

c_ll4 = ctypes.c_longlong * 4


class Shape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int), ("heads", ctypes.c_int), ("n", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("dtype", ctypes.c_int), ("per_head", ctypes.c_int)]


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride", c_ll4)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("shape", Shape), ("q", Tensor), ("k", Tensor), ("v", Tensor), ("abg", ctypes.c_void_p),
                ("prior", ctypes.c_void_p), ("o", ctypes.c_void_p), ("o_stride", c_ll4), ("stats", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("events", ctypes.c_void_p)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("shape", Shape), ("q", Tensor), ("k", Tensor), ("v", Tensor), ("o", Tensor), ("dout", Tensor),
                ("abg", ctypes.c_void_p), ("prior", ctypes.c_void_p), ("stats", ctypes.c_void_p),
                ("dq", ctypes.c_void_p), ("dq_stride", c_ll4), ("dk", ctypes.c_void_p), ("dk_stride", c_ll4),
                ("dv", ctypes.c_void_p), ("dv_stride", c_ll4), ("dabg", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("events", ctypes.c_void_p)]


class GeoAttnError(RuntimeError):
    """A non-zero status from libgeoattn (the message is geoattn_error_string(code))."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


_LIB = None


def lib():
    """Load libgeoattn.so once; raise if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libgeoattn.so is not built (run foreswe_gpu_optimization_b200.build.build()); "
                               "the geo-attention path has no fallback")
        L = ctypes.CDLL(LIB_PATH)
        sp = ctypes.POINTER(Shape)
        L.geoattn_version.restype = ctypes.c_int
        L.geoattn_error_string.restype = ctypes.c_char_p
        L.geoattn_error_string.argtypes = [ctypes.c_int]
        for fn in ("geoattn_prior_bytes", "geoattn_stats_bytes", "geoattn_fwd_workspace_bytes",
                   "geoattn_bwd_workspace_bytes"):
            getattr(L, fn).restype = ctypes.c_size_t
            getattr(L, fn).argtypes = [sp]
        L.geoattn_prior_from_dense.restype = ctypes.c_int
        L.geoattn_prior_from_dense.argtypes = [sp, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p,
                                               ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
        L.geoattn_prior_from_coords.restype = ctypes.c_int
        L.geoattn_prior_from_coords.argtypes = [sp] + [ctypes.c_void_p] * 7
        L.geoattn_fwd.restype = ctypes.c_int
        L.geoattn_fwd.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
        L.geoattn_bwd.restype = ctypes.c_int
        L.geoattn_bwd.argtypes = [ctypes.POINTER(BwdArgs), ctypes.c_void_p]
        L.geoattn_bwd_noalloc.restype = ctypes.c_int
        L.geoattn_bwd_noalloc.argtypes = [ctypes.POINTER(BwdArgs), ctypes.c_void_p]
        L.geoattn_read_status.restype = ctypes.c_int
        L.geoattn_read_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
        L.geoattn_wait_selftest.restype = ctypes.c_int
        L.geoattn_wait_selftest.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        if L.geoattn_version() != ABI_VERSION:  # argument structs of another layout: refuse before any call
            raise RuntimeError("%s has ABI version %d, this binding expects %d; rebuild it"
                               % (LIB_PATH, L.geoattn_version(), ABI_VERSION))
        _LIB = L
    return _LIB


def check(rc):
    if rc != GEOATTN_OK:
        raise GeoAttnError(rc, "libgeoattn: " + lib().geoattn_error_string(rc).decode())


def tensor_arg(t):
    return Tensor(ctypes.c_void_p(t.data_ptr()), c_ll4(*t.stride()))
