"""Fused geo-biased station attention on B200 -- drop-in for foreswe_bench/geo_attention_v2.py.

Public surface mirrored from the reference (foreswe_bench/geo_attention_v2.py):
  * ``fused_geo_attention_v2(q, k, v, dist, ang, alpha, beta, gamma)``   (:464-465)
  * ``patch_model(model, preset=...)``                                   (:468-478)
  * ``use_preset(name)``, ``PRESETS``, ``CFG``                           (:370-378)
  * ``FusedGeoAttentionV2`` autograd Function                           (:401-461)
plus the coordinate form ``geo_attention(q, k, v, geometry, alpha, beta, gamma)`` whose prior comes from a
``StationGeometry`` (no [N, N] matrix).

Semantics follow the reference: q/k/v are [B, H, N, D] (any strides, e.g. the transposed split_heads views,
custom_encoder_model.py:41-43); gradients are returned with the inputs' strides; alpha/beta/gamma are [1]
(reference) or [H] (per head); ``mask`` must be None (the reference asserts the same, :475). Unlike the reference,
the output dtype is the input dtype.

``precision`` selects the kernels: "auto" (default) follows the input dtype (bf16 inputs run the BF16 tensor-core
path, fp32 inputs the TF32 path); "bf16" runs the BF16 kernels on fp32 inputs too (inputs rounded to bf16, output
and gradients returned in the input dtype); "tf32" runs the TF32 kernels on bf16 inputs (widened to fp32). ``mode``
is "reference" (the operator above, the only one the reference has). The numerics presets of the reference are
accepted for compatibility; the kernels always use the accurate formulation (correctly repeated scaled scores,
delta2 consistent with the recomputed tiles, round-to-nearest TF32 operands, split 3-term TF32 for the
score-shaped products).
"""
import ctypes

import torch

from . import _lib
from .geometry import StationGeometry, prior_from_dense

# Optional per-kernel timing hook: lists of torch.cuda.Event (already recorded once, so their handles exist) that
# the library records around its kernels on the launching stream -- {"fwd": [2 events], "bwd": [4 events]}.
TIMING_EVENTS = {"fwd": None, "bwd": None}

PRESETS = {"accurate_experimental": dict(precision="auto"), "accurate_x3_experimental": dict(precision="auto"),
           "fast_experimental": dict(precision="auto")}
CFG = dict(PRESETS["accurate_experimental"])
LAUNCH_INFO = {}
PRECISIONS = ("auto", "bf16", "tf32")
MODES = ("reference",)


def _compute_dtype(q, precision, mode):
    """Storage dtype the kernels run in for `precision` ("auto" / None: q's dtype)."""
    if mode != "reference":
        raise NotImplementedError("mode=%r: only the reference operator (mode='reference') is implemented" % (mode,))
    precision = precision or CFG.get("precision", "auto")
    if precision not in PRECISIONS:
        raise ValueError("precision must be one of %s, got %r" % (PRECISIONS, precision))
    if precision == "bf16":
        return torch.bfloat16
    if precision == "tf32":
        return torch.float32
    if q.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("q, k, v must be bf16 or fp32 (or pass precision='bf16' / 'tf32')")
    return q.dtype


def _run(q, k, v, prior_fn, alpha, beta, gamma, precision, mode):
    """The autograd op in the kernels' dtype, with inputs converted and the output returned in q's dtype (the
    conversions are differentiable, so the gradients come back in the inputs' dtypes)."""
    cd = _compute_dtype(q, precision, mode)
    qc, kc, vc = (t if t.dtype == cd else t.to(cd) for t in (q, k, v))
    prior = prior_fn(cd) if q.numel() else torch.empty(0, dtype=torch.uint8, device=q.device)
    o = FusedGeoAttentionV2.apply(qc, kc, vc, prior, alpha, beta, gamma)
    return o if o.dtype == q.dtype else o.to(q.dtype)


def use_preset(name):
    CFG.update(PRESETS[name])


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _events(key):
    evs = TIMING_EVENTS.get(key)
    if not evs:
        return None
    arr = (ctypes.c_void_p * len(evs))(*[e.cuda_event for e in evs])
    return ctypes.cast(arr, ctypes.c_void_p), arr


def _tma_ready(t):
    """bf16 operands are read by TMA: head dim contiguous, base and other strides 16-byte aligned."""
    if t.dtype != torch.bfloat16:
        return t
    st = t.stride()
    ok = (st[3] == 1 and t.data_ptr() % 16 == 0 and all(s > 0 and (s * 2) % 16 == 0 for s in st[:3]))
    if ok:
        return t
    B, H, N, D = t.shape
    dp = (D + 7) // 8 * 8
    buf = torch.zeros(B, H, N, dp, dtype=t.dtype, device=t.device)
    buf[..., :D] = t
    return buf[..., :D]


def _abg(alpha, beta, gamma, H, device):
    sizes = {alpha.numel(), beta.numel(), gamma.numel()}
    if len(sizes) != 1 or sizes.pop() not in (1, H):
        raise ValueError("alpha, beta, gamma must all have 1 or H entries")
    per_head = int(alpha.numel() == H and H > 1)
    abg = torch.cat([t.detach().reshape(-1).to(device=device, dtype=torch.float32) for t in (alpha, beta, gamma)])
    return abg.contiguous(), per_head


def _same_device(q, **others):
    """Every tensor a launch reads or writes lives on q's device (the kernels dereference them there)."""
    for name, t in others.items():
        if t.device != q.device:
            raise ValueError("%s lives on %s, q on %s" % (name, t.device, q.device))


def _shape(q, per_head):
    B, H, N, D = q.shape
    return _lib.Shape(B, H, N, D, _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_FP32, per_head)


def _forward(q, k, v, prior, abg, per_head):
    """geoattn_fwd on torch tensors: returns (o, stats). q, k, v [B, H, N, D] bf16 or fp32 on one CUDA device."""
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must be [B, H, N, D] with equal shapes")
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must all be bf16 or all be fp32")
    if not q.is_cuda:
        raise RuntimeError("geo attention runs on CUDA tensors only (no CPU path)")
    _same_device(q, k=k, v=v, prior=prior, abg=abg)
    if q.numel() == 0:  # an empty batch, head or station set: nothing to launch
        return torch.empty_like(q), torch.empty(0, dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):  # the library launches on the current device's stream
        return _forward_launch(q, k, v, prior, abg, per_head)


def _forward_launch(q, k, v, prior, abg, per_head):
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    sh = _shape(q, per_head)
    L = _lib.lib()
    # O takes q's layout: for split_heads views of a [B, N, H*D] projection it is [B, N, H, D] in memory, so the
    # caller's combine_heads (transpose(1, 2).contiguous()) needs no copy and dO comes back as a strided view
    o = torch.empty_like(q)
    stats = torch.empty(L.geoattn_stats_bytes(ctypes.byref(sh)) // 4, dtype=torch.float32, device=q.device)
    ws = torch.empty(L.geoattn_fwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=q.device)
    args = _lib.FwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v),
                        ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                        ctypes.c_void_p(o.data_ptr()), _lib.c_ll4(*o.stride()),
                        ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(ws.data_ptr()))
    ev = _events("fwd")
    if ev:
        args.events = ev[0]
    _lib.check(L.geoattn_fwd(ctypes.byref(args), _stream()))
    return o, stats


def _backward(q, k, v, o, do, prior, abg, stats, per_head):
    """geoattn_bwd on torch tensors: returns (dq, dk, dv, dabg); dq/dk/dv keep the strides of q/k/v."""
    B, H, N, D = q.shape
    if q.numel() == 0:  # empty input: empty gradients, and the bias-parameter gradients are empty sums
        return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                torch.zeros(3 * (H if per_head else 1), dtype=torch.float32, device=q.device))
    _same_device(q, k=k, v=v, o=o, do=do, prior=prior, abg=abg, stats=stats)
    with torch.cuda.device(q.device):
        return _backward_launch(q, k, v, o, do, prior, abg, stats, per_head)


def _backward_launch(q, k, v, o, do, prior, abg, stats, per_head):
    H = q.shape[1]
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    do = _tma_ready(do.to(q.dtype))
    sh = _shape(q, per_head)
    L = _lib.lib()
    dq = torch.empty_strided(q.shape, q.stride(), dtype=q.dtype, device=q.device)
    dk = torch.empty_strided(k.shape, k.stride(), dtype=k.dtype, device=k.device)
    dv = torch.empty_strided(v.shape, v.stride(), dtype=v.dtype, device=v.device)
    nabg = H if per_head else 1
    dabg = torch.empty(3 * nabg, dtype=torch.float32, device=q.device)
    ws = torch.empty(L.geoattn_bwd_workspace_bytes(ctypes.byref(sh)), dtype=torch.uint8, device=q.device)
    args = _lib.BwdArgs(sh, _lib.tensor_arg(q), _lib.tensor_arg(k), _lib.tensor_arg(v), _lib.tensor_arg(o),
                        _lib.tensor_arg(do), ctypes.c_void_p(abg.data_ptr()), ctypes.c_void_p(prior.data_ptr()),
                        ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(dq.data_ptr()),
                        _lib.c_ll4(*dq.stride()), ctypes.c_void_p(dk.data_ptr()), _lib.c_ll4(*dk.stride()),
                        ctypes.c_void_p(dv.data_ptr()), _lib.c_ll4(*dv.stride()),
                        ctypes.c_void_p(dabg.data_ptr()), ctypes.c_void_p(ws.data_ptr()))
    ev = _events("bwd")
    if ev:
        args.events = ev[0]
    _lib.check(L.geoattn_bwd(ctypes.byref(args), _stream()))
    return dq, dk, dv, dabg


class FusedGeoAttentionV2(torch.autograd.Function):
    """O = softmax(alpha*softmax(QK^T/sqrt d) + beta*Dp + gamma*Ap) V on libgeoattn (fwd + bwd)."""

    @staticmethod
    def forward(ctx, q, k, v, prior, alpha, beta, gamma):
        abg, per_head = _abg(alpha, beta, gamma, q.shape[1], q.device)
        o, stats = _forward(q, k, v, prior, abg, per_head)
        ctx.save_for_backward(q, k, v, o, prior, abg, stats)
        ctx.per_head = per_head
        ctx.abg_meta = [(t.shape, t.dtype, t.device) for t in (alpha, beta, gamma)]
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, prior, abg, stats = ctx.saved_tensors
        dq, dk, dv, dabg = _backward(q, k, v, o, do, prior, abg, stats, ctx.per_head)
        nabg = q.shape[1] if ctx.per_head else 1
        grads = []
        for i, (shape, dtype, device) in enumerate(ctx.abg_meta):  # each gradient on its parameter's device
            grads.append(dabg[i * nabg:(i + 1) * nabg].reshape(shape).to(device=device, dtype=dtype))
        return dq, dk, dv, None, grads[0], grads[1], grads[2]


def fused_geo_attention_v2(q, k, v, dist, ang, alpha, beta, gamma, *, precision=None, mode="reference"):
    """The reference's call (dense [N, N] dist/ang): prior built on the device for this call."""
    return _run(q, k, v, lambda cd: prior_from_dense(dist, ang, cd), alpha, beta, gamma, precision, mode)


def geo_attention(q, k, v, geometry, alpha, beta, gamma, *, precision=None, mode="reference"):
    """Coordinate form: the prior comes from ``geometry`` (a StationGeometry), built once and cached."""
    if not isinstance(geometry, StationGeometry):
        raise TypeError("geometry must be a StationGeometry")
    if geometry.n != q.shape[2]:
        raise ValueError("geometry has %d stations, q has N = %d" % (geometry.n, q.shape[2]))
    return _run(q, k, v, geometry.prior, alpha, beta, gamma, precision, mode)


def patch_model(model, preset="accurate_experimental", geometry=None, precision=None, mode="reference"):
    """Swap every encoder layer's attention core for the B200 kernels (foreswe_bench/geo_attention_v2.py:468-478).

    With ``geometry`` (a StationGeometry) the layers ignore the dense (distances, angularities) arguments and use
    the coordinate prior; otherwise the prior is built from the dense arguments at each call. ``precision`` and
    ``mode`` are passed to every call (module docstring). ``preset="eager"`` restores the production method
    (foreswe_bench/geo_attention.py:326-328)."""
    if preset != "eager":
        if precision is not None and precision not in PRECISIONS:
            raise ValueError("precision must be one of %s, got %r" % (PRECISIONS, precision))
        if mode not in MODES:
            raise NotImplementedError("mode=%r: only the reference operator (mode='reference') is implemented" % (mode,))
    for layer in model.encoder_layers:
        att = layer.self_attn
        if preset == "eager":
            att.__dict__.pop("scaled_dot_product_attention", None)
            continue
        use_preset(preset)

        def core(Q, K, V, distances, angularities, mask=None, _att=att):
            assert mask is None, "ForeSWE never passes a mask"
            if geometry is not None:
                return geo_attention(Q, K, V, geometry, _att.alpha, _att.beta, _att.gamma, precision=precision,
                                     mode=mode)
            return fused_geo_attention_v2(Q, K, V, distances, angularities, _att.alpha, _att.beta, _att.gamma,
                                          precision=precision, mode=mode)
        att.scaled_dot_product_attention = core
    return model


def read_status(workspace):
    """Device status word of a workspace tensor (0 = ok); ``None`` reads the status word of the last
    ``geoattn_bwd_noalloc`` call on the current device. Synchronises the current stream."""
    st = ctypes.c_int(-1)
    ptr = ctypes.c_void_p(workspace.data_ptr() if workspace is not None else None)
    _lib.check(_lib.lib().geoattn_read_status(ptr, ctypes.byref(st), _stream()))
    return st.value
