"""Rotary embedding of q and k in one sm_100a launch (reference API:
solution/kernels/rope.py, ``fused_rope``; Qwen2 patch solution/rope.py:55-80).

    y = x * cos + rotate_half(x) * sin,   rotate_half(x) = cat(-x[D/2:], x[:D/2])

with eager PyTorch's rounding: each product is rounded to promote(x, cos)
before the sum, which is rounded again (solution/kernels/rope.py:1-15).  The
backward is the adjoint with products rounded to x's dtype.  q [B, Hq, S, D]
and k [B, Hk, S, D] may be strided views (the projections' transposed
[B, S, H, D] memory); cos/sin are [1 or B, S, D] with unit column stride and are
not differentiated.  Outputs are contiguous.  Only cos/sin and shapes are kept
for the backward (no activations).
"""

from __future__ import annotations

import ctypes

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .._spec import FLOATS, Operand, admit, refuse


def _strides(t, n):
    return (ctypes.c_int64 * n)(*t.stride()) if t is not None else None


def _launch(src_q, q_out, src_k, k_out, cos, sin, backward):
    b, hq, s, d = q_out.shape
    hk = k_out.shape[1] if k_out is not None else 0
    _lib.call("sb_rope",
              _lib.ptr(src_q), _lib.dtype_code(src_q.dtype) if src_q is not None else 0,
              _strides(src_q, 4), hq if src_q is not None else 0, _lib.ptr(q_out),
              _lib.dtype_code(q_out.dtype),
              _lib.ptr(src_k), _lib.dtype_code(src_k.dtype) if src_k is not None else 0,
              _strides(src_k, 4), hk if src_k is not None else 0, _lib.ptr(k_out),
              _lib.dtype_code(k_out.dtype) if k_out is not None else 0,
              cos.data_ptr(), sin.data_ptr(), _lib.dtype_code(cos.dtype), _strides(cos, 3),
              _strides(sin, 3), cos.shape[0], b, s, d, int(backward), _lib.stream_of(cos.device))


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cos, sin):
        yq = torch.empty(q.shape, device=q.device, dtype=torch.promote_types(q.dtype, cos.dtype))
        yk = torch.empty(k.shape, device=k.device, dtype=torch.promote_types(k.dtype, cos.dtype))
        if q.numel() or k.numel():
            _launch(q, yq, k, yk, cos, sin, backward=False)
        ctx.save_for_backward(cos, sin)
        ctx.shapes = (q.shape, k.shape)
        ctx.dtypes = (q.dtype, k.dtype)
        ctx.set_materialize_grads(False)
        frozen = [y for y, needed in zip((yq, yk), ctx.needs_input_grad[:2]) if not needed]
        if frozen:
            ctx.mark_non_differentiable(*frozen)
        return yq, yk

    @staticmethod
    @once_differentiable
    def backward(ctx, gq, gk):
        cos, sin = ctx.saved_tensors
        (q_shape, k_shape), (q_dtype, k_dtype) = ctx.shapes, ctx.dtypes
        want_q = gq is not None and ctx.needs_input_grad[0]
        want_k = gk is not None and ctx.needs_input_grad[1]
        dq = torch.empty(q_shape, device=cos.device, dtype=q_dtype) if want_q else None
        dk = torch.empty(k_shape, device=cos.device, dtype=k_dtype) if want_k else None
        if (want_q and dq.numel()) or (want_k and dk.numel()):
            # A side without a gradient is passed with zero heads.
            q_side = dq if want_q else torch.empty((q_shape[0], 0, q_shape[2], q_shape[3]),
                                                   device=cos.device, dtype=q_dtype)
            _launch(gq if want_q else None, q_side, gk if want_k else None, dk, cos, sin, backward=True)
        return dq, dk, None, None


def rope_fault(q, k, cos, sin):
    """Why (q, k, cos, sin) cannot take the fused kernel, or None."""
    try:
        device = q.device if isinstance(q, torch.Tensor) else None
        admit("fused_rope", device, q=(q, Operand(*FLOATS, ndim=4, layout="rows")),
              k=(k, Operand(*FLOATS, ndim=4, layout="rows")),
              cos=(cos, Operand(*FLOATS, ndim=3, layout="rows", frozen=True)),
              sin=(sin, Operand(*FLOATS, ndim=3, layout="rows", frozen=True)))
        b, _, s, d = q.shape
        if d == 0 or d % 2:
            refuse("fused_rope", f"head dimension {d} is not a positive even number")
        if k.shape[0] != b or tuple(k.shape[2:]) != (s, d):
            refuse("fused_rope", f"k {tuple(k.shape)} does not pair with q {tuple(q.shape)}")
        if cos.dtype != sin.dtype or cos.shape != sin.shape or cos.shape[0] not in (1, b) \
                or tuple(cos.shape[1:]) != (s, d):
            refuse("fused_rope", f"cos/sin {tuple(cos.shape)} do not match [1|{b}, {s}, {d}]")
        if torch.cuda.get_device_capability(q.device)[0] != 10:
            refuse("fused_rope", "not an sm_100 device")
    except ValueError as err:
        return str(err)
    return None


def fused_rope(q, k, cos, sin):
    """(q_rotated, k_rotated) for CUDA q/k [B, H, S, even D] and detached cos/sin
    [1|B, S, D] (unit last-dimension stride everywhere); ValueError otherwise."""
    fault = rope_fault(q, k, cos, sin)
    if fault is not None:
        raise ValueError(fault)
    with torch.cuda.device(q.device):
        return _Rotary.apply(q, k, cos, sin)
