"""Residual addition fused with the Qwen2 RMSNorm that follows it (reference API:
solution/kernels/add_rmsnorm.py, ``add_rms_norm``).

Arithmetic and cast order, which the reference pins against eager PyTorch
(solution/kernels/add_rmsnorm.py:37-81):

    s    = cast(residual + delta, promote(residual, delta))
    rstd = 1 / sqrt(mean(s^2) + eps)                         (fp32)
    y    = weight * cast(s * rstd, s.dtype)   in promote(s, weight), or fp16 if asked

    backward:  u = cast(g_y * weight, s.dtype),  a = s * rstd
               ds = g_s + cast(rstd * (u - a * mean(u * a)), s.dtype)
               d_residual = cast(ds, residual.dtype), d_delta = cast(ds, delta.dtype)

One sm_100a row kernel per direction (``sb_add_rmsnorm_fwd`` / ``_bwd``: the row
stays in registers, 16-byte vectors for fp16); the weight gradient is the
shared two-stage reduction.  Autograd keeps s, weight and rstd only.
"""

from __future__ import annotations

import math

import torch
from torch.autograd.function import once_differentiable

from .._spec import FLOATS, HALF, Choice, Number, Operand, admit, refuse
from . import _rownorm


class _ResidualNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, residual, delta, weight, eps, out_dtype):
        width = residual.shape[-1]
        rows = math.prod(residual.shape[:-1])
        sum_dtype = torch.promote_types(residual.dtype, delta.dtype)
        norm_dtype = torch.promote_types(sum_dtype, weight.dtype)
        s = torch.empty(residual.shape, device=residual.device, dtype=sum_dtype)
        y = torch.empty(residual.shape, device=residual.device, dtype=out_dtype or norm_dtype)
        rstd = torch.empty(rows, device=residual.device, dtype=torch.float32)
        if rows:
            _rownorm.residual_norm_forward(residual, delta, weight, eps, s, y, rstd, rows, width)
        ctx.save_for_backward(s, weight, rstd)
        ctx.dtypes = (residual.dtype, delta.dtype)
        ctx.half_products = norm_dtype == HALF
        ctx.set_materialize_grads(False)
        return s, y

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_s, grad_y):
        s, weight, rstd = ctx.saved_tensors
        width = s.shape[-1]
        rows = s.numel() // width if width else 0
        want_residual, want_delta, want_weight = ctx.needs_input_grad[:3]
        residual_dtype, delta_dtype = ctx.dtypes
        d_residual = torch.empty(s.shape, device=s.device, dtype=residual_dtype) if want_residual else None
        d_delta = torch.empty(s.shape, device=s.device, dtype=delta_dtype) if want_delta else None
        gs = None if grad_s is None else grad_s.reshape(rows, width)
        gy = None if grad_y is None else grad_y.reshape(rows, width)
        if rows and (want_residual or want_delta):
            _rownorm.residual_norm_backward(s, weight, rstd, gs, gy, d_residual, residual_dtype,
                                            d_delta, delta_dtype, rows, width)
        d_weight = None
        if want_weight:
            if gy is None:
                d_weight = torch.zeros(weight.shape, device=weight.device, dtype=weight.dtype)
            else:
                d_weight = _rownorm.weight_grad(s.reshape(rows, width), gy, rstd, weight,
                                                ctx.half_products)
        return d_residual, d_delta, d_weight, None, None


def add_rms_norm(residual, delta, weight, eps, out_dtype=None):
    """(residual + delta, RMSNorm(residual + delta) * weight) for contiguous CUDA
    fp16/fp32 inputs [..., H] and weight [H]; ``out_dtype`` None keeps PyTorch's
    promotion for y, torch.float16 casts it.  First derivatives only."""
    entry = "add_rms_norm"
    device = residual.device if isinstance(residual, torch.Tensor) else None
    admit(entry, device, residual=(residual, Operand(*FLOATS)), delta=(delta, Operand(*FLOATS)),
          weight=(weight, Operand(*FLOATS, ndim=1, layout=None)),
          eps=(eps, Number(minimum=0)), out_dtype=(out_dtype, Choice(None, HALF)))
    if residual.shape != delta.shape or residual.ndim == 0 or residual.shape[-1] == 0:
        refuse(entry, f"residual {tuple(residual.shape)} and delta {tuple(delta.shape)} must be "
                      f"equal [..., H] shapes with H > 0")
    if weight.shape[0] != residual.shape[-1]:
        refuse(entry, f"weight has {weight.shape[0]} entries for rows of {residual.shape[-1]}")
    with torch.cuda.device(residual.device):
        return _ResidualNorm.apply(residual, delta, weight, eps, out_dtype)
