"""Qwen2 RMSNorm with the reference's cast order (reference API:
solution/kernels/rmsnorm.py, ``rms_norm``).

    rstd = 1 / sqrt(mean(x^2) + eps)      a = x * rstd (fp32)      q = cast(a, x.dtype)
    y    = weight * q   in promote(x, weight), or fp16 when asked

    backward:  u = cast(g * weight, x.dtype),  dx = rstd * (u - a * mean(u * a))
               dweight = sum over rows of g * q (products rounded to fp16 when the
               norm's exact output is fp16), reduced in a fixed order

Kernels ``sb_rmsnorm_fwd`` / ``sb_rmsnorm_input_grad`` / ``sb_rmsnorm_weight_grad``
(csrc/rowwise.cuh).  The input may be a 2-D view whose rows are strided; any
other input must be contiguous.
"""

from __future__ import annotations

import math

import torch
from torch.autograd.function import once_differentiable

from .._spec import FLOATS, HALF, Choice, Number, Operand, admit, refuse
from . import _rownorm


def _matrix(t, rows, width):
    return t if t.ndim == 2 else t.reshape(rows, width)


class _Norm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype):
        width = x.shape[-1]
        rows = math.prod(x.shape[:-1])
        norm_dtype = torch.promote_types(x.dtype, weight.dtype)
        y = torch.empty(x.shape, device=x.device, dtype=out_dtype or norm_dtype)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        if rows:
            _rownorm.norm_forward(_matrix(x, rows, width), weight, eps, y, rstd)
        ctx.save_for_backward(x, weight, rstd)
        ctx.half_products = norm_dtype == HALF
        ctx.set_materialize_grads(False)
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        if grad is None:
            return None, None, None, None
        x, weight, rstd = ctx.saved_tensors
        width = x.shape[-1]
        rows = rstd.numel()
        x2d, g2d = _matrix(x, rows, width), grad.reshape(rows, width)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(x.shape, device=x.device, dtype=x.dtype)
            if rows:
                _rownorm.norm_input_grad(x2d, weight, g2d, rstd, dx)
        if ctx.needs_input_grad[1]:
            dw = _rownorm.weight_grad(x2d, g2d, rstd, weight, ctx.half_products)
        return dx, dw, None, None


def rms_norm(x, weight, eps, out_dtype=None):
    """RMSNorm over the last dimension of CUDA fp16/fp32 ``x`` with weight [H]."""
    entry = "rms_norm"
    device = x.device if isinstance(x, torch.Tensor) else None
    admit(entry, device, x=(x, Operand(*FLOATS, layout="rows")),
          weight=(weight, Operand(*FLOATS, ndim=1, layout=None)),
          eps=(eps, Number(minimum=0)), out_dtype=(out_dtype, Choice(None, HALF)))
    if x.ndim == 0 or x.shape[-1] == 0 or weight.shape[0] != x.shape[-1]:
        refuse(entry, f"x {tuple(x.shape)} and weight {tuple(weight.shape)} must be [..., H] and [H], H > 0")
    if x.ndim != 2 and not x.is_contiguous():
        refuse(entry, "strided rows are accepted for 2-D inputs only")
    with torch.cuda.device(x.device):
        return _Norm.apply(x, weight, eps, out_dtype)
