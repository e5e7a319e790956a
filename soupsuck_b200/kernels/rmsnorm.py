"""Qwen2 RMSNorm with explicit cast order and an optional weight gradient.

Mirror of solution/kernels/rmsnorm.py: r = rsqrt(mean(x^2) + eps), a = x*r in
fp32, q = cast(a, x.dtype), y = weight * q in promote(x, weight) (or fp16).
Backward: u = cast(g * weight, x.dtype), dx = r * (u - a * mean(u * a));
dweight = sum(g * q) (each product rounded to fp16 when the exact output is
fp16), two-stage and atomic-free.  Kernels: sb_rmsnorm_fwd /
sb_rmsnorm_input_grad / sb_rmsnorm_weight_grad.
"""

from __future__ import annotations

import math
import numbers

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .add_rmsnorm import _weight_grad


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype):
        h = x.shape[-1]
        rows = math.prod(x.shape[:-1])
        ctx.exact_dtype = torch.promote_types(x.dtype, weight.dtype)
        out = torch.empty(x.shape, device=x.device, dtype=out_dtype or ctx.exact_dtype)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        if rows:
            matrix = x if x.ndim == 2 else x.view(rows, h)
            _lib.call("sb_rmsnorm_fwd", matrix.data_ptr(), _lib.dtype_code(x.dtype), matrix.stride(0),
                      weight.data_ptr(), _lib.dtype_code(weight.dtype), weight.stride(0),
                      out.data_ptr(), _lib.dtype_code(out.dtype), rstd.data_ptr(), rows, h,
                      float(eps), _lib.stream_of(x.device))
        ctx.save_for_backward(x, weight, rstd)
        ctx.rows = rows
        ctx.set_materialize_grads(False)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        if grad is None:
            return None, None, None, None
        x, weight, rstd = ctx.saved_tensors
        h, rows = x.shape[-1], ctx.rows
        dx = dw = None
        matrix = x if x.ndim == 2 else x.view(rows, h)
        gmatrix = grad.reshape(rows, h)
        if ctx.needs_input_grad[0]:
            dx = torch.empty(x.shape, device=x.device, dtype=x.dtype)
            if rows:
                _lib.call("sb_rmsnorm_input_grad", matrix.data_ptr(), _lib.dtype_code(x.dtype),
                          matrix.stride(0), weight.data_ptr(), _lib.dtype_code(weight.dtype),
                          weight.stride(0), gmatrix.data_ptr(), _lib.dtype_code(gmatrix.dtype),
                          gmatrix.stride(0), gmatrix.stride(1), rstd.data_ptr(), dx.data_ptr(),
                          rows, h, _lib.stream_of(x.device))
        if ctx.needs_input_grad[1]:
            if rows:
                dw = _weight_grad(matrix, gmatrix, rstd, weight, ctx.exact_dtype == torch.float16)
            else:
                dw = torch.zeros(weight.shape, device=weight.device, dtype=weight.dtype)
        return dx, dw, None, None


def rms_norm(x, weight, eps, out_dtype=None):
    """Normalize the last contiguous dimension, preserving Qwen2 cast semantics."""
    if x.ndim < 1 or x.shape[-1] == 0 or weight.ndim != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError("Expected x[...,H] and weight[H] with positive H")
    if not x.is_cuda or weight.device != x.device:
        raise ValueError("x and weight must be on the same CUDA device")
    if x.stride(-1) != 1:
        raise ValueError("The last input dimension must be contiguous")
    if not x.is_contiguous() and x.ndim != 2:
        raise ValueError("Noncontiguous leading dimensions require a 2-D input")
    if x.dtype not in (torch.float16, torch.float32) or weight.dtype not in (torch.float16, torch.float32):
        raise ValueError("RMSNorm supports only fp16/fp32 input and weight")
    if not isinstance(eps, numbers.Real) or not math.isfinite(eps) or eps < 0:
        raise ValueError("eps must be a finite nonnegative scalar")
    if out_dtype not in (None, torch.float16):
        raise ValueError("out_dtype must be None or torch.float16")
    with torch.cuda.device(x.device):
        return _RMSNorm.apply(x, weight, eps, out_dtype)
