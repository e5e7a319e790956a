"""Residual addition and Qwen2 RMSNorm in one forward/backward row pass.

Mirror of solution/kernels/add_rmsnorm.py.  Let s = cast(residual + delta,
promote(residual, delta)), r = rsqrt(mean(s^2) + eps), q = cast(s*r, s.dtype),
y = weight * q in promote(s, weight) (or fp16 when out_dtype=torch.float16).
Backward: u = cast(g_y * w, s.dtype), a = s * r,
ds = g_s + cast(r * (u - a * mean(u * a)), s.dtype), cast to each input dtype;
the optional weight gradient uses the two-stage atomic-free reduction.
Kernels: sb_add_rmsnorm_fwd / sb_add_rmsnorm_bwd / sb_rmsnorm_weight_grad.
"""

from __future__ import annotations

import math
import numbers

import torch
from torch.autograd.function import once_differentiable

from .. import _lib


def _weight_grad(s2d, gy2d, rstd, weight, exact_is_half):
    rows, h = s2d.shape
    dw = torch.empty(weight.shape, device=weight.device, dtype=weight.dtype)
    nbytes = _lib.query("sb_rmsnorm_weight_grad_workspace_bytes", rows, h)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=weight.device)
    _lib.call("sb_rmsnorm_weight_grad", s2d.data_ptr(), _lib.dtype_code(s2d.dtype), s2d.stride(0),
              gy2d.data_ptr(), _lib.dtype_code(gy2d.dtype), gy2d.stride(0), gy2d.stride(1),
              rstd.data_ptr(), dw.data_ptr(), _lib.dtype_code(dw.dtype), rows, h, int(exact_is_half),
              ws.data_ptr(), nbytes, _lib.stream_of(weight.device))
    return dw


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, residual, delta, weight, eps, out_dtype):
        h = residual.shape[-1]
        rows = math.prod(residual.shape[:-1])
        sum_dtype = torch.promote_types(residual.dtype, delta.dtype)
        exact_dtype = torch.promote_types(sum_dtype, weight.dtype)
        new_residual = torch.empty(residual.shape, device=residual.device, dtype=sum_dtype)
        normed = torch.empty(residual.shape, device=residual.device, dtype=out_dtype or exact_dtype)
        rstd = torch.empty(rows, device=residual.device, dtype=torch.float32)
        if rows:
            _lib.call("sb_add_rmsnorm_fwd", residual.data_ptr(), _lib.dtype_code(residual.dtype),
                      delta.data_ptr(), _lib.dtype_code(delta.dtype), weight.data_ptr(),
                      _lib.dtype_code(weight.dtype), weight.stride(0), new_residual.data_ptr(),
                      normed.data_ptr(), _lib.dtype_code(normed.dtype), rstd.data_ptr(), rows, h,
                      float(eps), _lib.stream_of(residual.device))
        ctx.save_for_backward(new_residual, weight, rstd)
        ctx.residual_dtype, ctx.delta_dtype = residual.dtype, delta.dtype
        ctx.exact_dtype, ctx.rows = exact_dtype, rows
        ctx.set_materialize_grads(False)
        return new_residual, normed

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_residual, grad_normed):
        s, weight, rstd = ctx.saved_tensors
        rows, h = ctx.rows, s.shape[-1]
        need_r, need_d, need_w = ctx.needs_input_grad[:3]
        dr = torch.empty(s.shape, device=s.device, dtype=ctx.residual_dtype) if need_r else None
        dd = torch.empty(s.shape, device=s.device, dtype=ctx.delta_dtype) if need_d else None
        dw = None
        if rows and (need_r or need_d):
            gs = grad_residual.reshape(rows, h) if grad_residual is not None else None
            gy = grad_normed.reshape(rows, h) if grad_normed is not None else None
            _lib.call("sb_add_rmsnorm_bwd", s.data_ptr(), _lib.dtype_code(s.dtype), weight.data_ptr(),
                      _lib.dtype_code(weight.dtype), weight.stride(0), rstd.data_ptr(),
                      _lib.ptr(gs), _lib.dtype_code(gs.dtype) if gs is not None else 0,
                      gs.stride(0) if gs is not None else 0, gs.stride(1) if gs is not None else 0,
                      _lib.ptr(gy), _lib.dtype_code(gy.dtype) if gy is not None else 0,
                      gy.stride(0) if gy is not None else 0, gy.stride(1) if gy is not None else 0,
                      _lib.ptr(dr), _lib.dtype_code(ctx.residual_dtype), _lib.ptr(dd),
                      _lib.dtype_code(ctx.delta_dtype), rows, h, _lib.stream_of(s.device))
        if need_w:
            if rows and grad_normed is not None:
                dw = _weight_grad(s.reshape(rows, h), grad_normed.reshape(rows, h), rstd, weight,
                                  ctx.exact_dtype == torch.float16)
            else:
                dw = torch.zeros(weight.shape, device=weight.device, dtype=weight.dtype)
        return dr, dd, dw, None, None


def add_rms_norm(residual, delta, weight, eps, out_dtype=None):
    """Return residual+delta and its Qwen2 RMSNorm; inputs must be contiguous CUDA.

    residual/delta/weight support fp16/fp32.  Shapes of the two inputs must
    agree, and weight is [H].  out_dtype is None (exact eager promotion) or
    torch.float16 (cast the exact result).  Only first derivatives are supported.
    """
    if residual.shape != delta.shape or residual.ndim < 1 or residual.shape[-1] == 0:
        raise ValueError("Expected matching residual/delta [...,H] with positive H")
    if weight.ndim != 1 or weight.shape[0] != residual.shape[-1]:
        raise ValueError("Expected weight[H]")
    if not residual.is_cuda or delta.device != residual.device or weight.device != residual.device:
        raise ValueError("All inputs must be on the same CUDA device")
    if not residual.is_contiguous() or not delta.is_contiguous():
        raise ValueError("residual and delta must be contiguous")
    if any(t.dtype not in (torch.float16, torch.float32) for t in (residual, delta, weight)):
        raise ValueError("Only fp16/fp32 inputs are supported")
    if out_dtype not in (None, torch.float16):
        raise ValueError("out_dtype must be None or torch.float16")
    if not isinstance(eps, numbers.Real) or not math.isfinite(eps) or eps < 0:
        raise ValueError("eps must be a finite nonnegative scalar")
    with torch.cuda.device(residual.device):
        return _AddRMSNorm.apply(residual, delta, weight, eps, out_dtype)
