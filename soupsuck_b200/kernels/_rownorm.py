"""Launch helpers for the row-normalisation kernels (csrc/rowwise.cuh).

One place that turns row-major matrices into the C-ABI calls of the residual
add-RMSNorm and the plain RMSNorm, forward and backward, and the deterministic
weight-gradient reduction they share.  Shapes and dtypes are validated by the
public entries (``add_rmsnorm.py``, ``rmsnorm.py``) before these are called.
"""

from __future__ import annotations

import torch

from .. import _lib


def _code(t):
    return _lib.dtype_code(t.dtype)


def _strides(t):
    return (t.stride(0), t.stride(1)) if t is not None else (0, 0)


def residual_norm_forward(residual, delta, weight, eps, s, y, rstd, rows, width):
    _lib.call("sb_add_rmsnorm_fwd", residual.data_ptr(), _code(residual), delta.data_ptr(), _code(delta),
              weight.data_ptr(), _code(weight), weight.stride(0), s.data_ptr(), y.data_ptr(), _code(y),
              rstd.data_ptr(), rows, width, float(eps), _lib.stream_of(residual.device))


def residual_norm_backward(s, weight, rstd, grad_s, grad_y, d_residual, residual_dtype, d_delta,
                           delta_dtype, rows, width):
    gs_rs, gs_cs = _strides(grad_s)
    gy_rs, gy_cs = _strides(grad_y)
    _lib.call("sb_add_rmsnorm_bwd", s.data_ptr(), _code(s), weight.data_ptr(), _code(weight),
              weight.stride(0), rstd.data_ptr(),
              _lib.ptr(grad_s), _code(grad_s) if grad_s is not None else 0, gs_rs, gs_cs,
              _lib.ptr(grad_y), _code(grad_y) if grad_y is not None else 0, gy_rs, gy_cs,
              _lib.ptr(d_residual), _lib.dtype_code(residual_dtype), _lib.ptr(d_delta),
              _lib.dtype_code(delta_dtype), rows, width, _lib.stream_of(s.device))


def norm_forward(x2d, weight, eps, y, rstd):
    rows, width = x2d.shape
    _lib.call("sb_rmsnorm_fwd", x2d.data_ptr(), _code(x2d), x2d.stride(0), weight.data_ptr(),
              _code(weight), weight.stride(0), y.data_ptr(), _code(y), rstd.data_ptr(), rows, width,
              float(eps), _lib.stream_of(x2d.device))


def norm_input_grad(x2d, weight, g2d, rstd, dx):
    rows, width = x2d.shape
    _lib.call("sb_rmsnorm_input_grad", x2d.data_ptr(), _code(x2d), x2d.stride(0), weight.data_ptr(),
              _code(weight), weight.stride(0), g2d.data_ptr(), _code(g2d), g2d.stride(0), g2d.stride(1),
              rstd.data_ptr(), dx.data_ptr(), rows, width, _lib.stream_of(x2d.device))


def weight_grad(x2d, g2d, rstd, weight, half_products):
    """dweight[j] = sum_rows g[row, j] * q[row, j], q the normalised input before the
    weight; ``half_products`` rounds each product to fp16 (when the norm's exact
    output dtype is fp16, as eager PyTorch does).  Two stages, fixed order."""
    rows, width = x2d.shape
    dw = torch.empty(weight.shape, device=weight.device, dtype=weight.dtype)
    if rows == 0:
        return dw.zero_()
    nbytes = _lib.query("sb_rmsnorm_weight_grad_workspace_bytes", rows, width)
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=weight.device)
    _lib.call("sb_rmsnorm_weight_grad", x2d.data_ptr(), _code(x2d), x2d.stride(0), g2d.data_ptr(),
              _code(g2d), g2d.stride(0), g2d.stride(1), rstd.data_ptr(), dw.data_ptr(), _code(dw),
              rows, width, int(half_products), scratch.data_ptr(), nbytes, _lib.stream_of(weight.device))
    return dw
