"""Vanilla LoRA scale/add, preserving eager intermediate rounding.

Mirror of solution/kernels/lora_epilogue.py: out = base + cast_A(adapter * s)
(optionally cast to the base dtype first), computed by ``sb_lora_scale_add``;
backward casts the gradient to the adapter dtype before scaling
(``sb_lora_scale_grad``).  Bit-exact with eager PyTorch for fp16/fp32 combinations.
The fused QLoRA projection (nf4_gemm.nf4_lora_linear) folds this epilogue into
the GEMM accumulator instead; this module serves the patched PEFT path that
keeps PEFT's own LoRA modules.
"""

from __future__ import annotations

import math
import numbers

import torch
from torch.autograd.function import once_differentiable

from .. import _lib


class _LoRAEpilogue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, result, lora_out, scaling, cast_to_result):
        dtype = result.dtype if cast_to_result else torch.promote_types(result.dtype, lora_out.dtype)
        out = torch.empty(result.shape, device=result.device, dtype=dtype)
        if result.numel():
            _lib.call("sb_lora_scale_add", result.data_ptr(), _lib.dtype_code(result.dtype),
                      lora_out.data_ptr(), _lib.dtype_code(lora_out.dtype), out.data_ptr(),
                      _lib.dtype_code(dtype), result.numel(), float(scaling), int(cast_to_result),
                      _lib.stream_of(result.device))
        ctx.result_dtype, ctx.adapter_dtype = result.dtype, lora_out.dtype
        ctx.scaling, ctx.shape = float(scaling), result.shape
        ctx.set_materialize_grads(False)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        if grad is None:
            return None, None, None, None
        d_result = grad.to(ctx.result_dtype) if ctx.needs_input_grad[0] else None
        d_adapter = None
        if ctx.needs_input_grad[1]:
            grad = grad.contiguous()
            d_adapter = torch.empty(ctx.shape, device=grad.device, dtype=ctx.adapter_dtype)
            if grad.numel():
                _lib.call("sb_lora_scale_grad", grad.data_ptr(), _lib.dtype_code(grad.dtype),
                          d_adapter.data_ptr(), _lib.dtype_code(ctx.adapter_dtype), grad.numel(),
                          ctx.scaling, _lib.stream_of(grad.device))
        return d_result, d_adapter, None, None


def lora_epilogue(result, lora_out, scaling, *, cast_to_result=False):
    """Return result + rounded(scaling * lora_out), with optional PEFT cast."""
    if (not result.is_cuda or result.device != lora_out.device
            or result.shape != lora_out.shape):
        raise ValueError("Expected equal-shaped result/LoRA tensors on one CUDA device")
    if result.dtype not in (torch.float16, torch.float32) or lora_out.dtype not in (torch.float16, torch.float32):
        raise ValueError("LoRA epilogue supports fp16/fp32 tensors")
    if not isinstance(scaling, numbers.Real) or not math.isfinite(scaling):
        raise ValueError("scaling must be a finite real scalar")
    if not isinstance(cast_to_result, bool):
        raise ValueError("cast_to_result must be bool")
    with torch.cuda.device(result.device):
        return _LoRAEpilogue.apply(result.contiguous(), lora_out.contiguous(), scaling, cast_to_result)
