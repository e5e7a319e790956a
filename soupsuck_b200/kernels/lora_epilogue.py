"""The LoRA scale/add epilogue of PEFT's forward with eager PyTorch rounding
(reference API: solution/kernels/lora_epilogue.py, ``lora_epilogue``).

    forward:   out = base + cast_adapter(adapter * s)        in promote(base, adapter),
               or cast to base's dtype first when cast_to_result (PEFT's no-autocast path)
    backward:  d_base = cast_base(g),  d_adapter = cast_adapter(g) * s

(solution/kernels/lora_epilogue.py:24-43: the scaled adapter output is rounded
to its own dtype before the addition, as ``result + lora_out * scaling`` does
eagerly.)  Element-wise sm_100a kernels ``sb_lora_scale_add`` /
``sb_lora_scale_grad``.  The fused projection ``nf4_lora_linear`` needs none of
this: its LoRA product is accumulated with the NF4 product in one accumulator.
"""

from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .._spec import FLOATS, Choice, Number, Operand, admit, refuse


class _ScaledAdd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, base, adapter, scaling, cast_to_result):
        dtype = base.dtype if cast_to_result else torch.promote_types(base.dtype, adapter.dtype)
        out = torch.empty(base.shape, device=base.device, dtype=dtype)
        if out.numel():
            _lib.call("sb_lora_scale_add", base.data_ptr(), _lib.dtype_code(base.dtype),
                      adapter.data_ptr(), _lib.dtype_code(adapter.dtype), out.data_ptr(),
                      _lib.dtype_code(dtype), out.numel(), float(scaling), int(cast_to_result),
                      _lib.stream_of(base.device))
        ctx.base_dtype, ctx.adapter_dtype, ctx.scaling = base.dtype, adapter.dtype, float(scaling)
        ctx.set_materialize_grads(False)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        if grad is None:
            return None, None, None, None
        d_base = grad.to(ctx.base_dtype) if ctx.needs_input_grad[0] else None
        d_adapter = None
        if ctx.needs_input_grad[1]:
            g = grad.contiguous()
            d_adapter = torch.empty(g.shape, device=g.device, dtype=ctx.adapter_dtype)
            if g.numel():
                _lib.call("sb_lora_scale_grad", g.data_ptr(), _lib.dtype_code(g.dtype),
                          d_adapter.data_ptr(), _lib.dtype_code(ctx.adapter_dtype), g.numel(),
                          ctx.scaling, _lib.stream_of(g.device))
        return d_base, d_adapter, None, None


def lora_epilogue(result, lora_out, scaling, *, cast_to_result=False):
    """result + rounded(scaling * lora_out) for equal-shaped CUDA fp16/fp32 tensors."""
    entry = "lora_epilogue"
    device = result.device if isinstance(result, torch.Tensor) else None
    admit(entry, device, result=(result, Operand(*FLOATS, layout=None)),
          lora_out=(lora_out, Operand(*FLOATS, layout=None)), scaling=(scaling, Number()),
          cast_to_result=(cast_to_result, Choice(False, True)))
    if result.shape != lora_out.shape:
        refuse(entry, f"result {tuple(result.shape)} and lora_out {tuple(lora_out.shape)} differ in shape")
    with torch.cuda.device(result.device):
        return _ScaledAdd.apply(result.contiguous(), lora_out.contiguous(), scaling, cast_to_result)
