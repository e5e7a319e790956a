"""PEFT ``Linear4bit.forward`` as one fused NF4 + LoRA projection.

Reference: solution/lora.py:135-164 patches peft/tuners/lora/bnb.py's
``Linear4bit.forward`` to run ``base_layer(x)`` (bnb NF4), then
``lora_B(lora_A(dropout(fp32(x))))`` under fp16 autocast, then the rounded
scale/add epilogue.  Here the whole projection

    Y = X . deq(W)^T + s * (X . A^T) . B^T (+ bias)

is ``nf4_lora_linear`` (one LoRA-factor kernel and one tcgen05 GEMM with the
LoRA product in the same TMEM accumulator; the backward gives dX through the
same GEMM and dA / dB through the rank-r reductions).  When LoRA dropout is
active (training with p > 0) the dropout runs first, on the reference's fp32
LoRA input (so the RNG stream is the reference's), and the same fused GEMM
takes the dropped activation for the LoRA factors and X for the NF4 base; the
backward adds the LoRA branch's input gradient through that dropout.

Numerics: the reference rounds the base result to fp16 and adds the fp16
rounded LoRA term in fp32; the fused kernel accumulates both in fp32 and rounds
once, so outputs agree to fp16 rounding (the GEMM gate: 2e-3 abs + 2e-3 rel).
Output dtype follows the reference: the input's dtype (bnb returns the input
dtype, and the epilogue promotes it with the fp16 adapter output or casts back).
"""

from functools import wraps
import math
import numbers
import sys

from .utils import enabled, no_hooks, supported_tensor

_MARKER = "_solution_lora_4bit_original"


def _nf4_base(layer):
    """The packed weight and quant_state of a bnb Linear4bit base, or None."""
    base = layer.base_layer
    if (type(base).__module__ != "bitsandbytes.nn.modules" or type(base).__name__ != "Linear4bit"
            or not no_hooks(base)):
        return None
    weight = getattr(base, "weight", None)
    state = getattr(weight, "quant_state", None)
    if state is None or getattr(weight, "requires_grad", True):
        return None
    import torch

    if getattr(base, "compute_dtype", torch.float16) not in (None, torch.float16):
        return None
    bias = getattr(base, "bias", None)
    if bias is not None and (bias.requires_grad or bias.dtype != torch.float16):
        return None
    from .kernels.nf4 import nested_shape

    packed = weight.data if weight.is_contiguous() else None
    if packed is None:
        return None
    packed = packed.reshape(-1, 1)
    try:
        n, k = nested_shape(packed, state, entry="Linear4bit")
    except ValueError:
        return None
    return packed, state, bias, n, k


def _eligible(layer, x, kwargs):
    """Structural and dtype conditions of the fused path (reference lora.py:70-108)."""
    import torch

    if (not enabled() or not supported_tensor(x) or x.ndim == 0 or x.data_ptr() % 16
            or kwargs.get("adapter_names") is not None or kwargs.get("alora_offsets") is not None
            or layer.disable_adapters or layer.merged or len(layer.active_adapters) != 1):
        return None
    adapter = layer.active_adapters[0]
    if (adapter not in layer.lora_A or adapter not in layer.lora_B
            or adapter in getattr(layer, "lora_variant", {})
            or getattr(layer, "use_dora", {}).get(adapter, False)):
        return None
    a, b = layer.lora_A[adapter], layer.lora_B[adapter]
    dropout, scaling = layer.lora_dropout[adapter], layer.scaling[adapter]
    if (type(a) is not torch.nn.Linear or type(b) is not torch.nn.Linear
            or a.bias is not None or b.bias is not None
            or type(dropout) not in (torch.nn.Dropout, torch.nn.Identity)
            or getattr(dropout, "inplace", False)
            or not all(no_hooks(m) for m in (a, b, dropout))
            or not supported_tensor(a.weight) or not supported_tensor(b.weight)
            or a.weight.device != x.device or b.weight.device != x.device
            or not isinstance(scaling, numbers.Real) or not math.isfinite(scaling)
            or a.weight.shape[0] > 64):
        return None
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") != torch.float16:
        return None
    base = _nf4_base(layer)
    if base is None:
        return None
    packed, state, bias, n, k = base
    if (x.shape[-1] != k or a.weight.shape[1] != k or b.weight.shape[0] != n
            or k % 32 or n % 32 or packed.device != x.device):
        return None
    return adapter, a, b, dropout, float(scaling), packed, state, bias


def _patch_class(cls, variant_kwarg_keys):
    original = cls.forward
    if hasattr(original, _MARKER):
        return

    @wraps(original)
    def forward(self, x, *args, **kwargs):
        import torch

        found = _eligible(self, x, kwargs) if not args else None
        if found is None:
            return original(self, x, *args, **kwargs)
        self._check_forward_args(x, *args, **kwargs)
        adapter, a, b, dropout, scaling, packed, state, bias = found
        from .kernels.nf4_gemm import nf4_lora_linear

        x16 = x if x.dtype == torch.float16 else x.to(torch.float16)
        active_dropout = (type(dropout) is torch.nn.Dropout and dropout.p > 0 and dropout.training)
        dropped = None
        if active_dropout:
            # The dropout mask is drawn exactly as the reference's LoRA branch draws
            # it (same input dtype, same point in the RNG stream); the fused GEMM
            # then feeds the dropped activation to the LoRA factors and the raw
            # input to the NF4 base in one accumulator.
            lora_input = x.float() if x.dtype == torch.float16 else x
            if not torch.is_autocast_enabled("cuda"):
                lora_input = lora_input.to(a.weight.dtype)
            dropped = dropout(lora_input)
        y = nf4_lora_linear(x16, packed, state, a.weight, b.weight, scaling, bias=bias,
                            lora_input=dropped)
        return y.to(x.dtype)

    setattr(forward, _MARKER, original)
    cls.forward = forward


def patch_lora_4bit():
    """Register on PEFT's bnb Linear4bit when PEFT is importable."""
    module = sys.modules.get("peft.tuners.lora.bnb")
    if module is None:
        try:
            import importlib

            module = importlib.import_module("peft.tuners.lora.bnb")
        except (ImportError, AttributeError):
            return False
    cls = getattr(module, "Linear4bit", None)
    if not isinstance(cls, type):
        return False
    _patch_class(cls, tuple(getattr(module, "VARIANT_KWARG_KEYS", ())))
    return True
