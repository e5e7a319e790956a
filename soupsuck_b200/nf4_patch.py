"""bitsandbytes 0.50.2 NF4 entry points redirected to the sm_100a kernels.

Four library functions are replaced by wrappers that first try the library
here and otherwise call the function they replaced (kept on the wrapper under
the contract's marker attribute, ``_solution_fused_original``):

  bitsandbytes.functional.dequantize_4bit          nested fp16 NF4 -> sb_nf4_dequant_nested
  bitsandbytes.backends.cuda.ops._dequant_linear_fallback
                                                    records whether its fp32 scales were
                                                    rebuilt from a nested state
  bitsandbytes.backends.cuda.ops._dequantize_4bit_impl
                                                    inside such a call -> sb_nf4_dequant_flat
  bitsandbytes.matmul_4bit                          fp16 X . NF4 W^T as the fused tcgen05
                                                    GEMM (forward and dX); SOUP_EXP_NF4_GEMM=0
                                                    keeps bitsandbytes' own

Reference behaviour kept (solution/nf4_patch.py:43-125, solution/kernels/nf4_gemm.py:121-154):
only canonical nested fp16 NF4/block64 states are taken, anything the argument
contracts refuse (a ValueError) runs the replaced function, and an error from
a kernel launch propagates.  The nested-scales flag travels in a ContextVar,
because only the linear fallback knows where its scales came from while the
flat decoder it calls cannot tell.  Nothing here imports torch or the kernels
until a wrapper runs.
"""

from contextvars import ContextVar
from functools import wraps
import importlib
import os
from types import ModuleType

from .utils import enabled

_MARKER = "_solution_fused_original"
_PINNED_VERSION = "0.50.2"
# True only while bitsandbytes' linear fallback that rebuilt fp32 scales from a
# nested state is on the stack.
_NESTED_BACKEND = ContextVar("soupsuck_b200_nested_scales", default=False)


def _with_nested_flag(value, fn, *args, **kwargs):
    token = _NESTED_BACKEND.set(value)
    try:
        return fn(*args, **kwargs)
    finally:
        _NESTED_BACKEND.reset(token)


def _redirect(owner, attr, make):
    """Install ``make(original)`` as ``owner.attr`` unless a wrapper is already there."""
    original = getattr(owner, attr)
    if hasattr(original, _MARKER):
        return
    wrapper = wraps(original)(make(original))
    setattr(wrapper, _MARKER, original)
    setattr(owner, attr, wrapper)


def _cuda_tensor(value):
    import torch
    return isinstance(value, torch.Tensor) and value.is_cuda


# ------------------------------------------------------------------ the four routes
def _functional_route(original):
    def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=None, quant_type="fp4"):
        def library():
            # bitsandbytes' own decode reaches _dequantize_4bit_impl too; that
            # call must not be mistaken for the nested linear fallback.
            return _with_nested_flag(False, original, A, quant_state=quant_state, absmax=absmax,
                                     out=out, blocksize=blocksize, quant_type=quant_type)

        if not enabled() or not _cuda_tensor(A):
            return library()
        from .kernels.nf4 import check_out, dequantize_nf4, nested_shape
        try:
            n, k = nested_shape(A, quant_state)
            check_out(out, n, k, A.device)
        except ValueError:
            return library()
        return dequantize_nf4(A, quant_state, out=out)

    return dequantize_4bit


def _backend_route(original):
    def _dequantize_4bit_impl(A, absmax, blocksize, quant_type, dtype, out):
        import torch

        if (enabled() and _NESTED_BACKEND.get() and quant_type == "nf4" and blocksize == 64
                and dtype == torch.float16):
            from .kernels.nf4 import decode_flat_into, flat_fault
            if flat_fault(A, absmax, out) is None:
                decode_flat_into(A, absmax, out)
                return None  # bitsandbytes' helper fills `out` and returns nothing
        return original(A, absmax, blocksize, quant_type, dtype, out)

    return _dequantize_4bit_impl


def _linear_fallback_route(original):
    def _dequant_linear_fallback(A, B, shapeB, absmax, blocksize, quant_type, bias=None,
                                 absmax_8bit=None, absmax_code=None, absmax_offset=None):
        # absmax_8bit is present exactly when the fp32 scales were rebuilt from
        # a nested state (the only case the flat route accepts).
        return _with_nested_flag(absmax_8bit is not None, original, A, B, shapeB, absmax,
                                 blocksize, quant_type, bias=bias, absmax_8bit=absmax_8bit,
                                 absmax_code=absmax_code, absmax_offset=absmax_offset)

    return _dequant_linear_fallback


def _matmul_fault(A, B, quant_state, out, bias):
    """None when matmul_4bit can run as the fused GEMM, else why not."""
    import torch

    from ._spec import HALF, Operand, admit
    from .kernels.nf4 import nested_shape

    if out is not None:
        return "an out= buffer was given"
    try:
        admit("matmul_4bit", None, A=(A, Operand(HALF, ndim=None, layout=None)),
              B=(B, Operand(layout=None, frozen=True)))
        if A.ndim < 2:
            return "A is not a batch of rows"
        packed = (B if B.is_contiguous() else B.contiguous()).reshape(-1, 1)
        n, k = nested_shape(packed, quant_state, entry="matmul_4bit")
        if A.shape[-1] != k:
            return f"A has {A.shape[-1]} features, the weight {k}"
        admit("matmul_4bit", A.device,
              bias=(bias, Operand(HALF, ndim=1, frozen=True, exactly=n, optional=True)))
        if torch.cuda.get_device_capability(A.device)[0] != 10:
            return "not an sm_100 device"
    except ValueError as err:
        return str(err)
    return None


def make_matmul_4bit(original):
    """Wrapper for ``bitsandbytes.matmul_4bit(A, B, quant_state, out=None, bias=None)``.

    ``Linear4bit`` passes B = weight.t(), a [1, n*k/2] view of the packed codes;
    the weight is frozen, so the autograd graph needs dX only."""
    def matmul_4bit(A, B, quant_state, out=None, bias=None):
        if (enabled() and os.environ.get("SOUP_EXP_NF4_GEMM", "1") != "0"
                and _cuda_tensor(A) and _matmul_fault(A, B, quant_state, out, bias) is None):
            from .kernels.nf4_gemm import nf4_lora_linear
            packed = (B if B.is_contiguous() else B.contiguous()).reshape(-1, 1)
            return nf4_lora_linear(A, packed, quant_state, bias=bias)
        return original(A, B, quant_state, out=out, bias=bias)

    out = wraps(original)(matmul_4bit)
    setattr(out, _MARKER, original)
    return out


def patch_bnb_dequant():
    """Install the routes on bitsandbytes 0.50.2 (idempotent); False for any other version."""
    try:
        bnb = importlib.import_module("bitsandbytes")
        functional = importlib.import_module("bitsandbytes.functional")
        backend = importlib.import_module("bitsandbytes.backends.cuda.ops")
    except (ImportError, AttributeError):
        return False
    if not all(isinstance(m, ModuleType) for m in (bnb, functional, backend)):
        return False
    if getattr(bnb, "__version__", None) != _PINNED_VERSION:
        return False
    targets = ((functional, "dequantize_4bit", _functional_route),
               (backend, "_dequantize_4bit_impl", _backend_route),
               (backend, "_dequant_linear_fallback", _linear_fallback_route))
    if not all(callable(getattr(owner, attr, None)) for owner, attr, _ in targets):
        return False
    for owner, attr, make in targets:
        _redirect(owner, attr, make)
    if callable(getattr(bnb, "matmul_4bit", None)) and not hasattr(bnb.matmul_4bit, _MARKER):
        bnb.matmul_4bit = make_matmul_4bit(bnb.matmul_4bit)
    return True
