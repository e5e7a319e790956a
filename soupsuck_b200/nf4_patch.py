"""Route bitsandbytes 0.50.2's NF4 paths through the sm_100a kernels.

Mirror of the reference's solution/nf4_patch.py:43-125 (same three patched
symbols, same marker attribute, same fallback rules) plus the matmul patch of
solution/kernels/nf4_gemm.py:121-154, which here is on by default because the
fused tcgen05 GEMM is the hot path (SOUP_EXP_NF4_GEMM=0 turns it off):

* ``bitsandbytes.functional.dequantize_4bit`` - canonical nested fp16 NF4
  states decode with ``sb_nf4_dequant_nested`` (into ``out`` when given);
* ``bitsandbytes.backends.cuda.ops._dequantize_4bit_impl`` - inside a nested
  ``_dequant_linear_fallback`` scope, decodes with ``sb_nf4_dequant_flat``;
* ``..._dequant_linear_fallback`` - only marks that scope;
* ``bitsandbytes.matmul_4bit`` - fp16 X against a canonical nested NF4 weight
  runs the fused dequant-GEMM forward and dX (``sb_nf4_linear_fwd/dx``).

Every unsupported input takes the saved original; only ``ValueError`` from
validation is treated as "unsupported" and nothing raised by a kernel launch
is swallowed.  Imports of torch and of the kernels are lazy.
"""

from contextlib import contextmanager
from contextvars import ContextVar
from functools import wraps
import importlib
import os
from types import ModuleType

from .utils import enabled

_MARKER = "_solution_fused_original"
_NESTED_BACKEND = ContextVar("soupsuck_b200_nf4_nested_backend", default=False)


@contextmanager
def _nested_backend_scope(nested):
    token = _NESTED_BACKEND.set(nested)
    try:
        yield
    finally:
        _NESTED_BACKEND.reset(token)


def _gemm_enabled():
    return os.environ.get("SOUP_EXP_NF4_GEMM", "1") != "0"


def _make_dequantize(original_f):
    @wraps(original_f)
    def dequantize(A, quant_state=None, absmax=None, out=None, blocksize=None, quant_type="fp4"):
        import torch

        arguments = dict(quant_state=quant_state, absmax=absmax, out=out,
                         blocksize=blocksize, quant_type=quant_type)

        def fallback():
            with _nested_backend_scope(False):
                return original_f(A, **arguments)

        if not enabled() or not isinstance(A, torch.Tensor) or not A.is_cuda:
            return fallback()
        from .kernels.nf4 import _validate_state, dequantize_nf4

        try:
            shape = _validate_state(A, quant_state, torch.float16)
        except ValueError:
            return fallback()
        if out is not None and (not isinstance(out, torch.Tensor) or tuple(out.shape) != shape
                                or out.dtype != torch.float16 or out.device != A.device
                                or not out.is_contiguous() or out.requires_grad):
            return fallback()
        return dequantize_nf4(A, quant_state, out=out)

    setattr(dequantize, _MARKER, original_f)
    return dequantize


def _make_backend(original_backend):
    @wraps(original_backend)
    def dequantize_backend(A, absmax, blocksize, quant_type, dtype, out):
        import torch

        if (not _NESTED_BACKEND.get() or not enabled() or blocksize != 64
                or quant_type != "nf4" or dtype != torch.float16):
            return original_backend(A, absmax, blocksize, quant_type, dtype, out)
        from .kernels.nf4 import _dequantize_flat_into, _validate_flat

        try:
            _validate_flat(A, absmax, out)
        except ValueError:
            return original_backend(A, absmax, blocksize, quant_type, dtype, out)
        _dequantize_flat_into(A, absmax, out)
        return None  # the original helper writes ``out`` and returns None

    setattr(dequantize_backend, _MARKER, original_backend)
    return dequantize_backend


def _make_linear_fallback(original_linear):
    @wraps(original_linear)
    def linear_fallback(A, B, shapeB, absmax, blocksize, quant_type, bias=None,
                        absmax_8bit=None, absmax_code=None, absmax_offset=None):
        with _nested_backend_scope(absmax_8bit is not None):
            return original_linear(A, B, shapeB, absmax, blocksize, quant_type, bias=bias,
                                   absmax_8bit=absmax_8bit, absmax_code=absmax_code,
                                   absmax_offset=absmax_offset)

    setattr(linear_fallback, _MARKER, original_linear)
    return linear_fallback


def make_matmul_4bit(original):
    """``bitsandbytes.matmul_4bit(A, B, quant_state, out=None, bias=None)`` replacement.

    bnb's Linear4bit passes ``B = weight.t()`` (a [1, nk/2] view of the packed
    bytes); the weight is frozen, so autograd needs only dX (and no dW).
    """
    @wraps(original)
    def matmul(A, B, quant_state, out=None, bias=None):
        import torch

        shape = getattr(quant_state, "shape", ())
        if (not enabled() or not _gemm_enabled() or len(shape) != 2
                or not isinstance(A, torch.Tensor) or not A.is_cuda or A.dtype != torch.float16
                or A.ndim < 2 or A.shape[-1] != shape[1] or out is not None
                or not isinstance(B, torch.Tensor) or B.requires_grad
                or (bias is not None and (not isinstance(bias, torch.Tensor) or bias.requires_grad
                                          or bias.dtype != torch.float16 or bias.device != A.device
                                          or tuple(bias.shape) != (shape[0],)))):
            return original(A, B, quant_state, out=out, bias=bias)
        from .kernels.nf4 import _validate_state
        from .kernels.nf4_gemm import nf4_lora_linear
        from .utils import supported_tensor

        if not supported_tensor(A.contiguous() if not A.is_contiguous() else A):
            return original(A, B, quant_state, out=out, bias=bias)
        packed = B.reshape(-1, 1) if B.is_contiguous() else B.contiguous().reshape(-1, 1)
        try:
            _validate_state(packed, quant_state, torch.float16)
        except ValueError:
            return original(A, B, quant_state, out=out, bias=bias)
        return nf4_lora_linear(A, packed, quant_state, bias=bias)

    setattr(matmul, _MARKER, original)
    return matmul


def patch_bnb_dequant():
    """Idempotently patch bitsandbytes 0.50.2; return whether it was patched."""
    try:
        bnb = importlib.import_module("bitsandbytes")
        functional = importlib.import_module("bitsandbytes.functional")
        backend = importlib.import_module("bitsandbytes.backends.cuda.ops")
    except (ImportError, AttributeError):
        return False
    if (not all(isinstance(m, ModuleType) for m in (bnb, functional, backend))
            or getattr(bnb, "__version__", None) != "0.50.2"
            or not callable(getattr(functional, "dequantize_4bit", None))
            or not callable(getattr(backend, "_dequantize_4bit_impl", None))
            or not callable(getattr(backend, "_dequant_linear_fallback", None))):
        return False
    if not hasattr(functional.dequantize_4bit, _MARKER):
        functional.dequantize_4bit = _make_dequantize(functional.dequantize_4bit)
    if not hasattr(backend._dequantize_4bit_impl, _MARKER):
        backend._dequantize_4bit_impl = _make_backend(backend._dequantize_4bit_impl)
    if not hasattr(backend._dequant_linear_fallback, _MARKER):
        backend._dequant_linear_fallback = _make_linear_fallback(backend._dequant_linear_fallback)
    original = getattr(bnb, "matmul_4bit", None)
    if callable(original) and not hasattr(original, _MARKER):
        bnb.matmul_4bit = make_matmul_4bit(original)
    return True
