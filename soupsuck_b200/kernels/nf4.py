"""NF4/block64 + double-quant/block256 decoder (bitsandbytes 0.50.2 storage format).

Mirror of the reference module solution/kernels/nf4.py: same public names,
argument meaning and ValueError behaviour; the decode itself is the sm_100a
kernel ``sb_nf4_dequant_*`` (bit-exact fp16 output, see csrc/nf4_dequant.cuh).

Scale for output i is fp32(fp32(state2.code[qabs[i//64]] * state2.absmax[(i//64)//256])
+ offset); multiply by the NF4 code value in fp32, round once to fp16.
A byte stores the earlier value in its HIGH nibble.
"""

from __future__ import annotations

import math

import torch

from .. import _lib

# Format data: the sixteen NF4 code values (reference solution/kernels/nf4.py:32-37).
_NF4_VALUES = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _tensor(t, dtype, device, minimum):
    return (isinstance(t, torch.Tensor) and t.device == device and t.dtype == dtype
            and t.is_contiguous() and t.numel() >= minimum and not t.requires_grad)


def _validate_state(packed, state, out_dtype):
    """Accept only the nested fp16 NF4/block64 state (reference nf4.py:140-168)."""
    if not isinstance(packed, torch.Tensor) or not packed.is_cuda or packed.dtype != torch.uint8:
        raise ValueError("NF4 storage must be uint8 CUDA")
    if not packed.is_contiguous() or packed.ndim not in (1, 2):
        raise ValueError("NF4 storage must be contiguous and one- or two-dimensional")
    if out_dtype != torch.float16:
        raise ValueError("Only fp16 NF4 output is supported")
    if (getattr(state, "quant_type", None) != "nf4" or getattr(state, "blocksize", None) != 64
            or getattr(state, "dtype", None) != torch.float16 or not getattr(state, "nested", False)):
        raise ValueError("Expected fp16 NF4/block64 with compressed statistics")
    shape = getattr(state, "shape", None)
    if not isinstance(shape, (tuple, list, torch.Size)) or len(shape) != 2:
        raise ValueError("Expected a matrix shape in quant_state")
    if any(not isinstance(d, int) or d <= 0 for d in shape):
        raise ValueError("quant_state dimensions must be positive integers")
    n = math.prod(shape)
    blocks = _cdiv(n, 64)
    second = getattr(state, "state2", None)
    if (getattr(second, "blocksize", None) != 256 or getattr(second, "dtype", None) != torch.float32
            or getattr(second, "nested", False)):
        raise ValueError("Expected non-nested fp32 state2/block256")
    if (packed.numel() * 2 < n
            or not _tensor(getattr(state, "absmax", None), torch.uint8, packed.device, blocks)
            or not _tensor(getattr(second, "absmax", None), torch.float32, packed.device, _cdiv(blocks, 256))
            or not _tensor(getattr(second, "code", None), torch.float32, packed.device, 256)
            or not _tensor(getattr(state, "offset", None), torch.float32, packed.device, 1)
            or state.offset.numel() != 1):
        raise ValueError("Invalid packed length or nested scale/code/offset buffers")
    return tuple(shape)


def _validate_flat(packed, absmax, out):
    """Backend flat path buffers (reference nf4.py:171-178)."""
    if (not isinstance(packed, torch.Tensor) or not packed.is_cuda or packed.dtype != torch.uint8
            or not packed.is_contiguous() or packed.ndim not in (1, 2)
            or not isinstance(out, torch.Tensor) or out.dtype != torch.float16
            or out.device != packed.device or not out.is_contiguous() or out.ndim != 2 or out.requires_grad
            or packed.numel() * 2 < out.numel()
            or not _tensor(absmax, torch.float32, packed.device, _cdiv(out.numel(), 64))):
        raise ValueError("Unsupported flat NF4 dequantization buffers")


def _dequantize_flat_into(packed, absmax, out):
    """Backend entry: fp32 absmax was already reconstructed by bitsandbytes."""
    _validate_flat(packed, absmax, out)
    with torch.cuda.device(packed.device):
        if out.numel():
            _lib.call("sb_nf4_dequant_flat", packed.data_ptr(), absmax.data_ptr(), out.data_ptr(),
                      out.numel(), _lib.stream_of(packed.device))
    return out


def dequantize_nf4(packed, quant_state, out_dtype=torch.float16, *, out=None):
    """Decode directly into out (canonical state.shape), then apply the BC view."""
    shape = _validate_state(packed, quant_state, out_dtype)
    if out is not None and (not isinstance(out, torch.Tensor) or tuple(out.shape) != shape
                            or out.device != packed.device or out.dtype != out_dtype
                            or not out.is_contiguous() or out.requires_grad):
        raise ValueError("Expected a contiguous non-grad out buffer matching quant_state")
    with torch.cuda.device(packed.device):
        if out is None:
            out = torch.empty(shape, device=packed.device, dtype=out_dtype)
        st = quant_state
        _lib.call("sb_nf4_dequant_nested", packed.data_ptr(), st.absmax.data_ptr(),
                  st.state2.absmax.data_ptr(), st.state2.code.data_ptr(), st.offset.data_ptr(),
                  out.data_ptr(), out.numel(), _lib.stream_of(packed.device))
    return out.t() if packed.shape[0] == 1 else out
