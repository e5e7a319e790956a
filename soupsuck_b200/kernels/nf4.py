"""NF4 decoding of bitsandbytes weights on sm_100a (reference API: solution/kernels/nf4.py).

Storage read as bitsandbytes 0.50.2 writes it (format description at
solution/kernels/nf4.py:1-16): two 4-bit codes per byte, the earlier element
in the high nibble; one uint8 scale index per 64 elements, decoded through the
256-entry fp32 table ``state2.code`` and multiplied by one fp32 ``state2.absmax``
per 256 scale indices, then ``offset`` is added.  Element i therefore decodes to

    fp16( NF4[code_i] * ( fp32(code2[qabs[i/64]] * absmax2[i/16384]) + offset ) )

with one rounding and no fused multiply-add (solution/kernels/nf4.py:41-59); the
sm_100a kernels ``sb_nf4_dequant_nested`` / ``sb_nf4_dequant_flat`` produce
these fp16 bits exactly.  The flat form (fp32 scales already reconstructed by
bitsandbytes' backend) is the same rule without the nested step.
"""

from __future__ import annotations

import math

import torch

from .. import _lib
from .._spec import BYTE, HALF, SINGLE, Choice, Operand, admit, refuse

# Format data: the sixteen NF4 levels, code 0 = -1.0 ... code 7 = 0.0 ... code 15 = 1.0
# (solution/kernels/nf4.py:32-37); the decoder kernel carries the same constants.
NF4_LEVELS = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)

ELEMENTS_PER_SCALE = 64      # one uint8 scale index per 64 codes
SCALES_PER_GROUP = 256       # one fp32 group scale per 256 scale indices

# What the decoder requires of a QuantState: attribute path -> accepted value.
_NESTED_LAYOUT = (
    ("quant_type", Choice("nf4")),
    ("blocksize", Choice(ELEMENTS_PER_SCALE)),
    ("dtype", Choice(HALF)),
    ("nested", Choice(True)),
    ("state2__blocksize", Choice(SCALES_PER_GROUP)),
    ("state2__dtype", Choice(SINGLE)),
    ("state2__nested", Choice(False)),
)

_MISSING = object()


def _field(obj, path):
    for part in path.split("__"):
        obj = getattr(obj, part, _MISSING)
        if obj is _MISSING:
            return _MISSING
    return obj


def _groups(count, size):
    return -(-count // size)


def nested_shape(packed, state, out_dtype=HALF, entry="dequantize_nf4"):
    """(n, k) of a supported nested NF4 weight; ValueError for anything else."""
    admit(entry, None, packed=(packed, Operand(BYTE, ndim=(1, 2))))
    if out_dtype != HALF:
        refuse(entry, f"output dtype {out_dtype} requested; the decoder writes fp16 only")
    for path, rule in _NESTED_LAYOUT:
        value = _field(state, path)
        admit(entry, None, **{f"quant_state__{path}": (None if value is _MISSING else value, rule)})
    shape = getattr(state, "shape", None)
    if (not isinstance(shape, (tuple, list, torch.Size)) or len(shape) != 2
            or not all(isinstance(d, int) and not isinstance(d, bool) and d > 0 for d in shape)):
        refuse(entry, f"quant_state.shape is {shape!r}; two positive integers are required")
    elements = math.prod(shape)
    scales = _groups(elements, ELEMENTS_PER_SCALE)
    if 2 * packed.numel() < elements:
        refuse(entry, f"packed holds {packed.numel()} bytes, {elements} codes need {_groups(elements, 2)}")
    second = state.state2
    admit(entry, packed.device,
          quant_state__absmax=(state.absmax, Operand(BYTE, frozen=True, at_least=scales)),
          quant_state__state2__absmax=(second.absmax, Operand(
              SINGLE, frozen=True, at_least=_groups(scales, SCALES_PER_GROUP))),
          quant_state__state2__code=(second.code, Operand(SINGLE, frozen=True, at_least=256)),
          quant_state__offset=(state.offset, Operand(SINGLE, frozen=True, exactly=1)))
    return int(shape[0]), int(shape[1])


def flat_fault(packed, absmax, out):
    """None when the flat decoder can fill ``out`` from (packed, absmax), else the reason."""
    try:
        admit("nf4 flat decode", packed.device if isinstance(packed, torch.Tensor) else None,
              packed=(packed, Operand(BYTE, ndim=(1, 2))),
              out=(out, Operand(HALF, ndim=2, frozen=True)))
        admit("nf4 flat decode", packed.device,
              absmax=(absmax, Operand(SINGLE, frozen=True,
                                      at_least=_groups(out.numel(), ELEMENTS_PER_SCALE))))
        if 2 * packed.numel() < out.numel():
            refuse("nf4 flat decode", f"packed holds {packed.numel()} bytes for {out.numel()} outputs")
    except ValueError as err:
        return str(err)
    return None


def decode_flat_into(packed, absmax, out):
    """Fill fp16 ``out`` from packed codes and bitsandbytes' reconstructed fp32 scales."""
    fault = flat_fault(packed, absmax, out)
    if fault is not None:
        raise ValueError(fault)
    if out.numel():
        with torch.cuda.device(packed.device):
            _lib.call("sb_nf4_dequant_flat", packed.data_ptr(), absmax.data_ptr(), out.data_ptr(),
                      out.numel(), _lib.stream_of(packed.device))
    return out


def check_out(out, n, k, device, entry="dequantize_nf4"):
    """A caller's out= buffer must be a contiguous fp16 [n, k] on `device` without grad."""
    if out is None:
        return
    admit(entry, device, out=(out, Operand(HALF, ndim=2, frozen=True)))
    if tuple(out.shape) != (n, k):
        refuse(entry, f"out has shape {tuple(out.shape)}, the weight is {(n, k)}")


def dequantize_nf4(packed, quant_state, out_dtype=torch.float16, *, out=None):
    """Decode a nested NF4 weight to fp16 [n, k] (reference: solution/kernels/nf4.py:190-203).

    ``out``, when given, must be a contiguous fp16 [n, k] tensor on packed's
    device without grad; it is written in place and nothing else is allocated.
    bitsandbytes hands ``Linear4bit`` weights over as a transposed [1, bytes]
    view; for that view the decoded matrix is returned transposed as well.
    """
    n, k = nested_shape(packed, quant_state, out_dtype)
    check_out(out, n, k, packed.device)
    with torch.cuda.device(packed.device):
        target = out if out is not None else torch.empty((n, k), device=packed.device, dtype=HALF)
        st = quant_state
        _lib.call("sb_nf4_dequant_nested", packed.data_ptr(), st.absmax.data_ptr(),
                  st.state2.absmax.data_ptr(), st.state2.code.data_ptr(), st.offset.data_ptr(),
                  target.data_ptr(), target.numel(), _lib.stream_of(packed.device))
    # The contract's rule for the view: a leading dimension of one means the
    # caller passed bitsandbytes' transposed storage view.
    return target.t() if packed.shape[0] == 1 else target
