"""NF4 + double-quant quantizer that produces the bitsandbytes 0.50.2 storage format.

This is data preparation (synthetic weights for tests and the benchmark), not
part of the hot path.  The reference never quantizes itself: bitsandbytes'
``quantize_4bit(..., quant_type="nf4", compress_statistics=True, blocksize=64)``
does, and bitsandbytes is not installed here.  The quantizer below is written
from the published method (Dettmers et al., "QLoRA", 2023, NF4 + double
quantization; Dettmers et al., "8-bit Optimizers via Block-wise Quantization",
2022, for the signed dynamic 8-bit code):

* per 64-element block of the row-major flattened weight, ``absmax`` = max |w|;
  each element is mapped to the nearest of the 16 NF4 code values of
  ``w / absmax``; two codes per byte, the EARLIER element in the HIGH nibble;
* double quantization: ``offset = mean(absmax)``; the centred absmax values are
  quantized per 256-block group with fp32 scale ``state2.absmax`` to the index
  of the nearest entry of a 256-entry signed dynamic code ``state2.code``.

The storage layout matches what the reference's decoder reads
(solution/kernels/nf4.py:140-168): packed uint8 ``[ceil(n/2), 1]``, uint8
absmax, fp32 state2.absmax/code/offset.  Because the decoder takes the code
table as an input, its bit-exactness does not depend on matching bitsandbytes'
own code table, which this module does not claim to reproduce.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch

NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


@dataclass
class NestedState:
    """Second-level state: fp32 absmax per 256 blocks and the 8-bit code table."""
    absmax: torch.Tensor
    code: torch.Tensor
    blocksize: int = 256
    dtype: torch.dtype = torch.float32
    nested: bool = False


@dataclass
class QuantState:
    """Mirror of the bitsandbytes QuantState fields the reference validates."""
    absmax: torch.Tensor
    shape: Tuple[int, int]
    state2: Optional[NestedState]
    offset: Optional[torch.Tensor]
    quant_type: str = "nf4"
    blocksize: int = 64
    dtype: torch.dtype = torch.float16
    nested: bool = True
    code: Optional[torch.Tensor] = field(default=None)


def dynamic_code_map(device=None) -> torch.Tensor:
    """Signed 256-entry dynamic code: 0, +-fractions over seven decades, and 1.

    Decade e (scale 10**-e) carries 2**(6-e) linearly spaced fractions in
    (0.1, 1], so small magnitudes get fewer, coarser codes.  Sorted ascending.
    """
    values = []
    for e in range(7):
        count = 2 ** (6 - e)
        for k in range(count):
            frac = 0.1 + 0.9 * (k + 0.5) / count
            values.append(frac * 10.0 ** (-e))
    values = sorted(values)
    code = [-v for v in reversed(values)] + [0.0] + values + [1.0]
    assert len(code) == 256
    return torch.tensor(code, dtype=torch.float32, device=device)


def _nearest(values: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Index of the nearest entry of an ascending table (ties -> lower index)."""
    right = torch.searchsorted(table, values.contiguous()).clamp(1, table.numel() - 1)
    left = right - 1
    pick_right = (table[right] - values).abs() < (values - table[left]).abs()
    return torch.where(pick_right, right, left)


def quantize_nf4(weight: torch.Tensor, blocksize: int = 64,
                 nested_blocksize: int = 256) -> Tuple[torch.Tensor, QuantState]:
    """Quantize a 2-D weight to packed NF4 with double-quantized block scales."""
    if weight.ndim != 2:
        raise ValueError("expected a 2-D weight")
    if blocksize != 64 or nested_blocksize != 256:
        raise ValueError("only NF4/block64 with block256 double quantization is produced")
    device = weight.device
    n = weight.numel()
    blocks = (n + blocksize - 1) // blocksize
    flat = weight.reshape(-1).to(torch.float32)
    padded = torch.zeros(blocks * blocksize, dtype=torch.float32, device=device)
    padded[:n] = flat
    grid = padded.view(blocks, blocksize)
    absmax = grid.abs().amax(dim=1)
    safe = torch.where(absmax > 0, absmax, torch.ones_like(absmax))
    normalized = (grid / safe[:, None]).clamp(-1.0, 1.0)
    table = torch.tensor(NF4_CODE, dtype=torch.float32, device=device)
    codes = _nearest(normalized.reshape(-1), table)[:n].to(torch.uint8)
    if n % 2:
        codes = torch.cat([codes, torch.zeros(1, dtype=torch.uint8, device=device)])
    pairs = codes.view(-1, 2)
    packed = ((pairs[:, 0] << 4) | pairs[:, 1]).to(torch.uint8).view(-1, 1)

    offset = absmax.mean()
    centred = absmax - offset
    groups = (blocks + nested_blocksize - 1) // nested_blocksize
    cpad = torch.zeros(groups * nested_blocksize, dtype=torch.float32, device=device)
    cpad[:blocks] = centred
    cgrid = cpad.view(groups, nested_blocksize)
    absmax2 = cgrid.abs().amax(dim=1)
    safe2 = torch.where(absmax2 > 0, absmax2, torch.ones_like(absmax2))
    code2 = dynamic_code_map(device)
    q = _nearest((cgrid / safe2[:, None]).reshape(-1), code2)[:blocks].to(torch.uint8)
    state = QuantState(
        absmax=q.contiguous(), shape=(int(weight.shape[0]), int(weight.shape[1])),
        state2=NestedState(absmax=absmax2.contiguous(), code=code2.contiguous()),
        offset=offset.reshape(1).to(torch.float32).contiguous(),
    )
    return packed.contiguous(), state


def fixture_state(shape, offset: float, device=None):
    """The reference's deterministic decoder fixture (solution/tests/test_nf4_fast.py:96-110):
    packed bytes and absmax codes cycle through 0..255, code = linspace(-1, 1, 256),
    state2.absmax = 1.125 + 0.375 k.  Used for golden-vector parity."""
    n = math.prod(shape)
    blocks = (n + 63) // 64
    packed = (torch.arange((n + 1) // 2, device=device, dtype=torch.int64) % 256).to(torch.uint8).view(-1, 1)
    qabs = (torch.arange(blocks, device=device, dtype=torch.int64) % 256).to(torch.uint8)
    second = NestedState(
        absmax=1.125 + 0.375 * torch.arange((blocks + 255) // 256, device=device, dtype=torch.float32),
        code=torch.linspace(-1, 1, 256, device=device, dtype=torch.float32))
    state = QuantState(absmax=qabs, shape=tuple(shape), state2=second,
                       offset=torch.tensor([offset], device=device, dtype=torch.float32))
    return packed, state
