"""Right-padded training batches packed to their real tokens, and back (reference:
solution/unpad.py:76-200 -- mask validation, ``_batch_metadata``,
``_indices_from_lengths``, ``_pack``, ``_scatter``).

A batch of B rows padded to S tokens carries an attention mask [B, S] of ones
(real tokens, a prefix of each row) and zeros (padding); every padded position's
label must be the ignore index.  ``pack_batch`` checks exactly that on the
device (``sb_unpad_metadata``: one CTA per row, then one CTA for the offsets)
and reads back the row offsets ``cu_seqlens`` [B + 1] (the varlen-attention
convention) and a validity word in ONE device-to-host copy.  ``pack`` gathers
the real rows of any [B, S, ...] tensor into [T, ...] and ``scatter`` writes
[T, ...] back into a [B, S, ...] tensor whose padded rows are zero; each is
the other's gradient.  The projections then run on exactly T rows.

``right_padding_lengths`` is the host-side check of the same rules for a mask
given as nested lists (no device, no torch).
"""

from __future__ import annotations

from dataclasses import dataclass


def right_padding_lengths(rows):
    """Lengths of the real prefixes of a binary right-padded mask given as nested
    lists, or None if any row is empty, not binary or has a one after a zero."""
    if not rows or not rows[0]:
        return None
    width = len(rows[0])
    lengths = []
    for row in rows:
        if len(row) != width or any(v not in (0, 1) for v in row):
            return None
        real = sum(1 for v in row if v == 1)
        if real == 0 or any(v != 1 for v in row[:real]):
            return None
        lengths.append(real)
    return tuple(lengths)


_MASK_CODES = None


def _mask_code(dtype):
    import torch
    global _MASK_CODES
    if _MASK_CODES is None:
        _MASK_CODES = {torch.int64: 0, torch.int32: 1, torch.uint8: 2, torch.bool: 2,
                       torch.float16: 3, torch.float32: 4}
    return _MASK_CODES.get(dtype)


# Validity bits of sb_unpad_metadata.
_FAULTS = {1: "the mask is not binary", 2: "a row is not right-padded",
           4: "a padded position has a label other than the ignore index", 8: "a row has no real token"}


@dataclass(frozen=True)
class PackedBatch:
    """Geometry of one packed batch: per-row real lengths (host), offsets
    ``cu_seqlens`` [B + 1] int32 on the device, B, S and T."""
    batch: int
    sequence: int
    lengths: tuple
    cu_seqlens: object

    @property
    def tokens(self):
        return sum(self.lengths)


def pack_batch(mask, labels=None, ignore_index=-100):
    """Validate a right-padded batch on the device and return its PackedBatch, or
    raise ValueError naming the first broken rule."""
    import torch

    from . import _lib
    from ._spec import LONG, Operand, admit, refuse

    admit("pack_batch", mask.device if isinstance(mask, torch.Tensor) else None,
          mask=(mask, Operand(ndim=2)), labels=(labels, Operand(LONG, ndim=2, optional=True)))
    code = _mask_code(mask.dtype)
    if code is None:
        refuse("pack_batch", f"mask dtype {mask.dtype} is not supported")
    if labels is not None and labels.shape != mask.shape:
        refuse("pack_batch", f"labels {tuple(labels.shape)} do not match the mask {tuple(mask.shape)}")
    b, s = mask.shape
    if b == 0 or s == 0:
        refuse("pack_batch", "empty batch")
    dev = mask.device
    with torch.cuda.device(dev):
        nbytes = _lib.query("sb_unpad_workspace_bytes", b)
        scratch = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=dev)
        meta = torch.empty(b + 2, dtype=torch.int32, device=dev)
        _lib.call("sb_unpad_metadata", mask.data_ptr(), code, _lib.ptr(labels), int(ignore_index), b, s,
                  meta.data_ptr(), scratch.data_ptr(), nbytes, _lib.stream_of(dev))
        host = meta.cpu().tolist()  # the one device-to-host transfer
    flags = host[-1]
    if flags:
        refuse("pack_batch", "; ".join(text for bit, text in _FAULTS.items() if flags & bit))
    offsets = host[:-1]
    lengths = tuple(offsets[i + 1] - offsets[i] for i in range(b))
    return PackedBatch(b, s, lengths, meta[:b + 1])


def _row_bytes(t, batch_dims):
    import math
    return math.prod(t.shape[batch_dims:]) * t.element_size()


def _pack_raw(x, pb):
    import torch

    from . import _lib
    tail = tuple(x.shape[2:])
    src = x.contiguous()
    out = torch.empty((pb.tokens, *tail), device=x.device, dtype=x.dtype)
    _lib.call("sb_unpad_pack", src.data_ptr(), pb.batch, pb.sequence, _row_bytes(src, 2),
              pb.cu_seqlens.data_ptr(), pb.tokens, out.data_ptr(), _lib.stream_of(x.device))
    return out


def _scatter_raw(packed, pb):
    import torch

    from . import _lib
    tail = tuple(packed.shape[1:])
    src = packed.contiguous()
    out = torch.empty((pb.batch, pb.sequence, *tail), device=packed.device, dtype=packed.dtype)
    _lib.call("sb_unpad_scatter", src.data_ptr(), pb.batch, pb.sequence, _row_bytes(src, 1),
              pb.cu_seqlens.data_ptr(), out.data_ptr(), _lib.stream_of(packed.device))
    return out


def _functions():
    import torch

    class _Pack(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, pb):
            ctx.pb = pb
            return _pack_raw(x, pb)

        @staticmethod
        def backward(ctx, grad):
            return _scatter_raw(grad, ctx.pb), None

    class _Scatter(torch.autograd.Function):
        @staticmethod
        def forward(ctx, packed, pb):
            ctx.pb = pb
            return _scatter_raw(packed, pb)

        @staticmethod
        def backward(ctx, grad):
            return _pack_raw(grad, ctx.pb), None

    return _Pack, _Scatter


_FNS = None


def pack(x, pb):
    """[B, S, ...] -> [T, ...]: the real rows in batch order (differentiable)."""
    global _FNS
    if _FNS is None:
        _FNS = _functions()
    if tuple(x.shape[:2]) != (pb.batch, pb.sequence):
        raise ValueError(f"pack: x {tuple(x.shape)} does not match the batch [{pb.batch}, {pb.sequence}]")
    return _FNS[0].apply(x, pb)


def scatter(packed, pb):
    """[T, ...] -> [B, S, ...] with zero padded rows (differentiable)."""
    global _FNS
    if _FNS is None:
        _FNS = _functions()
    if packed.shape[0] != pb.tokens:
        raise ValueError(f"scatter: {packed.shape[0]} rows for a batch of {pb.tokens} tokens")
    return _FNS[1].apply(packed, pb)
