"""Cross-entropy through a frozen linear head without materialising the logits
(reference API: solution/kernels/cross_entropy.py, ``fused_linear_cross_entropy``).

Semantics the reference pins (solution/kernels/cross_entropy.py:1-43, 51-211):
the logits are fp16(fp16(hidden) . fp16(W)^T) -- rounded to fp16 before any
statistic -- and per row

    lse = m + log(sum exp(z - m)),  loss = lse - z[target] (0 for ignore_index),
    entropy = lse - sum(z exp(z - lse)),  argmax = first index of the maximum.

Only ``loss`` has a gradient: dZ = (softmax(z) - onehot(target)) * g, formed
per vocabulary chunk in fp16 after dividing by gain = max(|g|, 1e-30) / 1024,
multiplied into the head in fp32 and multiplied by the gain again; ignored rows
get exact zeros whatever their upstream value.

sm_100a path: ``sb_ce_forward`` folds the statistics into the epilogue of the
tcgen05 logits GEMM (128 x 256 tiles; the logits never reach memory) and
merges the per-tile statistics per row; ``sb_ce_backward`` compacts the
labelled rows on the device and, per vocabulary chunk (32768 columns up to a
256 MiB dZ chunk, 8192 from T = 16384 on), recomputes the logits into dZ and
accumulates dZ . W_chunk in fp32.  The hidden size is zero-padded to a
multiple of 8 for the tensor maps.
"""

from __future__ import annotations

import ctypes

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .._spec import FLOATS, LONG, Number, Operand, admit, refuse


def _half_padded(t, width):
    """fp16 copy of t [rows, h] with zero columns up to `width` (t itself when it fits)."""
    t16 = t.to(torch.float16)
    if t16.shape[1] == width:
        return t16.contiguous()
    out = torch.zeros((t16.shape[0], width), dtype=torch.float16, device=t16.device)
    out[:, :t16.shape[1]] = t16
    return out


def _scratch(name, device, *sizes):
    nbytes = _lib.query(name, *sizes)
    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device), nbytes


class _HeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, ignore_index):
        rows, width = hidden.shape
        vocab = weight.shape[0]
        padded = -(-width // 8) * 8
        h16 = _half_padded(hidden, padded)
        w16 = _half_padded(weight, padded)
        targets = targets.contiguous()
        dev = hidden.device
        loss = torch.empty(rows, device=dev, dtype=torch.float32)
        entropy = torch.empty(rows, device=dev, dtype=torch.float32)
        lse = torch.empty(rows, device=dev, dtype=torch.float32)
        argmax = torch.empty(rows, device=dev, dtype=torch.int64)
        if rows:
            scratch, nbytes = _scratch("sb_ce_forward_workspace_bytes", dev, rows, padded, vocab)
            _lib.call("sb_ce_forward", h16.data_ptr(), rows, padded, w16.data_ptr(), vocab,
                      targets.data_ptr(), int(ignore_index), loss.data_ptr(), entropy.data_ptr(),
                      argmax.data_ptr(), lse.data_ptr(), scratch.data_ptr(), nbytes, _lib.stream_of(dev))
        ctx.save_for_backward(h16, w16, targets, lse)
        ctx.meta = (hidden.dtype, width, int(ignore_index))
        ctx.mark_non_differentiable(entropy, argmax, lse)
        ctx.set_materialize_grads(False)
        return loss, entropy, argmax, lse

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_loss, *_unused):
        if grad_loss is None or not ctx.needs_input_grad[0]:
            return None, None, None, None
        h16, w16, targets, lse = ctx.saved_tensors
        hidden_dtype, width, ignore_index = ctx.meta
        rows, padded = h16.shape
        vocab = w16.shape[0]
        dev = h16.device
        grad_dtype = hidden_dtype if hidden_dtype in FLOATS else torch.float32
        dx = torch.empty((rows, padded), device=dev, dtype=grad_dtype)
        if rows:
            g = grad_loss.to(torch.float32).contiguous()
            scratch, nbytes = _scratch("sb_ce_backward_workspace_bytes", dev, rows, padded, vocab)
            _lib.call("sb_ce_backward", h16.data_ptr(), rows, padded, w16.data_ptr(), vocab,
                      targets.data_ptr(), ignore_index, lse.data_ptr(), g.data_ptr(), dx.data_ptr(),
                      _lib.dtype_code(grad_dtype), scratch.data_ptr(), nbytes, _lib.stream_of(dev))
        dx = dx[:, :width]
        return (dx if dx.dtype == hidden_dtype else dx.to(hidden_dtype)), None, None, None


def check_targets(targets, vocab, ignore_index):
    """ValueError if a target other than ignore_index lies outside [0, vocab).
    (The reference asserts this asynchronously; this check waits for the device.)"""
    outside = ctypes.c_int64(0)
    _lib.call("sb_ce_check_targets", targets.data_ptr(), targets.numel(), vocab, int(ignore_index),
              ctypes.byref(outside), _lib.stream_of(targets.device))
    if outside.value:
        raise ValueError(f"fused_linear_cross_entropy: {outside.value} targets lie outside "
                         f"the vocabulary [0, {vocab})")


def fused_linear_cross_entropy(hidden, weight, targets, ignore_index=-100, *, validate=True):
    """(loss, entropy, argmax, lse) per row for CUDA hidden [N, H], a frozen head
    weight [V, H] (fp16/fp32) and already shifted int64 targets [N].  Only loss
    is differentiable, with respect to hidden."""
    entry = "fused_linear_cross_entropy"
    device = hidden.device if isinstance(hidden, torch.Tensor) else None
    admit(entry, device, hidden=(hidden, Operand(*FLOATS, ndim=2, layout=None)),
          weight=(weight, Operand(*FLOATS, ndim=2, layout=None, frozen=True)),
          targets=(targets, Operand(LONG, ndim=1, layout=None)),
          ignore_index=(ignore_index, Number(integral=True)))
    if weight.shape[0] == 0 or weight.shape[1] == 0:
        refuse(entry, f"weight {tuple(weight.shape)} has an empty vocabulary or hidden size")
    if hidden.shape[1] != weight.shape[1] or hidden.shape[0] != targets.shape[0]:
        refuse(entry, f"hidden {tuple(hidden.shape)}, weight {tuple(weight.shape)} and "
                      f"targets {tuple(targets.shape)} do not line up")
    with torch.cuda.device(hidden.device):
        if validate and targets.numel():
            check_targets(targets.contiguous(), weight.shape[0], ignore_index)
        return _HeadCrossEntropy.apply(hidden, weight, targets, ignore_index)
