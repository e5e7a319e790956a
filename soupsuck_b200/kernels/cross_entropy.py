"""Frozen linear head, cross entropy and metrics without full vocabulary logits.

Mirror of solution/kernels/cross_entropy.py (``fused_linear_cross_entropy``):
logits are fp16(fp16(hidden) . fp16(W)^T) formed tile by tile on the tensor
cores (sb_ce_forward) and never stored; per row the online statistics give
lse = m + log s, loss = lse - z_target (0 when ignored), entropy = lse - t/s and
the first argmax.  Only ``loss`` is differentiable; the backward
(sb_ce_backward) compacts labelled rows on the device, recomputes logits per
8192-wide vocabulary chunk, forms dz = (softmax - onehot) * g / gain in fp16 and
accumulates dz . W_chunk in fp32 before undoing the gain.  Ignored rows get
exact zeros whatever their (possibly non-finite) upstream value.
"""

from __future__ import annotations

import ctypes

import torch
from torch.autograd.function import once_differentiable

from .. import _lib


def _pad_h(t, h8):
    if t.shape[1] == h8:
        return t.contiguous()
    out = torch.zeros((t.shape[0], h8), dtype=t.dtype, device=t.device)
    out[:, :t.shape[1]] = t
    return out


class _FrozenLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, ignore_index):
        ctx.hidden_dtype = hidden.dtype
        n, h = hidden.shape
        v = weight.shape[0]
        h8 = (h + 7) // 8 * 8
        hidden16 = _pad_h(hidden.to(torch.float16), h8)
        weight16 = _pad_h(weight.to(torch.float16), h8)
        targets = targets.contiguous()
        loss = torch.empty(n, device=hidden.device, dtype=torch.float32)
        entropy, lse = torch.empty_like(loss), torch.empty_like(loss)
        best = torch.empty(n, device=hidden.device, dtype=torch.int64)
        if n:
            nbytes = _lib.query("sb_ce_forward_workspace_bytes", n, h8, v)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=hidden.device)
            _lib.call("sb_ce_forward", hidden16.data_ptr(), n, h8, weight16.data_ptr(), v,
                      targets.data_ptr(), int(ignore_index), loss.data_ptr(), entropy.data_ptr(),
                      best.data_ptr(), lse.data_ptr(), ws.data_ptr(), nbytes,
                      _lib.stream_of(hidden.device))
        ctx.save_for_backward(hidden16, weight16, targets, lse)
        ctx.ignore_index, ctx.h = ignore_index, h
        ctx.mark_non_differentiable(entropy, best, lse)
        ctx.set_materialize_grads(False)
        return loss, entropy, best, lse

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_loss, _grad_entropy, _grad_best, _grad_lse):
        if grad_loss is None or not ctx.needs_input_grad[0]:
            return None, None, None, None
        hidden16, weight16, targets, lse = ctx.saved_tensors
        n, h8 = hidden16.shape
        v = weight16.shape[0]
        out_dtype = ctx.hidden_dtype if ctx.hidden_dtype in (torch.float16, torch.float32) else torch.float32
        dx = torch.empty((n, h8), device=hidden16.device, dtype=out_dtype)
        if n:
            grad = grad_loss.to(torch.float32).contiguous()
            nbytes = _lib.query("sb_ce_backward_workspace_bytes", n, h8, v)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=hidden16.device)
            _lib.call("sb_ce_backward", hidden16.data_ptr(), n, h8, weight16.data_ptr(), v,
                      targets.data_ptr(), int(ctx.ignore_index), lse.data_ptr(), grad.data_ptr(),
                      dx.data_ptr(), _lib.dtype_code(out_dtype), ws.data_ptr(), nbytes,
                      _lib.stream_of(hidden16.device))
        dx = dx[:, :ctx.h]
        if dx.dtype != ctx.hidden_dtype:
            dx = dx.to(ctx.hidden_dtype)
        return dx, None, None, None


def check_targets(targets, vocab, ignore_index):
    """Raise ValueError for targets outside [0, vocab) other than ignore_index
    (the reference checks this with torch._assert_async; this one synchronises)."""
    bad = ctypes.c_int64(0)
    _lib.call("sb_ce_check_targets", targets.data_ptr(), targets.numel(), vocab, int(ignore_index),
              ctypes.byref(bad), _lib.stream_of(targets.device))
    if bad.value:
        raise ValueError("Target outside vocabulary")


def fused_linear_cross_entropy(hidden, weight, targets, ignore_index=-100, *, validate=True):
    """Return per-token loss, entropy, first argmax and lse for a frozen head.

    Inputs are CUDA hidden[N,H] fp16/fp32, weight[V,H] fp16/fp32 and targets[N]
    int64 on the same device.  Targets are already shifted.  Only loss has an
    autograd edge, and only first derivatives with respect to hidden are supported.
    """
    if weight.requires_grad:
        raise ValueError("fused_linear_cross_entropy requires frozen weight")
    if hidden.ndim != 2 or weight.ndim != 2 or targets.ndim != 1:
        raise ValueError("Expected hidden[N,H], weight[V,H], targets[N]")
    if hidden.shape[1] != weight.shape[1] or hidden.shape[0] != targets.shape[0]:
        raise ValueError("Incompatible hidden, weight and targets shapes")
    if weight.shape[0] == 0 or weight.shape[1] == 0:
        raise ValueError("Vocabulary and hidden dimensions must be positive")
    if hidden.dtype not in (torch.float16, torch.float32) or weight.dtype not in (torch.float16, torch.float32):
        raise ValueError("Expected fp16/fp32 hidden and weight")
    if targets.dtype != torch.int64:
        raise ValueError("Expected int64 targets")
    if not hidden.is_cuda or weight.device != hidden.device or targets.device != hidden.device:
        raise ValueError("Inputs must be on the same CUDA device")
    if not isinstance(ignore_index, int):
        raise ValueError("ignore_index must be an integer")
    with torch.cuda.device(hidden.device):
        if validate and targets.numel():
            check_targets(targets.contiguous(), weight.shape[0], ignore_index)
        return _FrozenLinearCrossEntropy.apply(hidden, weight, targets, ignore_index)
