"""Fused NF4 dequantize -> tcgen05 GEMM with the LoRA term in the same accumulator.

Reference counterparts: nf4_tile_matmul_kernel / nf4_matmul / _NF4Linear
(solution/kernels/nf4_gemm.py:35-118, never enabled there because it lost to
decode + cuBLAS on T4), the base projection bnb MatMul4Bit (forward F.linear,
backward dequantize + torch.matmul, solution/nf4_patch.py:62-120) and the PEFT
LoRA branch with its scale/add epilogue (solution/lora.py:135-164,
solution/kernels/lora_epilogue.py).

    forward   Y  = X . deq(W)^T + s * (X . A^T) . B^T (+ bias)
    backward  dX = dY . deq(W) + s * (dY . B) . A
              dA = (s * dY . B)^T . X,   dB = s * dY^T . (X . A^T)

X and dY are fp16; the LoRA factors are used in fp16 (the reference runs them
under fp16 autocast); dA / dB are accumulated in fp32 and returned in the
parameters' dtype.  GEMM results are toleranced against the dense product (the
reference's preregistered gate: rtol = atol = 2e-3, relative L2 <= 1e-3).
"""

from __future__ import annotations

import ctypes

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .nf4 import _validate_state

_SUPPORTED_RANKS = (16, 32, 64)


def _weight_struct(packed, state):
    n, k = state.shape
    return _lib.NF4Weight(packed.data_ptr(), state.absmax.data_ptr(), state.state2.absmax.data_ptr(),
                          state.state2.code.data_ptr(), state.offset.data_ptr(), n, k)


def _workspace(m, n, k, dx, device):
    nbytes = _lib.query("sb_nf4_linear_workspace_bytes", m, n, k, int(dx))
    buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device) if nbytes else None
    return buf, nbytes


def _padded_rank(r):
    for cand in _SUPPORTED_RANKS:
        if r <= cand:
            return cand
    raise ValueError("LoRA rank above 64 is not supported")


def _pad_cols(t, width):
    if t.shape[-1] == width:
        return t.contiguous()
    out = torch.zeros((*t.shape[:-1], width), dtype=t.dtype, device=t.device)
    out[..., :t.shape[-1]] = t
    return out


def nf4_linear_raw(x2d, packed, state, *, transpose=False, bias=None, lora_a=None, lora_b=None):
    """One launch of the fused GEMM.  lora_a [m, r] and lora_b [width, r] are the
    already-scaled fp16 low-rank factors (r padded to 16/32/64); no autograd."""
    n, k = state.shape
    m = x2d.shape[0]
    width = k if transpose else n
    out = torch.empty((m, width), dtype=torch.float16, device=x2d.device)
    if m == 0:
        return out
    r = 0 if lora_a is None else lora_a.shape[1]
    w = _weight_struct(packed, state)
    ws, nbytes = _workspace(m, n, k, transpose, x2d.device)
    stream = _lib.stream_of(x2d.device)
    if transpose:
        _lib.call("sb_nf4_linear_dx", x2d.data_ptr(), m, ctypes.byref(w), _lib.ptr(lora_a),
                  _lib.ptr(lora_b), r, out.data_ptr(), _lib.ptr(ws), nbytes, stream)
    else:
        _lib.call("sb_nf4_linear_fwd", x2d.data_ptr(), m, ctypes.byref(w), _lib.ptr(bias),
                  _lib.ptr(lora_a), _lib.ptr(lora_b), r, out.data_ptr(), _lib.ptr(ws), nbytes, stream)
    return out


def nf4_matmul(x, packed, state, *, transpose=False, bias=None, config=None):
    """Direct entry with the reference's signature (solution/kernels/nf4_gemm.py:74-96):
    X[.., K] . deq(W)^T (+bias) or, with transpose=True, dY[.., N] . deq(W).
    ``config`` is accepted for signature compatibility and ignored (one kernel)."""
    n, k = _validate_state(packed, state, torch.float16)
    if (not isinstance(x, torch.Tensor) or x.device != packed.device
            or x.dtype != torch.float16 or not x.is_contiguous() or x.ndim < 2
            or x.shape[-1] != (n if transpose else k)):
        raise ValueError("Expected contiguous CUDA fp16 X matching canonical nested NF4 weight")
    width = k if transpose else n
    if bias is not None and (transpose or not isinstance(bias, torch.Tensor)
            or bias.device != x.device or bias.dtype != torch.float16
            or bias.shape != (width,) or not bias.is_contiguous() or bias.requires_grad):
        raise ValueError("Only frozen contiguous fp16 forward bias is supported")
    with torch.cuda.device(x.device):
        out = nf4_linear_raw(x.reshape(-1, x.shape[-1]), packed, state, transpose=transpose, bias=bias)
    return out.reshape(*x.shape[:-1], width)


def _lora_factors_fwd(x2d, a16, b16, scaling):
    """zs = fp16(s * X . A^T) [m, rp] and z = fp16(X . A^T) [m, r] (saved for dB)."""
    m, k = x2d.shape
    r = a16.shape[0]
    rp = _padded_rank(r)
    z = torch.empty((m, r), dtype=torch.float16, device=x2d.device)
    zs = torch.zeros((m, rp), dtype=torch.float16, device=x2d.device) if rp != r else \
        torch.empty((m, r), dtype=torch.float16, device=x2d.device)
    if m:
        if rp == r:
            _lib.call("sb_lora_down", x2d.data_ptr(), m, k, a16.data_ptr(), r, float(scaling),
                      z.data_ptr(), zs.data_ptr(), _lib.stream_of(x2d.device))
        else:
            tmp = torch.empty((m, r), dtype=torch.float16, device=x2d.device)
            _lib.call("sb_lora_down", x2d.data_ptr(), m, k, a16.data_ptr(), r, float(scaling),
                      z.data_ptr(), tmp.data_ptr(), _lib.stream_of(x2d.device))
            zs[:, :r] = tmp
    return z, zs, rp


class _NF4LoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, packed, state, lora_a, lora_b, scaling, bias):
        n, k = state.shape
        x2d = x.reshape(-1, k)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        has_lora = lora_a is not None
        z = None
        if has_lora:
            a16 = lora_a.detach().to(torch.float16).contiguous()
            b16 = lora_b.detach().to(torch.float16).contiguous()
            z, zs, rp = _lora_factors_fwd(x2d, a16, b16, scaling)
            y = nf4_linear_raw(x2d, packed, state, bias=bias, lora_a=zs, lora_b=_pad_cols(b16, rp))
        else:
            y = nf4_linear_raw(x2d, packed, state, bias=bias)
        ctx.save_for_backward(x2d, packed, z, lora_a, lora_b)
        ctx.state, ctx.scaling, ctx.has_lora = state, float(scaling), has_lora
        ctx.x_shape = x.shape
        return y.reshape(*x.shape[:-1], n)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        x2d, packed, z, lora_a, lora_b = ctx.saved_tensors
        state = ctx.state
        n, k = state.shape
        g = grad.reshape(-1, n).to(torch.float16).contiguous()
        m = g.shape[0]
        dx = da = db = None
        stream = _lib.stream_of(g.device)
        if ctx.has_lora:
            r = lora_a.shape[0]
            rp = _padded_rank(r)
            b16 = lora_b.detach().to(torch.float16).contiguous()
            a16 = lora_a.detach().to(torch.float16).contiguous()
            u32 = torch.empty((m, r), dtype=torch.float32, device=g.device)
            u16 = torch.empty((m, r), dtype=torch.float16, device=g.device)
            if m:
                _lib.call("sb_lora_up_grad", g.data_ptr(), m, n, b16.data_ptr(), r, ctx.scaling,
                          u16.data_ptr(), u32.data_ptr(), stream)
            at = torch.empty((k, r), dtype=torch.float16, device=g.device)
            _lib.call("sb_lora_transpose_a", a16.data_ptr(), r, k, at.data_ptr(), stream)
            if ctx.needs_input_grad[0]:
                dx = nf4_linear_raw(g, packed, state, transpose=True,
                                    lora_a=_pad_cols(u16, rp), lora_b=_pad_cols(at, rp))
            if ctx.needs_input_grad[3]:
                da = torch.empty((r, k), dtype=torch.float32, device=g.device)
                nb = _lib.query("sb_lora_grad_workspace_bytes", m, k, r)
                ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=g.device)
                _lib.call("sb_lora_grad_a", u32.data_ptr(), x2d.data_ptr(), m, k, r, da.data_ptr(),
                          ws.data_ptr(), nb, stream)
                da = da.to(lora_a.dtype)
            if ctx.needs_input_grad[4]:
                db = torch.empty((n, r), dtype=torch.float32, device=g.device)
                nb = _lib.query("sb_lora_grad_workspace_bytes", m, n, r)
                ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=g.device)
                _lib.call("sb_lora_grad_b", g.data_ptr(), z.data_ptr(), m, n, r, ctx.scaling,
                          db.data_ptr(), ws.data_ptr(), nb, stream)
                db = db.to(lora_b.dtype)
        elif ctx.needs_input_grad[0]:
            dx = nf4_linear_raw(g, packed, state, transpose=True)
        if dx is not None:
            dx = dx.reshape(ctx.x_shape)
        return dx, None, None, da, db, None, None


def nf4_lora_linear(x, packed, state, lora_a=None, lora_b=None, scaling=1.0, bias=None):
    """Differentiable fused QLoRA projection (the north-star hot path).

    x: fp16 [..., K] CUDA; packed/state: nested NF4 weight W[N, K];
    lora_a: [r, K] (lora_A.weight), lora_b: [N, r] (lora_B.weight), trainable;
    bias: optional frozen fp16 [N].  Returns fp16 [..., N].
    """
    n, k = _validate_state(packed, state, torch.float16)
    if (not isinstance(x, torch.Tensor) or x.device != packed.device or x.dtype != torch.float16
            or x.ndim < 1 or x.shape[-1] != k):
        raise ValueError("Expected CUDA fp16 X[..., K] matching the NF4 weight")
    if (lora_a is None) != (lora_b is None):
        raise ValueError("lora_a and lora_b must be given together")
    if lora_a is not None:
        if (lora_a.ndim != 2 or lora_b.ndim != 2 or lora_a.shape[1] != k or lora_b.shape[0] != n
                or lora_a.shape[0] != lora_b.shape[1] or lora_a.device != x.device
                or lora_b.device != x.device):
            raise ValueError("Expected lora_a[r, K] and lora_b[N, r] on the input's device")
        _padded_rank(lora_a.shape[0])
    if bias is not None and (bias.dtype != torch.float16 or bias.shape != (n,) or bias.requires_grad
                             or bias.device != x.device):
        raise ValueError("Only frozen fp16 bias[N] is supported")
    with torch.cuda.device(x.device):
        return _NF4LoRALinear.apply(x, packed, state, lora_a, lora_b, scaling,
                                    None if bias is None else bias.contiguous())
