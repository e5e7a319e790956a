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


def _aligned16(t):
    """The kernels take 16-byte aligned operands; copy the rare misaligned view."""
    if t is None or t.data_ptr() % 16 == 0:
        return t
    return t.clone()


def nf4_linear_raw(x2d, packed, state, *, transpose=False, bias=None, lora_a=None, lora_b=None):
    """One launch of the fused GEMM.  lora_a [m, r] and lora_b [width, r] are the
    already-scaled fp16 low-rank factors (r padded to 16/32/64); no autograd."""
    n, k = state.shape
    m = x2d.shape[0]
    x2d, packed, lora_a, lora_b = (_aligned16(t) for t in (x2d, packed, lora_a, lora_b))
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


def _round16(m):
    return (m + 15) // 16 * 16


class _LoRAFactors:
    """fp16 copies of the LoRA weights, zero-padded to a supported rank:
    a16 [rp, K], at16 [K, rp], b16 [N, rp], bt16 [rp, N] (one sb_lora_prepare launch)."""

    def __init__(self, lora_a, lora_b):
        r, k = lora_a.shape
        n = lora_b.shape[0]
        rp = _padded_rank(r)
        a, b = lora_a.detach(), lora_b.detach()
        if rp != r:
            a = torch.cat([a, a.new_zeros((rp - r, k))])
            b = torch.cat([b, b.new_zeros((n, rp - r))], dim=1)
        a, b = a.contiguous(), b.contiguous()
        dev = a.device
        self.r, self.rp = r, rp
        self.a16 = torch.empty((rp, k), dtype=torch.float16, device=dev)
        self.at16 = torch.empty((k, rp), dtype=torch.float16, device=dev)
        self.b16 = torch.empty((n, rp), dtype=torch.float16, device=dev)
        self.bt16 = torch.empty((rp, n), dtype=torch.float16, device=dev)
        _lib.call("sb_lora_prepare", a.data_ptr(), _lib.dtype_code(a.dtype), b.data_ptr(),
                  _lib.dtype_code(b.dtype), rp, k, n, self.a16.data_ptr(), self.at16.data_ptr(),
                  self.b16.data_ptr(), self.bt16.data_ptr(), _lib.stream_of(dev))


def _project(x2d, w16, rp, scale_rows, want_rows, scale_t, want_t):
    """rows = fp16(scale_rows * X.W^T) [m, rp]; t = fp16(scale_t * X.W^T)^T [rp, m16]."""
    m, k = x2d.shape
    rows = torch.empty((m, rp), dtype=torch.float16, device=x2d.device) if want_rows else None
    ldt = _round16(m)
    tr = torch.empty((rp, ldt), dtype=torch.float16, device=x2d.device) if want_t else None
    if m:
        _lib.call("sb_lora_project", x2d.data_ptr(), m, k, w16.data_ptr(), rp, float(scale_rows),
                  _lib.ptr(rows), rp, float(scale_t), _lib.ptr(tr), ldt, _lib.stream_of(x2d.device))
    return rows, tr


def _reduce(pt, q2d, rp, scale, transpose, out_dtype):
    """scale * (pt[:, :m] . q)  -> [rp, w] (or [w, rp] when transposed) in out_dtype."""
    m, w = q2d.shape
    shape = (w, rp) if transpose else (rp, w)
    out = torch.empty(shape, dtype=out_dtype, device=q2d.device)
    nbytes = _lib.query("sb_lora_reduce_workspace_bytes", m, w, rp)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q2d.device)
    _lib.call("sb_lora_reduce", _lib.ptr(pt), pt.shape[1] if pt is not None else _round16(m),
              q2d.data_ptr(), m, w, rp, float(scale), int(transpose), out.data_ptr(),
              _lib.dtype_code(out_dtype), ws.data_ptr(), nbytes, _lib.stream_of(q2d.device))
    return out


class _NF4LoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, packed, state, lora_a, lora_b, scaling, bias):
        n, k = state.shape
        x2d = x.reshape(-1, k)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        has_lora = lora_a is not None
        f = zt = None
        if has_lora:
            f = _LoRAFactors(lora_a, lora_b)
            zs, zt = _project(x2d, f.a16, f.rp, scaling, True, 1.0, True)
            y = nf4_linear_raw(x2d, packed, state, bias=bias, lora_a=zs, lora_b=f.b16)
            ctx.a_dtype, ctx.b_dtype = lora_a.dtype, lora_b.dtype
            ctx.save_for_backward(x2d, packed, zt, f.at16, f.bt16)
        else:
            y = nf4_linear_raw(x2d, packed, state, bias=bias)
            ctx.save_for_backward(x2d, packed)
        ctx.state, ctx.scaling, ctx.has_lora = state, float(scaling), has_lora
        ctx.r = f.r if has_lora else 0
        ctx.x_shape = x.shape
        return y.reshape(*x.shape[:-1], n)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        state = ctx.state
        n, k = state.shape
        g = grad.reshape(-1, n)
        if g.dtype != torch.float16 or not g.is_contiguous():
            g = g.to(torch.float16).contiguous()
        dx = da = db = None
        if ctx.has_lora:
            x2d, packed, zt, at16, bt16 = ctx.saved_tensors
            rp, r, s = at16.shape[1], ctx.r, ctx.scaling
            need_x, need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[3], ctx.needs_input_grad[4]
            u, ut = _project(g, bt16, rp, s, need_x, s, need_a)
            if need_x:
                dx = nf4_linear_raw(g, packed, state, transpose=True, lora_a=u, lora_b=at16)
            if need_a:
                da = _reduce(ut, x2d, rp, 1.0, False, ctx.a_dtype)[:r]
            if need_b:
                db = _reduce(zt, g, rp, s, True, ctx.b_dtype)[:, :r]
        else:
            x2d, packed = ctx.saved_tensors
            if ctx.needs_input_grad[0]:
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
        if lora_a.dtype not in (torch.float16, torch.float32) or lora_b.dtype not in (torch.float16, torch.float32):
            raise ValueError("LoRA weights must be fp16 or fp32")
        if k % 32 or n % 32:
            raise ValueError("The fused LoRA path needs K and N multiples of 32")
        _padded_rank(lora_a.shape[0])
    if bias is not None and (bias.dtype != torch.float16 or bias.shape != (n,) or bias.requires_grad
                             or bias.device != x.device):
        raise ValueError("Only frozen fp16 bias[N] is supported")
    with torch.cuda.device(x.device):
        return _NF4LoRALinear.apply(x, packed, state, lora_a, lora_b, scaling,
                                    None if bias is None else bias.contiguous())
