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
import weakref

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .._spec import FLOATS, HALF, Operand, admit, refuse
from .nf4 import nested_shape

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
    raise ValueError(f"LoRA rank {r} is above the largest supported rank {_SUPPORTED_RANKS[-1]}")


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
    """Reference signature (solution/kernels/nf4_gemm.py:74-96): X[.., K] . deq(W)^T
    (+ bias), or with transpose=True dY[.., N] . deq(W), as one fused launch.
    ``config`` (a Triton tile choice there) is accepted and has no effect."""
    n, k = nested_shape(packed, state, entry="nf4_matmul")
    width, depth = (k, n) if transpose else (n, k)
    admit("nf4_matmul", packed.device, x=(x, Operand(HALF, ndim=tuple(range(2, 9)))))
    if x.shape[-1] != depth:
        refuse("nf4_matmul", f"x has {x.shape[-1]} features, the weight takes {depth}")
    if bias is not None and transpose:
        refuse("nf4_matmul", "a bias applies to the forward product only")
    admit("nf4_matmul", x.device,
          bias=(bias, Operand(HALF, ndim=1, frozen=True, exactly=width, optional=True)))
    with torch.cuda.device(x.device):
        out = nf4_linear_raw(x.reshape(-1, depth), packed, state, transpose=transpose, bias=bias)
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


# Eager calls reuse the fp16 factor copies while the LoRA parameters are unchanged
# (same storage, same in-place version counter): with several micro-batches per
# optimizer step, or a layer called more than once, sb_lora_prepare runs once per
# weight update.  Inside a CUDA-graph capture the conversion is always part of the
# graph, because a replay has to see the parameters of its own time.
_FACTOR_CACHE = {}


def _factors(lora_a, lora_b):
    if torch.cuda.is_current_stream_capturing():
        return _LoRAFactors(lora_a, lora_b)
    key = (id(lora_a), id(lora_b))
    stamp = (lora_a.data_ptr(), lora_a._version, lora_a.dtype, tuple(lora_a.shape),
             lora_b.data_ptr(), lora_b._version, lora_b.dtype, tuple(lora_b.shape),
             torch.cuda.current_stream(lora_a.device).cuda_stream)
    hit = _FACTOR_CACHE.get(key)
    if hit is not None and hit[0] == stamp and hit[1]() is lora_a and hit[2]() is lora_b:
        return hit[3]
    f = _LoRAFactors(lora_a, lora_b)
    if len(_FACTOR_CACHE) > 4096:
        _FACTOR_CACHE.clear()
    _FACTOR_CACHE[key] = (stamp, weakref.ref(lora_a), weakref.ref(lora_b), f)
    return f


# Rows at least this long are projected by the tiled one-pass kernel of
# sb_lora_dual (u only): [32 x 256] tiles of X staged by cp.async, partials per
# 256-column block summed in order by a second kernel.
_WIDE_PROJECT_K = 4096


def _project(x2d, w16, rp, scale_rows, want_rows, scale_t, want_t):
    """rows = fp16(scale_rows * X.W^T) [m, rp]; t = fp16(scale_t * X.W^T)^T [rp, m16]."""
    m, k = x2d.shape
    if m and k >= _WIDE_PROJECT_K and (want_rows or want_t) and _dual_ok(x2d, None, w16, rp, 0):
        rows, tr, _ = _dual(x2d, None, w16, rp, 0, 1.0, None, scale_rows, want_rows, scale_t, want_t)
        return rows, tr
    rows = torch.empty((m, rp), dtype=torch.float16, device=x2d.device) if want_rows else None
    ldt = _round16(m)
    tr = torch.empty((rp, ldt), dtype=torch.float16, device=x2d.device) if want_t else None
    if m:
        _lib.call("sb_lora_project", x2d.data_ptr(), m, k, w16.data_ptr(), rp, float(scale_rows),
                  _lib.ptr(rows), rp, float(scale_t), _lib.ptr(tr), ldt, _lib.stream_of(x2d.device))
    return rows, tr


def _dual_ok(q2d, pt, bt, rp, wsplit):
    w = q2d.shape[1]
    if wsplit:
        if rp not in (32, 64) or wsplit % 256 or not 0 < wsplit < w:
            return False
    elif rp not in (16, 32):
        return False
    if pt is not None and (pt.shape[1] % 16 or pt.data_ptr() % 16):
        return False
    return (w % 8 == 0 and q2d.is_contiguous() and bt.is_contiguous() and tuple(bt.shape) == (rp, w)
            and q2d.data_ptr() % 16 == 0 and bt.data_ptr() % 16 == 0)


def _dual(q2d, pt, bt, rp, wsplit, scale_b, b_dtype, scale_rows, want_rows, scale_t, want_t):
    """One pass over q2d [m, w] for both backward products of a LoRA factor pair:
    rows / t as ``_project(q2d, bt, rp, ...)`` (U = Q.Bt^T) and
    db = scale_b * (pt[:, :m] . Q)^T [w, rh] in b_dtype, rh = rp, or rp / 2 for a
    block-diagonal pair split at column wsplit (each column's rows of its block).
    pt = None: U only (db is None)."""
    m, w = q2d.shape
    rh = rp // 2 if wsplit else rp
    dev = q2d.device
    rows = torch.empty((m, rp), dtype=torch.float16, device=dev) if want_rows else None
    ldt = _round16(m)
    tr = torch.empty((rp, ldt), dtype=torch.float16, device=dev) if want_t else None
    db = torch.empty((w, rh), dtype=b_dtype, device=dev) if pt is not None else None
    nbytes = _lib.query("sb_lora_dual_workspace_bytes", m, w, rp, wsplit)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.call("sb_lora_dual", q2d.data_ptr(), m, w, _lib.ptr(pt), 0 if pt is None else pt.shape[1],
              bt.data_ptr(), rp, wsplit, float(scale_b), 1, _lib.ptr(db),
              _lib.dtype_code(b_dtype if pt is not None else torch.float32), float(scale_rows), _lib.ptr(rows), rp,
              float(scale_t), _lib.ptr(tr), ldt, ws.data_ptr(), nbytes, _lib.stream_of(dev))
    return rows, tr, db


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
    """Y = X.deq(W)^T + s (D.A^T).B^T (+ bias) with D = X, or D = the caller's
    dropped LoRA input (a separate differentiable input: the LoRA branch of a
    PEFT layer in training sees dropout(X), the base projection sees X)."""

    @staticmethod
    def forward(ctx, x, packed, state, lora_a, lora_b, scaling, bias, lora_input):
        n, k = state.shape
        x2d = x.reshape(-1, k)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        has_lora = lora_a is not None
        separate = lora_input is not None
        f = zt = None
        if has_lora:
            f = _factors(lora_a, lora_b)
            d2d = x2d
            if separate:
                d2d = lora_input.reshape(-1, k).to(torch.float16).contiguous()
            zs, zt = _project(d2d, f.a16, f.rp, scaling, True, 1.0, True)
            y = nf4_linear_raw(x2d, packed, state, bias=bias, lora_a=zs, lora_b=f.b16)
            ctx.a_dtype, ctx.b_dtype = lora_a.dtype, lora_b.dtype
            if separate:
                ctx.d_dtype, ctx.d_shape = lora_input.dtype, lora_input.shape
                ctx.save_for_backward(d2d, packed, zt, f.at16, f.bt16, f.a16)
            else:
                ctx.save_for_backward(x2d, packed, zt, f.at16, f.bt16)
        else:
            y = nf4_linear_raw(x2d, packed, state, bias=bias)
            ctx.save_for_backward(x2d, packed)
        ctx.state, ctx.scaling, ctx.has_lora, ctx.separate = state, float(scaling), has_lora, separate
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
        dx = da = db = dd = None
        need_x = ctx.needs_input_grad[0]
        if ctx.has_lora:
            if ctx.separate:
                d2d, packed, zt, at16, bt16, a16 = ctx.saved_tensors
            else:
                d2d, packed, zt, at16, bt16 = ctx.saved_tensors
            rp, r, s = at16.shape[1], ctx.r, ctx.scaling
            need_a, need_b = ctx.needs_input_grad[3], ctx.needs_input_grad[4]
            need_d = ctx.separate and ctx.needs_input_grad[7]
            # u = s dY.B: the rank-r factor of the LoRA input gradient (and of dA);
            # with dB = s (Z^T.dY)^T from the same pass over dY when both are wanted.
            want_u = need_x or need_d or need_a
            if need_b and want_u and _dual_ok(g, zt, bt16, rp, 0):
                u, ut, db_full = _dual(g, zt, bt16, rp, 0, s, ctx.b_dtype, s, need_x or need_d, s, need_a)
                db = db_full[:, :r]
                need_b = False
            elif want_u:
                u, ut = _project(g, bt16, rp, s, need_x or need_d, s, need_a)
            else:
                u = ut = None
            if need_x:
                if ctx.separate:
                    dx = nf4_linear_raw(g, packed, state, transpose=True)
                else:
                    dx = nf4_linear_raw(g, packed, state, transpose=True, lora_a=u, lora_b=at16)
            if need_d:
                # d(loss)/dD = u . A, rank r: the expansion is one small fp16 product.
                dd = torch.mm(u, a16).to(ctx.d_dtype).reshape(ctx.d_shape)
            if need_a:
                da = _reduce(ut, d2d, rp, 1.0, False, ctx.a_dtype)[:r]
            if need_b:
                db = _reduce(zt, g, rp, s, True, ctx.b_dtype)[:, :r]
        else:
            x2d, packed = ctx.saved_tensors
            if need_x:
                dx = nf4_linear_raw(g, packed, state, transpose=True)
        if dx is not None:
            dx = dx.reshape(ctx.x_shape)
        return dx, None, None, da, db, None, None, dd


def nf4_lora_linear(x, packed, state, lora_a=None, lora_b=None, scaling=1.0, bias=None,
                    lora_input=None):
    """Differentiable fused QLoRA projection (the north-star hot path).

    x: fp16 [..., K] CUDA; packed/state: nested NF4 weight W[N, K];
    lora_a: [r, K] (lora_A.weight), lora_b: [N, r] (lora_B.weight), trainable;
    bias: optional frozen fp16 [N]; lora_input: optional tensor of x's shape
    (fp16 or fp32) that the LoRA branch reads instead of x -- a PEFT layer's
    dropout(x) in training, whose gradient flows back through that dropout.
    Returns fp16 [..., N].
    """
    entry = "nf4_lora_linear"
    n, k = nested_shape(packed, state, entry=entry)
    admit(entry, packed.device, x=(x, Operand(HALF, layout=None)))
    if x.ndim < 1 or x.shape[-1] != k:
        refuse(entry, f"x has shape {tuple(x.shape)}, the weight takes {k} features")
    if (lora_a is None) != (lora_b is None):
        refuse(entry, "lora_a and lora_b come together or not at all")
    if lora_a is not None:
        admit(entry, x.device, lora_a=(lora_a, Operand(*FLOATS, ndim=2, layout=None)),
              lora_b=(lora_b, Operand(*FLOATS, ndim=2, layout=None)))
        r = lora_a.shape[0]
        if lora_a.shape[1] != k or tuple(lora_b.shape) != (n, r):
            refuse(entry, f"LoRA factors {tuple(lora_a.shape)} / {tuple(lora_b.shape)} do not "
                          f"fit a [{n}, {k}] weight")
        if k % 32 or n % 32:
            refuse(entry, f"the fused LoRA step needs both weight sides divisible by 32, got {(n, k)}")
        _padded_rank(r)
    admit(entry, x.device, bias=(bias, Operand(HALF, ndim=1, frozen=True, exactly=n, layout=None,
                                                optional=True)))
    if lora_input is not None:
        if lora_a is None:
            refuse(entry, "lora_input without LoRA factors")
        admit(entry, x.device, lora_input=(lora_input, Operand(*FLOATS, layout=None)))
        if lora_input.shape != x.shape:
            refuse(entry, f"lora_input has shape {tuple(lora_input.shape)}, x {tuple(x.shape)}")
    with torch.cuda.device(x.device):
        return _NF4LoRALinear.apply(x, packed, state, lora_a, lora_b, scaling,
                                    None if bias is None else bias.contiguous(), lora_input)
