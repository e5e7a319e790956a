"""CPU oracle for the QLoRA hot path -- TEST INFRASTRUCTURE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline
leg and ``--impl reference``) may import this module, and only as the checker or
the timed CPU baseline.  The shipped path (``soupsuck_b200``) never calls it.

Each function restates one reference kernel of Khasuetolog/soupsuck in numpy,
with the exact cast order of the Triton source it cites (paths are relative to
the reference project root).  Floating-point arithmetic is float32 where the
reference computes in float32, so the byte-level results of elementwise kernels
(NF4 decode, LoRA epilogue, the residual sum of add-RMSNorm) are bit-exact.
Reductions (RMSNorm statistics, GEMMs, softmax sums) are computed in float64
here; they are compared against the CUDA path with the tolerances stated in the
tests, as the reference's own tests do.

Parity pin: the NF4 decoder, LoRA epilogue and add-RMSNorm/CE statistics are
pinned against outputs of the reference's own ``@triton.jit`` kernels executed
with ``TRITON_INTERPRET=1`` (``tests/golden/make_golden.py`` writes the
fixtures; ``tests/test_oracle_golden.py`` checks this module against them).
"""

from __future__ import annotations

import numpy as np

F16 = np.float16
F32 = np.float32
F64 = np.float64

# NF4 format data: the sixteen normal-float code values, code 0 = -1.0,
# code 7 = 0.0, code 15 = 1.0 (solution/kernels/nf4.py:32-37).
NF4_VALUES = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
], dtype=F32)


# --------------------------------------------------------------------------
# NF4 dequantisation (solution/kernels/nf4.py:41-59, flat variant :181-187)
# --------------------------------------------------------------------------

def nf4_codes(packed: np.ndarray, n: int) -> np.ndarray:
    """Nibble of element i: byte i//2, HIGH nibble for even i (nf4.py:46-47)."""
    packed = np.ascontiguousarray(packed).reshape(-1)
    idx = np.arange(n, dtype=np.int64)
    byte = packed[idx >> 1].astype(np.int32)
    return np.where((idx & 1) == 0, byte >> 4, byte & 15)


def nf4_block_scales_nested(qabs, absmax2, code2, offset, n: int) -> np.ndarray:
    """fp32(fp32(code2[qabs[b]] * absmax2[b // 256]) + offset), no FMA (nf4.py:50-55)."""
    blocks = (n + 63) // 64
    b = np.arange(blocks, dtype=np.int64)
    q = np.asarray(qabs).reshape(-1)[:blocks].astype(np.int64)
    code_value = np.asarray(code2, dtype=F32).reshape(-1)[q]
    scale_value = np.asarray(absmax2, dtype=F32).reshape(-1)[b >> 8]
    decoded = (code_value * scale_value).astype(F32)
    off = F32(np.asarray(offset, dtype=F32).reshape(-1)[0])
    return (decoded + off).astype(F32)


def nf4_dequant_nested(packed, qabs, absmax2, code2, offset, n: int) -> np.ndarray:
    """Bit-exact restatement of ``nf4_decode_kernel`` with NESTED=True."""
    if n == 0:
        return np.zeros(0, dtype=F16)
    codes = nf4_codes(packed, n)
    scales = nf4_block_scales_nested(qabs, absmax2, code2, offset, n)
    idx = np.arange(n, dtype=np.int64)
    value = (NF4_VALUES[codes] * scales[idx >> 6]).astype(F32)
    return value.astype(F16)


def nf4_dequant_flat(packed, absmax, n: int) -> np.ndarray:
    """``nf4_decode_kernel`` with NESTED=False: fp32 absmax[i // 64] (nf4.py:56-57)."""
    if n == 0:
        return np.zeros(0, dtype=F16)
    codes = nf4_codes(packed, n)
    idx = np.arange(n, dtype=np.int64)
    scales = np.asarray(absmax, dtype=F32).reshape(-1)[idx >> 6]
    return (NF4_VALUES[codes] * scales).astype(F32).astype(F16)


# --------------------------------------------------------------------------
# LoRA epilogue (solution/kernels/lora_epilogue.py:24-43)
# --------------------------------------------------------------------------

def _promote(a, b):
    return np.promote_types(a, b)


def lora_scale_add(base, adapter, scaling: float, cast_to_base: bool = False):
    """out = f32(base) + f32(cast_A(f32(adapter) * s)) [cast to base dtype first].

    Output dtype is base's dtype when cast_to_base, else promote(base, adapter)
    (lora_epilogue.py:24-34 and :58).
    """
    base = np.asarray(base)
    adapter = np.asarray(adapter)
    s = F32(scaling)
    scaled = (adapter.astype(F32) * s).astype(F32).astype(adapter.dtype).astype(F32)
    if cast_to_base:
        scaled = scaled.astype(base.dtype).astype(F32)
        out_dtype = base.dtype
    else:
        out_dtype = _promote(base.dtype, adapter.dtype)
    return (base.astype(F32) + scaled).astype(F32).astype(out_dtype)


def lora_scale_gradient(grad, adapter_dtype, scaling: float):
    """dAdapter = f32(cast_A(grad)) * s, stored in the adapter dtype (:37-43)."""
    g = np.asarray(grad).astype(adapter_dtype).astype(F32)
    return (g * F32(scaling)).astype(F32).astype(adapter_dtype)


# --------------------------------------------------------------------------
# Residual add + RMSNorm (solution/kernels/add_rmsnorm.py:37-81)
# --------------------------------------------------------------------------

def add_rmsnorm_forward(residual, delta, weight, eps: float, out_dtype=None):
    """Return (s, y, rstd) with the reference's cast order.

    s = cast_S(f32(r) + f32(d)); rstd = rsqrt(mean(f32(s)^2) + eps);
    q = cast_S(f32(s) * rstd); y = f32(q) * f32(w) stored in promote(S, W) or
    ``out_dtype`` (add_rmsnorm.py:43-51, dtypes :89-92).
    """
    residual = np.asarray(residual)
    delta = np.asarray(delta)
    weight = np.asarray(weight)
    s_dtype = _promote(residual.dtype, delta.dtype)
    y_dtype = out_dtype or _promote(s_dtype, weight.dtype)
    s = (residual.astype(F32) + delta.astype(F32)).astype(F32).astype(s_dtype)
    sf = s.astype(F64)
    h = s.shape[-1]
    rstd = (1.0 / np.sqrt((sf * sf).sum(-1) / h + eps)).astype(F32)
    q = (s.astype(F32) * rstd[..., None]).astype(F32).astype(s_dtype).astype(F32)
    y = (q * weight.astype(F32)).astype(F32).astype(y_dtype)
    return s, y, rstd


def add_rmsnorm_backward(s, weight, rstd, grad_s=None, grad_y=None,
                         residual_dtype=None, delta_dtype=None):
    """ds = cast_S(cast_S(rstd*(u - a*mean(u*a))) + g_s), u = cast_S(g_y*w), a = s*rstd.

    Returned once per requested input dtype (add_rmsnorm.py:63-81, :112-122).
    """
    s = np.asarray(s)
    s_dtype = s.dtype
    h = s.shape[-1]
    if grad_y is not None:
        sf = s.astype(F32)
        r = np.asarray(rstd, dtype=F32)[..., None]
        a = (sf * r).astype(F32)
        u = (np.asarray(grad_y).astype(F32) * np.asarray(weight).astype(F32)).astype(F32)
        u = u.astype(s_dtype).astype(F32)
        proj = ((u.astype(F64) * a.astype(F64)).sum(-1) / h)[..., None]
        ds = (r.astype(F64) * (u.astype(F64) - a.astype(F64) * proj))
        ds = ds.astype(F32).astype(s_dtype).astype(F32)
    else:
        ds = np.zeros(s.shape, dtype=F32)
    if grad_s is not None:
        ds = (ds + np.asarray(grad_s).astype(F32)).astype(F32)
    ds = ds.astype(s_dtype).astype(F32)
    out = []
    for dt in (residual_dtype, delta_dtype):
        out.append(None if dt is None else ds.astype(dt))
    return tuple(out)


def rmsnorm_weight_grad(s, rstd, grad_y, exact_is_half: bool):
    """dgamma = sum_rows(g * cast_S(s*rstd)) with optional fp16 product rounding
    (solution/kernels/rmsnorm.py:73-102)."""
    s = np.asarray(s)
    q = (s.astype(F32) * np.asarray(rstd, dtype=F32)[:, None]).astype(F32).astype(s.dtype).astype(F32)
    prod = (np.asarray(grad_y).astype(F32) * q).astype(F32)
    if exact_is_half:
        prod = prod.astype(F16).astype(F32)
    return prod.astype(F64).sum(0).astype(F32)


def rmsnorm_forward(x, weight, eps: float, out_dtype=None):
    """Qwen2 RMSNorm (solution/kernels/rmsnorm.py:42-52)."""
    x = np.asarray(x)
    weight = np.asarray(weight)
    h = x.shape[-1]
    xf = x.astype(F64)
    rstd = (1.0 / np.sqrt((xf * xf).sum(-1) / h + eps)).astype(F32)
    q = (x.astype(F32) * rstd[..., None]).astype(F32).astype(x.dtype).astype(F32)
    y_dtype = out_dtype or _promote(x.dtype, weight.dtype)
    return (q * weight.astype(F32)).astype(F32).astype(y_dtype), rstd


def rmsnorm_input_grad(x, weight, rstd, grad):
    """dx = rstd*(u - a*mean(u*a)), u = cast_X(g*w), a = x*rstd (rmsnorm.py:55-70)."""
    x = np.asarray(x)
    h = x.shape[-1]
    r = np.asarray(rstd, dtype=F32)[..., None]
    a = (x.astype(F32) * r).astype(F32)
    u = (np.asarray(grad).astype(F32) * np.asarray(weight).astype(F32)).astype(F32)
    u = u.astype(x.dtype).astype(F32)
    proj = ((u.astype(F64) * a.astype(F64)).sum(-1) / h)[..., None]
    return (r.astype(F64) * (u.astype(F64) - a.astype(F64) * proj)).astype(F32).astype(x.dtype)


# --------------------------------------------------------------------------
# Fused linear cross-entropy (solution/kernels/cross_entropy.py:51-211)
# --------------------------------------------------------------------------

def fp16_logits(hidden, weight):
    """Logits of fp16 operands, accumulated exactly, rounded once to fp16
    (the reference's torch.mm with fp16 inputs and output, :146-149)."""
    h = np.asarray(hidden).astype(F16).astype(F64)
    w = np.asarray(weight).astype(F16).astype(F64)
    return (h @ w.T).astype(F16)


def ce_forward(hidden, weight, targets, ignore_index: int = -100, chunk: int = 4096):
    """(loss, entropy, argmax, lse) via the reference's chunked online statistics.

    Per chunk: tile max, first argmax (ties -> lowest index), rescaled sum of
    exp and of exp*z, target logit (:51-89); then lse = m + log s,
    entropy = lse - t/s, loss = lse - z_t or 0 when ignored (:92-105).
    """
    targets = np.asarray(targets, dtype=np.int64)
    n = targets.shape[0]
    v = np.asarray(weight).shape[0]
    m = np.full(n, -np.inf)
    s = np.zeros(n)
    t = np.zeros(n)
    tz = np.zeros(n)
    best = np.full(n, np.iinfo(np.int64).max, dtype=np.int64)
    rows = np.arange(n)
    for start in range(0, v, chunk):
        z = fp16_logits(hidden, np.asarray(weight)[start:start + chunk]).astype(F64)
        width = z.shape[1]
        tile_max = z.max(axis=1) if width else np.full(n, -np.inf)
        tile_arg = z.argmax(axis=1) + start
        new_m = np.maximum(m, tile_max)
        rescale = np.exp(m - new_m)
        p = np.exp(z - new_m[:, None])
        s = s * rescale + p.sum(1)
        t = t * rescale + (p * z).sum(1)
        inside = (targets >= start) & (targets < start + width) & (targets != ignore_index)
        col = np.clip(targets - start, 0, max(width - 1, 0))
        tz = tz + np.where(inside, z[rows, col], 0.0)
        best = np.where(tile_max > m, tile_arg,
                        np.where(tile_max == m, np.minimum(best, tile_arg), best))
        m = new_m
    lse = m + np.log(s)
    entropy = lse - t / s
    loss = np.where(targets != ignore_index, lse - tz, 0.0)
    return loss.astype(F32), entropy.astype(F32), best.astype(np.int64), lse.astype(F32)


def ce_backward_ideal(hidden, weight, targets, grad, ignore_index: int = -100,
                      chunk: int = 8192):
    """Analytic dX of CE at the fp16-rounded logits: (softmax - onehot)*g @ W16.

    This is the 'ideal' gradient of solution/tests/test_cross_entropy.py:89-98
    that the reference's own tests bound its result against.  Two passes over
    vocabulary chunks (exact float64 log-sum-exp, then the weighted sum), so a
    full 151,936-row head never has to be widened to float64 at once.
    """
    targets = np.asarray(targets, dtype=np.int64)
    weight = np.asarray(weight)
    n, v = targets.shape[0], weight.shape[0]
    m = np.full(n, -np.inf)
    s = np.zeros(n)
    for start in range(0, v, chunk):
        z = fp16_logits(hidden, weight[start:start + chunk]).astype(F64)
        new_m = np.maximum(m, z.max(1))
        s = s * np.exp(m - new_m) + np.exp(z - new_m[:, None]).sum(1)
        m = new_m
    lse = m + np.log(s)
    valid = targets != ignore_index
    g = np.where(valid, np.asarray(grad, dtype=F64), 0.0)
    rows = np.arange(n)
    out = np.zeros((n, weight.shape[1]), dtype=F64)
    for start in range(0, v, chunk):
        wc = weight[start:start + chunk].astype(F16).astype(F64)
        p = np.exp(fp16_logits(hidden, weight[start:start + chunk]).astype(F64) - lse[:, None])
        inside = valid & (targets >= start) & (targets < start + wc.shape[0])
        p[rows[inside], targets[inside] - start] -= 1.0
        out += (p * g[:, None]) @ wc
    return out


def ce_backward_reference(hidden, weight, targets, lse, grad, ignore_index: int = -100,
                          chunk: int = 4096):
    """The reference's own backward arithmetic (:164-211): gain-scaled fp16 dZ.

    gain = max(|g|, 1e-30) / 1024 per valid row; dz = fp16((exp(z - lse) -
    onehot) * g / gain); dx = sum_chunks(dz @ W16) in fp32, then dx *= gain.
    """
    targets = np.asarray(targets, dtype=np.int64)
    hidden16 = np.asarray(hidden).astype(F16)
    n, h = hidden16.shape
    out = np.zeros((n, h), dtype=F32)
    valid = np.nonzero(targets != ignore_index)[0]
    if valid.size == 0:
        return out
    hv = hidden16[valid]
    tv = targets[valid]
    lv = np.asarray(lse, dtype=F32)[valid].astype(F64)
    g = np.asarray(grad, dtype=F32)[valid]
    gain = (np.maximum(np.abs(g), F32(1e-30)) / F32(1024.0)).astype(F32)
    dx = np.zeros((valid.size, h), dtype=F64)
    w16 = np.asarray(weight).astype(F16)
    for start in range(0, w16.shape[0], chunk):
        wc = w16[start:start + chunk]
        z = fp16_logits(hv, wc).astype(F64)
        cols = np.arange(start, start + wc.shape[0])
        onehot = (cols[None, :] == tv[:, None]).astype(F64)
        dz = ((np.exp(z - lv[:, None]) - onehot) * g[:, None].astype(F64)) / gain[:, None].astype(F64)
        dz16 = dz.astype(F32).astype(F16).astype(F64)
        dx += dz16 @ wc.astype(F64)
    out[valid] = (dx.astype(F32) * gain[:, None]).astype(F32)
    return out


# --------------------------------------------------------------------------
# NF4 linear with LoRA (north-star GEMM; reference semantics of
# solution/lora.py:135-164 + bnb MatMul4Bit, mirrored at
# solution/kernels/nf4_gemm.py:35-71 and :109-118)
# --------------------------------------------------------------------------

def nf4_linear_forward(x, w16, lora_a=None, lora_b=None, scaling=0.0, bias=None):
    """Y = X @ deq(W)^T + s * (X @ A^T) @ B^T (+ bias), exact in float64."""
    xf = np.asarray(x).astype(F64)
    y = xf @ np.asarray(w16).astype(F64).T
    if bias is not None:
        y = y + np.asarray(bias).astype(F64)
    if lora_a is not None:
        z = xf @ np.asarray(lora_a).astype(F64).T
        y = y + scaling * (z @ np.asarray(lora_b).astype(F64).T)
    return y


def nf4_linear_dx(dy, w16, lora_a=None, lora_b=None, scaling=0.0):
    """dX = dY @ deq(W) + s * (dY @ B) @ A, exact in float64."""
    g = np.asarray(dy).astype(F64)
    dx = g @ np.asarray(w16).astype(F64)
    if lora_a is not None:
        u = g @ np.asarray(lora_b).astype(F64)
        dx = dx + scaling * (u @ np.asarray(lora_a).astype(F64))
    return dx


def lora_weight_grads(x, dy, lora_a, lora_b, scaling):
    """dA = (s * dY @ B)^T @ X and dB = (s * dY)^T @ (X @ A^T), float64."""
    xf = np.asarray(x).astype(F64)
    g = np.asarray(dy).astype(F64) * scaling
    z = xf @ np.asarray(lora_a).astype(F64).T
    u = g @ np.asarray(lora_b).astype(F64)
    return u.T @ xf, g.T @ z


def gemm_gate(actual, expected, rtol=2e-3, atol=2e-3, rel_l2=1e-3):
    """The reference's preregistered NF4-GEMM gate (experiments/reports/EXP-002.md:57-72):
    elementwise |a - e| <= atol + rtol*|e|, finite, and relative L2 <= 1e-3.
    Returns (ok, max_abs_err, rel_l2_err)."""
    a = np.asarray(actual, dtype=F64)
    e = np.asarray(expected, dtype=F64)
    err = np.abs(a - e)
    finite = bool(np.isfinite(a).all())
    close = bool((err <= atol + rtol * np.abs(e)).all())
    denom = float(np.linalg.norm(e)) or 1.0
    rel = float(np.linalg.norm(a - e)) / denom
    return finite and close and rel <= rel_l2, float(err.max(initial=0.0)), rel


# --------------------------------------------------------------------------
# Joint q/k rotary embedding (solution/kernels/rope.py:24-105)
# --------------------------------------------------------------------------

def _rope_rows(x, cos, sin, out_dtype, backward):
    """x [B, H, S, D] (any float dtype), cos/sin [1|B, S, D]; products rounded to
    out_dtype before the sum, the sum rounded on store (rope.py:55-58, :91-93)."""
    x = np.asarray(x).astype(F32)
    half = x.shape[-1] // 2
    c = np.asarray(cos).astype(F32)[:, None]
    s = np.asarray(sin).astype(F32)[:, None]
    c1, c2, s1, s2 = c[..., :half], c[..., half:], s[..., :half], s[..., half:]
    x1, x2 = x[..., :half], x[..., half:]
    r = lambda v: v.astype(F32).astype(out_dtype).astype(F32)
    if not backward:
        lo = r(x1 * c1) + r((-x2) * s1)
        hi = r(x2 * c2) + r(x1 * s2)
    else:
        lo = r(x1 * c1) + r(x2 * s2)
        hi = r(x2 * c2) - r(x1 * s1)
    return np.concatenate([lo.astype(F32), hi.astype(F32)], axis=-1).astype(out_dtype)


def rope_forward(q, k, cos, sin):
    """(yq, yk): y = x*cos + rotate_half(x)*sin in promote(x, cos), eager rounding."""
    cdt = np.asarray(cos).dtype
    return (_rope_rows(q, cos, sin, np.promote_types(np.asarray(q).dtype, cdt), False),
            _rope_rows(k, cos, sin, np.promote_types(np.asarray(k).dtype, cdt), False))


def rope_backward(gq, gk, cos, sin, q_dtype, k_dtype):
    """(dq, dk): dx1 = g1*c1 + g2*s2, dx2 = g2*c2 - g1*s1, products rounded to x's dtype."""
    return (_rope_rows(gq, cos, sin, q_dtype, True), _rope_rows(gk, cos, sin, k_dtype, True))


# --------------------------------------------------------------------------
# SwiGLU tile engine (solution/kernels/swiglu_fused.py:21-46)
# --------------------------------------------------------------------------

def _sigmoid32(g):
    return (F32(1.0) / (F32(1.0) + np.exp(-g).astype(F32))).astype(F32)


def swiglu_forward(gate, up, out_dtype=None):
    """a = g * sigmoid(g) * u in fp32, stored in gate's dtype (swiglu_fused.py:29-46)."""
    gate = np.asarray(gate)
    g = gate.astype(F32)
    u = np.asarray(up).astype(F32)
    p = _sigmoid32(g)
    return ((g * p).astype(F32) * u).astype(F32).astype(out_dtype or gate.dtype)


def swiglu_backward(gate, up, grad, gate_dtype=None, up_dtype=None):
    """dg = (da*u) * (p + a*(1-p)), du = da * a with p = sigmoid(g), a = g*p (:35-41)."""
    gate = np.asarray(gate)
    up = np.asarray(up)
    g = gate.astype(F32)
    u = up.astype(F32)
    da = np.asarray(grad).astype(F32)
    p = _sigmoid32(g)
    act = (g * p).astype(F32)
    slope = (p + (act * (F32(1.0) - p)).astype(F32)).astype(F32)
    dg = ((da * u).astype(F32) * slope).astype(F32)
    du = (da * act).astype(F32)
    return dg.astype(gate_dtype or gate.dtype), du.astype(up_dtype or up.dtype)


# --------------------------------------------------------------------------
# Right-padding removal (solution/unpad.py:51-72, :149-200)
# --------------------------------------------------------------------------

def unpad_lengths(mask, labels=None, ignore_index: int = -100):
    """Real-token count per row of a binary right-padded mask whose padded positions
    carry ignore_index labels, or None when any rule fails (a value other than 0/1,
    a one after a zero, a padded label, an empty row) -- _batch_metadata (:164-183)
    followed by right_padding_lengths (:51-72)."""
    mask = np.asarray(mask)
    if mask.ndim != 2 or mask.shape[0] == 0 or mask.shape[1] == 0:
        return None
    real = mask == 1
    if not ((mask == 0) | real).all():
        return None
    if labels is not None and not (real | (np.asarray(labels) == ignore_index)).all():
        return None
    lengths = real.sum(axis=1)
    if (lengths == 0).any():
        return None
    prefix = np.arange(mask.shape[1])[None, :] < lengths[:, None]
    if not np.array_equal(prefix, real):
        return None
    return tuple(int(x) for x in lengths)


def unpad_indices(lengths, sequence: int):
    """Row-major positions b*S + t of the real tokens (_indices_from_lengths :186-200)."""
    return np.concatenate([b * sequence + np.arange(n) for b, n in enumerate(lengths)]).astype(np.int64)


def unpad_pack(x, lengths):
    """[B, S, ...] -> [T, ...] (the index_select of _pack :149-150)."""
    x = np.asarray(x)
    flat = x.reshape(x.shape[0] * x.shape[1], *x.shape[2:])
    return flat[unpad_indices(lengths, x.shape[1])]


def unpad_scatter(packed, lengths, sequence: int):
    """[T, ...] -> zero-padded [B, S, ...] (the index_copy of _scatter :153-161)."""
    packed = np.asarray(packed)
    out = np.zeros((len(lengths) * sequence, *packed.shape[1:]), dtype=packed.dtype)
    out[unpad_indices(lengths, sequence)] = packed
    return out.reshape(len(lengths), sequence, *packed.shape[1:])
