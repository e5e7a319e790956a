"""The Qwen2 MLP on NF4 weights with SwiGLU inside the GEMM epilogues
(reference: the frozen MLP boundary solution/mlp.py:500-593 and the SwiGLU tile
engine solution/kernels/swiglu_fused.py:21-78).

    gate, up = X.deq(Wg)^T + s(X.Ag^T).Bg^T,  X.deq(Wu)^T + s(X.Au^T).Bu^T
    act      = SwiGLU(gate, up) = gate * sigmoid(gate) * up          (fp32 math on fp16 gate/up)
    Y        = act.deq(Wd)^T + s(act.Ad^T).Bd^T

Forward: ONE pair-kernel launch computes gate and up together -- each 256-wide
tile holds 128 gate and the same 128 up columns (one CTA of the pair decodes
Wg, the other Wu) -- and its epilogue writes gate|up [T, 2N] (kept for the
backward) and act [T, N]; then the down projection.  Backward: the down
projection's dX kernel applies the SwiGLU derivatives in its epilogue against
the saved gate|up and writes dgate|dup [T, 2N]; the gate and up input gradients
are ONE GEMM whose reduction runs over both weights (dX = dgate.Wg + dup.Wu),
with both LoRA terms as one rank-2r step.  The LoRA factors of gate and up
travel as one rank-2r pair (block-diagonal where they must not mix), so their
projections and weight-gradient reductions are one launch each.

``swiglu_fused_forward`` / ``swiglu_fused_backward`` keep the reference's
element-wise API (sb_swiglu_fwd / sb_swiglu_bwd) for gate/up tensors that come
from elsewhere.
"""

from __future__ import annotations

import ctypes
import weakref

import torch
from torch.autograd.function import once_differentiable

from .. import _lib
from .._spec import HALF, Operand, admit, refuse
from .nf4 import nested_shape
from .nf4_gemm import (_dual, _dual_ok, _factors, _padded_rank, _project, _reduce, _weight_struct,
                       nf4_linear_raw)


# ------------------------------------------------------------------ element-wise SwiGLU
def _matrix(t):
    return t.reshape(-1, t.shape[-1]) if t.ndim != 2 else t


def swiglu_fused_forward(gate, up, out=None):
    """act = gate * sigmoid(gate) * up for fp16 CUDA tensors of one shape (last
    dimension unit-strided); fills ``out`` when given."""
    admit("swiglu_fused_forward", gate.device if isinstance(gate, torch.Tensor) else None,
          gate=(gate, Operand(HALF, layout="rows")), up=(up, Operand(HALF, layout="rows")),
          out=(out, Operand(HALF, layout="rows", optional=True)))
    if gate.shape != up.shape or (out is not None and out.shape != gate.shape):
        refuse("swiglu_fused_forward", "gate, up and out must have one shape")
    if out is None:
        out = torch.empty_like(gate, memory_format=torch.contiguous_format)
    g, u, a = _matrix(gate), _matrix(up), _matrix(out)
    if g.numel():
        with torch.cuda.device(gate.device):
            _lib.call("sb_swiglu_fwd", g.data_ptr(), g.stride(0), u.data_ptr(), u.stride(0), a.data_ptr(),
                      a.stride(0), g.shape[0], g.shape[1], _lib.stream_of(gate.device))
    return out


def swiglu_fused_backward(gate, up, grad, gate_dtype=None, up_dtype=None):
    """(dgate, dup) of act = SwiGLU(gate, up) for the upstream ``grad`` (fp16)."""
    admit("swiglu_fused_backward", gate.device if isinstance(gate, torch.Tensor) else None,
          gate=(gate, Operand(HALF, layout="rows")), up=(up, Operand(HALF, layout="rows")),
          grad=(grad, Operand(HALF, layout="rows")))
    if gate.shape != up.shape or grad.shape != gate.shape:
        refuse("swiglu_fused_backward", "gate, up and grad must have one shape")
    if gate_dtype not in (None, HALF) or up_dtype not in (None, HALF):
        refuse("swiglu_fused_backward", "the derivatives are produced in fp16")
    dgate = torch.empty(gate.shape, device=gate.device, dtype=HALF)
    dup = torch.empty(gate.shape, device=gate.device, dtype=HALF)
    g, u, d, dg, du = (_matrix(t) for t in (gate, up, grad, dgate, dup))
    if g.numel():
        with torch.cuda.device(gate.device):
            _lib.call("sb_swiglu_bwd", g.data_ptr(), g.stride(0), u.data_ptr(), u.stride(0), d.data_ptr(),
                      d.stride(0), dg.data_ptr(), dg.stride(0), du.data_ptr(), du.stride(0), g.shape[0],
                      g.shape[1], _lib.stream_of(gate.device))
    return dgate, dup


# ------------------------------------------------------------------ gate/up LoRA as one rank-2r pair
class _PairFactors:
    """The gate and up adapters as one rank-2r adapter (rp = padded rank):
    a_cat [2rp, H] (both A stacked), at_cat [H, 2rp], b_gu [2N, 2rp] = [Bg 0; 0 Bu],
    bt_bd [2rp, 2N] = [Bg^T 0; 0 Bu^T].  Built by one sb_lora_prepare_pair launch
    when both ranks equal the padded rank and the factors share dtypes; otherwise
    from the per-adapter fp16 copies."""

    def __init__(self, ag, bg, au, bu):
        r, h = ag.shape
        n = bg.shape[0]
        rp = _padded_rank(r)
        dev = ag.device
        self.rp, self.r_gate, self.r_up = rp, r, au.shape[0]
        self.a_cat = torch.empty((2 * rp, h), device=dev, dtype=HALF)
        self.at_cat = torch.empty((h, 2 * rp), device=dev, dtype=HALF)
        self.b_gu = torch.empty((2 * n, 2 * rp), device=dev, dtype=HALF)
        self.bt_bd = torch.empty((2 * rp, 2 * n), device=dev, dtype=HALF)
        direct = (r == rp and au.shape[0] == rp and ag.dtype == au.dtype and bg.dtype == bu.dtype)
        if direct:
            tensors = [t.detach().contiguous() for t in (ag, au, bg, bu)]
            _lib.call("sb_lora_prepare_pair", tensors[0].data_ptr(), tensors[1].data_ptr(),
                      _lib.dtype_code(ag.dtype), tensors[2].data_ptr(), tensors[3].data_ptr(),
                      _lib.dtype_code(bg.dtype), rp, h, n, self.a_cat.data_ptr(), self.at_cat.data_ptr(),
                      self.b_gu.data_ptr(), self.bt_bd.data_ptr(), _lib.stream_of(dev))
            return
        fg, fu = _factors(ag, bg), _factors(au, bu)
        torch.cat([fg.a16, fu.a16], out=self.a_cat)
        torch.cat([fg.at16, fu.at16], dim=1, out=self.at_cat)
        self.b_gu.zero_()
        self.b_gu[:n, :rp] = fg.b16
        self.b_gu[n:, rp:] = fu.b16
        self.bt_bd.zero_()
        self.bt_bd[:rp, :n] = fg.bt16
        self.bt_bd[rp:, n:] = fu.bt16


_PAIR_CACHE = {}


def _pair_factors(ag, bg, au, bu):
    """Cached like _factors: reused while the four parameters are unchanged (same
    storage and version counters); rebuilt inside every CUDA-graph capture."""
    if torch.cuda.is_current_stream_capturing():
        return _PairFactors(ag, bg, au, bu)
    key = tuple(id(t) for t in (ag, bg, au, bu))
    stamp = tuple((t.data_ptr(), t._version, t.dtype, tuple(t.shape)) for t in (ag, bg, au, bu))
    stamp += (torch.cuda.current_stream(ag.device).cuda_stream,)
    hit = _PAIR_CACHE.get(key)
    if hit is not None and hit[0] == stamp and all(ref() is t for ref, t in zip(hit[1], (ag, bg, au, bu))):
        return hit[2]
    pf = _PairFactors(ag, bg, au, bu)
    if len(_PAIR_CACHE) > 1024:
        _PAIR_CACHE.clear()
    _PAIR_CACHE[key] = (stamp, tuple(weakref.ref(t) for t in (ag, bg, au, bu)), pf)
    return pf


_SIDE_STREAMS = {}


def _side_stream(dev):
    """One extra stream per device for work that only the optimizer waits for."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _SIDE_STREAMS.get(idx)
    if st is None:
        st = _SIDE_STREAMS[idx] = torch.cuda.Stream(device=torch.device("cuda", idx))
    return st


class _FusedMLP(torch.autograd.Function):
    """Forward/backward of the fused MLP.  The gate/up adapters come as a pair or
    not at all (r = 0 for the pair kernel), the down adapter independently."""

    @staticmethod
    def forward(ctx, x, scaling, g_packed, g_state, ag, bg, u_packed, u_state, au, bu, d_packed, d_state, ad, bd):
        n, h = g_state.shape
        x2d = x.reshape(-1, h)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        t = x2d.shape[0]
        dev = x.device
        s = float(scaling)
        stream = _lib.stream_of(dev)
        pf = _pair_factors(ag, bg, au, bu) if ag is not None else None
        fd = _factors(ad, bd) if ad is not None else None
        z_rows = z_t = None
        if pf is not None:
            z_rows, z_t = _project(x2d, pf.a_cat, 2 * pf.rp, s, True, 1.0, True)
        gate_up = torch.empty((t, 2 * n), device=dev, dtype=HALF)
        act = torch.empty((t, n), device=dev, dtype=HALF)
        wg, wu = _weight_struct(g_packed, g_state), _weight_struct(u_packed, u_state)
        if t:
            _lib.call("sb_nf4_mlp_gate_up_fwd", x2d.data_ptr(), t, ctypes.byref(wg), ctypes.byref(wu),
                      _lib.ptr(z_rows), None if pf is None else pf.b_gu.data_ptr(),
                      0 if pf is None else 2 * pf.rp, gate_up.data_ptr(), act.data_ptr(), stream)
        zd_t = None
        if fd is not None:
            zd_rows, zd_t = _project(act, fd.a16, fd.rp, s, True, 1.0, True)
            y = nf4_linear_raw(act, d_packed, d_state, lora_a=zd_rows, lora_b=fd.b16)
        else:
            y = nf4_linear_raw(act, d_packed, d_state)
        ctx.save_for_backward(x2d, gate_up, act, z_t, zd_t,
                              None if pf is None else pf.at_cat, None if pf is None else pf.bt_bd,
                              None if fd is None else fd.at16, None if fd is None else fd.bt16,
                              g_packed, u_packed, d_packed)
        ctx.states = (g_state, u_state, d_state)
        dtypes = tuple(None if p is None else p.dtype for p in (ag, bg, au, bu, ad, bd))
        ctx.meta = (s, None if pf is None else (pf.rp, pf.r_gate, pf.r_up),
                    None if fd is None else fd.r, x.shape, dtypes)
        return y.reshape(*x.shape[:-1], d_state.shape[0])

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        (x2d, gate_up, act, z_t, zd_t, at_cat, bt_bd, at_d, bt_d, g_packed, u_packed, d_packed) = ctx.saved_tensors
        g_state, u_state, d_state = ctx.states
        s, pair, r_down, x_shape, (ag_t, bg_t, au_t, bu_t, ad_t, bd_t) = ctx.meta
        n, h = g_state.shape
        hd = d_state.shape[0]
        g = grad.reshape(-1, hd)
        if g.dtype != HALF or not g.is_contiguous():
            g = g.to(HALF).contiguous()
        t = g.shape[0]
        dev = g.device
        stream = _lib.stream_of(dev)
        # down: dact (with its LoRA term) -> (dgate, dup) in one launch.  The down
        # adapter's U = s dY.B and dB = s (Z^T.dY)^T come from one pass over dY.
        ud = ud_t = d_bd = None
        rpd = 0
        if at_d is not None:
            rpd = at_d.shape[1]
            if _dual_ok(g, zd_t, bt_d, rpd, 0):
                ud, ud_t, d_bd = _dual(g, zd_t, bt_d, rpd, 0, s, bd_t, s, True, s, True)
                d_bd = d_bd[:, :r_down]
            else:
                ud, ud_t = _project(g, bt_d, rpd, s, True, s, True)
        dgate_up = torch.empty((t, 2 * n), device=dev, dtype=HALF)
        wd = _weight_struct(d_packed, d_state)
        if t:
            _lib.call("sb_nf4_mlp_down_dx", g.data_ptr(), t, ctypes.byref(wd), _lib.ptr(ud), _lib.ptr(at_d),
                      rpd, gate_up.data_ptr(), dgate_up.data_ptr(), stream)
        d_ad = None
        main = torch.cuda.current_stream(dev)
        side = None
        if at_d is not None:
            if d_bd is None:
                d_bd = _reduce(zd_t, g, rpd, s, True, bd_t)[:, :r_down]
            # The down adapter's dA = U_d^T . act only feeds the optimizer: it runs on a
            # side stream beside the gate/up factor pass below and joins before the
            # gate/up dX, which would otherwise leave it no SM.
            side = _side_stream(dev)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                d_ad = _reduce(ud_t, act, rpd, 1.0, False, ad_t)[:r_down]
            d_ad.record_stream(main)
        # gate + up: one reduction over both weights, both LoRA terms in one rank-2rp
        # step; U_cat = s dgate|dup . blockdiag(B_g, B_u) and the two dB blocks come
        # from one pass over dgate|dup.
        u_cat = u_cat_t = d_bgu = None
        r2 = 0
        if pair is not None:
            rp = pair[0]
            r2 = 2 * rp
            if _dual_ok(dgate_up, z_t, bt_bd, r2, n):
                u_cat, u_cat_t, d_bgu = _dual(dgate_up, z_t, bt_bd, r2, n, s, torch.float32, s, True, s, True)
            else:
                u_cat, u_cat_t = _project(dgate_up, bt_bd, r2, s, True, s, True)
        if side is not None:
            main.wait_stream(side)
        dx = torch.empty((t, h), device=dev, dtype=HALF)
        wg, wu = _weight_struct(g_packed, g_state), _weight_struct(u_packed, u_state)
        if t:
            nbytes = _lib.query("sb_nf4_linear_dx2_workspace_bytes", t, n, h)
            scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
            _lib.call("sb_nf4_linear_dx2", dgate_up.data_ptr(), t, ctypes.byref(wg), ctypes.byref(wu),
                      _lib.ptr(u_cat), _lib.ptr(at_cat), r2, dx.data_ptr(), scratch.data_ptr(), nbytes, stream)
        d_ag = d_bg = d_au = d_bu = None
        if pair is not None:
            rp, r_gate, r_up = pair
            d_acat = _reduce(u_cat_t, x2d, r2, 1.0, False, torch.float32)
            d_ag = d_acat[:r_gate].to(ag_t)
            d_au = d_acat[rp:rp + r_up].to(au_t)
            if d_bgu is not None:  # [2N, rp]: each half's rows of its own adapter
                d_bg = d_bgu[:n, :r_gate].to(bg_t)
                d_bu = d_bgu[n:, :r_up].to(bu_t)
            else:
                d_bgu = _reduce(z_t, dgate_up, r2, s, True, torch.float32)
                d_bg = d_bgu[:n, :r_gate].to(bg_t)
                d_bu = d_bgu[n:, rp:rp + r_up].to(bu_t)
        return (dx.reshape(x_shape), None, None, None, d_ag, d_bg, None, None, d_au, d_bu, None, None,
                d_ad, d_bd)


def nf4_swiglu_mlp(x, gate, up, down, scaling=1.0):
    """Differentiable Qwen2 MLP ``down(SwiGLU(gate(x), up(x)))`` on NF4 weights.
    x: fp16 [..., H] CUDA; gate / up / down: tuples (packed, quant_state, lora_a,
    lora_b) with gate/up [N, H] and down [H, N] (N a multiple of 128, H of 64);
    lora_a [r, in] / lora_b [out, r] are the adapter (r <= 32) or both None (a
    frozen projection; gate and up have adapters together or neither).
    Returns fp16 [..., H]."""
    entry = "nf4_swiglu_mlp"
    (gp, gs, ag, bg), (up_p, us, au, bu), (dp, ds, ad, bd) = gate, up, down
    n, h = nested_shape(gp, gs, entry=entry)
    if nested_shape(up_p, us, entry=entry) != (n, h) or nested_shape(dp, ds, entry=entry) != (h, n):
        refuse(entry, "gate/up must be [N, H] and down [H, N]")
    if n % 128 or h % 64:
        refuse(entry, f"intermediate size {n} must be a multiple of 128 and hidden size {h} of 64")
    admit(entry, gp.device, x=(x, Operand(HALF, layout=None)))
    if x.ndim < 1 or x.shape[-1] != h:
        refuse(entry, f"x has shape {tuple(x.shape)}, the MLP takes {h} features")
    if (ag is None) != (bg is None) or (au is None) != (bu is None) or (ad is None) != (bd is None):
        refuse(entry, "each adapter needs both factors or none")
    if (ag is None) != (au is None):
        refuse(entry, "gate and up carry adapters together or not at all")
    for name, (a, b, rows_in, rows_out) in {"gate": (ag, bg, h, n), "up": (au, bu, h, n),
                                            "down": (ad, bd, n, h)}.items():
        if a is None:
            continue
        admit(entry, x.device, **{f"{name}_lora_a": (a, Operand(torch.float16, torch.float32, ndim=2, layout=None)),
                                  f"{name}_lora_b": (b, Operand(torch.float16, torch.float32, ndim=2, layout=None))})
        if a.shape[1] != rows_in or b.shape[0] != rows_out or b.shape[1] != a.shape[0]:
            refuse(entry, f"{name} LoRA factors {tuple(a.shape)} / {tuple(b.shape)} do not fit")
        if _padded_rank(a.shape[0]) > 32:
            refuse(entry, f"{name} adapter rank {a.shape[0]} above 32")
    if ag is not None and _padded_rank(ag.shape[0]) != _padded_rank(au.shape[0]):
        refuse(entry, "gate and up adapters must pad to the same rank")
    with torch.cuda.device(x.device):
        return _FusedMLP.apply(x, scaling, gp, gs, ag, bg, up_p, us, au, bu, dp, ds, ad, bd)
