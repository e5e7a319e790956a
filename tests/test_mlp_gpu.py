"""The fused Qwen2 MLP (SwiGLU in the GEMM epilogues) against the float64 oracle.

Reference semantics: solution/mlp.py:500-593 runs gate/up (fp16 outputs), the
SwiGLU tile engine (solution/kernels/swiglu_fused.py:21-46, restated in
oracle.swiglu_forward / swiglu_backward), then down; backward: down dX (fp16),
the SwiGLU derivatives, and the sum of the gate and up input gradients.

Gates: GEMM outputs against the exact product of the same fp16 operands with
the reference's EXP-002 gate (rtol = atol = 2e-3, rel-L2 <= 1e-3); the SwiGLU
epilogues against the oracle applied to the kernel's own fp16 inputs within one
or two fp16 ulps (CUDA's expf against numpy's exp); LoRA weight gradients within a
relative L2 of 1e-2.  At the configs[1] shape (T = 3300, H = 1536, N = 8960) a
seeded subset of rows is checked; the kernels run at full size.
"""

import ctypes
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of, oracle_dequant

pytestmark = pytest.mark.gpu


def _weight(n, k, gen):
    from soupsuck_b200.quantize import quantize_nf4
    w = (torch.randn((n, k), device="cuda", generator=gen) * 0.02).to(torch.float16)
    packed, st = quantize_nf4(w)
    return packed, st, oracle_dequant(packed, st)


def _adapter(n_out, k_in, r, gen):
    a = ((torch.rand((r, k_in), device="cuda", generator=gen) * 2 - 1) / math.sqrt(k_in)).requires_grad_()
    b = (torch.randn((n_out, r), device="cuda", generator=gen) * 0.05).requires_grad_()
    return a, b


def _h64(t):
    return np_of(t.detach().half()).astype(np.float64)


def _gate(actual, expected, what):
    ok, max_abs, rel = O.gemm_gate(np.asarray(actual, dtype=np.float64), expected)
    assert ok, f"{what}: max abs err {max_abs:.3e}, rel-L2 {rel:.3e}"


def _ulps(a, b):
    a = np.asarray(a).astype(np.float16).view(np.int16).astype(np.int32)
    b = np.asarray(b).astype(np.float16).view(np.int16).astype(np.int32)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return np.abs(a - b)


def _rows(t, count, seed):
    rng = np.random.default_rng(seed)
    picked = set(range(0, min(t, 64))) | set(range(max(t - 64, 0), t))
    picked |= set(rng.choice(t, size=min(count, t), replace=False).tolist())
    return np.array(sorted(picked))


@pytest.mark.parametrize("t,h,n,r", [(300, 512, 1024, 16), (3300, 1536, 8960, 16), (77, 256, 384, 8)],
                         ids=["small", "configs1", "ragged"])
def test_fused_mlp_forward_backward_vs_oracle(t, h, n, r):
    from soupsuck_b200.kernels.mlp import nf4_swiglu_mlp
    gen = torch.Generator(device="cuda").manual_seed(t + n)
    gp, gs, wg = _weight(n, h, gen)
    up_p, us, wu = _weight(n, h, gen)
    dp, ds, wd = _weight(h, n, gen)
    ag, bg = _adapter(n, h, r, gen)
    au, bu = _adapter(n, h, r, gen)
    ad, bd = _adapter(h, n, r, gen)
    s = 2.0
    x = torch.randn((t, h), device="cuda", dtype=torch.float16, generator=gen).requires_grad_()
    dy = torch.randn((t, h), device="cuda", dtype=torch.float16, generator=gen)
    y = nf4_swiglu_mlp(x, (gp, gs, ag, bg), (up_p, us, au, bu), (dp, ds, ad, bd), s)
    y.backward(dy)
    torch.cuda.synchronize()

    rows = _rows(t, 160, seed=t)
    xr = np_of(x.detach())[rows].astype(np.float64)
    gate = O.nf4_linear_forward(xr, wg, _h64(ag), _h64(bg), s)
    up = O.nf4_linear_forward(xr, wu, _h64(au), _h64(bu), s)
    act = O.swiglu_forward(gate.astype(np.float16), up.astype(np.float16))
    y_ref = O.nf4_linear_forward(act, wd, _h64(ad), _h64(bd), s)
    _gate(np_of(y)[rows], y_ref, "y")

    dyr = np_of(dy)[rows]
    dact = O.nf4_linear_dx(dyr, wd, _h64(ad), _h64(bd), s).astype(np.float16)
    dg, du = O.swiglu_backward(gate.astype(np.float16), up.astype(np.float16), dact)
    dg64, du64 = dg.astype(np.float64), du.astype(np.float64)
    dx_ref = (O.nf4_linear_dx(dg64, wg, _h64(ag), _h64(bg), s)
              + O.nf4_linear_dx(du64, wu, _h64(au), _h64(bu), s))
    # the upstream of dX went through two fp16 roundings (gate/up, then dact);
    # compare with the gate's relative L2 and a looser elementwise bound
    got = np_of(x.grad)[rows].astype(np.float64)
    rel = np.linalg.norm(got - dx_ref) / np.linalg.norm(dx_ref)
    assert rel < 5e-3, rel

    if t <= 300:  # LoRA weight gradients need every row
        xf = np_of(x.detach()).astype(np.float64)
        gate_f = O.nf4_linear_forward(xf, wg, _h64(ag), _h64(bg), s).astype(np.float16)
        up_f = O.nf4_linear_forward(xf, wu, _h64(au), _h64(bu), s).astype(np.float16)
        act_f = O.swiglu_forward(gate_f, up_f)
        dact_f = O.nf4_linear_dx(np_of(dy), wd, _h64(ad), _h64(bd), s).astype(np.float16)
        dg_f, du_f = O.swiglu_backward(gate_f, up_f, dact_f)
        refs = (O.lora_weight_grads(xf, dg_f.astype(np.float64), _h64(ag), _h64(bg), s)
                + O.lora_weight_grads(xf, du_f.astype(np.float64), _h64(au), _h64(bu), s)
                + O.lora_weight_grads(act_f.astype(np.float64), np_of(dy).astype(np.float64), _h64(ad),
                                      _h64(bd), s))
        for got_g, ref_g, what in zip((ag.grad, bg.grad, au.grad, bu.grad, ad.grad, bd.grad), refs,
                                      ("dAg", "dBg", "dAu", "dBu", "dAd", "dBd")):
            assert got_g.dtype == torch.float32
            rel = np.linalg.norm(np_of(got_g).astype(np.float64) - ref_g) / np.linalg.norm(ref_g)
            assert rel < 1e-2, (what, rel)


def _struct(packed, st):
    from soupsuck_b200.kernels.nf4_gemm import _weight_struct
    return _weight_struct(packed, st)


@pytest.mark.parametrize("t,h,n", [(300, 512, 1024), (1000, 1536, 8960), (5, 256, 256)])
def test_gate_up_epilogue_and_down_dx_epilogue_without_lora(t, h, n):
    """The three C-ABI launches one by one: gate|up and act, the SwiGLU-derivative
    epilogue of the down dX, and the two-weight dX."""
    from soupsuck_b200 import _lib
    gen = torch.Generator(device="cuda").manual_seed(7 * t + h)
    gp, gs, wg = _weight(n, h, gen)
    up_p, us, wu = _weight(n, h, gen)
    dp, ds, wd = _weight(h, n, gen)
    x = torch.randn((t, h), device="cuda", dtype=torch.float16, generator=gen)
    gate_up = torch.empty((t, 2 * n), device="cuda", dtype=torch.float16)
    act = torch.empty((t, n), device="cuda", dtype=torch.float16)
    stream = _lib.stream_of(x.device)
    sg, su, sd = _struct(gp, gs), _struct(up_p, us), _struct(dp, ds)
    _lib.call("sb_nf4_mlp_gate_up_fwd", x.data_ptr(), t, ctypes.byref(sg), ctypes.byref(su), None, None, 0,
              gate_up.data_ptr(), act.data_ptr(), stream)
    dy = torch.randn((t, h), device="cuda", dtype=torch.float16, generator=gen)
    dgu = torch.empty((t, 2 * n), device="cuda", dtype=torch.float16)
    _lib.call("sb_nf4_mlp_down_dx", dy.data_ptr(), t, ctypes.byref(sd), None, None, 0, gate_up.data_ptr(),
              dgu.data_ptr(), stream)
    dx = torch.empty((t, h), device="cuda", dtype=torch.float16)
    nbytes = _lib.query("sb_nf4_linear_dx2_workspace_bytes", t, n, h)
    ws = torch.empty(max(nbytes, 1), device="cuda", dtype=torch.uint8)
    _lib.call("sb_nf4_linear_dx2", dgu.data_ptr(), t, ctypes.byref(sg), ctypes.byref(su), None, None, 0,
              dx.data_ptr(), ws.data_ptr(), nbytes, stream)
    torch.cuda.synchronize()
    rows = _rows(t, 96, seed=h)
    xr = np_of(x)[rows]
    gu = np_of(gate_up)[rows]
    _gate(gu[:, :n], O.nf4_linear_forward(xr, wg), "gate")
    _gate(gu[:, n:], O.nf4_linear_forward(xr, wu), "up")
    assert _ulps(np_of(act)[rows], O.swiglu_forward(gu[:, :n], gu[:, n:])).max() <= 1
    dact = O.nf4_linear_dx(np_of(dy)[rows], wd)
    d = np_of(dgu)[rows]
    # dact is rounded to fp16 in the epilogue and the oracle rounds the exact
    # product: the two may differ by one fp16 ulp of dact, which moves dgate by
    # up to |u| ulp(dact) and dup by |g sigmoid(g)| ulp(dact).  dgate's factor
    # sigmoid(g) (1 + g (1 - sigmoid(g))) also cancels near g = -1.28, where a
    # tiny result carries the absolute error of its O(da * u) terms.  Gates:
    # relative L2 <= 1e-3, 99.9 % of elements within two fp16 ulps, and every
    # element within four ulps plus 2^-8 of those magnitudes plus 1e-5.
    da16 = dact.astype(np.float16)
    rdg, rdu = O.swiglu_backward(gu[:, :n], gu[:, n:], da16)
    g64, u64, da64 = (a.astype(np.float64) for a in (gu[:, :n], gu[:, n:], da16))
    act_mag = np.abs(g64 / (1.0 + np.exp(-g64)))
    for got_d, ref_d, terms in ((d[:, :n], rdg, np.abs(da64 * u64)), (d[:, n:], rdu, np.abs(da64 * act_mag))):
        got64, ref64 = got_d.astype(np.float64), ref_d.astype(np.float64)
        assert np.linalg.norm(got64 - ref64) <= 1e-3 * np.linalg.norm(ref64)
        assert np.percentile(_ulps(got_d, ref_d), 99.9) <= 2
        ulp = np.spacing(np.abs(ref_d).astype(np.float16)).astype(np.float64)
        excess = np.abs(got64 - ref64) - 4 * ulp - terms * 2.0 ** -8
        assert (excess <= 1e-5).all(), float(excess.max())
    _gate(np_of(dx)[rows], O.nf4_linear_dx(d[:, :n], wg) + O.nf4_linear_dx(d[:, n:], wu), "dx2")
    assert _lib.take_device_error(x.device) == 0


def test_fused_mlp_rejects_unsupported_shapes_before_launch():
    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels.mlp import nf4_swiglu_mlp
    gen = torch.Generator(device="cuda").manual_seed(1)
    gp, gs, _ = _weight(192, 128, gen)  # 192 is not a multiple of 128
    dp, ds, _ = _weight(128, 192, gen)
    a, b = _adapter(192, 128, 16, gen)
    ad, bd = _adapter(128, 192, 16, gen)
    x = torch.randn((4, 128), device="cuda", dtype=torch.float16)
    before = _lib.launch_count()
    with pytest.raises(ValueError):
        nf4_swiglu_mlp(x, (gp, gs, a, b), (gp, gs, a, b), (dp, ds, ad, bd))
    assert _lib.launch_count() == before
