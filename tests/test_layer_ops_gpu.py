"""RoPE and element-wise SwiGLU on the B200 against the reference's goldens, the
oracle and eager PyTorch (the semantics the reference's own tests pin:
solution/tests/test_rope.py:51-120, solution/tests/test_mlp.py:12).

RoPE is bit-exact (every rounding explicit); SwiGLU computes exp and the
reciprocal with the fast hardware forms (as the reference's tl.exp does), so
its fp16 outputs may differ from the interpreter's numpy exp by one fp16 ulp.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "golden_layer_ops.npz")


def _bits(t):
    t = t.detach().contiguous()
    return t.view(torch.int16 if t.dtype == torch.float16 else torch.int32)


def _eager(q, k, cos, sin):
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)

    def rotate(x):
        h = x.shape[-1] // 2
        return torch.cat((-x[..., h:], x[..., :h]), dim=-1)
    return q * c + rotate(q) * s, k * c + rotate(k) * s


def _layout(arr, transposed):
    t = torch.from_numpy(arr).cuda()
    return t.transpose(1, 2).contiguous().transpose(1, 2) if transposed else t


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_rope_matches_reference_golden_bits(case):
    from soupsuck_b200.kernels.rope import fused_rope
    p = lambda key: GOLDEN[f"rope_{case}_{key}"]
    transposed = bool(p("meta")[6])
    q, k = _layout(p("q"), transposed), _layout(p("k"), transposed)
    cos, sin = torch.from_numpy(p("cos")).cuda(), torch.from_numpy(p("sin")).cuda()
    q.requires_grad_()
    k.requires_grad_()
    yq, yk = fused_rope(q, k, cos, sin)
    assert np.array_equal(np_of(yq).view(np.uint8), p("yq").view(np.uint8))
    assert np.array_equal(np_of(yk).view(np.uint8), p("yk").view(np.uint8))
    torch.autograd.backward([yq, yk], [torch.from_numpy(p("gq")).cuda(), torch.from_numpy(p("gk")).cuda()])
    assert np.array_equal(np_of(q.grad).view(np.uint8), p("dq").view(np.uint8))
    assert np.array_equal(np_of(k.grad).view(np.uint8), p("dk").view(np.uint8))


@pytest.mark.parametrize("shape", [(4, 12, 2, 512, 128, 1, True), (3, 5, 2, 17, 66, 3, True),
                                   (1, 3, 1, 7, 10, 1, False)])
@pytest.mark.parametrize("dtypes", [("float16", "float16", "float16"), ("float16", "float16", "float32"),
                                    ("float32", "float32", "float32"), ("float32", "float16", "float16")])
def test_rope_forward_bits_and_gradients_vs_eager(shape, dtypes):
    from soupsuck_b200.kernels.rope import fused_rope
    torch.manual_seed(347)
    batch, hq, hk, seq, dim, cb, transposed = shape
    qt, kt, ct = (getattr(torch, name) for name in dtypes)

    def tensor(heads, dtype):
        if transposed:
            return torch.randn(batch, seq, heads, dim, device="cuda", dtype=dtype).transpose(1, 2).detach().requires_grad_()
        return torch.randn(batch, heads, seq, dim, device="cuda", dtype=dtype, requires_grad=True)
    q, k = tensor(hq, qt), tensor(hk, kt)
    qr, kr = q.detach().clone().requires_grad_(), k.detach().clone().requires_grad_()
    cos = torch.randn(cb, seq, dim, device="cuda", dtype=ct)
    sin = torch.randn_like(cos)
    got, ref = fused_rope(q, k, cos, sin), _eager(qr, kr, cos, sin)
    for a, b in zip(got, ref):
        assert a.dtype == b.dtype and torch.equal(_bits(a), _bits(b))
    grads = [torch.randn_like(o) for o in got]
    torch.autograd.backward(got, grads)
    torch.autograd.backward(ref, grads)
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad)):
        tol = dict(rtol=2e-3, atol=2e-3) if a.dtype == torch.float16 else dict(rtol=2e-6, atol=2e-6)
        torch.testing.assert_close(a, b, **tol)
    # the oracle restates the reference kernel's adjoint bit for bit
    dq, dk = O.rope_backward(np_of(grads[0]), np_of(grads[1]), np_of(cos), np_of(sin),
                             np_of(q).dtype, np_of(k).dtype)
    assert np.array_equal(np_of(q.grad).view(np.uint8), dq.view(np.uint8))
    assert np.array_equal(np_of(k.grad).view(np.uint8), dk.view(np.uint8))


def test_rope_broadcast_strided_cos_and_optional_gradient():
    from soupsuck_b200.kernels.rope import fused_rope
    q = torch.randn(2, 3, 13, 128, device="cuda", requires_grad=True)
    k = torch.randn(2, 1, 13, 128, device="cuda", dtype=torch.float16, requires_grad=True)
    cos = torch.randn(1, 26, 128, device="cuda")[:, ::2].expand(2, -1, -1)
    sin = torch.randn(1, 13, 128, device="cuda").expand(2, -1, -1)
    got, ref = fused_rope(q, k, cos, sin), _eager(q.detach(), k.detach(), cos, sin)
    for a, b in zip(got, ref):
        assert torch.equal(_bits(a), _bits(b))
    for seq in (0, 7):
        q = torch.randn(2, 3, seq, 128, device="cuda")
        k = torch.randn(2, 1, seq, 128, device="cuda", requires_grad=True)
        c, s = torch.ones(1, seq, 128, device="cuda"), torch.zeros(1, seq, 128, device="cuda")
        qo, ko = fused_rope(q, k, c, s)
        assert not qo.requires_grad and ko.requires_grad
        ko.sum().backward()
        torch.testing.assert_close(k.grad, torch.ones_like(k), rtol=0, atol=0)


def test_rope_rejects_unsupported_before_launch():
    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels.rope import fused_rope
    q = torch.randn(1, 2, 4, 7, device="cuda")
    c = torch.randn(1, 4, 7, device="cuda")
    before = _lib.launch_count()
    with pytest.raises(ValueError):
        fused_rope(q, q, c, c)  # odd head dimension
    with pytest.raises(ValueError):
        fused_rope(q.cpu(), q.cpu(), c.cpu(), c.cpu())
    assert _lib.launch_count() == before


def _ulps(a, b):
    a = a.astype(np.float16).view(np.int16).astype(np.int32)
    b = b.astype(np.float16).view(np.int16).astype(np.int32)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return np.abs(a - b)


def _check_dgate(got, ref, da, u):
    """dgate's factor sigmoid(g)(1 + g(1 - sigmoid(g))) cancels near g = -1.28; there a
    tiny result carries the fp32 error of its O(|da u|) terms.  One fp16 ulp of the
    result plus 2^-12 |da u|."""
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    bound = ulp + np.abs(da.astype(np.float64) * u.astype(np.float64)) * 2.0 ** -12 + 1e-7
    assert (err <= bound).all(), float((err - bound).max())


@pytest.mark.parametrize("case", ["small", "wide"])
def test_swiglu_elementwise_matches_reference_golden(case):
    from soupsuck_b200.kernels.mlp import swiglu_fused_backward, swiglu_fused_forward
    p = lambda key: GOLDEN[f"swiglu_{case}_{key}"]
    g, u, da = (torch.from_numpy(p(k)).cuda() for k in ("gate", "up", "grad"))
    act = swiglu_fused_forward(g, u)
    assert _ulps(np_of(act), p("act")).max() <= 1
    dg, du = swiglu_fused_backward(g, u, da)
    _check_dgate(np_of(dg), p("dgate"), p("grad"), p("up"))
    assert _ulps(np_of(du), p("dup")).max() <= 1


def test_swiglu_elementwise_strided_rows_and_odd_width():
    from soupsuck_b200.kernels.mlp import swiglu_fused_backward, swiglu_fused_forward
    torch.manual_seed(3)
    base = torch.randn(33, 2 * 131, device="cuda").half()
    g, u = base[:, :131], base[:, 131:]
    act = swiglu_fused_forward(g, u)
    ref = O.swiglu_forward(np_of(g), np_of(u))
    assert _ulps(np_of(act), ref).max() <= 1
    da = torch.randn(33, 131, device="cuda").half()
    dg, du = swiglu_fused_backward(g, u, da)
    rdg, rdu = O.swiglu_backward(np_of(g), np_of(u), np_of(da))
    _check_dgate(np_of(dg), rdg, np_of(da), np_of(u))
    assert _ulps(np_of(du), rdu).max() <= 1
