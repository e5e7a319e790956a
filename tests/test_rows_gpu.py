"""LoRA epilogue, add-RMSNorm and RMSNorm kernels against the reference goldens and oracle.

Tolerances follow solution/tests/test_add_rmsnorm.py:16-22 (fp32 1e-5, fp16 2e-3)
and the exactness of solution/tests/test_lora.py:15-49.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import golden, manifest, np_of

pytestmark = pytest.mark.gpu

FP32_TOL = dict(rtol=1e-5, atol=1e-5)
FP16_TOL = dict(rtol=2e-3, atol=2e-3)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("tag", manifest()["lora"])
def test_lora_epilogue_bit_exact_with_reference(tag):
    from soupsuck_b200.kernels import lora_epilogue
    g = golden()
    result = _cuda(g[tag + "_result"]).requires_grad_()
    adapter = _cuda(g[tag + "_adapter"]).requires_grad_()
    out = lora_epilogue(result, adapter, 1.3, cast_to_result=tag.endswith("_1"))
    assert np.array_equal(np_of(out).view(np.uint8), g[tag + "_out"].view(np.uint8))
    out.backward(_cuda(g[tag + "_grad"]))
    assert np.array_equal(np_of(adapter.grad).view(np.uint8), g[tag + "_dadapter"].view(np.uint8))


def test_lora_epilogue_rounds_before_add():
    from soupsuck_b200.kernels import lora_epilogue
    adapter = torch.linspace(-2, 2, 2049, device="cuda", dtype=torch.float16)
    result = -(adapter * 1.3)
    assert torch.count_nonzero(lora_epilogue(result, adapter, 1.3)) == 0


@pytest.mark.parametrize("tag", manifest()["add_rmsnorm"])
def test_add_rmsnorm_matches_reference_kernel(tag):
    from soupsuck_b200.kernels import add_rms_norm
    g = golden()
    r, d, w = (_cuda(g[tag + k]) for k in ("_r", "_d", "_w"))
    r.requires_grad_(); d.requires_grad_()
    s, y = add_rms_norm(r, d, w, 1e-6)
    assert np.array_equal(np_of(s), g[tag + "_s"])  # the residual sum is exact
    tol = FP32_TOL if y.dtype == torch.float32 else FP16_TOL
    np.testing.assert_allclose(np_of(y).astype(np.float64), g[tag + "_y"].astype(np.float64), **tol)
    torch.autograd.backward((s, y), (_cuda(g[tag + "_gs"]), _cuda(g[tag + "_gy"])))
    for got, key, dt in ((r.grad, "_dr", r.dtype), (d.grad, "_dd", d.dtype)):
        assert got.dtype == dt
        t = FP32_TOL if dt == torch.float32 else FP16_TOL
        np.testing.assert_allclose(np_of(got).astype(np.float64), g[tag + key].astype(np.float64), **t)


@pytest.mark.parametrize("rows,h", [(3300, 1536), (5, 7), (1, 4096), (0, 1536)])
@pytest.mark.parametrize("out_dtype", [None, torch.float16])
def test_add_rmsnorm_vs_oracle(rows, h, out_dtype):
    from soupsuck_b200.kernels import add_rms_norm
    torch.manual_seed(rows + h)
    r = torch.randn(rows, h, device="cuda", dtype=torch.float16, requires_grad=True)
    d = torch.randn(rows, h, device="cuda", dtype=torch.float16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(h, device="cuda")).to(torch.float16).requires_grad_()
    s, y = add_rms_norm(r, d, w, 1e-6, out_dtype)
    es, ey, erstd = O.add_rmsnorm_forward(np_of(r), np_of(d), np_of(w), 1e-6,
                                          None if out_dtype is None else np.float16)
    assert np.array_equal(np_of(s), es)
    np.testing.assert_allclose(np_of(y).astype(np.float64), ey.astype(np.float64), **FP16_TOL)
    gs, gy = torch.randn_like(s), torch.randn_like(y)
    torch.autograd.backward((s, y), (gs, gy))
    dr, dd = O.add_rmsnorm_backward(es, np_of(w), erstd, np_of(gs), np_of(gy), np.float16, np.float16)
    np.testing.assert_allclose(np_of(r.grad).astype(np.float64), dr.astype(np.float64), **FP16_TOL)
    np.testing.assert_allclose(np_of(d.grad).astype(np.float64), dd.astype(np.float64), **FP16_TOL)
    if rows:
        dw = O.rmsnorm_weight_grad(es, erstd, np_of(gy), True)
        np.testing.assert_allclose(np_of(w.grad).astype(np.float64), dw.astype(np.float64),
                                   rtol=2e-3, atol=2e-3 * max(1.0, float(np.abs(dw).max())))


def test_add_rmsnorm_one_output_without_upstream():
    from soupsuck_b200.kernels import add_rms_norm
    r = torch.randn(9, 64, device="cuda", requires_grad=True)
    d = torch.randn(9, 64, device="cuda", dtype=torch.float16, requires_grad=True)
    w = torch.randn(64, device="cuda")
    s, y = add_rms_norm(r, d, w, 1e-6)
    y.sum().backward()
    es, _, erstd = O.add_rmsnorm_forward(np_of(r), np_of(d), np_of(w), 1e-6)
    dr, _ = O.add_rmsnorm_backward(es, np_of(w), erstd, None, np.ones((9, 64), np.float32),
                                   np.float32, np.float16)
    np.testing.assert_allclose(np_of(r.grad), dr, **FP32_TOL)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_rms_norm_vs_oracle(dtype):
    from soupsuck_b200.kernels import rms_norm
    torch.manual_seed(7)
    x = torch.randn(130, 1536, device="cuda", dtype=dtype, requires_grad=True)
    w = (1 + 0.1 * torch.randn(1536, device="cuda")).requires_grad_()
    y = rms_norm(x, w, 1e-6)
    ey, erstd = O.rmsnorm_forward(np_of(x), np_of(w), 1e-6)
    tol = FP32_TOL if dtype == torch.float32 else FP16_TOL
    np.testing.assert_allclose(np_of(y).astype(np.float64), ey.astype(np.float64), **tol)
    g = torch.randn_like(y)
    y.backward(g)
    edx = O.rmsnorm_input_grad(np_of(x), np_of(w), erstd, np_of(g))
    np.testing.assert_allclose(np_of(x.grad).astype(np.float64), edx.astype(np.float64), **tol)


def test_invalid_inputs_raise():
    from soupsuck_b200.kernels import add_rms_norm, rms_norm
    x = torch.randn(4, 8, device="cuda")
    with pytest.raises(ValueError):
        add_rms_norm(x, x[:, :4], torch.ones(8, device="cuda"), 1e-6)
    with pytest.raises(ValueError):
        add_rms_norm(x, x, torch.ones(8, device="cuda"), 1e-6, torch.bfloat16)
    with pytest.raises(ValueError):
        rms_norm(x.t(), torch.ones(4, device="cuda"), 1e-6)
