"""Fused NF4 dequant -> tcgen05 GEMM (+ LoRA) against the float64 oracle.

Gate (fixed in advance, the reference's EXP-002 gate, experiments/reports/EXP-002.md:57-72):
elementwise |a - e| <= 2e-3 + 2e-3 |e|, finite, relative L2 <= 1e-3, where e is
the exact product of the same fp16 operands (the decoded weight is bit-exact,
so only accumulation order and the final fp16 rounding differ).
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of, oracle_dequant

pytestmark = pytest.mark.gpu


def _weight(n, k, seed=0, std=0.02):
    from soupsuck_b200.quantize import quantize_nf4
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn((n, k), device="cuda", generator=g) * std).to(torch.float16)
    packed, st = quantize_nf4(w)
    return packed, st, oracle_dequant(packed, st)


def _gate(actual, expected):
    ok, max_abs, rel = O.gemm_gate(np_of(actual).astype(np.float64), expected)
    assert ok, f"max abs err {max_abs:.3e}, rel-L2 {rel:.3e}"


SHAPES = [
    (827, 8960, 1536),
    (1, 1536, 1536),
    (16, 256, 1536),
    (300, 1536, 8960),
    (257, 384, 640),
    (64, 512, 256),
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_forward_matches_dequant_matmul(m, n, k):
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, w16 = _weight(n, k, seed=m + n)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = nf4_matmul(x, packed, st)
    _gate(y, O.nf4_linear_forward(np_of(x), w16))


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_dx_matches_dequant_matmul(m, n, k):
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, w16 = _weight(n, k, seed=m + k)
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    dx = nf4_matmul(dy, packed, st, transpose=True)
    _gate(dx, O.nf4_linear_dx(np_of(dy), w16))


def test_forward_bias():
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, w16 = _weight(384, 512, seed=3)
    x = torch.randn((200, 512), device="cuda", dtype=torch.float16)
    bias = torch.randn(384, device="cuda", dtype=torch.float16)
    _gate(nf4_matmul(x, packed, st, bias=bias), O.nf4_linear_forward(np_of(x), w16, bias=np_of(bias)))


@pytest.mark.parametrize("m,n,k", [(7, 13, 17), (33, 65, 96), (5, 127, 130)])
def test_odd_shapes_use_fallback_and_match(m, n, k):
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, w16 = _weight(n, k, seed=11)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    _gate(nf4_matmul(x, packed, st), O.nf4_linear_forward(np_of(x), w16))
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    _gate(nf4_matmul(dy, packed, st, transpose=True), O.nf4_linear_dx(np_of(dy), w16))


@pytest.mark.parametrize("m,n,k,r", [(827, 8960, 1536, 16), (3300, 256, 1536, 16), (100, 640, 384, 8),
                                     (130, 256, 512, 32), (70, 128, 192, 64)])
def test_lora_linear_forward_backward(m, n, k, r):
    from soupsuck_b200.kernels import nf4_lora_linear
    packed, st, w16 = _weight(n, k, seed=r)
    torch.manual_seed(r)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16, requires_grad=True)
    a = ((torch.rand((r, k), device="cuda") * 2 - 1) / math.sqrt(k)).requires_grad_()
    b = (torch.randn((n, r), device="cuda") * 0.01).requires_grad_()
    s = 2.0
    y = nf4_lora_linear(x, packed, st, a, b, s)
    a16 = np_of(a.detach().half()).astype(np.float64)
    b16 = np_of(b.detach().half()).astype(np.float64)
    _gate(y, O.nf4_linear_forward(np_of(x), w16, a16, b16, s))
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    y.backward(dy)
    _gate(x.grad, O.nf4_linear_dx(np_of(dy), w16, a16, b16, s))
    da_ref, db_ref = O.lora_weight_grads(np_of(x.detach()), np_of(dy), a16, b16, s)
    for got, ref in ((a.grad, da_ref), (b.grad, db_ref)):
        assert got.dtype == torch.float32
        rel = np.linalg.norm(np_of(got).astype(np.float64) - ref) / np.linalg.norm(ref)
        assert rel < 2e-3, rel


def test_empty_rows():
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, _ = _weight(256, 512)
    x = torch.empty((0, 512), device="cuda", dtype=torch.float16)
    assert nf4_matmul(x, packed, st).shape == (0, 256)


def test_no_device_timeouts_recorded():
    from soupsuck_b200 import _lib
    assert _lib.take_device_error() == 0


@pytest.mark.parametrize("m,n,k", [(1, 3584, 3584), (5, 512, 3584), (16, 18944, 3584), (16, 3584, 18944),
                                   (3, 200, 128), (16, 1536, 1536)])
def test_small_m_forward_and_dx(m, n, k):
    """M <= 16 rows take the streaming small-M kernel (fp32 partials over reduction slices)."""
    from soupsuck_b200.kernels import nf4_matmul
    packed, st, w16 = _weight(n, k, seed=m + 7)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    _gate(nf4_matmul(x, packed, st), O.nf4_linear_forward(np_of(x), w16))
    if n % 8 == 0:
        dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
        _gate(nf4_matmul(dy, packed, st, transpose=True), O.nf4_linear_dx(np_of(dy), w16))


@pytest.mark.parametrize("m,r", [(1, 16), (16, 64), (7, 8)])
def test_small_m_lora_and_bias(m, r):
    from soupsuck_b200.kernels import nf4_lora_linear
    n, k = 512, 1536
    packed, st, w16 = _weight(n, k, seed=r)
    torch.manual_seed(m)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16, requires_grad=True)
    a = ((torch.rand((r, k), device="cuda") * 2 - 1) / math.sqrt(k)).requires_grad_()
    b = (torch.randn((n, r), device="cuda") * 0.01).requires_grad_()
    bias = torch.randn(n, device="cuda", dtype=torch.float16)
    y = nf4_lora_linear(x, packed, st, a, b, 2.0, bias=bias)
    a16 = np_of(a.detach().half()).astype(np.float64)
    b16 = np_of(b.detach().half()).astype(np.float64)
    _gate(y, O.nf4_linear_forward(np_of(x), w16, a16, b16, 2.0, bias=np_of(bias)))
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    y.backward(dy)
    _gate(x.grad, O.nf4_linear_dx(np_of(dy), w16, a16, b16, 2.0))
