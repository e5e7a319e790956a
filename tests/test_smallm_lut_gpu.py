"""The small-M (M <= 16) NF4 forward and dX kernels against the float64 product of the decoded weight.

nf4_lut.cuh in its exact mode (the default) expands every packed word through the
block's fp16(NF4[code] * scale) table, the reference decoder's values; in its
lookup mode (SB_SMALLM=lut) it multiplies fp16(alpha * NF4[code]) and applies each
64-block's scale in fp32, a different weight rounding; the mma.sync kernel
(SB_SMALLM=mma, nf4_smallm.cuh) multiplies the decoded weight tile.  All must
pass the GEMM gate of test_gemm_gpu (|a - e| <= 2e-3 + 2e-3 |e|, rel-L2 <= 1e-3)
against the exact product of the reference decoder's fp16 weight, across the
work splits the lookup kernel plans: one or several cluster ranks along the
reduction, 8 or 16 token columns, ragged weight rows, LoRA and bias.
"""

import math
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of, oracle_dequant

pytestmark = pytest.mark.gpu


@pytest.fixture
def kernel():
    saved = os.environ.get("SB_SMALLM")

    def set_(name):
        os.environ["SB_SMALLM"] = name

    yield set_
    if saved is None:
        os.environ.pop("SB_SMALLM", None)
    else:
        os.environ["SB_SMALLM"] = saved


def _weight(n, k, seed):
    from soupsuck_b200.quantize import quantize_nf4
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn((n, k), device="cuda", generator=g) * 0.02).to(torch.float16)
    packed, st = quantize_nf4(w)
    return packed, st, oracle_dequant(packed, st)


def _gate(actual, expected):
    ok, max_abs, rel = O.gemm_gate(np_of(actual).astype(np.float64), expected)
    assert ok, f"max abs err {max_abs:.3e}, rel-L2 {rel:.3e}"


@pytest.mark.parametrize("name", ["exact", "lut", "mma"])
@pytest.mark.parametrize("m,n,k", [(1, 18944, 3584), (8, 3584, 3584), (9, 512, 3584), (16, 1536, 8960),
                                   (4, 3584, 18944), (2, 200, 128), (13, 48, 64), (16, 4096, 2048)])
def test_small_m_forward_kernels(kernel, name, m, n, k):
    from soupsuck_b200.kernels import nf4_matmul
    kernel(name)
    packed, st, w16 = _weight(n, k, seed=m * 31 + n + k)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = nf4_matmul(x, packed, st)
    _gate(y, O.nf4_linear_forward(np_of(x), w16))
    # A second call on the same inputs gives the same bits (fixed reduction order).
    assert torch.equal(y, nf4_matmul(x, packed, st))


@pytest.mark.parametrize("name", ["exact", "lut", "mma"])
@pytest.mark.parametrize("m,r", [(1, 16), (12, 64), (7, 8)])
def test_small_m_forward_lora_bias(kernel, name, m, r):
    from soupsuck_b200.kernels.nf4_gemm import nf4_linear_raw
    kernel(name)
    n, k = 1536, 3584
    packed, st, w16 = _weight(n, k, seed=r + 100 * m)
    torch.manual_seed(m + r)
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    za = (torch.randn((m, r), device="cuda") * 0.5).half()
    lb = (torch.randn((n, r), device="cuda") * 0.05).half()
    bias = torch.randn(n, device="cuda", dtype=torch.float16)
    y = nf4_linear_raw(x, packed, st, bias=bias, lora_a=za, lora_b=lb)
    exp = O.nf4_linear_forward(np_of(x), w16) + np_of(za).astype(np.float64) @ np_of(lb).astype(np.float64).T
    _gate(y, exp + np_of(bias).astype(np.float64))


@pytest.mark.parametrize("name", ["exact", "mma"])
@pytest.mark.parametrize("m,n,k", [(1, 18944, 3584), (1, 3584, 18944), (8, 3584, 3584), (9, 512, 3584),
                                   (16, 1536, 8960), (2, 200, 128), (13, 48, 64), (16, 8, 4096),
                                   (5, 104, 192)])
def test_small_m_dx_kernels(kernel, name, m, n, k):
    """dX = dY . deq(W): the warp-staged kernel (default) and the decode-to-shared one
    (SB_SMALLM=mma), over one or several cluster ranks, row runs that end inside a
    warp step (n not a multiple of 32) and 8 or 16 token columns."""
    from soupsuck_b200.kernels import nf4_matmul
    kernel(name)
    packed, st, w16 = _weight(n, k, seed=m * 17 + n + k)
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    dx = nf4_matmul(dy, packed, st, transpose=True)
    _gate(dx, O.nf4_linear_dx(np_of(dy), w16))
    assert torch.equal(dx, nf4_matmul(dy, packed, st, transpose=True))


@pytest.mark.parametrize("name", ["exact", "mma"])
@pytest.mark.parametrize("m,r", [(1, 16), (12, 64), (7, 8)])
def test_small_m_dx_lora(kernel, name, m, r):
    from soupsuck_b200.kernels.nf4_gemm import nf4_linear_raw
    kernel(name)
    n, k = 1536, 3584
    packed, st, w16 = _weight(n, k, seed=r + 50 * m)
    torch.manual_seed(m * r)
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    u = (torch.randn((m, r), device="cuda") * 0.5).half()
    at = (torch.randn((k, r), device="cuda") * 0.05).half()
    dx = nf4_linear_raw(dy, packed, st, transpose=True, lora_a=u, lora_b=at)
    exp = O.nf4_linear_dx(np_of(dy), w16) + np_of(u).astype(np.float64) @ np_of(at).astype(np.float64).T
    _gate(dx, exp)


def test_small_m_no_device_errors():
    from soupsuck_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
