"""Both tensor-core NF4 GEMM kernels -- the 2-SM pair kernel (cta_group::2, 256x256
tiles; the default) and the one-SM kernel (256x128 tiles) -- under both schedules
(whole tiles, stream-K), against a float64 product of the same fp16 operands.

The kernel is chosen per call by SB_PAIR (1 pair, 0 one-SM) and the schedule by
SB_STREAMK (0 whole tiles, 1 stream-K); both are read by the library on every call.
Gate: the GEMM gate of test_gemm_gpu (|a - e| <= 2e-3 + 2e-3 |e|, rel-L2 <= 1e-3).
"""

import ctypes
import os

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture
def env():
    saved = {k: os.environ.get(k) for k in ("SB_PAIR", "SB_STREAMK")}

    def set_(**kv):
        for k, v in kv.items():
            os.environ[k] = str(v)

    yield set_
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


def _case(m, n, k, dx, r, bias, seed):
    from soupsuck_b200.kernels import dequantize_nf4
    from soupsuck_b200.quantize import quantize_nf4
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn((n, k), device="cuda", generator=g) * 0.02).half()
    packed, st = quantize_nf4(w)
    w64 = dequantize_nf4(packed, st).double()
    width, red = (k, n) if dx else (n, k)
    a = torch.randn((m, red), device="cuda", dtype=torch.float16, generator=g)
    la = lb = bb = None
    ref = a.double() @ (w64 if dx else w64.t())
    if r:
        la = (torch.randn((m, r), device="cuda", generator=g) * 0.5).half()
        lb = (torch.randn((width, r), device="cuda", generator=g) * 0.05).half()
        ref += la.double() @ lb.double().t()
    if bias:
        bb = torch.randn(width, device="cuda", dtype=torch.float16, generator=g)
        ref += bb.double()
    return packed, st, a, la, lb, bb, ref


def _gate(out, ref):
    from soupsuck_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    o = out.double()
    assert torch.isfinite(o).all()
    bad = (o - ref).abs() > 2e-3 + 2e-3 * ref.abs()
    assert not bad.any(), f"{int(bad.sum())} elements outside the gate"
    rel = ((o - ref).norm() / ref.norm()).item()
    assert rel <= 1e-3, rel


SHAPES = [
    # m, n, k, dx, r, bias
    (256, 256, 64, False, 0, False),      # one pair tile, one k-step
    (300, 384, 640, False, 16, True),     # ragged rows and columns, LoRA, bias
    (513, 640, 1536, True, 32, False),    # dX (MN-major decode), ragged
    (1000, 1280, 4096, False, 64, False),
    (700, 4096, 1280, True, 16, False),
]


@pytest.mark.parametrize("pair", [1, 0])
@pytest.mark.parametrize("streamk", [0, 1])
@pytest.mark.parametrize("m,n,k,dx,r,bias", SHAPES)
def test_kernels_and_schedules_match(env, pair, streamk, m, n, k, dx, r, bias):
    from soupsuck_b200.kernels.nf4_gemm import nf4_linear_raw
    env(SB_PAIR=pair, SB_STREAMK=streamk)
    packed, st, a, la, lb, bb, ref = _case(m, n, k, dx, r, bias, seed=m + n + k)
    out = nf4_linear_raw(a, packed, st, transpose=dx, bias=bb, lora_a=la, lora_b=lb)
    _gate(out, ref)


@pytest.mark.parametrize("dx", [False, True])
def test_pair_kernel_unaligned_output_rows(env, dx):
    """An output pointer that is not 16-byte aligned takes the pair kernel's
    direct-store epilogue instead of the bulk tensor stores."""
    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels.nf4_gemm import _weight_struct, _workspace
    env(SB_PAIR=1, SB_STREAMK=0)
    m, n, k = 300, 512, 768
    packed, st, a, _, _, _, ref = _case(m, n, k, dx, 0, False, seed=5)
    width = k if dx else n
    buf = torch.zeros(m * width + 8, dtype=torch.float16, device="cuda")
    out_ptr = buf.data_ptr() + 2  # 2-byte aligned only
    w = _weight_struct(packed, st)
    ws, nbytes = _workspace(m, n, k, dx, a.device)
    stream = _lib.stream_of(a.device)
    if dx:
        _lib.call("sb_nf4_linear_dx", a.data_ptr(), m, ctypes.byref(w), None, None, 0, out_ptr,
                  _lib.ptr(ws), nbytes, stream)
    else:
        _lib.call("sb_nf4_linear_fwd", a.data_ptr(), m, ctypes.byref(w), None, None, None, 0, out_ptr,
                  _lib.ptr(ws), nbytes, stream)
    out = buf[1:1 + m * width].view(m, width)
    _gate(out, ref)
    assert buf[0].item() == 0 and (buf[1 + m * width:] == 0).all()  # nothing written outside
