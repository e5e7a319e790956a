"""NF4 decode on the GPU: exact fp16 bits against the reference's own decoder.

The golden digests were produced by the reference's nf4_decode_kernel
(solution/kernels/nf4.py:41-59) under the Triton interpreter
(tests/golden/make_golden.py); the cases follow solution/tests/test_nf4.py and
solution/tests/test_nf4_fast.py.
"""

import copy
import hashlib
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import bits16, golden, manifest, oracle_dequant

pytestmark = pytest.mark.gpu


def _fixture(shape, offset):
    from soupsuck_b200.quantize import fixture_state
    packed, st = fixture_state(shape, offset, device="cuda")
    return packed, st


@pytest.mark.parametrize("entry", manifest()["nf4_nested"],
                         ids=lambda e: f"{e['shape'][0]}x{e['shape'][1]}-{e['offset']}")
def test_nested_bits_match_reference_goldens(entry):
    from soupsuck_b200.kernels import dequantize_nf4
    packed, st = _fixture(tuple(entry["shape"]), entry["offset"])
    out = dequantize_nf4(packed, st)
    if packed.shape[0] == 1:  # one packed byte: the reference returns the transposed view
        out = out.t()
    assert out.dtype == torch.float16 and tuple(out.shape) == tuple(entry["shape"])
    raw = bits16(out.contiguous()).reshape(-1)
    assert hashlib.sha256(raw.tobytes()).hexdigest() == entry["sha256"]
    if "key" in entry:
        assert np.array_equal(raw, golden()[entry["key"]])


@pytest.mark.parametrize("entry", manifest()["nf4_flat"], ids=lambda e: str(e["n"]))
def test_flat_signed_scales_and_unaligned_out(entry):
    from soupsuck_b200.kernels.nf4 import decode_flat_into
    n = entry["n"]
    packed, _ = _fixture((1, n), 0.0)
    blocks = (n + 63) // 64
    scales = torch.linspace(-2, 2, blocks, device="cuda", dtype=torch.float32)
    expected = golden()[entry["key"]]
    out = torch.empty((1, n), device="cuda", dtype=torch.float16)
    assert decode_flat_into(packed, scales, out).data_ptr() == out.data_ptr()
    assert np.array_equal(bits16(out).reshape(-1), expected)
    guarded = torch.full((n + 2,), 123.0, device="cuda", dtype=torch.float16)
    view = guarded[1:n + 1].view(1, n)  # contiguous but not vector-store aligned
    decode_flat_into(packed, scales, view)
    assert np.array_equal(bits16(view).reshape(-1), expected)
    assert guarded[0].item() == 123.0 and guarded[-1].item() == 123.0


@pytest.mark.parametrize("tag", manifest()["nf4_quantized"])
def test_quantized_weights_match_reference(tag):
    from soupsuck_b200.kernels import dequantize_nf4
    from soupsuck_b200.quantize import NestedState, QuantState
    g = golden()
    out_ref = g[tag + "_out"]
    shape = tuple(int(s) for s in tag.split("_")[1].split("x"))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = QuantState(absmax=dev(g[tag + "_qabs"]), shape=shape,
                    state2=NestedState(absmax=dev(g[tag + "_absmax2"]), code=dev(g[tag + "_code2"])),
                    offset=dev(g[tag + "_offset"]))
    packed = dev(g[tag + "_packed"]).view(-1, 1)
    out = dequantize_nf4(packed, st)
    assert np.array_equal(bits16(out).reshape(-1), out_ref)


@pytest.mark.parametrize("shape", [(1536, 1536), (8960, 1536), (1536, 8960), (256, 1536),
                                   (7, 13), (3, 65), (17, 127), (1, 1), (1, 3)])
def test_random_quantized_weights_match_oracle(shape):
    from soupsuck_b200.kernels import dequantize_nf4
    from soupsuck_b200.quantize import quantize_nf4
    torch.manual_seed(2026)
    w = torch.randn(shape, device="cuda", dtype=torch.float16)
    packed, st = quantize_nf4(w)
    out = dequantize_nf4(packed, st)
    assert np.array_equal(bits16(out), oracle_dequant(packed, st).view(np.uint16))


def test_zero_weight_sign_bits():
    from soupsuck_b200.kernels import dequantize_nf4
    from soupsuck_b200.quantize import quantize_nf4
    packed, st = quantize_nf4(torch.zeros((17, 127), device="cuda", dtype=torch.float16))
    # Force signed scales: negative code entries give -0.0 for the zero code.
    st.state2.code = torch.linspace(-1, 1, 256, device="cuda", dtype=torch.float32)
    out = dequantize_nf4(packed, st)
    assert np.array_equal(bits16(out), oracle_dequant(packed, st).view(np.uint16))


def test_packed_transpose_shim():
    from soupsuck_b200.kernels import dequantize_nf4
    packed, st = _fixture((256, 1536), 0.0625)
    expected = dequantize_nf4(packed, st)
    transposed = dequantize_nf4(packed.t(), st)
    assert transposed.shape == (1536, 256)
    assert torch.equal(transposed.contiguous().view(torch.int16), expected.t().contiguous().view(torch.int16))


def test_out_is_written_without_allocation(monkeypatch):
    from soupsuck_b200.kernels import dequantize_nf4
    packed, st = _fixture((256, 1536), 0.0625)
    expected = dequantize_nf4(packed, st)
    out = torch.empty_like(expected)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()

    def no_alloc(*args, **kwargs):
        raise AssertionError("out= allocated an extra tensor")
    monkeypatch.setattr(torch, "empty", no_alloc)
    monkeypatch.setattr(torch, "empty_like", no_alloc)
    assert dequantize_nf4(packed, st, out=out).data_ptr() == out.data_ptr()
    monkeypatch.undo()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    assert torch.equal(out.view(torch.int16), expected.view(torch.int16))


def test_unsupported_states_raise_before_launch():
    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels import dequantize_nf4
    packed, st = _fixture((17, 128), 0.0)
    before = _lib.launch_count()
    with pytest.raises(ValueError, match="fp16"):
        dequantize_nf4(packed, st, torch.float32)
    for field, value in (("quant_type", "fp4"), ("blocksize", 128), ("nested", False)):
        changed = copy.copy(st)
        setattr(changed, field, value)
        with pytest.raises(ValueError):
            dequantize_nf4(packed, changed)
    changed = copy.copy(st)
    changed.state2 = copy.copy(st.state2)
    changed.state2.blocksize = 64
    with pytest.raises(ValueError, match="state2"):
        dequantize_nf4(packed, changed)
    assert _lib.launch_count() == before
