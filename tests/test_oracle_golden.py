"""The CPU oracle against the reference's own kernel outputs (golden fixtures).

tests/golden/make_golden.py produced the fixtures by running the reference's
@triton.jit kernels under the Triton interpreter; these tests pin the numpy
and C restatements in oracle/ to them before anything is compared against the oracle.
"""

import ctypes
import hashlib
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import golden, manifest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def c_oracle():
    lib_path = ROOT / "oracle" / "_build" / "libnf4_oracle.so"
    if not lib_path.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "-s"], check=True)
    lib = ctypes.CDLL(str(lib_path))
    lib.nf4_oracle_dequant_nested.argtypes = [ctypes.c_void_p] * 4 + [
        ctypes.c_float, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int]
    lib.nf4_oracle_dequant_flat.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64, ctypes.c_int]
    lib.nf4_oracle_f32_to_f16.argtypes = [ctypes.c_float]
    lib.nf4_oracle_f32_to_f16.restype = ctypes.c_uint16
    return lib


def _fixture_np(shape, offset):
    """The reference's deterministic decoder fixture (solution/tests/test_nf4_fast.py:96-110)."""
    n = math.prod(shape)
    blocks = (n + 63) // 64
    packed = (np.arange((n + 1) // 2) % 256).astype(np.uint8)
    qabs = (np.arange(blocks) % 256).astype(np.uint8)
    code = np.linspace(-1, 1, 256, dtype=np.float64).astype(np.float32)
    absmax2 = (1.125 + 0.375 * np.arange((blocks + 255) // 256)).astype(np.float32)
    return packed, qabs, absmax2, code, np.array([offset], np.float32), n


def _torch_linspace_code():
    # torch.linspace(-1, 1, 256) in fp32 (the fixture's exact code table).
    import torch
    return torch.linspace(-1, 1, 256, dtype=torch.float32).numpy()


@pytest.mark.parametrize("entry", manifest()["nf4_nested"],
                         ids=lambda e: f"{e['shape'][0]}x{e['shape'][1]}-{e['offset']}")
def test_nested_decoder_matches_reference(entry, c_oracle):
    packed, qabs, absmax2, _, off, n = _fixture_np(tuple(entry["shape"]), entry["offset"])
    code = _torch_linspace_code()
    out = O.nf4_dequant_nested(packed, qabs, absmax2, code, off, n)
    assert hashlib.sha256(out.view(np.uint16).tobytes()).hexdigest() == entry["sha256"]
    cout = np.empty(n, np.uint16)
    c_oracle.nf4_oracle_dequant_nested(packed.ctypes.data, qabs.ctypes.data, absmax2.ctypes.data,
                                       code.ctypes.data, float(off[0]), cout.ctypes.data, n, 4)
    assert hashlib.sha256(cout.tobytes()).hexdigest() == entry["sha256"]


@pytest.mark.parametrize("entry", manifest()["nf4_flat"], ids=lambda e: str(e["n"]))
def test_flat_decoder_matches_reference(entry, c_oracle):
    import torch
    n = entry["n"]
    packed = (np.arange((n + 1) // 2) % 256).astype(np.uint8)
    scales = torch.linspace(-2, 2, (n + 63) // 64, dtype=torch.float32).numpy()
    expected = golden()[entry["key"]]
    assert np.array_equal(O.nf4_dequant_flat(packed, scales, n).view(np.uint16), expected)
    cout = np.empty(n, np.uint16)
    c_oracle.nf4_oracle_dequant_flat(packed.ctypes.data, scales.ctypes.data, cout.ctypes.data, n, 2)
    assert np.array_equal(cout, expected)


@pytest.mark.parametrize("tag", manifest()["nf4_quantized"])
def test_quantized_weight_decode_matches_reference(tag):
    g = golden()
    n = g[tag + "_out"].size
    out = O.nf4_dequant_nested(g[tag + "_packed"], g[tag + "_qabs"], g[tag + "_absmax2"],
                               g[tag + "_code2"], g[tag + "_offset"], n)
    assert np.array_equal(out.view(np.uint16), g[tag + "_out"])


def test_f16_rounding_of_the_c_oracle(c_oracle):
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
                           np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, -6e-8, np.inf, -np.inf], np.float32)])
    got = np.array([c_oracle.nf4_oracle_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        expected = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, expected)


@pytest.mark.parametrize("tag", manifest()["lora"])
def test_lora_epilogue_matches_reference(tag):
    g = golden()
    out = O.lora_scale_add(g[tag + "_result"], g[tag + "_adapter"], 1.3, tag.endswith("_1"))
    assert out.dtype == g[tag + "_out"].dtype
    assert np.array_equal(out.view(np.uint8), g[tag + "_out"].view(np.uint8))
    grad = O.lora_scale_gradient(g[tag + "_grad"], g[tag + "_adapter"].dtype, 1.3)
    assert np.array_equal(grad.view(np.uint8), g[tag + "_dadapter"].view(np.uint8))


@pytest.mark.parametrize("tag", manifest()["add_rmsnorm"])
def test_add_rmsnorm_matches_reference(tag):
    g = golden()
    r, d, w = g[tag + "_r"], g[tag + "_d"], g[tag + "_w"]
    s, y, rstd = O.add_rmsnorm_forward(r, d, w, 1e-6)
    assert np.array_equal(s, g[tag + "_s"])
    np.testing.assert_allclose(y.astype(np.float64), g[tag + "_y"].astype(np.float64), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(rstd, g[tag + "_rstd"], rtol=1e-6)
    dr, dd = O.add_rmsnorm_backward(s, w, rstd, g[tag + "_gs"], g[tag + "_gy"], r.dtype, d.dtype)
    np.testing.assert_allclose(dr.astype(np.float64), g[tag + "_dr"].astype(np.float64), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(dd.astype(np.float64), g[tag + "_dd"].astype(np.float64), rtol=1e-5, atol=1e-5)


def test_cross_entropy_statistics_match_reference():
    g = golden()
    loss, ent, best, lse = O.ce_forward(g["ce_hidden"], g["ce_weight"], g["ce_targets"])
    np.testing.assert_allclose(loss, g["ce_loss"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(ent, g["ce_entropy"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse, g["ce_lse"], rtol=1e-5, atol=1e-5)
    assert np.array_equal(best, g["ce_best"])


def test_cross_entropy_derivative_matches_reference():
    """dz = (exp(z - lse) - onehot) * g / gain, zero when ignored (cross_entropy.py:108-122)."""
    g = golden()
    hidden, weight, targets = g["ce_hidden"], g["ce_weight"], g["ce_targets"]
    lse, grad = g["ce_lse"].astype(np.float64), g["ce_grad"].astype(np.float64)
    gain = np.maximum(np.abs(g["ce_grad"]), np.float32(1e-30)) / np.float32(1024.0)
    z = O.fp16_logits(hidden, weight).astype(np.float64)
    cols = np.arange(z.shape[1])
    onehot = (cols[None, :] == targets[:, None]).astype(np.float64)
    dz = (np.exp(z - lse[:, None]) - onehot) * grad[:, None] / gain[:, None].astype(np.float64)
    dz[targets == -100] = 0.0
    np.testing.assert_allclose(dz.astype(np.float16).astype(np.float64),
                               g["ce_dz"].astype(np.float64), rtol=2e-3, atol=2e-3)
