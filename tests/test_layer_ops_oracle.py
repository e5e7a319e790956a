"""The oracle's RoPE and SwiGLU restatements against the reference's own kernels.

``tests/golden/golden_layer_ops.npz`` holds outputs of the reference's
``rope_pair_forward_kernel`` / ``rope_pair_backward_kernel`` and
``swiglu_tile_engine`` run under the Triton interpreter
(``tests/golden/make_golden_layer_ops.py``).  RoPE is elementwise with every
rounding explicit, so the oracle must match bit for bit.  SwiGLU uses exp();
the interpreter's numpy exp and the oracle's agree to the fp16 output in all
but rare ties, so at most one fp16 ulp is allowed there.
"""

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_layer_ops.npz"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_rope_oracle_matches_reference_kernels(g, case):
    p = lambda key: g[f"rope_{case}_{key}"]
    yq, yk = O.rope_forward(p("q"), p("k"), p("cos"), p("sin"))
    for got, ref in ((yq, p("yq")), (yk, p("yk"))):
        assert got.dtype == ref.dtype
        assert np.array_equal(got.view(np.uint8), ref.view(np.uint8))
    dq, dk = O.rope_backward(p("gq"), p("gk"), p("cos"), p("sin"), p("q").dtype, p("k").dtype)
    for got, ref in ((dq, p("dq")), (dk, p("dk"))):
        assert got.dtype == ref.dtype
        assert np.array_equal(got.view(np.uint8), ref.view(np.uint8))


def _ulps(a, b):
    a = a.astype(np.float16).view(np.int16).astype(np.int32)
    b = b.astype(np.float16).view(np.int16).astype(np.int32)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return np.abs(a - b)


@pytest.mark.parametrize("case", ["small", "wide"])
def test_swiglu_oracle_matches_reference_kernel(g, case):
    p = lambda key: g[f"swiglu_{case}_{key}"]
    act = O.swiglu_forward(p("gate"), p("up"))
    assert act.dtype == np.float16 and _ulps(act, p("act")).max() <= 1
    dg, du = O.swiglu_backward(p("gate"), p("up"), p("grad"))
    assert _ulps(dg, p("dgate")).max() <= 1
    assert _ulps(du, p("dup")).max() <= 1


@pytest.mark.parametrize("case", ["valid", "nonbinary", "leftpad", "labelpad", "empty"])
def test_unpad_oracle_matches_reference_metadata(g, case):
    p = lambda key: g[f"unpad_{case}_{key}"]
    got = O.unpad_lengths(p("mask"), p("labels"))
    ref = tuple(int(x) for x in p("lengths"))
    assert (got is None and ref == ()) or got == ref


def test_unpad_oracle_pack_scatter_and_float_mask(g):
    lengths = O.unpad_lengths(g["unpad_valid_mask"], g["unpad_valid_labels"])
    assert np.array_equal(O.unpad_indices(lengths, 5), g["unpad_valid_indices"])
    packed = O.unpad_pack(g["unpad_valid_x"], lengths)
    assert np.array_equal(packed, g["unpad_valid_packed"][0])  # the reference packs to [1, T, ...]
    assert np.array_equal(O.unpad_scatter(packed, lengths, 5), g["unpad_valid_scattered"])
    assert O.unpad_lengths(g["unpad_valid_mask"].astype(np.float32)) == tuple(g["unpad_float_lengths"])


def test_host_right_padding_check_matches_oracle(g):
    from soupsuck_b200.unpad import right_padding_lengths
    for case in ("valid", "nonbinary", "leftpad", "empty"):
        mask = g[f"unpad_{case}_mask"]
        assert right_padding_lengths(mask.tolist()) == O.unpad_lengths(mask)
