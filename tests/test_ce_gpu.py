"""Fused linear cross-entropy against the reference's kernels and preregistered gates.

Gates from solution/tests/test_cross_entropy.py:30-35 (METRIC 2e-3, GRAD 1e-2 of
the ideal gradient norm, argmax agreement >= 0.999) and its edge cases
(all ignored, non-finite upstream on ignored rows, empty rows, tails, ties).
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import golden, np_of

pytestmark = pytest.mark.gpu

METRIC = dict(rtol=2e-3, atol=2e-3)
GRAD_RTOL = 1e-2
ARGMAX_AGREEMENT = 0.999


def _inputs(n, h, v, ignored="some", scale=1.0, seed=123, hidden_dtype=torch.float16):
    torch.manual_seed(seed)
    x = (torch.randn(n, h, device="cuda", dtype=hidden_dtype) * scale).requires_grad_()
    w = (torch.randn(v, h, device="cuda") / math.sqrt(h)).to(torch.float16)
    y = torch.randint(v, (n,), device="cuda")
    if ignored == "some":
        y[::3] = -100
    elif ignored == "all":
        y.fill_(-100)
    return x, w, y


def _compare(x, w, y, upstream):
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    loss, entropy, argmax, lse = fused_linear_cross_entropy(x, w, y)
    rl, re, ra, rlse = O.ce_forward(np_of(x.detach()), np_of(w), np_of(y))
    for got, ref in ((loss, rl), (entropy, re), (lse, rlse)):
        assert got.dtype == torch.float32 and torch.isfinite(got).all()
        np.testing.assert_allclose(np_of(got), ref, **METRIC)
    assert (np_of(argmax) == ra).mean() >= ARGMAX_AGREEMENT
    assert torch.count_nonzero(loss[y == -100]).item() == 0
    assert loss.requires_grad and not entropy.requires_grad
    loss.backward(upstream)
    ideal = O.ce_backward_ideal(np_of(x.detach()), np_of(w), np_of(y), np_of(upstream))
    err = np.linalg.norm(np_of(x.grad).astype(np.float64) - ideal)
    assert err <= GRAD_RTOL * max(np.linalg.norm(ideal), 1e-30) + 1e-7, (err, np.linalg.norm(ideal))
    assert torch.count_nonzero(x.grad[y == -100]).item() == 0


def test_statistics_match_reference_kernel_golden():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    g = golden()
    hidden = torch.from_numpy(g["ce_hidden"]).cuda()
    weight = torch.from_numpy(g["ce_weight"]).cuda()
    targets = torch.from_numpy(g["ce_targets"]).cuda()
    loss, entropy, best, lse = fused_linear_cross_entropy(hidden, weight, targets)
    for got, key in ((loss, "ce_loss"), (entropy, "ce_entropy"), (lse, "ce_lse")):
        np.testing.assert_allclose(np_of(got), g[key], **METRIC)
    assert (np_of(best) == g["ce_best"]).mean() >= ARGMAX_AGREEMENT


@pytest.mark.parametrize("n,h,v,ignored,scale", [
    (77, 64, 1000, "some", 1.0),
    (1001, 96, 1000, "some", 1.0),
    (77, 64, 1000, "all", 1.0),
    (77, 64, 1000, "none", 20.0),
    (77, 80, 4103, "some", 1.0),
    (1, 33, 7, "none", 1.0),
    (300, 1536, 20000, "some", 1.0),
])
def test_forward_and_arbitrary_upstream(n, h, v, ignored, scale):
    x, w, y = _inputs(n, h, v, ignored, scale)
    _compare(x, w, y, torch.randn(n, device="cuda", dtype=torch.float32))


def test_fp32_hidden_returns_fp32_grad():
    x, w, y = _inputs(77, 64, 4103, hidden_dtype=torch.float32)
    _compare(x, w, y, torch.randn(77, device="cuda"))
    assert x.grad.dtype == torch.float32


@pytest.mark.parametrize("nonfinite", [float("inf"), -float("inf"), float("nan")])
def test_all_ignored_nonfinite_upstream_gives_zero_gradient(nonfinite):
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(6, 32, 1000, "all")
    loss = fused_linear_cross_entropy(x, w, y)[0]
    loss.backward(torch.full_like(loss, nonfinite))
    assert torch.isfinite(x.grad).all() and torch.count_nonzero(x.grad).item() == 0


def test_one_ignored_row_with_infinite_upstream_cannot_poison_valid_rows():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(6, 32, 1000, "none")
    y[2] = -100
    upstream = torch.randn(6, device="cuda")
    safe = upstream.clone()
    safe[2] = 0
    ideal = O.ce_backward_ideal(np_of(x.detach()), np_of(w), np_of(y), np_of(safe))
    upstream[2] = float("inf")
    fused_linear_cross_entropy(x, w, y)[0].backward(upstream)
    assert torch.isfinite(x.grad).all() and torch.count_nonzero(x.grad[2]).item() == 0
    assert np.linalg.norm(np_of(x.grad).astype(np.float64) - ideal) <= GRAD_RTOL * np.linalg.norm(ideal)


def test_logit_rounding_precedes_argmax():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x = torch.ones((1, 8), device="cuda", dtype=torch.float16)
    w = torch.zeros((2, 8), device="cuda", dtype=torch.float16)
    w[0, 0], w[0, 1] = 1.0, 0.0001
    w[1, 0], w[1, 1] = 1.0, 0.0002
    loss, entropy, argmax, lse = fused_linear_cross_entropy(x, w, torch.tensor([1], device="cuda"))
    assert argmax.item() == 0  # both logits round to 1.0 in fp16
    torch.testing.assert_close(loss, torch.full_like(loss, math.log(2)), rtol=1e-5, atol=1e-5)


def test_ties_pick_first_argmax_and_repeat_calls_agree():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(77, 64, 4103)
    w.zero_()
    first = fused_linear_cross_entropy(x, w, y)
    second = fused_linear_cross_entropy(x, w, y)
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    assert torch.count_nonzero(first[2]).item() == 0
    torch.testing.assert_close(first[1], torch.full_like(first[1], math.log(4103)), **METRIC)


def test_empty_rows():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(0, 32, 1000)
    outputs = fused_linear_cross_entropy(x, w, y)
    assert all(o.shape == (0,) for o in outputs)
    outputs[0].sum().backward()
    assert x.grad.shape == x.shape


def test_target_outside_vocabulary_raises():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(4, 32, 100)
    y[1] = 100
    with pytest.raises(ValueError, match="outside"):
        fused_linear_cross_entropy(x, w, y)


def test_trainable_weight_rejected():
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    x, w, y = _inputs(2, 32, 100)
    w.requires_grad_()
    with pytest.raises(ValueError, match="frozen"):
        fused_linear_cross_entropy(x, w, y)
