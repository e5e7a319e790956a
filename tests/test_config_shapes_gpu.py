"""Parity at the benchmark configurations' own shapes.

The kernels run at full size, exactly as ``bench.py`` launches them; the float64
oracle checks a seeded subset of rows (every row of Y / dX / the CE outputs
depends only on its own input row, so a subset is an exact check of those rows).

* the seven Qwen2.5-1.5B projections at T = 3300 with LoRA r = 16,
  forward and dX, through ``nf4_lora_linear`` (gate/up forward: whole 256x256
  tiles; gate/up dX and down forward: stream-K over 140 k-blocks), against the
  oracle's decode of the same NF4 weight and the EXP-002 gate.
* fused linear CE at T = 3300, V = 151936, H = 1536, 63 % of the
  targets ignored (the backward walks 5 vocabulary chunks of 32768), and at
  T = 16384 (19 chunks of 8192), against the reference's chunked statistics
  and its ideal gradient (solution/kernels/cross_entropy.py:51-211,
  solution/tests/test_cross_entropy.py:30-35).
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of, oracle_dequant

pytestmark = pytest.mark.gpu

HIDDEN, INTER, KV, T = 1536, 8960, 256, 3300
PROJ = [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
        ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]


def _rows(t, count, seed):
    """First tile, last (ragged) tile and a seeded spread of rows in between."""
    rng = np.random.default_rng(seed)
    picked = set(range(0, min(t, 128), 7)) | set(range(max(t - 128, 0), t, 5))
    picked |= set(rng.choice(t, size=min(count, t), replace=False).tolist())
    return np.array(sorted(picked))


def _gate(actual_rows, expected_rows, what):
    ok, max_abs, rel = O.gemm_gate(actual_rows.astype(np.float64), expected_rows)
    assert ok, f"{what}: max abs err {max_abs:.3e}, rel-L2 {rel:.3e}"


@pytest.mark.parametrize("name,n,k", PROJ, ids=[p[0] for p in PROJ])
def test_layer_projection_t3300_forward_dx_lora(name, n, k):
    from soupsuck_b200.kernels import nf4_lora_linear
    from soupsuck_b200.quantize import quantize_nf4
    r, s = 16, 2.0
    g = torch.Generator(device="cuda").manual_seed(n * 7 + k)
    w = (torch.randn((n, k), device="cuda", generator=g) * 0.02).to(torch.float16)
    packed, st = quantize_nf4(w)
    w16 = oracle_dequant(packed, st)
    x = torch.randn((T, k), device="cuda", dtype=torch.float16, generator=g).requires_grad_()
    a = ((torch.rand((r, k), device="cuda", generator=g) * 2 - 1) / math.sqrt(k)).requires_grad_()
    b = (torch.randn((n, r), device="cuda", generator=g) * 0.01).requires_grad_()
    dy = torch.randn((T, n), device="cuda", dtype=torch.float16, generator=g)
    y = nf4_lora_linear(x, packed, st, a, b, s)
    y.backward(dy)
    torch.cuda.synchronize()
    rows = _rows(T, 192, seed=n + k)
    a16 = np_of(a.detach().half()).astype(np.float64)
    b16 = np_of(b.detach().half()).astype(np.float64)
    xr, dyr = np_of(x.detach())[rows], np_of(dy)[rows]
    _gate(np_of(y)[rows], O.nf4_linear_forward(xr, w16, a16, b16, s), f"{name} forward")
    _gate(np_of(x.grad)[rows], O.nf4_linear_dx(dyr, w16, a16, b16, s), f"{name} dX")
    da_ref, db_ref = O.lora_weight_grads(np_of(x.detach()), np_of(dy), a16, b16, s)
    for got, ref, what in ((a.grad, da_ref, "dA"), (b.grad, db_ref, "dB")):
        rel = np.linalg.norm(np_of(got).astype(np.float64) - ref) / np.linalg.norm(ref)
        assert rel < 2e-3, (name, what, rel)


METRIC = dict(rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("t,v,count", [(3300, 151936, 96), (16384, 151936, 64)],
                         ids=["configs3_t3300", "t16384_chunk8192"])
def test_cross_entropy_full_vocabulary(t, v, count):
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    h = HIDDEN
    g = torch.Generator(device="cuda").manual_seed(t)
    x = torch.randn((t, h), device="cuda", dtype=torch.float16, generator=g).requires_grad_()
    w = (torch.randn((v, h), device="cuda", generator=g) * 0.02).to(torch.float16)
    y = torch.randint(v, (t,), device="cuda", generator=g)
    y[torch.rand(t, device="cuda", generator=g) < 0.63] = -100
    upstream = torch.randn(t, device="cuda", dtype=torch.float32, generator=g)
    loss, entropy, argmax, lse = fused_linear_cross_entropy(x, w, y)
    loss.backward(upstream)
    torch.cuda.synchronize()

    rows = _rows(t, count, seed=t)
    xr, yr, wn = np_of(x.detach())[rows], np_of(y)[rows], np_of(w)
    rl, re, ra, rlse = O.ce_forward(xr, wn, yr)
    for got, ref in ((loss, rl), (entropy, re), (lse, rlse)):
        np.testing.assert_allclose(np_of(got)[rows], ref, **METRIC)
    got_arg = np_of(argmax)[rows]
    agree = got_arg == ra
    # A disagreement is allowed only on a near tie: the chosen column's fp16 logit
    # must be within one fp16 ulp of the row maximum.
    for i in np.nonzero(~agree)[0]:
        z = O.fp16_logits(xr[i:i + 1], wn[[got_arg[i], ra[i]]]).astype(np.float64)[0]
        assert z[0] >= z[1] - float(np.spacing(np.float16(abs(z[1])))), (rows[i], got_arg[i], ra[i], z)
    assert agree.mean() >= 0.98
    assert torch.count_nonzero(loss[y == -100]).item() == 0
    grad = np_of(x.grad)
    assert np.isfinite(grad).all()
    assert np.count_nonzero(grad[np_of(y) == -100]) == 0
    ideal = O.ce_backward_ideal(xr, wn, yr, np_of(upstream)[rows])
    err = np.linalg.norm(grad[rows].astype(np.float64) - ideal)
    assert err <= 1e-2 * max(np.linalg.norm(ideal), 1e-30) + 1e-7, (err, np.linalg.norm(ideal))
