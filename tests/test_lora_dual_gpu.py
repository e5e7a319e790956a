"""sb_lora_dual: U = Q.Bt^T and dB = s (Pt.Q)^T from one pass over Q, against float64.

The two products are the LoRA backward's reads of its upstream gradient
(solution/lora.py:161 under autograd: lora_B's input gradient dY.B and its weight
gradient (Z^T.dY)^T).  Gates: U is stored in fp16, so within one fp16 ulp of the
exact product plus the fp32 accumulation bound; dB is fp32, within 1e-4 of the
sum of |terms|.  The block-diagonal mode (two adapters side by side, the MLP's
gate/up pair) is checked against the dense product with zero off-diagonal
factor blocks, and its dB against the diagonal blocks.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import np_of

pytestmark = pytest.mark.gpu


def _round16(m):
    return (m + 15) // 16 * 16


def _inputs(m, w, r, wsplit, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((m, w), device="cuda", dtype=torch.float16, generator=gen)
    ldp = _round16(m)
    pt = torch.zeros((r, ldp), device="cuda", dtype=torch.float16)
    pt[:, :m] = torch.randn((r, m), device="cuda", generator=gen).half()
    bt = (torch.randn((r, w), device="cuda", generator=gen) * 0.05).half()
    if wsplit:
        h = r // 2
        bt[:h, wsplit:] = 0
        bt[h:, :wsplit] = 0
    return q, pt, bt


def _run(q, pt, bt, r, wsplit, s, db_dtype=torch.float32):
    from soupsuck_b200 import _lib
    m, w = q.shape
    rh = r // 2 if wsplit else r
    rows = torch.full((m, r), float("nan"), device="cuda", dtype=torch.float16)
    ldt = _round16(m)
    tr = torch.full((r, ldt), float("nan"), device="cuda", dtype=torch.float16)
    db = torch.full((w, rh), float("nan"), device="cuda", dtype=db_dtype)
    nbytes = _lib.query("sb_lora_dual_workspace_bytes", m, w, r, wsplit)
    ws = torch.empty(max(nbytes, 1), device="cuda", dtype=torch.uint8)
    _lib.call("sb_lora_dual", q.data_ptr(), m, w, pt.data_ptr(), pt.shape[1], bt.data_ptr(), r, wsplit, s, 1,
              db.data_ptr(), _lib.dtype_code(db_dtype), s, rows.data_ptr(), r, s, tr.data_ptr(), ldt,
              ws.data_ptr(), nbytes, _lib.stream_of(q.device))
    torch.cuda.synchronize()
    assert _lib.take_device_error(q.device) == 0
    return rows, tr, db


def _check_u(rows, tr, q64, bt64, s, m):
    exact = s * (q64 @ bt64.T)
    bound = s * (np.abs(q64) @ np.abs(bt64).T) * 2.0 ** -20
    got = np_of(rows).astype(np.float64)
    ulp = np.spacing(np.abs(exact).astype(np.float16)).astype(np.float64)
    assert (np.abs(got - exact) <= ulp + bound).all(), float((np.abs(got - exact) - ulp - bound).max())
    t = np_of(tr)
    assert np.array_equal(t[:, :m], np_of(rows).T)
    assert (t[:, m:] == 0).all()


@pytest.mark.parametrize("m,w,r", [(300, 1536, 16), (3300, 1536, 16), (77, 256, 32), (1, 1536, 16),
                                   (33, 8960, 16), (3300, 8960, 32)])
def test_dual_dense_matches_float64(m, w, r):
    s = 2.0
    q, pt, bt = _inputs(m, w, r, 0, seed=m + w + r)
    rows, tr, db = _run(q, pt, bt, r, 0, s)
    q64, p64, b64 = (np_of(t).astype(np.float64) for t in (q, pt[:, :m], bt))
    _check_u(rows, tr, q64, b64, s, m)
    exact = s * (p64 @ q64).T
    bound = s * (np.abs(p64) @ np.abs(q64)).T * 1e-4 + 1e-12
    assert (np.abs(np_of(db).astype(np.float64) - exact) <= bound).all()


@pytest.mark.parametrize("m,n,r", [(3300, 8960, 32), (300, 1024, 32), (45, 512, 64)])
def test_dual_block_diagonal_pair(m, n, r):
    """Columns [0, n) pair with rows [0, r/2), columns [n, 2n) with rows [r/2, r)."""
    s = 2.0
    w, h = 2 * n, r // 2
    q, pt, bt = _inputs(m, w, r, n, seed=7 * m + n)
    rows, tr, db = _run(q, pt, bt, r, n, s)
    q64, p64, b64 = (np_of(t).astype(np.float64) for t in (q, pt[:, :m], bt))
    _check_u(rows, tr, q64, b64, s, m)
    got = np_of(db).astype(np.float64)
    for cols, prow in ((slice(0, n), slice(0, h)), (slice(n, w), slice(h, r))):
        exact = s * (p64[prow] @ q64[:, cols]).T
        bound = s * (np.abs(p64[prow]) @ np.abs(q64[:, cols])).T * 1e-4 + 1e-12
        assert (np.abs(got[cols] - exact) <= bound).all()


def test_dual_is_deterministic_and_fp16_db():
    q, pt, bt = _inputs(1000, 3072, 32, 1536, seed=3)
    a = _run(q, pt, bt, 32, 1536, 0.5)
    b = _run(q, pt, bt, 32, 1536, 0.5)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    rows16, _, db16 = _run(q, pt, bt, 32, 1536, 0.5, db_dtype=torch.float16)
    assert torch.equal(rows16, a[0])
    assert torch.equal(db16, a[2].half())


def test_dual_rejects_bad_arguments_before_launch():
    from soupsuck_b200 import _lib
    q, pt, bt = _inputs(64, 1000, 32, 0, seed=1)  # 1000 columns: a split at 500 is not a multiple of 256
    db = torch.empty((1000, 16), device="cuda")
    ws = torch.empty(1 << 20, device="cuda", dtype=torch.uint8)
    before = _lib.launch_count()
    with pytest.raises(ValueError):
        _lib.call("sb_lora_dual", q.data_ptr(), 64, 1000, pt.data_ptr(), pt.shape[1], bt.data_ptr(), 32, 500,
                  1.0, 1, db.data_ptr(), _lib.dtype_code(torch.float32), 1.0, 0, 32, 1.0, 0, 64,
                  ws.data_ptr(), ws.numel(), _lib.stream_of(q.device))
    with pytest.raises(ValueError):  # no U output requested
        _lib.call("sb_lora_dual", q.data_ptr(), 64, 1000, pt.data_ptr(), pt.shape[1], bt.data_ptr(), 16, 0,
                  1.0, 1, db.data_ptr(), _lib.dtype_code(torch.float32), 1.0, 0, 16, 1.0, 0, 64,
                  ws.data_ptr(), ws.numel(), _lib.stream_of(q.device))
    assert _lib.launch_count() == before


@pytest.mark.parametrize("m,w,r", [(3300, 8960, 16), (77, 4096, 32)])
def test_dual_u_only_equals_dual_u(m, w, r):
    """Without Pt the kernel computes U alone (the forward's Z = X.A^T for long
    rows): the same bits as the U of the two-product pass."""
    from soupsuck_b200 import _lib
    q, pt, bt = _inputs(m, w, r, 0, seed=11 + m)
    rows, tr, _ = _run(q, pt, bt, r, 0, 2.0)
    rows2 = torch.full_like(rows, float("nan"))
    ldt = _round16(m)
    tr2 = torch.full_like(tr, float("nan"))
    nbytes = _lib.query("sb_lora_dual_workspace_bytes", m, w, r, 0)
    ws = torch.empty(max(nbytes, 1), device="cuda", dtype=torch.uint8)
    _lib.call("sb_lora_dual", q.data_ptr(), m, w, None, 0, bt.data_ptr(), r, 0, 1.0, 1, None,
              _lib.dtype_code(torch.float32), 2.0, rows2.data_ptr(), r, 2.0, tr2.data_ptr(), ldt,
              ws.data_ptr(), nbytes, _lib.stream_of(q.device))
    torch.cuda.synchronize()
    assert torch.equal(rows2, rows) and torch.equal(tr2, tr)
