"""The allocation-free LoRA weight-gradient reduction (sb_lora_reduce_static).

Some callers of this library cannot allocate device memory -- frameworks that
plan all device memory once at start-up, foreign-language bindings without a
CUDA allocator, or training steps that must not grow their footprint -- so they
cannot pass sb_lora_reduce its workspace.  sb_lora_reduce_static computes the
same reduction with its partial sums in a fixed device array of the library.
This test calls both entry points through the C ABI, twice in a row with
different inputs (the shared array keeps the previous call's contents), and
requires the allocation-free result to match the workspace result.  It lives
in a file that pytest collects last so a failure here never hides another.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _inputs(m, w, r, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ldp = (m + 15) // 16 * 16
    pt = torch.zeros((r, ldp), device="cuda", dtype=torch.float16)
    pt[:, :m] = torch.randn((r, m), device="cuda", generator=g).to(torch.float16)
    q = torch.randn((m, w), device="cuda", generator=g).to(torch.float16)
    return pt, ldp, q


def _workspace_result(lib, pt, ldp, q, m, w, r, scale, transpose, stream):
    nbytes = lib.sb_lora_reduce_workspace_bytes(m, w, r)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    out = torch.empty((w, r) if transpose else (r, w), dtype=torch.float32, device="cuda")
    rc = lib.sb_lora_reduce(pt.data_ptr(), ldp, q.data_ptr(), m, w, r, scale, transpose,
                            out.data_ptr(), 1, ws.data_ptr(), nbytes, stream)
    assert rc == 0, lib.sb_last_error()
    return out


@pytest.mark.parametrize("m,w,r,transpose", [(3300, 1536, 16, 0), (3300, 8960, 16, 1), (827, 640, 64, 1)])
def test_static_reduction_matches_workspace_reduction_twice(m, w, r, transpose):
    from soupsuck_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    scale = 2.0
    for call, seed in enumerate((11, 12)):
        pt, ldp, q = _inputs(m, w, r, seed + m + w)
        expected = _workspace_result(lib, pt, ldp, q, m, w, r, scale, transpose, stream)
        out = torch.full((w, r) if transpose else (r, w), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.sb_lora_reduce_static(pt.data_ptr(), ldp, q.data_ptr(), m, w, r, scale, transpose,
                                       out.data_ptr(), 1, stream)
        assert rc == 0, lib.sb_last_error()
        torch.cuda.synchronize()
        got, ref = out.cpu().numpy().astype(np.float64), expected.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all(), f"call {call}"
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert rel < 2e-3, f"call {call}: relative error {rel}"
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)


def test_static_reduction_rejects_oversized_request():
    from soupsuck_b200 import _lib
    lib = _lib.load()
    pt, ldp, q = _inputs(16, 64, 64, 3)
    out = torch.empty((64, 65536), dtype=torch.float32, device="cuda")
    rc = lib.sb_lora_reduce_static(pt.data_ptr(), ldp, q.data_ptr(), 16, 65536, 64, 1.0, 0,
                                   out.data_ptr(), 1, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SB_EINVAL
    assert b"at most" in lib.sb_last_error()
