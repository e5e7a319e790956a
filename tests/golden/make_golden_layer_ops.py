"""Golden vectors of the reference's RoPE, SwiGLU and unpad code (run once, here).

Usage (in a container where the reference checkout exists):

    TRITON_INTERPRET=1 python tests/golden/make_golden_layer_ops.py /path/to/reference

Calls the reference's raw ``@triton.jit`` kernels with the launch arguments of
their wrappers under the Triton interpreter on CPU tensors:

* ``rope_pair_forward_kernel`` / ``rope_pair_backward_kernel``
  (solution/kernels/rope.py:24-105, launched as in ``_RoPE`` :110-146) on the
  shapes and dtype combinations of solution/tests/test_rope.py:51-56, with the
  transposed [B, S, H, D] projection view and a broadcast or per-batch cos/sin;
* ``swiglu_tile_engine`` (solution/kernels/swiglu_fused.py:21-46, launched as in
  :53-78) forward and backward on fp16 gate/up [37, 300] and [3, 2304];
* the unpad helpers (solution/unpad.py: ``right_padding_lengths`` :51-72,
  ``_batch_metadata`` :164-183, ``_indices_from_lengths`` :186-200, ``_pack`` /
  ``_scatter`` :149-161) on valid and invalid masks and a small hidden tensor.

Inputs are stored with the outputs in ``golden_layer_ops.npz``; nothing at test
time reads the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(reference_root: str) -> None:
    os.environ.setdefault("TRITON_INTERPRET", "1")
    sys.path.insert(0, reference_root)
    import torch
    import triton
    from solution.kernels import rope as rp
    from solution.kernels import swiglu_fused as sw

    arrays = {}
    torch.manual_seed(347)
    cases = [("a", 3, 5, 2, 17, 66, 3, True, (torch.float16, torch.float16, torch.float16)),
             ("b", 3, 5, 2, 17, 66, 1, True, (torch.float16, torch.float16, torch.float32)),
             ("c", 1, 3, 1, 7, 10, 1, False, (torch.float32, torch.float32, torch.float32)),
             ("d", 2, 4, 2, 9, 128, 1, True, (torch.float32, torch.float16, torch.float16))]
    for name, b, hq, hk, s, d, cb, transposed, (qt, kt, ct) in cases:
        def make(heads, dtype):
            if transposed:
                return torch.randn(b, s, heads, d, dtype=dtype).transpose(1, 2)
            return torch.randn(b, heads, s, d, dtype=dtype)
        q, k = make(hq, qt), make(hk, kt)
        cos = torch.randn(cb, s, d, dtype=ct)
        sin = torch.randn(cb, s, d, dtype=ct)
        yq = torch.empty(q.shape, dtype=torch.promote_types(qt, ct))
        yk = torch.empty(k.shape, dtype=torch.promote_types(kt, ct))
        width = triton.next_power_of_2(d // 2)
        grid = (triton.cdiv(b * (hq + hk) * s, 4),)
        rp.rope_pair_forward_kernel[grid](
            q, k, cos, sin, yq, yk, s, b, hq, hk, d // 2, cb,
            *q.stride()[:3], *k.stride()[:3], *cos.stride()[:2], *sin.stride()[:2],
            ROWS=4, WIDTH=width)
        gq, gk = torch.randn_like(yq), torch.randn_like(yk)
        dq = torch.empty(q.shape, dtype=qt)
        dk = torch.empty(k.shape, dtype=kt)
        rp.rope_pair_backward_kernel[grid](
            gq, gk, cos, sin, dq, dk, s, b, hq, hk, d // 2, cb,
            *gq.stride(), *gk.stride(), *cos.stride()[:2], *sin.stride()[:2],
            NEED_Q=True, NEED_K=True, ROWS=4, WIDTH=width)
        for key, t in (("q", q), ("k", k), ("cos", cos), ("sin", sin), ("yq", yq), ("yk", yk),
                       ("gq", gq), ("gk", gk), ("dq", dq), ("dk", dk)):
            arrays[f"rope_{name}_{key}"] = t.contiguous().numpy()
        arrays[f"rope_{name}_meta"] = np.array([b, hq, hk, s, d, cb, int(transposed)], dtype=np.int64)

    for name, rows, width in (("small", 37, 300), ("wide", 3, 2304)):
        g = (torch.randn(rows, width) * 3).to(torch.float16)
        u = torch.randn(rows, width).to(torch.float16)
        da = torch.randn(rows, width).to(torch.float16)
        a = torch.empty_like(g)
        grid = (triton.cdiv(rows, 4), triton.cdiv(width, 256))
        sw.swiglu_tile_engine[grid](g, u, a, g, g, u, rows, width, *g.stride(), *u.stride(),
                                    *a.stride(), *g.stride(), *g.stride(), *u.stride(),
                                    BACKWARD=False, ROWS=4, COLS=256)
        dg, du = torch.empty_like(g), torch.empty_like(u)
        sw.swiglu_tile_engine[grid](g, u, g, da, dg, du, rows, width, *g.stride(), *u.stride(),
                                    *g.stride(), *da.stride(), *dg.stride(), *du.stride(),
                                    BACKWARD=True, ROWS=4, COLS=256)
        for key, t in (("gate", g), ("up", u), ("act", a), ("grad", da), ("dgate", dg), ("dup", du)):
            arrays[f"swiglu_{name}_{key}"] = t.numpy()

    # Unpad metadata and packing (solution/unpad.py:51-72, :149-200) on masks that
    # are valid, non-binary, left-padded, with a label on padding, with an empty
    # row, and as fp32 values; then pack/scatter of a [B, S, 3] tensor.
    from solution import unpad as up
    masks = {
        "valid": ([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1], [1, 0, 0, 0, 0]], None),
        "nonbinary": ([[1, 2, 0, 0, 0], [1, 1, 1, 1, 1], [1, 0, 0, 0, 0]], None),
        "leftpad": ([[0, 1, 1, 0, 0], [1, 1, 1, 1, 1], [1, 0, 0, 0, 0]], None),
        "labelpad": ([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1], [1, 0, 0, 0, 0]], (0, 4)),
        "empty": ([[1, 1, 1, 0, 0], [0, 0, 0, 0, 0], [1, 0, 0, 0, 0]], None),
    }
    for name, (rows, bad_label) in masks.items():
        mask = torch.tensor(rows, dtype=torch.int64)
        labels = torch.where(mask == 1, torch.arange(mask.numel()).reshape(mask.shape), torch.full_like(mask, -100))
        if bad_label is not None:
            labels[bad_label] = 7
        meta = up._batch_metadata(mask, labels)
        lengths = up.right_padding_lengths(meta) if meta is not None else None
        arrays[f"unpad_{name}_mask"] = mask.numpy()
        arrays[f"unpad_{name}_labels"] = labels.numpy()
        arrays[f"unpad_{name}_lengths"] = np.array(lengths if lengths is not None else [], dtype=np.int64)
    float_mask = torch.tensor(masks["valid"][0], dtype=torch.float32)
    arrays["unpad_float_lengths"] = np.array(up.right_padding_lengths(
        up._batch_metadata(float_mask, torch.zeros_like(float_mask, dtype=torch.int64) - 100)), dtype=np.int64)
    lengths = up.right_padding_lengths(masks["valid"][0])
    indices = up._indices_from_lengths(lengths, 5, "cpu")

    class _Batch:
        batch, sequence, tokens = 3, 5, sum(lengths)
    _Batch.indices = indices
    x = torch.randn(3, 5, 3)
    packed = up._pack(x, _Batch)
    arrays["unpad_valid_indices"] = indices.numpy()
    arrays["unpad_valid_x"] = x.numpy()
    arrays["unpad_valid_packed"] = packed.numpy()
    arrays["unpad_valid_scattered"] = up._scatter(packed, _Batch).numpy()

    np.savez_compressed(HERE / "golden_layer_ops.npz", **arrays)
    print("wrote", HERE / "golden_layer_ops.npz", (HERE / "golden_layer_ops.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: TRITON_INTERPRET=1 python tests/golden/make_golden_layer_ops.py <reference checkout>")
    main(sys.argv[1])
