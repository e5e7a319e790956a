"""CPU restatement of the reference hot path, timed as the CPU baseline -- TEST INFRASTRUCTURE.

Only bench.py (its ``cpu_baseline`` leg and ``--impl reference``) and the tests
use this module.  It follows the reference's PyTorch/bitsandbytes path for one
quantized projection (solution/nf4_patch.py + bitsandbytes MatMul4Bit):
forward = dequantize (solution/kernels/nf4.py:41-59, here the C oracle
``nf4_oracle_dequant_nested`` on every host thread) then ``torch.matmul``; the
input gradient dequantizes again and multiplies by dY.  The LoRA branch is
X.A^T then .B^T scaled and added (solution/lora.py:135-164).  Arithmetic runs in
fp32 on the CPU (the host has no fast fp16 GEMM); the number of threads used is
reported with the timing.
"""

from __future__ import annotations

import ctypes
import os
import time
from pathlib import Path

import numpy as np
import torch

_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        path = Path(__file__).resolve().parent / "_build" / "libnf4_oracle.so"
        if not path.exists():
            raise RuntimeError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(path))
        lib.nf4_oracle_dequant_nested.argtypes = [ctypes.c_void_p] * 4 + [
            ctypes.c_float, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int]
        lib.nf4_oracle_dequant_nested.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def threads() -> int:
    return max(1, os.cpu_count() or 1)


def dequant_cpu(packed: np.ndarray, qabs, absmax2, code2, offset: float, shape) -> torch.Tensor:
    n = int(shape[0]) * int(shape[1])
    out = np.empty(n, dtype=np.uint16)
    packed = np.ascontiguousarray(packed.reshape(-1))
    qabs = np.ascontiguousarray(qabs)
    absmax2 = np.ascontiguousarray(absmax2, dtype=np.float32)
    code2 = np.ascontiguousarray(code2, dtype=np.float32)
    _lib().nf4_oracle_dequant_nested(packed.ctypes.data, qabs.ctypes.data, absmax2.ctypes.data,
                                     code2.ctypes.data, float(offset), out.ctypes.data, n, threads())
    return torch.from_numpy(out.view(np.float16).reshape(shape))


class CpuProjection:
    """One NF4 projection with LoRA held on the host (numpy state arrays)."""

    def __init__(self, packed, state, lora_a, lora_b, scaling):
        to_np = lambda t: t.detach().cpu().numpy()
        self.packed = to_np(packed).reshape(-1)
        self.qabs = to_np(state.absmax)
        self.absmax2 = to_np(state.state2.absmax)
        self.code2 = to_np(state.state2.code)
        self.offset = float(state.offset.reshape(-1)[0].item())
        self.shape = tuple(state.shape)
        self.a = lora_a.detach().float().cpu()
        self.b = lora_b.detach().float().cpu()
        self.s = float(scaling)

    def weight(self) -> torch.Tensor:
        return dequant_cpu(self.packed, self.qabs, self.absmax2, self.code2, self.offset, self.shape)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight().float()
        y = x @ w.t()
        return y + self.s * ((x @ self.a.t()) @ self.b.t())

    def backward_dx(self, dy: torch.Tensor) -> torch.Tensor:
        w = self.weight().float()
        return dy @ w + self.s * ((dy @ self.b) @ self.a)


def time_projections(projs, rows: int, budget_s: float = 10.0, min_reps: int = 1):
    """Run forward + dX of every projection on `rows` random rows until
    `budget_s` elapses (at least `min_reps` passes).  Returns (seconds per pass,
    algorithmic FLOPs per pass)."""
    torch.set_num_threads(threads())
    gen = torch.Generator().manual_seed(0)
    flops = 0
    inputs = []
    for p in projs:
        n, k = p.shape
        r = p.a.shape[0]
        x = torch.randn((rows, k), generator=gen)
        dy = torch.randn((rows, n), generator=gen)
        inputs.append((x, dy))
        flops += 2 * rows * n * k + 2 * rows * k * r + 2 * rows * r * n      # forward
        flops += 2 * rows * n * k + 2 * rows * n * r + 2 * rows * r * k      # dX
    reps = 0
    start = time.perf_counter()
    while True:
        for p, (x, dy) in zip(projs, inputs):
            p.forward(x)
            p.backward_dx(dy)
        reps += 1
        elapsed = time.perf_counter() - start
        if reps >= min_reps and elapsed >= budget_s:
            break
        if reps >= min_reps and elapsed * (reps + 1) / reps > 3 * budget_s:
            break
    return elapsed / reps, flops
