"""Shared test helpers: golden fixtures, oracle access and tensor conversions."""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden():
    return np.load(GOLDEN / "golden.npz")


def manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())


def np_of(t):
    """CPU numpy copy of a torch tensor (fp16 stays fp16)."""
    return t.detach().cpu().numpy()


def bits16(t):
    return np_of(t).view(np.uint16)


def state_numpy(packed, state):
    return (np_of(packed).reshape(-1), np_of(state.absmax), np_of(state.state2.absmax),
            np_of(state.state2.code), np_of(state.offset))


def oracle_dequant(packed, state):
    from oracle import oracle as O
    p, q, a2, c2, off = state_numpy(packed, state)
    n = math.prod(state.shape)
    return O.nf4_dequant_nested(p, q, a2, c2, off, n).reshape(state.shape)
