"""The C-ABI library loads and exports every entry point include/soupsuck_b200.h
declares, and the ctypes table matches the header (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "soupsuck_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from soupsuck_b200 import _lib
    if not _lib.LIB_PATH.exists():
        from soupsuck_b200 import build
        build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_covers_the_header():
    from soupsuck_b200 import _lib
    assert sorted(_lib.SIGNATURES) == _declared()


def test_invalid_arguments_fail_before_any_launch(lib):
    from soupsuck_b200 import _lib
    before = lib.sb_launch_count()
    assert lib.sb_nf4_dequant_nested(None, None, None, None, None, None, -1, None) == _lib.SB_EINVAL
    assert b"non-negative" in lib.sb_last_error()
    assert lib.sb_lora_project(None, 10, 33, None, 16, 1.0, None, 16, 1.0, None, 16, None) == _lib.SB_EINVAL
    assert lib.sb_lora_reduce_static(None, 16, None, 16, 65536, 64, 1.0, 0, ctypes.c_void_p(1), 1, None) == _lib.SB_EINVAL
    assert lib.sb_launch_count() == before


def test_workspace_queries_are_host_only(lib):
    # Qwen2.5 projections take the tcgen05 path: no decoded-weight workspace.
    assert lib.sb_nf4_linear_workspace_bytes(3300, 8960, 1536, 0) < 8960 * 1536 * 2
    # Odd shapes take the CUDA-core path, which needs the decoded weight.
    assert lib.sb_nf4_linear_workspace_bytes(7, 13, 17, 0) == 13 * 17 * 2
    assert lib.sb_ce_forward_workspace_bytes(3300, 1536, 151936) > 0
    assert lib.sb_lora_reduce_workspace_bytes(3300, 8960, 16) > 0
