"""The C-ABI library builds, loads without a GPU and exports every entry point include/h3b200.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "h3b200.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|size_t)\s+(h3_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from tfvideo import native
    import sys
    sys.path.insert(0, str(ROOT / "minimax-h3-tensorfold-rtx_b200"))
    from build import build   # noqa: E402  (the package's build script)
    build()
    return native.lib()


def test_header_declares_the_entry_points():
    names = declared()
    assert "h3_gemm_nvfp4" in names and "h3_attn_fp8" in names and "h3_norm_mod" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, f"declared in h3b200.h but not exported: {missing}"


def test_binding_covers_the_header():
    from tfvideo import native
    assert sorted(native.exported_symbols()) == declared()


def test_calls_without_gpu_work_fail_cleanly(lib):
    """Host-side argument checks run before any CUDA call: bad shapes return H3_ERR_SHAPE with a message."""

    from tfvideo import native
    assert lib.h3_version() == 1
    rc = lib.h3_gemm_nvfp4(None, None, None, None, None, 1.0, None, 128, 256, 100, None, None)
    assert rc == -1   # NULL pointers are rejected first
    assert "NULL" in native.last_error()
    assert lib.h3_sf_tiled_bytes(300, 5120) == 384 * 320
    assert lib.h3_attn_workspace_bytes(4096, 40) > 3 * 40 * 4096 * 128
