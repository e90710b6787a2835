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


def test_peer_entry_points_check_their_arguments(lib):
    """The multi-GPU entry points reject bad rank layouts and pointers on the host, before any CUDA call (the
    pointers below are aligned placeholders that are never dereferenced)."""

    from tfvideo import native as N

    fake = 1 << 20   # 16-byte aligned, never touched
    epi = N.H3Epilogue(kind=N.H3_EPI_STORE_PEERS, ranks=0, rank=0)
    rc = lib.h3_gemm_nvfp4(fake, fake, fake, fake, fake, 1.0, None, 256, 3 * 128 * 4, 256, ctypes.byref(epi), None)
    assert rc != 0 and "ranks" in N.last_error()
    epi = N.H3Epilogue(kind=N.H3_EPI_STORE_PEERS, ranks=2, rank=2)
    rc = lib.h3_gemm_nvfp4(fake, fake, fake, fake, fake, 1.0, None, 256, 3 * 128 * 4, 256, ctypes.byref(epi), None)
    assert rc != 0 and "rank" in N.last_error()
    epi = N.H3Epilogue(kind=N.H3_EPI_STORE_PEERS, ranks=4, rank=0)   # N = 3 * 128 * 2 does not split over 4
    rc = lib.h3_gemm_nvfp4(fake, fake, fake, fake, fake, 1.0, None, 256, 3 * 128 * 2, 256, ctypes.byref(epi), None)
    assert rc != 0 and "multiple" in N.last_error()
    epi = N.H3Epilogue(kind=N.H3_EPI_STORE_PEERS, ranks=2, rank=1)
    epi.peer[0] = fake
    epi.peer[1] = fake + 8   # misaligned
    rc = lib.h3_gemm_nvfp4(fake, fake, fake, fake, fake, 1.0, None, 256, 3 * 128 * 2, 256, ctypes.byref(epi), None)
    assert rc != 0 and "peer[1]" in N.last_error()

    peers = (ctypes.c_void_p * 2)(fake, fake)
    rc = lib.h3_attn_fp8_peers(fake, fake, fake, 384, 128, 1000, 1, None, None, peers, 3, 0, 128, fake, 1 << 30, None)
    assert rc != 0 and "ranks" in N.last_error()   # S = 1000 does not split over 3 ranks
    rc = lib.h3_attn_fp8_peers(fake, fake, fake, 384, 128, 1024, 2, None, None, peers, 2, 0, 128, fake, 1 << 30, None)
    assert rc != 0 and "H * 128" in N.last_error()   # receive rows shorter than this rank's heads
    rc = lib.h3_attn_fp8_peers(fake, fake, fake, 384, 128, 1024, 1, fake, None, peers, 2, 0, 128, fake, 1 << 30, None)
    assert rc != 0 and "tile list" in N.last_error()

    copies = (N.H3PeerCopy * 1)(N.H3PeerCopy(fake, fake + 4, 64))
    assert lib.h3_peer_push(copies, 1, None) != 0 and "aligned" in N.last_error()
    assert lib.h3_peer_push(copies, 0, None) != 0 and "1..8" in N.last_error()
    assert lib.h3_peer_copy(None, 1, None) != 0
    assert lib.h3_peer_alloc(0, None, None) != 0 and "zero" in N.last_error()
    assert lib.h3_peer_open(None, None) != 0


def test_noalloc_size_limit_edges(lib):
    """h3_attn_fp8_noalloc's limit is exact: at H = 40 the largest S whose scratch fits the fixed array (64 MiB minus
    the 1 KiB alignment step) is found by search, and S + 128 (the next size that needs more scratch) is refused with
    H3_ERR_SHAPE before any CUDA call; the limit is documented as S * H <= 170,000 (S = 4,096 at H = 40)."""

    from tfvideo import native as N

    cap = (64 << 20) - 1024
    H = 40
    S = 4096
    while N.attn_workspace_bytes(S + 1, H) <= cap:
        S += 1
    assert N.attn_workspace_bytes(S, H) <= cap < N.attn_workspace_bytes(S + 128, H)
    assert 4096 <= S and S * H <= 170_000
    fake = 1 << 20
    rc = lib.h3_attn_fp8_noalloc(fake, fake, fake, 3 * H * 128, 128, S + 128, H, fake, H * 128, None)
    assert rc == -2 and "scratch" in N.last_error() and "h3_attn_fp8_noalloc" in N.last_error()
    rc = lib.h3_attn_fp8_noalloc(fake, fake, fake, 3 * H * 128, 128, 0, H, fake, H * 128, None)
    assert rc == -2 and "h3_attn_fp8_noalloc" in N.last_error()
