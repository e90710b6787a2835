"""h3_attn_fp8_noalloc: the attention entry point for callers that cannot allocate device memory.

Some callers own no device allocator: code running inside a host framework that records and replays every device
allocation of a model block (ComfyUI's dynamic-VRAM mode does this around each block), or a plugin that is handed
only its input and output buffers.  For them the library keeps a fixed 64 MiB scratch array of its own, and this
entry point takes only q, k, v and out.  This test calls it through the C ABI, twice in a row (the array keeps the
last call's contents between calls), and checks both results against the allocating entry point h3_attn_fp8 on the
same inputs, with the attention tests' tolerance (cosine >= 0.998 against each other; identical kernels, so the
outputs are expected to be equal).  It also checks that a problem beyond the array's size is refused with a clear
error.  The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import need_gpu

pytestmark = pytest.mark.gpu


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


@pytest.mark.parametrize("S,H", [(1000, 4), (4096, 40)], ids=["small", "limit_example"])
def test_noalloc_attention_matches_allocating_entry_point(S, H):
    """Two calls in a row through the C ABI against h3_attn_fp8 on the same inputs; (4096, 40) is the documented
    example of a size at the array's limit (its scratch fills most of the 64 MiB)."""

    need_gpu()
    from tfvideo import native as N

    lib = N.lib()
    HD = H * 128
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = torch.randn(S, 3 * HD, generator=g, device="cuda").to(torch.bfloat16)
    q, k, v = qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:]
    stream = N.stream()

    ref = torch.empty(S, HD, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(N.attn_workspace_bytes(S, H) + 1024, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 1024
    rc = lib.h3_attn_fp8(q.data_ptr(), k.data_ptr(), v.data_ptr(), 3 * HD, 128, S, H, ref.data_ptr(), HD,
                         ws.data_ptr() + off, ws.numel() - off, stream)
    assert rc == 0, N.last_error()

    outs = []
    for _ in range(2):
        out = torch.full((S, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = lib.h3_attn_fp8_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 3 * HD, 128, S, H, out.data_ptr(), HD,
                                     stream)
        assert rc == 0, N.last_error()
        outs.append(out)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    for out in outs:
        assert torch.isfinite(out.float()).all()
        assert _cos(out, ref) >= 0.998
        assert torch.equal(out, ref)


def test_noalloc_attention_rejects_sizes_beyond_its_scratch():
    need_gpu()
    from tfvideo import native as N

    lib = N.lib()
    x = torch.zeros(8, 3 * 128, dtype=torch.bfloat16, device="cuda")
    rc = lib.h3_attn_fp8_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), 3 * 128, 128, 37760, 40, x.data_ptr(), 128,
                                 N.stream())
    assert rc == -2
    assert "scratch" in N.last_error()
    _ = ctypes
