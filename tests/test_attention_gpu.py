"""QK-RMSNorm + RoPE and the tcgen05 FP8 flash attention against the CPU oracle and fp32 SDPA.

Bars: QK-norm + RoPE bit-exact with the oracle (oracle/ops.py:qknorm_rope, the convention of the call at
tfvideo/minimax_h3.py:296-298); attention cosine >= 0.998 against fp32 SDPA (the north star's bar; the reference
compares its FP8 kernel the same way, tools/check_fp4attn.py:62-79), on ragged lengths too.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import block as OB
from oracle import nvfp4 as ON
from oracle import ops as OO

from helpers import bf16_array, device_ok, need_gpu, to_dev, to_np

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "reference_kernels.npz"


@pytest.fixture(autouse=True)
def _gpu():
    need_gpu()


def _ulps(a, b):
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64)) >> 16


@pytest.mark.parametrize("S,H,rot", [(37, 2, 128), (300, 4, 96), (129, 3, 64)])
def test_qknorm_rope(S, H, rot):
    from tfvideo import native as N

    HD = H * 128
    qkv = bf16_array((S, 3 * HD), seed=S, scale=3.0)
    rs = np.random.RandomState(1)
    qw, kw = (1 + 0.02 * rs.randn(128)).astype(np.float32), (1 + 0.02 * rs.randn(128)).astype(np.float32)
    rope = OB.rope_table(S, rot)
    t = to_dev(qkv)
    N.qknorm_rope(t[:, :HD], t[:, HD:2 * HD], 3 * HD, S, H, rot, to_dev(qw, torch.float32),
                  to_dev(kw, torch.float32), to_dev(rope, torch.float32), 1e-5)
    got = to_np(t)
    for j, w in ((0, qw), (1, kw)):
        ref = OO.qknorm_rope(qkv[:, j * HD:(j + 1) * HD].reshape(S, H, 128), w, rope, 1e-5).reshape(S, HD)
        assert np.array_equal(got[:, j * HD:(j + 1) * HD], ref)
    assert np.array_equal(got[:, 2 * HD:], qkv[:, 2 * HD:])       # v untouched
    device_ok()


def _normed(H, S, seed, bias=0.0):
    x = bf16_array((H, S, 128), seed, outliers=False)
    x = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True)).astype(np.float32)
    if bias:
        x = x + bias * np.random.RandomState(seed + 1).randn(H, 1, 128).astype(np.float32)
    return ON.bf16_round(x)


@pytest.mark.parametrize("S,H", [(128, 2), (200, 2), (1000, 3), (4096, 4)])
def test_attention_fp8_vs_sdpa(S, H):
    from tfvideo import attention as A

    q, k, v = _normed(H, S, 1), _normed(H, S, 2, bias=1.0), _normed(H, S, 3)
    o = A.fp8(*(to_dev(t)[None] for t in (q, k, v)))
    assert tuple(o.shape) == (1, H, S, 128)
    got = to_np(o[0])
    ref = OO.sdpa(q, k, v)
    assert np.isfinite(got).all()
    c = OO.cosine(got, ref)
    assert c >= 0.998, f"cos {c:.6f} rel_l2 {OO.rel_l2(got, ref):.4f}"
    assert OO.cosine(got, OO.attention_fp8(q, k, v)) >= 0.998
    device_ok()


def test_attention_on_reference_golden_inputs():
    """The q / k / v the reference's own FP8 kernel was run on (tests/golden, K with a channel bias)."""

    from tfvideo import attention as A

    z = np.load(GOLD)
    q, k, v = (z[n][0] for n in ("at_q", "at_k", "at_v"))
    got = to_np(A.fp8(*(to_dev(t)[None] for t in (q, k, v)))[0])
    ref = OO.sdpa(q, k, v)
    assert OO.cosine(got, ref) >= 0.998
    assert OO.cosine(got, z["at_o"][0]) >= 0.99


def test_attention_token_major_strided_views():
    """The block's call: q / k / v are column slices of one [S, 3 H 128] qkv buffer, out is [S, H 128]."""

    from tfvideo import attention as A

    S, H = 333, 2
    HD = H * 128
    qkv = bf16_array((S, 3 * HD), 7, outliers=False)
    t = to_dev(qkv)
    out = torch.empty((S, HD), dtype=torch.bfloat16, device="cuda")
    A.fp8_tokens(t[:, :HD], t[:, HD:2 * HD], t[:, 2 * HD:], S, H, 3 * HD, 128, out)
    q, k, v = (qkv[:, j * HD:(j + 1) * HD].reshape(S, H, 128).transpose(1, 0, 2) for j in range(3))
    ref = OO.sdpa(q, k, v).transpose(1, 0, 2).reshape(S, HD)
    assert OO.cosine(to_np(out), ref) >= 0.998
    device_ok()


def test_attention_deterministic():
    from tfvideo import attention as A

    q, k, v = (to_dev(_normed(2, 700, s))[None] for s in (4, 5, 6))
    a, b = A.fp8(q, k, v), A.fp8(q, k, v)
    assert torch.equal(a, b)
    _ = math


# ------------------------------------------------------------------------------------------------ block-sparse
def _random_lists(nt: int, seed: int, keep: float, empty_row: int | None = None):
    rs = np.random.RandomState(seed)
    lists = []
    for r in range(nt):
        if r == empty_row:
            lists.append([])
            continue
        row = {r} | set(rs.choice(nt, size=max(1, int(keep * nt)), replace=False).tolist())
        lists.append(sorted(row, reverse=bool(r % 2)))   # any order is allowed
    return lists


@pytest.mark.parametrize("S,H,keep", [(1000, 3, 0.4), (4096, 4, 0.25)])
def test_attention_block_sparse_vs_masked_references(S, H, keep):
    """Block-sparse FP8 attention against fp32 SDPA and the FP8 recipe under the same 128 x 128 tile mask."""

    from tfvideo import attention as A

    nt = (S + 127) // 128
    lists = _random_lists(nt, 5, keep, empty_row=1)
    m = A.TileMask(lists, S)
    q, k, v = _normed(H, S, 1), _normed(H, S, 2, bias=1.0), _normed(H, S, 3)
    got = to_np(A.fp8(*(to_dev(t)[None] for t in (q, k, v)), mask=m)[0])
    device_ok()
    assert np.isfinite(got).all()
    assert not got[:, 128:256].any()                      # the empty query tile gives zero rows
    live = np.ones(S, dtype=bool)
    live[128:256] = False
    ref = OO.sdpa(q, k, v, tile_lists=lists)
    c = OO.cosine(got[:, live], ref[:, live])
    assert c >= 0.998, f"cos {c:.6f}"
    assert OO.cosine(got[:, live], OO.attention_fp8(q, k, v, tile_lists=lists)[:, live]) >= 0.998


def test_attention_block_sparse_full_mask_equals_dense():
    """Every tile kept: the one-query-tile-per-CTA sparse launch computes each row exactly as the dense launch."""

    from tfvideo import attention as A

    S, H = 777, 2
    nt = (S + 127) // 128
    m = A.TileMask([list(range(nt))] * nt, S)
    q, k, v = (to_dev(_normed(H, S, s))[None] for s in (7, 8, 9))
    assert torch.equal(A.fp8(q, k, v, mask=m), A.fp8(q, k, v))
    device_ok()


def test_attention_block_sparse_config_mask():
    """BASELINE's sharded-config mask: 25% of tiles per query row, diagonal and text tiles kept."""

    from tfvideo import attention as A

    S, H = 2048, 2
    m = A.TileMask.block_sparse(S, keep=0.25, text_tokens=512, seed=4)
    assert all(r in row and {0, 1, 2, 3} <= set(row) for r, row in enumerate(m.lists))
    q, k, v = _normed(H, S, 11), _normed(H, S, 12), _normed(H, S, 13)
    got = to_np(A.fp8(*(to_dev(t)[None] for t in (q, k, v)), mask=m)[0])
    device_ok()
    assert OO.cosine(got, OO.sdpa(q, k, v, tile_lists=m.lists)) >= 0.998


def test_fp4attn_interface():
    """tfvideo.fp4attn.attention keeps the reference's signature (tfvideo/fp4attn.py:245-246): qk/pv "fp8" run the
    B200 kernel, "fp4" raises ValueError, ``out`` is written in place."""

    from tfvideo import attention as A
    from tfvideo import fp4attn

    S, H = 300, 2
    q, k, v = (to_dev(_normed(H, S, s))[None] for s in (31, 32, 33))
    ref = A.fp8(q, k, v)
    assert torch.equal(fp4attn.attention(q, k, v, qk="fp8", pv="fp8"), ref)
    assert torch.equal(fp4attn.attention(q, k, v, qk="fp8h", pv="fp8", pv_f16=True, smooth=False), ref)
    out = torch.empty(1, H, S, 128, dtype=torch.bfloat16, device="cuda")
    assert fp4attn.attention(q, k, v, qk="fp8", out=out) is out and torch.equal(out, ref)
    for bad in (dict(qk="fp4"), dict(pv="fp4"), dict(qk="int8")):
        with pytest.raises(ValueError):
            fp4attn.attention(q, k, v, **bad)
    device_ok()
