"""Block-sparse attention mask on the CPU: the seeded mask of BASELINE's sharded config and the masked oracle.

The mask is 128 x 128 tiles shared by all heads; BASELINE's config keeps 25% of the tiles of every query-tile row,
always including the diagonal tile and the text tiles (the first 512 tokens).  The reference gets sparse attention
from ComfyUI's BlockSparseAttention node (handed the block at tfvideo/minimax_h3.py:285-291), whose selection code is
not in the reference tree, so the seeded mask here is this build's stand-in with the config's shape.
"""

from __future__ import annotations

import numpy as np

from oracle import ops as OO


def _mask(S, **kw):
    from tfvideo import attention as A

    return A.TileMask.block_sparse(S, device="cpu", **kw)


def test_config_mask_shape():
    m = _mask(37760)
    assert m.tiles == 295
    assert all(len(row) == 74 for row in m.lists)            # 25% of 295 tiles per row
    assert all(r in row and {0, 1, 2, 3} <= set(row) for r, row in enumerate(m.lists))
    assert abs(m.density - 74 / 295) < 1e-9
    ptr = m.kv_ptr.tolist()
    assert ptr[0] == 0 and ptr[-1] == m.kept == 295 * 74 and len(ptr) == 296


def test_config_mask_is_seeded():
    a, b, c = _mask(4096, seed=4), _mask(4096, seed=4), _mask(4096, seed=5)
    assert a.lists == b.lists and a.lists != c.lists


def test_masked_oracle_full_mask_is_dense_and_masked_keys_do_not_matter():
    rs = np.random.RandomState(0)
    H, S = 2, 300
    q, k, v = (rs.randn(H, S, 128).astype(np.float32) for _ in range(3))
    nt = 3
    full = [list(range(nt))] * nt
    assert np.allclose(OO.sdpa(q, k, v, tile_lists=full), OO.sdpa(q, k, v), atol=1e-5)
    lists = [[0], [1, 2], [0, 2]]
    a = OO.sdpa(q, k, v, tile_lists=lists)
    k2, v2 = k.copy(), v.copy()
    k2[:, 0:128] *= 7.0                                          # key tile 0 only seen by query tiles 0 and 2
    v2[:, 0:128] += 3.0
    b = OO.sdpa(q, k2, v2, tile_lists=lists)
    assert np.allclose(a[:, 128:256], b[:, 128:256], atol=1e-6)  # query tile 1 does not see key tile 0
    f = OO.attention_fp8(q, k, v, tile_lists=lists)
    assert OO.cosine(f, a) >= 0.99
