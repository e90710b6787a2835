"""The CPU oracle against the reference's own kernels (golden fixtures) and known-answer tables.

Fixtures: tests/golden/reference_kernels.npz, made by tests/golden/make_golden.py from the reference's Triton
kernels run under TRITON_INTERPRET=1.  The interpreter differs from GPU hardware in two documented ways, both
handled explicitly below: it converts fp32 -> bf16 by truncation, and its fp32 -> e4m3 conversion rounds exact
ties away from zero and drops the carry when the mantissa rounds up to 2.0.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4 as N
from oracle import ops as O

GOLD = Path(__file__).resolve().parent / "golden" / "reference_kernels.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


# ------------------------------------------------------------------------------------------ tables
def test_e2m1_nearest_value_table():
    """tools/check_fp4attn.py:24-34: a code dequantises to the nearest e2m1 value (saturating at 6); at exact
    midpoints the oracle must pick the even code (round half to even)."""

    x = np.linspace(-7, 7, 2801, dtype=np.float32)
    deq = N.e2m1_value(N.e2m1_code(x))
    grid = N.E2M1[:8]
    d = np.abs(np.abs(x)[:, None] - grid[None, :])
    ref = np.sign(x) * grid[d.argmin(1)]
    srt = np.sort(d, 1)
    tie = np.abs(srt[:, 0] - srt[:, 1]) < 1e-7
    assert np.all((np.abs(deq - ref) < 1e-6) | tie)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    assert list(N.e2m1_value(N.e2m1_code(mids))) == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0]
    assert N.e2m1_code(np.float32(-0.0)) == 0 and N.e2m1_code(np.float32(100.0)) == 7
    assert N.e2m1_code(np.float32(-100.0)) == 15


def test_e4m3_matches_torch_rne():
    rs = np.random.RandomState(0)
    x = (rs.randn(300000) * np.exp2(rs.uniform(-14, 9, 300000))).astype(np.float32)
    x = x[np.abs(x) < 464]
    ours = N.e4m3_rne(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)
    allb = np.arange(256, dtype=np.uint8)
    v = N.e4m3_to_f32(allb)
    t = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(v), np.isnan(t)) and np.array_equal(v[~np.isnan(v)], t[~np.isnan(t)])
    # satfinite, as the hardware cvt.rn.satfinite does (torch gives NaN above 464)
    assert list(N.e4m3_rne(np.array([448, 470, 1e9, np.inf, -1e9], np.float32))) == [126, 126, 126, 126, 254]


def test_bf16_round_matches_torch():
    x = (np.random.RandomState(1).randn(100000) * 100).astype(np.float32)
    assert np.array_equal(N.bf16_round(x), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


# ------------------------------------------------------------------------------------------ fixtures
def _ulps(a, b):
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64)) >> 16


@pytest.mark.parametrize("part", [0, 1])
def test_norm_mod_matches_reference_kernel(gold, part):
    """tfvideo/kernels.py:15-40 run by the reference's Triton code; bit-exact before the bf16 rounding."""

    a = O.norm_mod(gold["ew_x"], gold["ew_w"], gold["ew_mod"], part, gold["ew_idx"], 1e-5, rnd=N.bf16_trunc)
    assert np.array_equal(a, gold[f"norm_mod_p{part}"])
    rne = O.norm_mod(gold["ew_x"], gold["ew_w"], gold["ew_mod"], part, gold["ew_idx"], 1e-5)
    assert _ulps(rne, gold[f"norm_mod_p{part}"]).max() <= 1


@pytest.mark.parametrize("part", [0, 1])
def test_gate_add_matches_reference_kernel(gold, part):
    a = O.gate_add(gold["ew_x"], gold["ew_y"], gold["ew_mod"], part, gold["ew_idx"], rnd=N.bf16_trunc)
    assert np.array_equal(a, gold[f"gate_add_p{part}"])


def test_swiglu_matches_reference_kernel(gold):
    assert np.array_equal(O.swiglu(gold["ew_gu"], rnd=N.bf16_trunc), gold["swiglu"])


def test_nvfp4_rows_match_reference_quantiser(gold):
    """tfvideo/fp4attn.py:95-115 (_quant_qk_kernel, two-level NVFP4 per row) against oracle.nvfp4.quantize with
    the row scale as global scale.  Group scales may differ only where the interpreter's e4m3 conversion is known
    to be off (an exact tie it rounds away from zero, or a dropped carry at a power of two); the oracle's scale
    must then equal torch's RNE conversion, and every code outside those groups must match."""

    x = gold["qk_x"][0]
    H, S, Dh = x.shape
    tie = carry = 0
    for h in range(H):
        for s in range(S):
            row = x[h, s][None]
            rs = np.maximum(np.float32(np.abs(row).max()), np.float32(1e-30)) / np.float32(2688)
            assert rs == gold["qk_rs"][h, s]
            c, sf = N.quantize(row, rs)
            ref_sf = gold["qk_scales"][h, s]
            xs = (row * (np.float32(1) / rs)).astype(np.float32).reshape(-1, 16)
            v = (np.abs(xs).max(1) / np.float32(6)).astype(np.float32)
            torch_sf = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            assert np.array_equal(sf[0], torch_sf)
            diff = sf[0] != ref_sf
            for gi in np.nonzero(diff)[0]:
                ours, theirs = N.e4m3_to_f32(np.array([sf[0, gi], ref_sf[gi]], np.uint8)).astype(np.float64)
                if abs(int(sf[0, gi]) - int(ref_sf[gi])) == 1 and float(v[gi]) == (ours + theirs) / 2:
                    assert sf[0, gi] % 2 == 0 and abs(theirs) > abs(ours)
                    tie += 1
                else:
                    assert ours == 2 * theirs and (ours.item() == 2 ** np.round(np.log2(ours)))
                    carry += 1
            cm = (c[0] != gold["qk_codes"][h, s]).reshape(-1, 8)
            assert not cm[~diff].any()
    assert tie + carry < 0.02 * H * S * (Dh // 16)


def test_fp8_attention_recipe_matches_reference_kernel(gold):
    """tfvideo/fp4attn.py:245-290 with qk="fp8", pv="fp8": the oracle's recipe tracks both the reference kernel's
    output and fp32 SDPA (tools/check_fp4attn.py:62-79 compares by cosine)."""

    q, k, v = (gold[n][0] for n in ("at_q", "at_k", "at_v"))
    ours = O.attention_fp8(q, k, v)
    ref = O.sdpa(q, k, v)
    assert O.cosine(ours, gold["at_o"][0]) > 0.99
    assert O.cosine(ours, ref) > 0.998
    assert O.cosine(gold["at_o"][0], ref) > 0.99


# ------------------------------------------------------------------------------------------ quantiser properties
def test_quantize_dequantize_bounds():
    rs = np.random.RandomState(3)
    x = N.bf16_round(rs.randn(64, 256).astype(np.float32))
    g = N.global_scale(np.abs(x).max())
    codes, sf = N.quantize(x, g)
    y = N.dequantize(codes, sf, g)
    assert O.rel_l2(y, x) < 0.12
    assert np.all(N.e4m3_to_f32(sf) <= 448)
    z, zs = N.quantize(np.zeros((2, 32), np.float32), N.global_scale(0.0))
    assert not z.any() and not zs.any()


def test_sf_tiled_roundtrip():
    rs = np.random.RandomState(4)
    sf = rs.randint(0, 127, size=(300, 16)).astype(np.uint8)
    t = N.sf_to_tiled(sf)
    assert t.size == 384 * 16
    assert np.array_equal(N.sf_from_tiled(t, 300, 16), sf)
    # atom layout: row 33 of block 0, group 2 sits at 16 * 1 + 4 * 1 + 2
    assert N.sf_tiled_offset(33, 2, 16) == 22


def test_delayed_scale_policy():
    """tfvideo/linear.py:192-210: next = max(amax, 1e-6) / 2688 * margin; a clipped linear doubles its margin."""

    nxt, m, clipped = N.update_delayed(np.array([10.0, 10.0, 0.0]), np.array([10 / 2688 / 2, 1.0, 0.0]),
                                       np.array([0.0, 4.0, 16.0]), np.array([True, True, False]))
    assert clipped == 1
    assert list(m) == [4.0, 4.0, 16.0]
    assert np.allclose(nxt, [10 / 2688 * 4, 10 / 2688 * 4, 1e-6 / 2688 * 16])


# ------------------------------------------------------------------------------------------------ torch CPU path
def test_torch_path_fake_quant_equals_oracle_quantiser():
    """The torch restatement the CPU baseline times dequantises to exactly the oracle quantiser's values."""

    import torch

    from oracle import torch_path as TP

    rs = np.random.RandomState(3)
    x = N.bf16_round(rs.randn(96, 512).astype(np.float32) * np.where(rs.rand(512) < 0.02, 20.0, 1.0))
    x[5, :16] = 0.0                                       # an all-zero group
    got = TP.fake_quant(torch.from_numpy(x)).numpy()
    g = N.global_scale(float(np.abs(x).max()))
    ref = N.dequantize(*N.quantize(x, g), g)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_torch_path_block_matches_oracle_block():
    """The timed CPU block computes the oracle's NVFP4 + SDPA block (same weights, inputs): cosine >= 0.999."""

    import torch

    from oracle import block as OB
    from oracle import torch_path as TP

    shape = OB.BlockShape(dim=256, heads=2, head_dim=128, ffn=512, act="gelu", rot_dim=128)
    p = OB.make_params(shape, t_dim=8, seed=4)
    S = 96
    x = N.bf16_round(np.random.RandomState(5).randn(S, shape.dim).astype(np.float32))
    t_emb = np.random.RandomState(6).randn(1, 8).astype(np.float32)
    segs = [(0, S, 0)]
    rope = OB.rope_table(S, 128)
    ref = OB.block_forward(shape, p, x, t_emb, segs, rope, linears="nvfp4", attn="sdpa")
    mod = torch.from_numpy(O.modulation(t_emb, p.ada_w, p.ada_b, shape.dim))
    W = {n: torch.from_numpy(N.dequantize(*p.quantized()[n])) for n in ("qkv", "out", "fc1", "fc2")}
    norms = {n: torch.from_numpy(getattr(p, n)) for n in ("norm1", "norm2", "q_norm", "k_norm")}
    got = TP.block(torch.from_numpy(x), W, norms, mod, torch.zeros(S, dtype=torch.long), torch.from_numpy(rope),
                   shape.heads).numpy()
    assert O.cosine(got - x, ref - x) >= 0.999
