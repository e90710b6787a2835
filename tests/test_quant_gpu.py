"""NVFP4 quantisation, fused norm_mod and the device scale policy against the CPU oracle, bit for bit.

The oracle (oracle/nvfp4.py, oracle/ops.py) is pinned to the reference's own kernels by tests/test_oracle.py; here
the CUDA kernels must reproduce it exactly: e2m1 codes and e4m3 scales (tfvideo/fp4attn.py:52-78 under the linear
path's per-tensor scale, tfvideo/linear.py:30-38,141-151) and norm_mod's bf16 output (tfvideo/kernels.py:15-40).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ON
from oracle import ops as OO

from helpers import bf16_array, device_ok, need_gpu, to_dev, to_np, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    need_gpu()


@pytest.mark.parametrize("R,K", [(1, 16), (7, 64), (128, 256), (300, 5120), (129, 20480)])
@pytest.mark.parametrize("tiled", [False, True])
def test_quant_bit_exact(R, K, tiled):
    from tfvideo import linear as L

    x = bf16_array((R, K), seed=R * 7 + K)
    x[0, :16] = 0.0                                            # an all-zero group
    if R > 2:
        x[2, :32] = np.float32(2.0 ** -120)                    # groups whose e4m3 scale rounds to 0
    g = ON.global_scale(float(np.abs(x).max()))
    codes, sf = L.quantize(to_dev(x), g=float(g), tiled=tiled)
    ref_c, ref_s = ON.quantize(x, g)
    assert np.array_equal(u8(codes), ref_c)
    got_s = ON.sf_from_tiled(u8(sf), R, K // 16) if tiled else u8(sf)
    assert np.array_equal(got_s, ref_s)
    device_ok()


def test_quant_saturation_and_negative_zero():
    """Inputs beyond the global scale's range (a clipped delayed scale) saturate like the oracle; -0.0 codes as +0."""

    from tfvideo import linear as L

    x = bf16_array((64, 256), seed=5, outliers=False)
    x[3, 5] = -0.0
    x[4, :16] = 0.0
    x[4, 3] = -0.0
    g = ON.global_scale(float(np.abs(x).max()) / 8)           # 8x too small: many values clip
    codes, sf = L.quantize(to_dev(x), g=float(g), tiled=False)
    ref_c, ref_s = ON.quantize(x, g)
    assert np.array_equal(u8(codes), ref_c) and np.array_equal(u8(sf), ref_s)
    assert (ref_s == 0x7E).any()                               # some scales saturated at 448


def test_nvfp4_weight_layout_matches_reference_api():
    """linear.nvfp4_weight returns ModelOpt's layout: codes [N, K/2], e4m3 scales [N, K/16], fp32 global scale."""

    from tfvideo import linear as L

    w = bf16_array((256, 512), seed=11, scale=0.02, outliers=False)
    codes, sf, g = L.nvfp4_weight(to_dev(w))
    ref_c, ref_s, ref_g = OO.nvfp4_weight(w)
    assert np.float32(g) == ref_g
    assert sf.dtype == torch.float8_e4m3fn and tuple(sf.shape) == (256, 32)
    assert np.array_equal(u8(codes), ref_c) and np.array_equal(u8(sf), ref_s)


@pytest.mark.parametrize("S,D,R", [(1, 256, 1), (37, 768, 4), (300, 5120, 4), (64, 5376, 3)])
@pytest.mark.parametrize("part", [0, 1])
def test_norm_mod_bit_exact(S, D, R, part):
    from tfvideo import kernels as K

    x = bf16_array((S, D), seed=S + D)
    rs = np.random.RandomState(S)
    w = (1 + 0.02 * rs.randn(D)).astype(np.float32)
    mod = (0.1 * rs.randn(R, 6, D)).astype(np.float32)
    idx = rs.randint(0, R, size=S).astype(np.int32)
    out = K.norm_mod(to_dev(x), to_dev(w, torch.float32), to_dev(mod, torch.float32), part,
                     to_dev(idx, torch.int32), 1e-5)
    ref = OO.norm_mod(x, w, mod, part, idx, 1e-5)
    assert np.array_equal(to_np(out), ref)
    device_ok()


@pytest.mark.parametrize("S,D,segments", [(5, 256, False), (300, 5120, False), (129, 5376, False),
                                           (1000, 5120, True), (77, 768, True)])
def test_fused_norm_mod_quant_bit_exact(S, D, segments):
    """norm_mod + NVFP4 in one kernel (the delayed-scale path): codes / scales equal the oracle's quantisation of the
    oracle's norm_mod output, and the slot's amax equals max |y|.  segments: contiguous runs of one modulation row
    (as in a video's token segments), else a random modulation row per token."""

    from tfvideo import linear as L
    from tfvideo import native as N

    x = bf16_array((S, D), seed=3 * S + D)
    rs = np.random.RandomState(D)
    w = (1 + 0.02 * rs.randn(D)).astype(np.float32)
    mod = (0.1 * rs.randn(4, 6, D)).astype(np.float32)
    idx = rs.randint(0, 4, size=S).astype(np.int32)
    if segments:
        idx = np.sort(idx).astype(np.int32)
    ref_y = OO.norm_mod(x, w, mod, 1, idx, 1e-5)
    g = ON.global_scale(float(np.abs(ref_y).max()) * 1.5)
    slots = L.new_slots(1, "cuda")
    slots[0, 1] = float(g)
    codes = torch.empty((S, D // 2), dtype=torch.uint8, device="cuda")
    sf = torch.zeros(N.sf_tiled_bytes(S, D), dtype=torch.uint8, device="cuda")
    N.norm_mod(to_dev(x), to_dev(w, torch.float32), to_dev(mod, torch.float32), to_dev(idx, torch.int32), 1, 1e-5,
               codes=codes, sf=sf, slot=N.slot_ptr(slots, 0))
    ref_c, ref_s = ON.quantize(ref_y, g)
    assert np.array_equal(u8(codes), ref_c)
    assert np.array_equal(ON.sf_from_tiled(u8(sf), S, D // 16), ref_s)
    assert to_np(slots)[0, 0] == np.abs(ref_y).max()
    device_ok()


def test_absmax_and_dynamic_scale():
    from tfvideo import linear as L
    from tfvideo import native as N

    x = bf16_array((333, 1024), seed=9)
    assert float(L.absmax(to_dev(x))) == np.abs(x).max()
    slots = L.new_slots(1, "cuda")
    N.absmax_into(to_dev(x), N.slot_ptr(slots, 0))
    N.scales_dynamic(N.slot_ptr(slots, 0))
    assert to_np(slots)[0, 1] == ON.global_scale(float(np.abs(x).max()))


def test_delayed_scale_policy_matches_reference():
    """h3_scales_begin(delayed) == tfvideo/linear.py:192-210 (oracle.nvfp4.update_delayed) on a batch of slots."""

    from tfvideo import linear as L
    from tfvideo import native as N

    rs = np.random.RandomState(1)
    n = 64
    amax = (rs.rand(n) * 50).astype(np.float32)
    used = np.where(rs.rand(n) < 0.5, amax / 2688 * rs.choice([0.5, 2.0], n), 0).astype(np.float32)
    margin = rs.choice([0.0, 2.0, 4.0, 16.0], n).astype(np.float32)
    slots = L.new_slots(n, "cuda")
    slots[:, 0] = torch.from_numpy(amax).cuda()
    slots[:, 2] = torch.from_numpy(used).cuda()
    slots[:, 3] = torch.from_numpy(margin).cuda()
    clipped = torch.zeros((), dtype=torch.int32, device="cuda")
    N.scales_begin(slots, True, clipped)
    nxt, m, nclip = ON.update_delayed(amax, used, margin, used > 0)
    s = to_np(slots)
    assert np.array_equal(s[:, 1], nxt) and np.array_equal(s[:, 3], m.astype(np.float32))
    assert int(clipped.item()) == nclip
    assert (s[:, 0] == -1).all()
    N.scales_begin(slots, False)
    assert (to_np(slots)[:, 0] == -1).all() and (to_np(slots)[:, 1:] == 0).all()


def test_gate_add_and_activations():
    from tfvideo import kernels as K

    S, D = 77, 512
    x, y = bf16_array((S, D), 1), bf16_array((S, D), 2, outliers=False)
    rs = np.random.RandomState(0)
    mod = (0.1 * rs.randn(3, 6, D)).astype(np.float32)
    idx = rs.randint(0, 3, size=S).astype(np.int32)
    xt = to_dev(x)
    K.gate_add(xt, to_dev(y), to_dev(mod, torch.float32), 1, to_dev(idx, torch.int32))
    assert np.array_equal(to_np(xt), OO.gate_add(x, y, mod, 1, idx))
    gu = bf16_array((S, 2 * 256), 3, scale=2.0, outliers=False)
    sw = to_np(K.swiglu(to_dev(gu)))
    assert np.abs(sw - OO.swiglu(gu)).max() <= 2 ** -7 * np.abs(OO.swiglu(gu)).max()
    ge = to_np(K.gelu_tanh(to_dev(gu)))
    ref = OO.gelu_tanh(gu)
    assert (np.abs(ge - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-30).all()     # relative, also in the far negative tail
    assert (ge == ref).mean() > 0.95
