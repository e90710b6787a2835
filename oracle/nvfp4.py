"""NVFP4 arithmetic on the CPU (numpy) -- test infrastructure only.

Two-level NVFP4 as the reference computes it:
  * global (per-tensor) scale g = max(amax, floor) / (6 * 448)
    (tfvideo/linear.py:35 for weights, :148 for activations), held as fp32;
  * x is multiplied by the IEEE fp32 reciprocal of g (tfvideo/fp4attn.py:73-75);
  * one e4m3 scale per 16 consecutive elements = e4m3_RNE(max|x/g| / 6)
    (tfvideo/fp4attn.py:76), saturating at 448;
  * code = e2m1 of (x/g) * (1 / max(scale, 1e-30)) by the RNE thresholds of
    tfvideo/fp4attn.py:60-63 (ties to even, saturating at 6, sign from v < 0);
  * two codes a byte, the even element in the low nibble (tfvideo/fp4attn.py:78,
    tools/check_fp4attn.py:28).
Every division is an IEEE fp32 division; numpy float32 arithmetic is round to
nearest even, so this module is bit-exact by construction.
"""

from __future__ import annotations

import numpy as np

FP4_MAX = 6.0
E4M3_MAX = 448.0
# tools/check_fp4attn.py:13
E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)

F32 = np.float32


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


# ------------------------------------------------------------------------------------------ bf16
def bf16_round(x) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, NaN kept quiet."""

    # In 32-bit words: the largest non-NaN pattern is 0xFF800000 (-inf), and adding at most 0x8000 to it stays below
    # 2^32, so the rounding carry never wraps; NaN patterns are replaced afterwards.
    x = f32(x)
    if not x.flags.c_contiguous:
        x = x.copy()
    b = x.view(np.uint32)
    r = ((b >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((b + r) & np.uint32(0xFFFF0000)).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.float32(np.nan), out)
    return out.astype(np.float32, copy=False)


def bf16_trunc(x) -> np.ndarray:
    """fp32 -> bf16 by truncation (what the Triton CPU interpreter does) -> fp32."""

    x = f32(x)
    return ((x.view(np.uint32) >> 16) << 16).view(np.float32)


def bf16_bits(x) -> np.ndarray:
    """fp32 (already bf16-representable) -> uint16 bits."""

    return (f32(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------------------------------ e4m3
def e4m3_rne(x) -> np.ndarray:
    """fp32 -> e4m3fn bits (uint8): round to nearest even, saturating at +-448 (satfinite), NaN -> 0x7F.

    Normal values: code = (e + 7) * 8 + RNE(8 * (|x| / 2^e - 1)); the contiguous encoding carries a rounded-up
    mantissa into the exponent.  Below 2^-6 the subnormal step is 2^-9 and code = RNE(|x| * 512)."""

    x = f32(x)
    a = np.abs(x).astype(np.float64)          # exact
    sign = (np.signbit(x)).astype(np.uint8) << 7
    code = np.zeros(x.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    code = np.where(sub, np.rint(np.where(sub, a, 0.0) * 512.0).astype(np.int64), code)
    big = ~(a < 448.0)                        # >= 448, inf and NaN
    fr, ex = np.frexp(np.where(sub | big, 1.0, a))  # a = fr * 2^ex, fr in [0.5, 1)
    e = ex - 1
    mant = np.rint((2.0 * fr - 1.0) * 8.0).astype(np.int64)
    normal = (e + 7) * 8 + mant
    code = np.where(sub, code, normal)
    code = np.where(big, 0x7E, np.minimum(code, 0x7E))   # satfinite: anything at or beyond 448 -> 448
    out = (code.astype(np.uint8) | sign)
    out = np.where(np.isnan(x), np.uint8(0x7F), out)
    return out.astype(np.uint8)


def e4m3_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


# ------------------------------------------------------------------------------------------ e2m1
def e2m1_code(v) -> np.ndarray:
    """fp32 (already divided by its scales) -> e2m1 code in the low 4 bits (tfvideo/fp4attn.py:52-63)."""

    v = f32(v)
    a = np.abs(v)
    m = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5)
         + (a > 5.0)).astype(np.uint8)
    return (m | ((v < 0).astype(np.uint8) << 3)).astype(np.uint8)


def e2m1_value(code) -> np.ndarray:
    return E2M1[np.asarray(code, dtype=np.int64) & 15]


# ------------------------------------------------------------------------------------------ scales
def global_scale(amax: float, floor: float = 1e-6) -> np.float32:
    """g = max(amax, floor) / (6 * 448) in float64, held as fp32 (tfvideo/linear.py:35,148)."""

    return np.float32(max(float(amax), floor) / (FP4_MAX * E4M3_MAX))


def weight_scale(w) -> np.float32:
    return global_scale(float(np.abs(f32(w)).max()), 1e-12)


# ------------------------------------------------------------------------------------------ quantiser
def quantize(x, g) -> tuple[np.ndarray, np.ndarray]:
    """x [R, K] fp32 (bf16 values), g fp32 -> (codes [R, K/2] uint8, e4m3 scales [R, K/16] uint8 bits)."""

    x = f32(x)
    R, K = x.shape
    assert K % 16 == 0
    inv_g = F32(1.0) / F32(g)
    xs = (x * inv_g).astype(np.float32).reshape(R, K // 16, 16)
    gmax = np.abs(xs).max(axis=2)
    sf = e4m3_rne((gmax / F32(6.0)).astype(np.float32))
    inv = (F32(1.0) / np.maximum(e4m3_to_f32(sf), F32(1e-30))).astype(np.float32)
    q = (xs * inv[:, :, None]).astype(np.float32)
    c = e2m1_code(q).reshape(R, K)
    codes = (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)
    return codes, sf


def dequantize(codes, sf, g) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    R, K2 = codes.shape
    vals = np.empty((R, K2 * 2), dtype=np.float32)
    vals[:, 0::2] = e2m1_value(codes & 15)
    vals[:, 1::2] = e2m1_value(codes >> 4)
    s = e4m3_to_f32(sf).astype(np.float64)
    out = vals.reshape(R, -1, 16).astype(np.float64) * s[:, :, None] * float(g)
    return out.reshape(R, K2 * 2).astype(np.float32)


# ------------------------------------------------------------------------------------------ SF tile layout
def sf_tiled_offset(r, k16, kgroups: int) -> np.ndarray:
    """Byte offset of scale (row r, group k16) in the tiled layout the GEMM reads: 512-byte atoms of 128 rows x
    4 groups, atoms ordered [row block][group block], inside an atom (r % 32) * 16 + (r // 32 % 4) * 4 + k16 % 4."""

    r = np.asarray(r, dtype=np.int64)
    k16 = np.asarray(k16, dtype=np.int64)
    kb = kgroups // 4
    return ((r // 128) * kb + k16 // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + (k16 % 4)


def sf_to_tiled(sf) -> np.ndarray:
    """[R, K/16] -> flat tiled bytes of ceil(R/128) * (K/64) * 512 (padding rows zero)."""

    sf = np.asarray(sf, dtype=np.uint8)
    R, G = sf.shape
    assert G % 4 == 0
    rp = (R + 127) // 128 * 128
    out = np.zeros(rp * G, dtype=np.uint8)
    r, k = np.meshgrid(np.arange(R), np.arange(G), indexing="ij")
    out[sf_tiled_offset(r, k, G)] = sf
    return out


def sf_from_tiled(buf, R: int, G: int) -> np.ndarray:
    buf = np.asarray(buf, dtype=np.uint8).reshape(-1)
    r, k = np.meshgrid(np.arange(R), np.arange(G), indexing="ij")
    return buf[sf_tiled_offset(r, k, G)]


# ------------------------------------------------------------------------------------------ delayed scales
DELAY_MARGIN = 2.0


def update_delayed(amax: np.ndarray, used_act: np.ndarray, margin: np.ndarray, has_used: np.ndarray):
    """tfvideo/linear.py:192-210 on arrays: returns (next_act fp32, new margin, clipped count).

    margin 0 means "unset" (DELAY_MARGIN); a linear whose input absmax exceeded used_act * 2688 doubles its margin,
    capped at 16."""

    amax = np.asarray(amax, dtype=np.float64)
    m = np.where(np.asarray(margin) > 0, margin, DELAY_MARGIN).astype(np.float64)
    clip = np.asarray(has_used, bool) & (amax > np.asarray(used_act, np.float64) * FP4_MAX * E4M3_MAX)
    m = np.where(clip, np.minimum(m * 2, 16.0), m)
    nxt = np.maximum(amax, 1e-6) / (FP4_MAX * E4M3_MAX) * m
    return nxt.astype(np.float32), m, int(clip.sum())
