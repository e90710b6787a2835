"""Block-level ops on the CPU -- test infrastructure only (see oracle/__init__.py).

Every function cites the reference code it restates.  Arrays are numpy float32 holding bf16 values where the
reference holds bf16 tensors; ``bf16_round`` marks each point where the reference writes a bf16 tensor.

Two functions fix a summation order so that the CUDA kernels can be compared bit for bit:
  * ``norm_mod``: the sum of squares of a row is accumulated per lane of a 32-lane group over 16-byte chunks
    (lane l owns columns it*256 + l*8 + j) and combined by a butterfly (xor 16, 8, 4, 2, 1); products and sums are
    separately rounded fp32 operations, 1/sqrt is an IEEE fp32 sqrt followed by an IEEE fp32 division.
  * ``gate_add``: x + y * gate as a rounded product then a rounded sum.
The reference's Triton kernels (tfvideo/kernels.py) reduce in a compiler-chosen order with an approximate rsqrt.
Its CPU interpreter (which made the committed fixtures) converts fp32 -> bf16 by truncation where the GPU rounds to
nearest even, so the fixture tests pass ``rnd=bf16_trunc`` to compare the fp32 arithmetic before that rounding.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .nvfp4 import F32, bf16_round, dequantize, f32, global_scale, quantize

LOG2E = 1.4426950408889634


# ------------------------------------------------------------------------------------------ reductions
def _row_sumsq_lanes(x: np.ndarray) -> np.ndarray:
    """Sum of squares of each row of x [S, D] in the lane order described in the module docstring."""

    S, D = x.shape
    lanes = np.arange(32)
    acc = np.zeros((S, 32), dtype=np.float32)
    for it in range((D + 255) // 256):
        for j in range(8):
            c = it * 256 + lanes * 8 + j
            ok = c < D
            v = x[:, np.minimum(c, D - 1)]
            acc = np.where(ok[None, :], (acc + (v * v).astype(np.float32)).astype(np.float32), acc)
    for k in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, lanes ^ k]).astype(np.float32)
    return acc[:, 0]


# ------------------------------------------------------------------------------------------ elementwise
def norm_mod(x, w, mod, part: int, idx, eps: float, rnd=bf16_round) -> np.ndarray:
    """RMSNorm(x) * w * (1 + scale[idx]) + shift[idx], bf16 out (tfvideo/kernels.py:15-40).

    x [S, D] (bf16 values), w [D] fp32, mod [R, 6, D] fp32, idx [S] int; part 0 uses chunks (0, 1), part 1 (3, 4)."""

    x = f32(x)
    S, D = x.shape
    ss = _row_sumsq_lanes(x)
    var = ((ss / F32(D)).astype(np.float32) + F32(eps)).astype(np.float32)
    r = (F32(1.0) / np.sqrt(var)).astype(np.float32)
    mod = f32(mod)
    idx = np.asarray(idx, dtype=np.int64)
    shift = mod[idx, 3 * part]
    scale = mod[idx, 3 * part + 1]
    y = (x * r[:, None]).astype(np.float32)
    y = (y * f32(w)[None, :]).astype(np.float32)
    y = (y * (F32(1.0) + scale).astype(np.float32)).astype(np.float32)
    y = (y + shift).astype(np.float32)
    return rnd(y)


def gate_add(x, y, mod, part: int, idx, rnd=bf16_round) -> np.ndarray:
    """x + y * gate[idx], bf16 out (tfvideo/kernels.py:43-63); part 0 = chunk 2, part 1 = chunk 5."""

    g = f32(mod)[np.asarray(idx, dtype=np.int64), 3 * part + 2]
    return rnd((f32(x) + (f32(y) * g).astype(np.float32)).astype(np.float32))


def swiglu(gu, rnd=bf16_round) -> np.ndarray:
    """[M, 2F] = [gate | up] -> silu(gate) * up, bf16 out (tfvideo/kernels.py:66-84)."""

    gu = f32(gu)
    F = gu.shape[1] // 2
    g, u = gu[:, :F].astype(np.float64), gu[:, F:].astype(np.float64)
    return rnd((g / (1.0 + np.exp(-g)) * u).astype(np.float32))


def gelu_tanh(u) -> np.ndarray:
    """GELU with the tanh approximation, bf16 out; BASELINE's FFN activation (torch's gelu(approximate="tanh")).

    0.5 u (1 + tanh(z)) with z = sqrt(2/pi) (u + 0.044715 u^3), evaluated in float64 as u / (1 + exp(-2 z)) -- the
    same function, without the cancellation of 1 + tanh(z) that flushes the far negative tail to zero."""

    u = f32(u).astype(np.float64)
    z = math.sqrt(2.0 / math.pi) * (u + 0.044715 * u ** 3)
    with np.errstate(over="ignore"):
        return bf16_round((u / (1.0 + np.exp(-2.0 * z))).astype(np.float32))


# ------------------------------------------------------------------------------------------ qk norm + rope
def _head_sumsq_lanes(x: np.ndarray) -> np.ndarray:
    """Sum of squares over the last dim (128) in the CUDA kernel's order: lane l owns dims 4l..4l+3, accumulated in
    order as rounded fp32 products and sums, then combined by an xor butterfly (16, 8, 4, 2, 1)."""

    lanes = np.arange(32)
    v = x.reshape(*x.shape[:-1], 32, 4)
    acc = np.zeros(v.shape[:-1], dtype=np.float32)
    for e in range(4):
        acc = (acc + (v[..., e] * v[..., e]).astype(np.float32)).astype(np.float32)
    for k in (16, 8, 4, 2, 1):
        acc = (acc + acc[..., lanes ^ k]).astype(np.float32)
    return acc[..., 0]


def qknorm_rope(x, w, rope, eps: float) -> np.ndarray:
    """Per-head RMSNorm with weight w [Dh = 128], then split-half RoPE over the first rot_dim dims, bf16 out.

    Restates the call ``ck.rms_rope_split_half_(q, k, rope_freqs, q_norm, k_norm, epsilon, rot_dim)``
    (tfvideo/minimax_h3.py:296-298): x [S, H, 128]; rope [S, rot/2, 2, 2] holds one 2x2 rotation per (token, pair)
    as built in tools/profile_block.py:41-45 (``[[cos, -sin], [sin, cos]]``).  Pair i couples dims i and
    i + rot/2:  o_i = f00 * y_i + f01 * y_{i+half},  o_{i+half} = f10 * y_i + f11 * y_{i+half}.  Dims at and past
    rot_dim only get the norm.  fp32 inside (the sum of squares in the lane order of ``_head_sumsq_lanes``, an IEEE
    sqrt and division, rounded products and sums), one bf16 rounding at the end -- comfy-kitchen's own rounding is
    not in the reference tree; this is the convention the CUDA kernel follows bit for bit."""

    x = f32(x)
    S, H, Dh = x.shape
    rope = f32(rope)
    half = rope.shape[1]
    ss = _head_sumsq_lanes(x)
    var = ((ss / F32(Dh)).astype(np.float32) + F32(eps)).astype(np.float32)
    r = (F32(1.0) / np.sqrt(var)).astype(np.float32)
    y = (x * r[..., None]).astype(np.float32)
    y = (y * f32(w)[None, None, :]).astype(np.float32)
    out = y.copy()
    f = rope[:, None, :, :, :]                       # [S, 1, half, 2, 2]
    y1, y2 = y[..., :half], y[..., half:2 * half]
    out[..., :half] = ((f[..., 0, 0] * y1).astype(np.float32) + (f[..., 0, 1] * y2).astype(np.float32))
    out[..., half:2 * half] = ((f[..., 1, 0] * y1).astype(np.float32) + (f[..., 1, 1] * y2).astype(np.float32))
    return bf16_round(out)


# ------------------------------------------------------------------------------------------ modulation
def row_index(mod_segments, S: int) -> np.ndarray:
    """int32 [S]: each row's modulation row (tfvideo/minimax_h3.py:252-263)."""

    idx = np.zeros(S, dtype=np.int32)
    for a, b, row in mod_segments:
        idx[a:b] = np.asarray(row, dtype=np.int32) if not np.isscalar(row) else int(row)
    return idx


def modulation(t_emb, ada_w, ada_b, D: int) -> np.ndarray:
    """ada_b + t_emb @ ada_w^T viewed [M * 3, 6, D] fp32 (tfvideo/minimax_h3.py:265-269)."""

    m = f32(ada_b).astype(np.float64)[None, :] + f32(t_emb).astype(np.float64) @ f32(ada_w).astype(np.float64).T
    return m.astype(np.float32).reshape(-1, 6, D)


# ------------------------------------------------------------------------------------------ linears
def nvfp4_weight(w):
    """bf16 [N, K] -> (codes, scales, g): tfvideo/linear.py:30-38 with the quantiser of oracle.nvfp4."""

    w = bf16_round(w)
    g = global_scale(float(np.abs(w).max()), 1e-12)
    codes, sf = quantize(w, g)
    return codes, sf, g


def linear_nvfp4(x, wq, g_act=None, bias=None) -> np.ndarray:
    """Nvfp4Linear.__call__ (tfvideo/linear.py:141-151) in fake-quant: quantise x under its dynamic per-tensor scale
    (or ``g_act``), dequantise both operands, fp64 matmul, bf16 out."""

    x = f32(x)
    if g_act is None:
        g_act = global_scale(float(np.abs(x).max()))
    ca, sa = quantize(x, g_act)
    a = dequantize(ca, sa, g_act).astype(np.float64)
    codes, sf, g = wq
    b = dequantize(codes, sf, g).astype(np.float64)
    y = torch.from_numpy(a) @ torch.from_numpy(b).T
    y = y.numpy()
    if bias is not None:
        y = y + f32(bias).astype(np.float64)[None, :]
    return bf16_round(y.astype(np.float32))


def linear_bf16(x, w, bias=None) -> np.ndarray:
    """Bf16Linear (tfvideo/linear.py:62-74), accumulated in fp64."""

    y = torch.from_numpy(f32(x).astype(np.float64)) @ torch.from_numpy(bf16_round(w).astype(np.float64)).T
    y = y.numpy()
    if bias is not None:
        y = y + f32(bias).astype(np.float64)[None, :]
    return bf16_round(y.astype(np.float32))


# ------------------------------------------------------------------------------------------ attention
def tile_key_mask(lists, S: int, tile: int = 128) -> torch.Tensor:
    """Boolean [S, S] key mask of a block-sparse tile mask: query tile r keeps the KV tiles in lists[r].  The block-
    sparse mask of BASELINE's sharded config (128 x 128 tiles, shared by all heads); the reference takes its sparse
    attention from ComfyUI's BlockSparseAttention node (called through tfvideo/minimax_h3.py:285-291)."""

    keep = torch.zeros(S, S, dtype=torch.bool)
    for r, row in enumerate(lists):
        for c in row:
            keep[r * tile:(r + 1) * tile, c * tile:(c + 1) * tile] = True
    return keep


def sdpa(q, k, v, tile_lists=None) -> np.ndarray:
    """softmax(q k^T / sqrt(Dh)) v in fp32 (torch CPU), [H, S, Dh] (tfvideo/attention.py:17-26); under a block-sparse
    tile mask when ``tile_lists`` is given (rows with no kept key give zeros)."""

    q, k, v = (torch.from_numpy(f32(t)) for t in (q, k, v))
    keep = None if tile_lists is None else tile_key_mask(tile_lists, q.shape[1])
    return softmax_attention(q, k, v, keep).numpy()


def softmax_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, keep: torch.Tensor | None = None,
                      rows: int = 2048) -> torch.Tensor:
    """softmax(q k^T / sqrt(Dh)) v in fp32, [H, Sq, Dh] x [H, Sk, Dh] -> [H, Sq, Dh], one head and ``rows`` query
    rows at a time (explicit matmul -> softmax -> matmul: what SDPA's math backend computes; torch's fused CPU kernel
    runs far slower than these matmuls on some hosts).  ``keep`` [Sq, Sk] masks keys; a row with no kept key gives
    zeros."""

    H, Sq, Dh = q.shape
    out = torch.empty(H, Sq, v.shape[2], dtype=torch.float32)
    scale = 1.0 / math.sqrt(Dh)
    for h in range(H):
        kh, vh = k[h].float(), v[h].float()
        for r0 in range(0, Sq, rows):
            s = (q[h, r0:r0 + rows].float() @ kh.T) * scale
            if keep is not None:
                s = s.masked_fill(~keep[r0:r0 + rows], float("-inf"))
            p = torch.softmax(s, -1)
            if keep is not None:
                p = p.nan_to_num(0.0)
            out[h, r0:r0 + rows] = p @ vh
    return out


def _e4m3(t: torch.Tensor) -> torch.Tensor:
    return t.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float()


def attention_fp8(q, k, v, blk: int = 128, tile_lists=None) -> np.ndarray:
    """The FP8 attention recipe of the CUDA kernel, with exact (not online) softmax, [H, S, Dh] -> bf16 values.

    Follows tfvideo/fp4attn.py:82-147,170-238 (qk="fp8", pv="fp8"): K smoothed by its per-channel mean over the
    sequence; Q scaled by log2(e)/sqrt(Dh) and quantised per row (rowmax/448); V per channel (448/vmax); P * 448 to
    FP8; out = acc * vmax / 448^2 / l.  One difference by design: K is quantised per 128-key block (one fp32 scale
    per block, the form BASELINE's config names) instead of per row."""

    q, k, v = (torch.from_numpy(f32(t)) for t in (q, k, v))
    H, S, Dh = q.shape
    kmean = k.mean(1, keepdim=True)
    vmax = v.abs().amax(1, keepdim=True).clamp_min(1e-30)
    qs = q * (LOG2E / math.sqrt(Dh))
    qr = qs.abs().amax(-1, keepdim=True).clamp_min(1e-30) / 448.0
    q8 = _e4m3(qs * (1.0 / qr))
    ks = k - kmean
    nb = (S + blk - 1) // blk
    pad = nb * blk - S
    kp = torch.nn.functional.pad(ks, (0, 0, 0, pad))
    kr = kp.view(H, nb, blk, Dh).abs().amax((-1, -2)).clamp_min(1e-30) / 448.0       # [H, nb]
    krow = kr.repeat_interleave(blk, 1)[:, :S, None]
    k8 = _e4m3(ks * (1.0 / krow))
    v8 = _e4m3(v * (448.0 / vmax))
    s = (q8 @ k8.transpose(1, 2)) * qr * krow.transpose(1, 2)
    if tile_lists is not None:   # block-sparse: the softmax runs over the kept keys only
        s = s.masked_fill(~tile_key_mask(tile_lists, S, blk), float("-inf"))
    m = s.amax(-1, keepdim=True)
    p = torch.exp2(s - m).nan_to_num(0.0)
    l = p.sum(-1, keepdim=True)
    p8 = _e4m3(p * 448.0)
    o = (p8 @ v8) * (vmax / (448.0 * 448.0)) / l.clamp_min(1e-30)
    return bf16_round(o.numpy())


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def rel_l2(a, ref) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - ref) / (np.linalg.norm(ref) + 1e-300))
