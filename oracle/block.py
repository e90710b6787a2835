"""One MiniMax H3 DiT block on the CPU -- test infrastructure only (see oracle/__init__.py).

``block_forward`` runs the block in the order of tfvideo/minimax_h3.py:275-324:
  norm_mod(part 0) -> qkv -> q/k RMSNorm + RoPE -> attention -> out -> gate_add(part 0)
  -> norm_mod(part 1) -> fc1 -> activation -> fc2 -> gate_add(part 1)
with bf16 roundings where the reference writes bf16 tensors.  ``linears`` selects NVFP4 fake-quant with dynamic
per-call activation scales (the reference's first forward, tfvideo/linear.py:141-151) or plain bf16
(tfvideo/linear.py:62-74); ``attn`` selects fp32 SDPA or the FP8 recipe.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import ops
from .nvfp4 import bf16_round, f32


@dataclass
class BlockShape:
    dim: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 20480
    act: str = "gelu"            # "gelu" or "swiglu" (MiniMax H3: fc1 emits [gate | up])
    rot_dim: int = 128
    eps: float = 1e-5
    qk_eps: float = 1e-5


@dataclass
class BlockParams:
    w: dict                      # name -> bf16-valued fp32 [N, K]: qkv, out, fc1, fc2
    norm1: np.ndarray
    norm2: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    ada_w: np.ndarray
    ada_b: np.ndarray
    wq: dict = field(default_factory=dict)   # name -> (codes, scales, g)

    def quantized(self):
        if not self.wq:
            self.wq = {n: ops.nvfp4_weight(w) for n, w in self.w.items()}
        return self.wq


def fc1_rows(shape: BlockShape) -> int:
    return 2 * shape.ffn if shape.act == "swiglu" else shape.ffn


def make_params(shape: BlockShape, t_dim: int, seed: int = 1) -> BlockParams:
    """Seeded synthetic block: W ~ N(0, 0.02) (bf16), norms 1 + N(0, 0.02), ada_w ~ N(0, 0.1 / sqrt(t_dim))."""

    rs = np.random.RandomState(seed)
    D, HD = shape.dim, shape.heads * shape.head_dim
    dims = {"qkv": (3 * HD, D), "out": (D, HD), "fc1": (fc1_rows(shape), D), "fc2": (D, shape.ffn)}
    w = {n: bf16_round((rs.randn(*s) * 0.02).astype(np.float32)) for n, s in dims.items()}
    return BlockParams(
        w=w,
        norm1=(1 + 0.02 * rs.randn(D)).astype(np.float32),
        norm2=(1 + 0.02 * rs.randn(D)).astype(np.float32),
        q_norm=(1 + 0.02 * rs.randn(shape.head_dim)).astype(np.float32),
        k_norm=(1 + 0.02 * rs.randn(shape.head_dim)).astype(np.float32),
        ada_w=(rs.randn(18 * D, t_dim) * (0.1 / np.sqrt(t_dim))).astype(np.float32),
        ada_b=np.zeros(18 * D, dtype=np.float32),
    )


def _linear(p: BlockParams, name: str, x, linears: str):
    if linears == "nvfp4":
        return ops.linear_nvfp4(x, p.quantized()[name])
    return ops.linear_bf16(x, p.w[name])


def block_forward(shape: BlockShape, p: BlockParams, x, t_emb, mod_segments, rope, linears: str = "nvfp4",
                  attn: str = "fp8", trace: dict | None = None) -> np.ndarray:
    """x [S, D] bf16 values -> x after the block (a new array).  rope [S, rot/2, 2, 2].  ``trace`` collects
    intermediate tensors by name when given."""

    x = f32(x).copy()
    S, D = x.shape
    H, Dh = shape.heads, shape.head_dim
    HD = H * Dh
    tr = trace if trace is not None else {}
    idx = ops.row_index(mod_segments, S)
    mod = ops.modulation(t_emb, p.ada_w, p.ada_b, D)
    tr["mod"] = mod
    h = ops.norm_mod(x, p.norm1, mod, 0, idx, shape.eps)
    tr["h1"] = h
    qkv = _linear(p, "qkv", h, linears)
    tr["qkv"] = qkv
    q = ops.qknorm_rope(qkv[:, :HD].reshape(S, H, Dh), p.q_norm, rope, shape.qk_eps)
    k = ops.qknorm_rope(qkv[:, HD:2 * HD].reshape(S, H, Dh), p.k_norm, rope, shape.qk_eps)
    v = qkv[:, 2 * HD:].reshape(S, H, Dh)
    tr["q"], tr["k"], tr["v"] = q, k, v
    qh, kh, vh = (t.transpose(1, 0, 2) for t in (q, k, v))
    o = ops.attention_fp8(qh, kh, vh) if attn == "fp8" else bf16_round(ops.sdpa(qh, kh, vh))
    o = o.transpose(1, 0, 2).reshape(S, HD)
    tr["attn"] = o
    h = _linear(p, "out", o, linears)
    tr["out"] = h
    x = ops.gate_add(x, h, mod, 0, idx)
    tr["x_mid"] = x
    h = ops.norm_mod(x, p.norm2, mod, 1, idx, shape.eps)
    tr["h2"] = h
    u = _linear(p, "fc1", h, linears)
    a = ops.swiglu(u) if shape.act == "swiglu" else ops.gelu_tanh(u)
    tr["act"] = a
    h = _linear(p, "fc2", a, linears)
    tr["fc2"] = h
    return ops.gate_add(x, h, mod, 1, idx)


def rope_table(S: int, rot_dim: int = 128, splits=(44, 42, 42), grid=None, theta: float = 10000.0) -> np.ndarray:
    """[S, rot/2, 2, 2] 3D (t, h, w) rotary table, pairs split per axis in proportion to ``splits`` dims.

    Positions: tokens enumerate a (T, Hg, Wg) grid in order (the packing ComfyUI builds for the video segment);
    ``grid`` defaults to the smallest cube-ish grid covering S."""

    half = rot_dim // 2
    tot = sum(splits)
    parts = [int(round(s * half / tot)) for s in splits]
    parts[-1] = half - sum(parts[:-1])
    if grid is None:
        w = max(1, int(round(S ** (1 / 3))))
        grid = (-(-S // (w * w)), w, w)
    T, Hg, Wg = grid
    s = np.arange(S)
    pos = [s // (Hg * Wg), (s // Wg) % Hg, s % Wg]
    angles = []
    for p_axis, n in zip(pos, parts):
        freqs = theta ** (-np.arange(n, dtype=np.float64) / max(n, 1))
        angles.append(p_axis[:, None].astype(np.float64) * freqs[None, :])
    ang = np.concatenate(angles, 1)                      # [S, half]
    c, sn = np.cos(ang), np.sin(ang)
    return np.stack([np.stack([c, -sn], -1), np.stack([sn, c], -1)], -2).astype(np.float32)
