"""The reference's block as a torch CPU program -- test infrastructure only (see oracle/__init__.py).

This is what the benchmark times as its CPU baseline: one MiniMax H3-shaped block through the reference's torch path
with NVFP4 fake-quant, written with multi-threaded torch CPU ops the way the reference's own torch
code would run on a host: tfvideo/kernels.py:15-84 as torch elementwise math, tfvideo/linear.py:141-151 as fake-quant
(quantise the input to NVFP4 under its per-tensor scale, dequantise, fp32 matmul with the dequantised weight), QK-norm
+ split-half RoPE as at the call tfvideo/minimax_h3.py:296-298, attention as softmax(q k^T / sqrt(Dh)) v in fp32,
bf16 roundings where the reference writes bf16 tensors (torch's fp32 -> bf16 conversion rounds to nearest even).

``fake_quant`` is the NVFP4 quantiser of oracle/nvfp4.py (tfvideo/fp4attn.py:52-78 under a per-tensor scale) in torch
ops; tests/test_oracle.py checks that its dequantised values equal oracle.nvfp4's bit for bit.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .ops import softmax_attention

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def fake_quant(a: torch.Tensor, floor: float = 1e-6) -> torch.Tensor:
    """fp32 [R, K] (bf16 values) -> dequantised NVFP4 of it under g = max(amax, floor) / 2688, fp32."""

    R, K = a.shape
    g = torch.tensor(max(float(a.abs().max()), floor) / 2688.0, dtype=torch.float32)
    xs = (a * (1.0 / g)).view(R, K // 16, 16)
    sf = (xs.abs().amax(-1, keepdim=True) / 6.0).clamp(max=448.0).to(torch.float8_e4m3fn).float()
    q = xs * (1.0 / sf.clamp_min(1e-30))
    m = q.abs()
    idx = ((m > 0.25).to(torch.uint8) + (m >= 0.75) + (m > 1.25) + (m >= 1.75) + (m > 2.5) + (m >= 3.5)
           + (m > 5.0)).long()
    v = _E2M1[idx].copysign(torch.where(q < 0, -1.0, 1.0))
    return (v * sf * g).view(R, K)


def linear(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return bf16(fake_quant(a) @ w.T)


def norm_mod(x, w, mod, part: int, idx, eps: float) -> torch.Tensor:
    shift, scale = mod[idx, 3 * part], mod[idx, 3 * part + 1]
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return bf16(x * r * w * (1.0 + scale) + shift)


def gate_add(x, y, mod, part: int, idx) -> torch.Tensor:
    return bf16(x + y * mod[idx, 3 * part + 2])


def qknorm_rope(t: torch.Tensor, w: torch.Tensor, rope: torch.Tensor, eps: float) -> torch.Tensor:
    """t [S, H, Dh]; rope [S, rot/2, 2, 2]: pair i couples dims i and i + rot/2."""

    y = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w
    half = rope.shape[1]
    f = rope[:, None]
    y1, y2 = y[..., :half], y[..., half:2 * half]
    out = y.clone()
    out[..., :half] = f[..., 0, 0] * y1 + f[..., 0, 1] * y2
    out[..., half:2 * half] = f[..., 1, 0] * y1 + f[..., 1, 1] * y2
    return bf16(out)


def block(x, W: dict, norms: dict, mod, idx, rope, heads: int, kv_buffer=None, eps: float = 1e-5):
    """One block for the rows of x [rows, D] (fp32, bf16 values).  W: qkv / out / fc1 / fc2 fp32 [N, K]; norms: norm1,
    norm2 [D], q_norm, k_norm [Dh].  ``kv_buffer`` (K, V), each [H, S, Dh] with S > rows: a sampled block of an
    S-token sequence -- the rows' own keys and values are written into the first ``rows`` positions and the rows attend
    over all S (the other positions stand for the rest of the sequence); None: the exact block of these rows."""

    rows, D = x.shape
    HD = W["qkv"].shape[0] // 3
    Dh = HD // heads
    h = norm_mod(x, norms["norm1"], mod, 0, idx, eps)
    qkv = linear(h, W["qkv"])
    q = qknorm_rope(qkv[:, :HD].reshape(rows, heads, Dh), norms["q_norm"], rope, eps)
    k = qknorm_rope(qkv[:, HD:2 * HD].reshape(rows, heads, Dh), norms["k_norm"], rope, eps)
    v = qkv[:, 2 * HD:].reshape(rows, heads, Dh)
    kt, vt = k.transpose(0, 1), v.transpose(0, 1)
    if kv_buffer is not None:
        kb, vb = kv_buffer
        kb[:, :rows] = kt
        vb[:, :rows] = vt
        kt, vt = kb, vb
    o = bf16(softmax_attention(q.transpose(0, 1), kt, vt).transpose(0, 1).reshape(rows, HD))
    xm = gate_add(x, linear(o, W["out"]), mod, 0, idx)
    a = bf16(F.gelu(linear(norm_mod(xm, norms["norm2"], mod, 1, idx, eps), W["fc1"]), approximate="tanh"))
    return gate_add(xm, linear(a, W["fc2"]), mod, 1, idx)
