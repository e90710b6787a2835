"""``tfvideo.fp4attn`` on B200: the reference's low-precision attention entry point (tfvideo/fp4attn.py:245-290),
backed by libh3b200's tcgen05 FP8 flash attention.

``attention(q, k, v, qk="fp8", pv="fp8")`` is the path the B200 build carries: K smoothed by its per-channel mean,
Q and K in e4m3 (Q one fp32 scale per row, K one per 128-key block), P and V in e4m3 (V one scale per channel), fp32
accumulation in TMEM.  q, k, v are [1, H, S, 128] bf16 views with a contiguous last dim; the result is [1, H, S, 128]
bf16 (a view of token-major memory unless ``out`` is given).

Arguments kept from the reference and how they map here:
  qk       "fp8" runs; "fp8h" (Q/K quantised to a max of 16 instead of 448 on sm_120) runs as "fp8", whose e4m3
           range the B200 kernel uses in full; "fp4" (NVFP4 Q/K) has no B200 build and raises ValueError.
  pv       "fp8" runs; "fp4" (NVFP4 V) raises ValueError.
  pv_f16   accepted; the reference's fp16 PV accumulation (an sm_120 speed option) does not apply, the B200 kernel
           accumulates PV in fp32.
  smooth   accepted; the B200 kernel always subtracts K's per-channel mean.  The shift adds the same constant to
           every logit of a query row, so the softmax is unchanged and only the FP8 rounding of K improves.
  out      optional [1, H, S, 128] bf16 output; written in place and returned.
"""

from __future__ import annotations

import torch

from . import attention as A


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, qk: str = "fp8", pv: str = "fp8",
              pv_f16: bool = False, smooth: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
    if qk not in ("fp8", "fp8h", "fp4"):
        raise ValueError(f"fp4attn.attention: qk={qk!r}: one of 'fp4', 'fp8', 'fp8h'")
    if pv not in ("fp8", "fp4"):
        raise ValueError(f"fp4attn.attention: pv={pv!r}: one of 'fp8', 'fp4'")
    if qk == "fp4" or pv == "fp4":
        raise ValueError("fp4attn.attention: NVFP4 Q/K or V has no B200 build; use qk='fp8', pv='fp8'")
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError(f"fp4attn.attention: q must be [1, H, S, 128], got {tuple(q.shape)}")
    _ = pv_f16, smooth
    o = A.fp8(q, k, v)
    if out is None:
        return o
    if tuple(out.shape) != tuple(o.shape) or out.dtype != torch.bfloat16:
        raise ValueError(f"fp4attn.attention: out must be bf16 {tuple(o.shape)}, got {tuple(out.shape)} {out.dtype}")
    out.copy_(o)
    return out
