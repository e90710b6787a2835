"""Generate golden vectors from the reference's own code (run once in the build container, outputs committed).

Runs the reference's Triton kernels on the CPU under ``TRITON_INTERPRET=1``, importing ``tfvideo`` from the
reference checkout (path given by ``--reference``, default the sibling checkout used to build this repository):
  * tfvideo/kernels.py:15-84   norm_mod, gate_add, swiglu on seeded inputs with per-token modulation rows
  * tfvideo/fp4attn.py:95-115  _quant_qk_kernel: two-level NVFP4 rows (e2m1 codes, e4m3 group scales, fp32 row
                               scale), including zero rows, outliers and values on e2m1 rounding boundaries
  * tfvideo/fp4attn.py:245-290 attention(qk="fp8", pv="fp8") on a small sequence
Writes tests/golden/reference_kernels.npz.  The interpreter rounds fp32 -> e4m3 ties away from zero (hardware and
torch round them to even), so tests/test_oracle.py accepts a differing group scale only where the value is an
exact e4m3 tie, and checks that the oracle picked the even neighbour there.

Usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("H3_REFERENCE"),
                    help="checkout of the reference repository (or set H3_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "reference_kernels.npz"))
    a = ap.parse_args()
    if not a.reference:
        sys.exit("pass --reference (or H3_REFERENCE): the reference repository's checkout")
    if os.environ.get("TRITON_INTERPRET") != "1":
        sys.exit("set TRITON_INTERPRET=1 (the reference kernels run on the CPU interpreter)")
    sys.path.insert(0, a.reference)
    import torch
    import triton
    from tfvideo import fp4attn as FA
    from tfvideo import kernels as K

    out = {}
    g = torch.Generator().manual_seed(0)

    # ---------------------------------------------------------------- elementwise (kernels.py)
    S, D, R = 48, 768, 4
    x = torch.randn(S, D, generator=g).to(torch.bfloat16)
    x[:, torch.randperm(D, generator=g)[:D // 100]] *= 20
    w = (1 + 0.02 * torch.randn(D, generator=g)).float()
    mod = (0.1 * torch.randn(R, 6, D, generator=g)).float()
    idx = torch.tensor([0] * 5 + [1] * 17 + [2] * 6 + [3] * 20, dtype=torch.int32)
    y = (torch.randn(S, D, generator=g) * 1.5).to(torch.bfloat16)
    for part in (0, 1):
        out[f"norm_mod_p{part}"] = K.norm_mod(x, w, mod, part, idx, 1e-5).float().numpy()
        xx = x.clone()
        K.gate_add(xx, y, mod, part, idx)
        out[f"gate_add_p{part}"] = xx.float().numpy()
    gu = (torch.randn(S, 2 * 384, generator=g) * 2).to(torch.bfloat16)
    out["swiglu"] = K.swiglu(gu).float().numpy()
    out.update(ew_x=x.float().numpy(), ew_w=w.numpy(), ew_mod=mod.numpy(), ew_idx=idx.numpy(),
               ew_y=y.float().numpy(), ew_gu=gu.float().numpy())

    # ---------------------------------------------------------------- NVFP4 rows (fp4attn._quant_qk_kernel)
    H, Sq, Dh, BS = 2, 256, 128, 128
    q = torch.randn(1, H, Sq, Dh, generator=g)
    q[0, 0, 3] = 0.0                                           # an all-zero row
    q[0, 1, :, 7] *= 40.0                                      # an outlier channel
    e2 = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 3.0])
    q[0, 0, 10, :10] = e2 * (q[0, 0, 10].abs().max() / 6.0)     # values on rounding boundaries
    q = q.to(torch.bfloat16)
    SP = triton.cdiv(Sq, BS) * BS
    codes = torch.empty((H, SP, Dh // 2), dtype=torch.uint8)
    scales = torch.empty((H, SP, Dh // 16), dtype=torch.float8_e4m3fn)
    rs = torch.empty((H, SP), dtype=torch.float32)
    kmean = torch.zeros((H, Dh), dtype=torch.float32)
    FA._quant_qk_kernel[(triton.cdiv(Sq, BS), H)](q, kmean, codes, scales, rs, Sq, SP, q.stride(2), q.stride(1), 1.0,
                                                  Dh, BS, False, num_warps=8)
    out.update(qk_x=q.float().numpy(), qk_codes=codes.numpy(), qk_scales=scales.view(torch.uint8).numpy(),
               qk_rs=rs.numpy())

    # ---------------------------------------------------------------- FP8 attention (fp4attn.attention)
    Sa, Ha = 200, 2
    qa, ka, va = (torch.randn(1, Ha, Sa, Dh, generator=g).to(torch.bfloat16) for _ in range(3))
    ka = (ka.float() + 2.0 * torch.randn(1, Ha, 1, Dh, generator=g)).to(torch.bfloat16)   # channel bias
    oa = FA.attention(qa, ka, va, qk="fp8", pv="fp8")
    out.update(at_q=qa.float().numpy(), at_k=ka.float().numpy(), at_v=va.float().numpy(), at_o=oa.float().numpy())

    np.savez_compressed(a.out, **out)
    print(f"wrote {a.out}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in out.items()))
    _ = math


if __name__ == "__main__":
    main()
