"""Linear layers for the DiT blocks on B200: NVFP4 W4A4 on the tcgen05 block-scaled GEMM of libh3b200.

Mirrors tfvideo/linear.py of the reference (same names, arguments and error behaviour where the B200 path keeps
them): ``nvfp4_weight`` (:30-38), ``absmax`` (:41-45), ``Linear`` (:48-59), ``Bf16Linear`` (:62-74),
``Nvfp4Linear`` (:113-154), ``update_delayed`` / ``reset_delayed`` (:189-216) and ``make`` (:236-246).

Activation scales live on the device in H3ScaleSlot records (amax / act / used / margin), so the delayed-scale
policy runs with no host read: ``MiniMaxH3Engine.begin_forward`` updates every slot in one kernel.  A standalone
``Nvfp4Linear`` call quantises under its input's own absmax (the reference's dynamic mode), also without a host sync.
"""

from __future__ import annotations

from functools import lru_cache

import torch

from . import native as N

FP4_MAX, E4M3_MAX = 6.0, 448.0
DELAY_MARGIN = 2.0


@lru_cache(maxsize=1)
def nvfp4_supported() -> bool:
    """The tcgen05 block-scaled GEMM needs a compute-capability 10.x GPU (B200)."""

    return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10


def new_slots(n: int, device) -> torch.Tensor:
    """n H3ScaleSlot records as a float32 [n, 4] device tensor, all "no history" (amax = -1)."""

    s = torch.zeros((n, N.SLOT_FLOATS), dtype=torch.float32, device=device)
    s[:, 0] = -1.0
    return s


def quantize(x: torch.Tensor, g: float | None = None, g_ptr: int | None = None, tiled: bool = True,
             amax_ptr: int | None = None):
    """bf16 [R, K] -> (codes [R, K/2] uint8, e4m3 scales (tiled for the GEMM, else [R, K/16]))."""

    R, K = x.shape
    codes = torch.empty((R, K // 2), dtype=torch.uint8, device=x.device)
    sf = (torch.zeros(N.sf_tiled_bytes(R, K), dtype=torch.uint8, device=x.device) if tiled
          else torch.empty((R, K // 16), dtype=torch.uint8, device=x.device))
    N.nvfp4_quant(x, codes, sf, g_ptr=g_ptr, g=0.0 if g is None else g, sf_tiled=tiled, amax_ptr=amax_ptr)
    return codes, sf


def nvfp4_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """bf16 [N, K] -> (e2m1 codes [N, K/2], e4m3 scales [N, K/16], global scale): ModelOpt's NVFP4 layout."""

    w = w.to(device="cuda", dtype=torch.bfloat16).contiguous()
    g = max(float(w.float().abs().amax()), 1e-12) / (FP4_MAX * E4M3_MAX)
    codes, sf = quantize(w, g=g, tiled=False)
    return codes, sf.view(torch.float8_e4m3fn), g


def absmax(x: torch.Tensor) -> torch.Tensor:
    """max |x| as an fp32 scalar tensor on x's device (one pass, no |x| materialised)."""

    out = torch.zeros((), dtype=torch.float32, device=x.device)
    N.absmax_into(x, out.data_ptr())
    return out


class Linear:
    """y = x @ W^T for 2-D bf16 rows; ``kind`` names the backend."""

    kind = "base"
    n: int
    k: int

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        raise NotImplementedError

    def nbytes(self) -> int:
        raise NotImplementedError


class Bf16Linear(Linear):
    """bf16 weights on torch.matmul: the reference's ``bf16-check`` precision (a checker, not the fast path)."""

    kind = "bf16"

    def __init__(self, w: torch.Tensor):
        self.w = w.to(torch.bfloat16).contiguous()
        self.n, self.k = self.w.shape

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        w = self.w if self.w.device == x.device else self.w.to(x.device, non_blocking=True)
        return torch.matmul(x, w.t(), out=out)

    def nbytes(self) -> int:
        return self.w.numel() * 2


class Nvfp4Linear(Linear):
    """W4A4 NVFP4 (e2m1 values, e4m3 scale per 16, fp32 global) on the tcgen05 block-scaled GEMM.

    ``act``: a fixed input scale (static, no absmax), or None for the measured one.  ``slots`` / ``slot``: the
    H3ScaleSlot array and index that hold this linear's input-scale state (the engine passes one shared array; a
    standalone linear makes its own).  ``interleave16``: store the rows of a [gate | up] weight interleaved in blocks
    of 16 so that the GEMM epilogue can apply SwiGLU (``act_kind`` 1)."""

    kind = "nvfp4"

    def __init__(self, w: torch.Tensor, act: float | None = None, slots: torch.Tensor | None = None, slot: int = 0,
                 bias: torch.Tensor | None = None, interleave16: bool = False):
        if not nvfp4_supported():
            raise RuntimeError("Nvfp4Linear needs a B200 (compute capability 10.x)")
        w = w.to(device="cuda", dtype=torch.bfloat16)
        self.n, self.k = w.shape
        if self.k % 256 or self.n % 128:
            raise ValueError(f"NVFP4 GEMM needs K % 256 == 0 and N % 128 == 0, got {tuple(w.shape)}")
        if interleave16:
            f = self.n // 2
            w = torch.stack([w[:f].view(f // 16, 16, self.k), w[f:].view(f // 16, 16, self.k)], 1).reshape(self.n,
                                                                                                           self.k)
        self.interleaved = interleave16
        self.g = max(float(w.float().abs().amax()), 1e-12) / (FP4_MAX * E4M3_MAX)
        self.codes, self.sf = quantize(w.contiguous(), g=self.g, tiled=True)
        self.bias = None if bias is None else bias.to(device="cuda", dtype=torch.float32).contiguous()
        self.slots = new_slots(1, w.device) if slots is None else slots
        self.slot = slot
        self.dynamic = act is None
        if act is not None:
            self.set_act(act)

    @classmethod
    def from_quantized(cls, codes: torch.Tensor, sf: torch.Tensor, g: float, n: int, k: int,
                       interleaved: bool = False, slots: torch.Tensor | None = None, slot: int = 0,
                       bias: torch.Tensor | None = None) -> "Nvfp4Linear":
        """A linear from already quantised weights (codes [N, K/2] u8, tiled scales, global scale g): how a converted
        engine is loaded back."""

        if not nvfp4_supported():
            raise RuntimeError("Nvfp4Linear needs a B200 (compute capability 10.x)")
        lin = cls.__new__(cls)
        lin.n, lin.k, lin.g, lin.interleaved = int(n), int(k), float(g), bool(interleaved)
        lin.codes = codes.to(device="cuda", dtype=torch.uint8).contiguous()
        lin.sf = sf.to(device="cuda", dtype=torch.uint8).contiguous()
        if tuple(lin.codes.shape) != (lin.n, lin.k // 2) or lin.sf.numel() != N.sf_tiled_bytes(lin.n, lin.k):
            raise ValueError(f"Nvfp4Linear.from_quantized: tensors do not match [{n}, {k}]")
        lin.bias = None if bias is None else bias.to(device="cuda", dtype=torch.float32).contiguous()
        lin.slots = new_slots(1, lin.codes.device) if slots is None else slots
        lin.slot = slot
        lin.dynamic = True
        return lin

    def slot_ptr(self) -> int:
        return N.slot_ptr(self.slots, self.slot)

    def set_act(self, act: float | None) -> None:
        self.dynamic = act is None
        if act is not None:
            self.slots[self.slot, 1] = float(act)

    @property
    def amax_dev(self) -> torch.Tensor:
        return self.slots[self.slot, 0]

    def quantize_input(self, x: torch.Tensor):
        """x bf16 [M, K] -> (codes, tiled scales, slot tensor, slot index) under this linear's input scale.

        Dynamic: the scale is this call's own absmax (tfvideo/linear.py:146-149), measured into a one-call slot
        (and folded into this linear's amax for the delayed policy); static / delayed: this linear's slot act."""

        if self.dynamic:
            call = new_slots(1, x.device)
            N.absmax_into(x, N.slot_ptr(call, 0))
            N.scales_dynamic(N.slot_ptr(call, 0))
            N.absmax_into(x, self.slot_ptr())
            slots, i = call, 0
        else:
            slots, i = self.slots, self.slot
        codes, sf = quantize(x, g_ptr=N.slot_ptr(slots, i) + 4, tiled=True)
        return codes, sf, slots, i

    def gemm(self, a_codes, a_sf, M: int, epi: N.H3Epilogue, a_slot: int | None = None) -> None:
        """The GEMM on an already-quantised input (global scale in slot a_slot, default this linear's) with a fused
        epilogue."""

        N.gemm_nvfp4(a_codes, a_sf, self.slot_ptr() if a_slot is None else a_slot, self.codes, self.sf, self.g, M,
                     self.n, self.k, epi, bias=self.bias)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.k or x.dtype != torch.bfloat16:
            raise ValueError(f"Nvfp4Linear expects bf16 [M, {self.k}], got {tuple(x.shape)} {x.dtype}")
        x = x.contiguous()
        M = x.shape[0]
        codes, sf, slots, i = self.quantize_input(x)
        out = torch.empty((M, self.n), dtype=torch.bfloat16, device=x.device) if out is None else out
        self.gemm(codes, sf, M, N.H3Epilogue(kind=N.H3_EPI_STORE, out=out.data_ptr(), ldo=out.stride(0)),
                  a_slot=N.slot_ptr(slots, i))
        return out

    def nbytes(self) -> int:
        return self.codes.numel() + self.sf.numel() + 4


def update_delayed(lins, margin: float = DELAY_MARGIN) -> int:
    """After a forward: each dynamic NVFP4 linear's next input scale becomes its absmax * margin (margin doubled for a
    linear whose input exceeded the range it was quantised under, capped at 16), on the device.  Returns how many
    linears clipped (one host read, as in the reference)."""

    del margin   # the device policy uses DELAY_MARGIN, as the reference's default
    clipped = None
    for slots in {id(l.slots): l.slots for l in lins if isinstance(l, Nvfp4Linear) and l.dynamic}.values():
        clipped = torch.zeros((), dtype=torch.int32, device=slots.device) if clipped is None else clipped
        N.scales_begin(slots, True, clipped)
    return 0 if clipped is None else int(clipped.item())


def reset_delayed(lins) -> None:
    for slots in {id(l.slots): l.slots for l in lins if isinstance(l, Nvfp4Linear)}.values():
        N.scales_begin(slots, False)


def make(kind: str, w: torch.Tensor, act: float | None = None) -> Linear:
    """A backend by name for a bf16 [N, K] weight: "nvfp4" (the B200 GEMM) or "bf16"."""

    if kind == "nvfp4":
        return Nvfp4Linear(w, act)
    if kind in ("bf16", "bf16-check"):
        return Bf16Linear(w)
    raise ValueError(f"linear kind {kind!r}: one of nvfp4, bf16")
