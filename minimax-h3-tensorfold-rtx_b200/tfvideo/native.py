"""ctypes binding of libh3b200.so, the C ABI declared in include/h3b200.h.

The library is the product: every op in this package runs through it.  It is loaded from this package's
``_native/`` directory (built in-tree by ``minimax-h3-tensorfold-rtx_b200/build.py``); there is no fallback, so a
missing or unloadable library raises ``RuntimeError`` on first use.  Tensors cross the boundary as raw device
pointers; the stream is torch's current stream.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("H3B200_LIB") or Path(__file__).resolve().parent / "_native" / "libh3b200.so")

H3_EPI_STORE, H3_EPI_GATE_RESID, H3_EPI_ACT_BF16, H3_EPI_ACT_Q, H3_EPI_STORE_PEERS = 0, 1, 2, 3, 4
ACT_GELU, ACT_SWIGLU = 0, 1
SLOT_FLOATS = 4   # H3ScaleSlot: amax, act, used, margin

vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_longlong, C.c_float, C.c_size_t


class H3Epilogue(C.Structure):
    _fields_ = [("kind", i32), ("out", vp), ("ldo", i64), ("x", vp), ("ldx", i64), ("mod", vp), ("idx", vp),
                ("gate_part", i32), ("act_kind", i32), ("qcodes", vp), ("qsf", vp), ("q_slot", vp),
                ("peer", vp * 8), ("ranks", i32), ("rank", i32)]


class H3PeerCopy(C.Structure):
    _fields_ = [("src", vp), ("dst", vp), ("bytes", sz)]


# name -> argtypes (restype int unless noted)
_SIGS = {
    "h3_version": [],
    "h3_last_error": [C.c_char_p, i32],
    "h3_device_status": [C.POINTER(i32), i32],
    "h3_status_publish": [vp, vp],
    "h3_sf_tiled_bytes": ([i32, i32], sz),
    "h3_scales_begin": [vp, i32, i32, vp, vp],
    "h3_scales_dynamic": [vp, vp],
    "h3_absmax_bf16": [vp, i64, i32, i32, vp, vp],
    "h3_norm_mod": [vp, i32, vp, vp, vp, i32, i32, i32, f32, vp, i32, vp, vp, i32, vp, vp],
    "h3_nvfp4_quant": [vp, i64, i32, i64, i32, i32, vp, f32, vp, vp, i32, vp, vp],
    "h3_gate_add": [vp, i32, vp, i32, vp, vp, i32, i32, i32, vp],
    "h3_act": [vp, i32, vp, i32, i32, i32, i32, vp, vp],
    "h3_modulation": [vp, i32, i32, vp, vp, i32, vp, vp],
    "h3_gemm_nvfp4": [vp, vp, vp, vp, vp, f32, vp, i32, i32, i32, C.POINTER(H3Epilogue), vp],
    "h3_qknorm_rope": [vp, vp, i64, i32, i32, i32, vp, vp, vp, f32, vp],
    "h3_attn_workspace_bytes": ([i32, i32], sz),
    "h3_attn_fp8": [vp, vp, vp, i64, i64, i32, i32, vp, i64, vp, sz, vp],
    "h3_attn_fp8_noalloc": [vp, vp, vp, i64, i64, i32, i32, vp, i64, vp],
    "h3_attn_fp8_sparse": [vp, vp, vp, i64, i64, i32, i32, vp, vp, vp, i64, vp, sz, vp],
    "h3_attn_fp8_peers": [vp, vp, vp, i64, i64, i32, i32, vp, vp, C.POINTER(vp), i32, i32, i64, vp, sz, vp],
    "h3_peer_alloc": [sz, C.POINTER(vp), vp],
    "h3_peer_open": [vp, C.POINTER(vp)],
    "h3_peer_close": [vp],
    "h3_peer_free": [vp],
    "h3_peer_push": [C.POINTER(H3PeerCopy), i32, vp],
    "h3_peer_copy": [C.POINTER(H3PeerCopy), i32, vp],
}

_lib = None
# kernels launched through this binding (each wrapper adds the number of kernels its entry point launches)
LAUNCHES = 0


def _count(n: int) -> None:
    global LAUNCHES
    LAUNCHES += n


def lib() -> C.CDLL:
    """The loaded library (loads it on first call; raises if it is missing)."""

    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"libh3b200.so not found at {LIB_PATH}: build it with "
                               "`python minimax-h3-tensorfold-rtx_b200/build.py` (there is no CPU fallback)")
        h = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
        for name, sig in _SIGS.items():
            fn = getattr(h, name)
            if isinstance(sig, tuple):
                fn.argtypes, fn.restype = sig
            else:
                fn.argtypes, fn.restype = sig, i32
        _lib = h
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().h3_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")


def device_status(reset: bool = False) -> int:
    st = i32(0)
    check(lib().h3_device_status(C.byref(st), int(reset)), "h3_device_status")
    return st.value


def status_publish(dst: torch.Tensor) -> None:
    """dst[0] = max(dst[0], this device's status word), in stream order (fp32 device tensor)."""

    _count(1)
    check(lib().h3_status_publish(ptr(dst), stream()), "h3_status_publish")


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libh3b200 takes CUDA tensors")
    return t.data_ptr()


def sf_tiled_bytes(rows: int, cols: int) -> int:
    return int(lib().h3_sf_tiled_bytes(rows, cols))


def attn_workspace_bytes(S: int, H: int) -> int:
    return int(lib().h3_attn_workspace_bytes(S, H))


def slot_ptr(slots: torch.Tensor, i: int) -> int:
    """Address of H3ScaleSlot i in a float32 [n, 4] device tensor."""

    return slots.data_ptr() + 16 * i


# ------------------------------------------------------------------------------------------------ thin wrappers
def scales_begin(slots: torch.Tensor, delayed: bool, clipped: torch.Tensor | None = None) -> None:
    _count(1)
    check(lib().h3_scales_begin(ptr(slots), slots.shape[0], int(delayed), ptr(clipped), stream()), "h3_scales_begin")


def scales_dynamic(slot: int) -> None:
    _count(1)
    check(lib().h3_scales_dynamic(slot, stream()), "h3_scales_dynamic")


def absmax_into(x: torch.Tensor, out_ptr: int) -> None:
    R, K = x.shape
    _count(1)
    check(lib().h3_absmax_bf16(ptr(x), x.stride(0), R, K, out_ptr, stream()), "h3_absmax_bf16")


def norm_mod(x, w, mod, idx, part, eps, out=None, codes=None, sf=None, sf_tiled=True, slot=None) -> None:
    S, D = x.shape
    _count(1)
    check(lib().h3_norm_mod(ptr(x), x.stride(0), ptr(w), ptr(mod), ptr(idx), S, D, part, eps, ptr(out),
                            out.stride(0) if out is not None else 0, ptr(codes), ptr(sf), int(sf_tiled), slot,
                            stream()), "h3_norm_mod")


def nvfp4_quant(x, codes, sf, g_ptr=None, g=0.0, sf_tiled=True, amax_ptr=None, K=None, cblk=None,
                blk_stride=0, R=None, ldx=None) -> None:
    R = x.shape[0] if R is None else R
    K = x.shape[1] if K is None else K
    ldx = x.stride(0) if ldx is None else ldx
    _count(1)
    check(lib().h3_nvfp4_quant(ptr(x), ldx, cblk or K, blk_stride, R, K, g_ptr, float(g), ptr(codes), ptr(sf),
                               int(sf_tiled), amax_ptr, stream()), "h3_nvfp4_quant")


def gate_add(x, y, mod, idx, part) -> None:
    S, D = x.shape
    _count(1)
    check(lib().h3_gate_add(ptr(x), x.stride(0), ptr(y), y.stride(0), ptr(mod), ptr(idx), S, D, part, stream()),
          "h3_gate_add")


def act(u, out, act_kind, amax_ptr=None) -> None:
    M, F = out.shape
    _count(1)
    check(lib().h3_act(ptr(u), u.stride(0), ptr(out), out.stride(0), M, F, act_kind, amax_ptr, stream()), "h3_act")


def modulation(t_emb, ada_w, ada_b, out) -> None:
    M, t_dim = t_emb.shape
    _count(1)
    check(lib().h3_modulation(ptr(t_emb), M, t_dim, ptr(ada_w), ptr(ada_b), ada_w.shape[0], ptr(out), stream()),
          "h3_modulation")


def gemm_nvfp4(a_codes, a_sf, a_slot: int, b_codes, b_sf, g_b: float, M: int, N: int, K: int, epi: H3Epilogue,
               bias=None) -> None:
    _count(1)
    check(lib().h3_gemm_nvfp4(ptr(a_codes), ptr(a_sf), a_slot, ptr(b_codes), ptr(b_sf), float(g_b), ptr(bias), M, N,
                              K, C.byref(epi), stream()), "h3_gemm_nvfp4")


def qknorm_rope(q, k, ld, S, H, rot, qw, kw, rope, eps) -> None:
    _count(1)
    check(lib().h3_qknorm_rope(ptr(q), ptr(k), ld, S, H, rot, ptr(qw), ptr(kw), ptr(rope), eps, stream()),
          "h3_qknorm_rope")


def attn_fp8(q, k, v, ld, hstride, S, H, out, ldo, workspace) -> None:
    _count(4)
    check(lib().h3_attn_fp8(ptr(q), ptr(k), ptr(v), ld, hstride, S, H, ptr(out), ldo, ptr(workspace),
                            workspace.numel() * workspace.element_size(), stream()), "h3_attn_fp8")


def attn_fp8_sparse(q, k, v, ld, hstride, S, H, kv_ptr, kv_idx, out, ldo, workspace) -> None:
    _count(4)
    check(lib().h3_attn_fp8_sparse(ptr(q), ptr(k), ptr(v), ld, hstride, S, H, ptr(kv_ptr), ptr(kv_idx), ptr(out), ldo,
                                   ptr(workspace), workspace.numel() * workspace.element_size(), stream()),
          "h3_attn_fp8_sparse")


def attn_fp8_peers(q, k, v, ld, hstride, S, H, peers: list[int], rank: int, ldo, workspace, kv_ptr=None,
                   kv_idx=None) -> None:
    """Attention of this rank's H heads over all S tokens, each output row stored to the receive buffer of the rank
    that owns the token (``peers``: every rank's buffer as mapped here)."""

    _count(4)
    arr = (vp * len(peers))(*peers)
    check(lib().h3_attn_fp8_peers(ptr(q), ptr(k), ptr(v), ld, hstride, S, H, ptr(kv_ptr), ptr(kv_idx), arr,
                                  len(peers), rank, ldo, ptr(workspace), workspace.numel() * workspace.element_size(),
                                  stream()), "h3_attn_fp8_peers")


# ---- device buffers shared between the processes of one node (CUDA IPC), for the fused Ulysses exchanges
IPC_HANDLE_BYTES = 64


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """A device allocation of the current device and its IPC handle (free it with peer_free)."""

    p = vp()
    h = C.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().h3_peer_alloc(nbytes, C.byref(p), h), "h3_peer_alloc")
    return p.value, h.raw


def peer_open(handle: bytes) -> int:
    """Maps another process's peer_alloc buffer into this one (close it with peer_close)."""

    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    p = vp()
    check(lib().h3_peer_open(C.create_string_buffer(handle, IPC_HANDLE_BYTES), C.byref(p)), "h3_peer_open")
    return p.value


def peer_push(copies: list[tuple[int, int, int]], stream_handle: int | None = None) -> None:
    """(src, dst, bytes) contiguous copies in one kernel, e.g. into other ranks' buffers, on torch's current stream
    unless given."""

    _count(1)
    arr = (H3PeerCopy * len(copies))(*[H3PeerCopy(s, d, b) for s, d, b in copies])
    check(lib().h3_peer_push(arr, len(copies), stream() if stream_handle is None else stream_handle), "h3_peer_push")


def peer_copy(copies: list[tuple[int, int, int]], stream_handle: int | None = None) -> None:
    """(src, dst, bytes) copies by the copy engines (cudaMemcpyAsync), on torch's current stream unless given."""

    if not copies:
        return
    arr = (H3PeerCopy * len(copies))(*[H3PeerCopy(s, d, b) for s, d, b in copies])
    check(lib().h3_peer_copy(arr, len(copies), stream() if stream_handle is None else stream_handle), "h3_peer_copy")


def peer_close(p: int) -> None:
    check(lib().h3_peer_close(p), "h3_peer_close")


def peer_free(p: int) -> None:
    check(lib().h3_peer_free(p), "h3_peer_free")


class _DeviceArray:
    """__cuda_array_interface__ of a raw device allocation, so torch can view it without a copy."""

    def __init__(self, p: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (p, False), "version": 3,
                                         "strides": None}


_TYPESTR = {torch.bfloat16: "<i2", torch.int16: "<i2", torch.uint8: "|u1", torch.float32: "<f4"}


def tensor_at(p: int, shape: tuple[int, ...], dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over the device memory at p (no copy; the caller keeps the memory alive).  bf16 has no
    array-interface type string: the 2-byte words are viewed as int16 and reinterpreted."""

    t = torch.as_tensor(_DeviceArray(p, shape, _TYPESTR[dtype]), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t
