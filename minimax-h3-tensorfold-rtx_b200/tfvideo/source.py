"""Reading a MiniMax H3 DiT checkpoint as ComfyUI stores it (the reference's tfvideo/source.py:1-109).

The block linears are either floats or ComfyUI's ``int8_tensorwise`` format with ConvRot: int8 rows with one fp32
scale per row, quantised in a rotated basis in which every 256-wide group of inputs was multiplied by a normalised
regular Hadamard matrix H (symmetric, its own inverse).  The weight in the model's basis is therefore
W[:, group] = (q * s)[:, group] @ H.  A linear's format is the JSON in its ``<name>.comfy_quant`` byte tensor, e.g.
``{"format": "int8_tensorwise", "convrot": true, "convrot_groupsize": 256}``.

The file is read with plain file I/O (header + byte offsets), as the reference does: ComfyUI patches file loading
for its own models, so no second memory map is opened on the checkpoint.
"""

from __future__ import annotations

import json
import math
import re
import struct
from functools import lru_cache
from pathlib import Path

import torch

# the four block linears and the block's small tensors, by their checkpoint names
LINEARS = ("attn.qkv_proj", "attn.out_proj", "mlp.fc1", "mlp.fc2")
SMALL = {"norm1": "norm1.weight", "norm2": "norm2.weight", "q_norm": "attn.q_norm.weight",
         "k_norm": "attn.k_norm.weight", "ada_w": "adaln_proj.linear.weight", "ada_b": "adaln_proj.linear.bias"}

# comfy-kitchen's ConvRot building block: the 4 x 4 regular Hadamard matrix (all row sums 2)
_H4 = ((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1))


@lru_cache(maxsize=8)
def hadamard(size: int, device: str = "cpu") -> torch.Tensor:
    """The normalised ConvRot matrix of a ``size``-wide group: the Kronecker power of _H4 of that size, / sqrt(size).
    ``size`` must be a power of 4 (ConvRot's groups are 256 wide)."""

    if size < 4 or 4 ** round(math.log(size, 4)) != size:
        raise ValueError(f"ConvRot group size must be a power of 4, got {size}")
    base = torch.tensor(_H4, dtype=torch.float32)
    h = base
    while h.shape[0] < size:
        h = torch.kron(h, base)
    return (h / math.sqrt(size)).to(device)


_DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
           "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
           "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2}


class SafeTensors:
    """A .safetensors file: an 8-byte little-endian header length, a JSON header (name -> dtype, shape, byte
    offsets; ``__metadata__`` -> str -> str), then the raw tensor bytes."""

    def __init__(self, path: str | Path):
        self.path = str(path)
        with open(self.path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
        self.metadata = header.pop("__metadata__", None) or {}
        self.header = header
        self.data_start = 8 + n

    def keys(self):
        return self.header.keys()

    def shape(self, name: str) -> list[int]:
        return list(self.header[name]["shape"])

    def get(self, name: str) -> torch.Tensor:
        entry = self.header[name]
        start, end = entry["data_offsets"]
        dtype = _DTYPES[entry["dtype"]]
        if end == start:
            return torch.empty(entry["shape"], dtype=dtype)
        with open(self.path, "rb") as f:
            f.seek(self.data_start + start)
            raw = bytearray(f.read(end - start))
        return torch.frombuffer(raw, dtype=dtype).reshape(entry["shape"])


class Checkpoint:
    """A MiniMax H3 DiT safetensors file: tensors by name (with or without ComfyUI's ``model.diffusion_model.``
    prefix) and the block linears as fp32 weights in the model's basis."""

    def __init__(self, path: str | Path):
        self.path = str(path)
        self.f = SafeTensors(self.path)
        names = set(self.f.keys())
        p = "model.diffusion_model."
        self.prefix = p if any(k.startswith(p + "blocks.") for k in names) else ""
        self._names = names
        blocks = {int(m.group(1)) for k in names if (m := re.match(re.escape(self.prefix) + r"blocks\.(\d+)\.", k))}
        if not blocks:
            raise ValueError(f"{self.path}: no DiT blocks found")
        self.layers = max(blocks) + 1

    def has(self, name: str) -> bool:
        return self.prefix + name in self._names

    def get(self, name: str) -> torch.Tensor:
        return self.f.get(self.prefix + name)

    def quant_conf(self, lin: str) -> dict | None:
        """The ComfyUI quantisation record of block linear ``lin`` (e.g. ``blocks.3.mlp.fc1``), or None for floats."""

        if not self.has(lin + ".comfy_quant"):
            return None
        return json.loads(bytes(self.get(lin + ".comfy_quant").to(torch.uint8).tolist()).decode())

    def linear(self, lin: str, device="cuda") -> torch.Tensor:
        """Block linear ``lin`` as fp32 [N, K] in the model's basis, on ``device``."""

        w = self.get(lin + ".weight").to(device)
        conf = self.quant_conf(lin)
        if conf is None:
            return w.float()
        if conf.get("format") != "int8_tensorwise":
            raise ValueError(f"{lin}: unsupported ComfyUI quantisation {conf}")
        s = self.get(lin + ".weight_scale").to(device).float()
        w = w.float() * (s.reshape(-1, 1) if s.numel() > 1 else s)
        if conf.get("convrot"):
            g = int(conf.get("convrot_groupsize", 256))
            n, k = w.shape
            if k % g:
                raise ValueError(f"{lin}: K = {k} is not a multiple of the ConvRot group {g}")
            w = (w.view(n, k // g, g) @ hadamard(g, str(torch.device(device)))).view(n, k)
        return w

    def small(self, i: int, device="cuda") -> dict[str, torch.Tensor]:
        """Block i's norms and adaLN projection as fp32 device tensors."""

        return {k: self.get(f"blocks.{i}.{v}").to(device=device, dtype=torch.float32) for k, v in SMALL.items()}

    def config(self):
        """The engine Config this checkpoint's shapes imply (dims, heads, FFN width and activation, t_dim)."""

        from .minimax_h3 import Config

        dim = self.f.shape(self.prefix + "blocks.0.norm1.weight")[0]
        head_dim = self.f.shape(self.prefix + "blocks.0.attn.q_norm.weight")[0]
        qkv_n = self.f.shape(self.prefix + "blocks.0.attn.qkv_proj.weight")[0]
        fc1_n = self.f.shape(self.prefix + "blocks.0.mlp.fc1.weight")[0]
        ffn = self.f.shape(self.prefix + "blocks.0.mlp.fc2.weight")[1]
        t_dim = self.f.shape(self.prefix + "blocks.0.adaln_proj.linear.weight")[1]
        return Config(layers=self.layers, dim=dim, heads=qkv_n // (3 * head_dim), head_dim=head_dim, ffn=ffn,
                      act="swiglu" if fc1_n == 2 * ffn else "gelu", t_dim=t_dim)
