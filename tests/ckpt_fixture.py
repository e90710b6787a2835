"""A small MiniMax H3-shaped checkpoint in ComfyUI's layout, for the checkpoint / conversion tests.

Block linears are stored the way ComfyUI's int8 + ConvRot quantisation stores them (int8 rows, fp32 row scale,
256-wide Hadamard groups, a ``comfy_quant`` JSON byte tensor), except a float linear per block to cover both formats.
``model_weights`` returns the weights the file encodes, in the model's basis, computed independently in float64.
"""

from __future__ import annotations

import json
import math

import numpy as np
import torch
from safetensors.torch import save_file

H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)


def hadamard64(size: int) -> np.ndarray:
    h = H4
    while h.shape[0] < size:
        h = np.kron(h, H4)
    return h / math.sqrt(size)


def write(path, layers=2, dim=512, heads=4, head_dim=128, ffn=1024, act="gelu", t_dim=8, prefix="model.diffusion_model.",
          seed=0):
    rs = np.random.RandomState(seed)
    hd = heads * head_dim
    shapes = {"attn.qkv_proj": (3 * hd, dim), "attn.out_proj": (dim, hd),
              "mlp.fc1": ((2 * ffn) if act == "swiglu" else ffn, dim), "mlp.fc2": (dim, ffn)}
    H = hadamard64(256)
    t, model = {}, {}
    for i in range(layers):
        p = f"{prefix}blocks.{i}."
        for j, (name, (n, k)) in enumerate(shapes.items()):
            w = rs.randn(n, k) * 0.02
            if j == 3 and i == 0:               # one float linear: stored as-is (bf16)
                wb = torch.from_numpy(w.astype(np.float32)).to(torch.bfloat16)
                t[p + name + ".weight"] = wb
                model[f"blocks.{i}.{name}"] = wb.double().numpy()
                continue
            rot = (w.reshape(n, k // 256, 256) @ H).reshape(n, k)        # the rotated basis (H is its own inverse)
            s = np.abs(rot).max(1, keepdims=True) / 127.0
            q = np.clip(np.round(rot / s), -127, 127).astype(np.int8)
            t[p + name + ".weight"] = torch.from_numpy(q)
            t[p + name + ".weight_scale"] = torch.from_numpy(s.astype(np.float32))
            conf = {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256}
            t[p + name + ".comfy_quant"] = torch.tensor(list(json.dumps(conf).encode()), dtype=torch.uint8)
            deq = q.astype(np.float64) * s.astype(np.float32).astype(np.float64)
            model[f"blocks.{i}.{name}"] = (deq.reshape(n, k // 256, 256) @ H).reshape(n, k)
        t[p + "norm1.weight"] = torch.from_numpy((1 + 0.02 * rs.randn(dim)).astype(np.float32))
        t[p + "norm2.weight"] = torch.from_numpy((1 + 0.02 * rs.randn(dim)).astype(np.float32))
        t[p + "attn.q_norm.weight"] = torch.from_numpy((1 + 0.02 * rs.randn(head_dim)).astype(np.float32))
        t[p + "attn.k_norm.weight"] = torch.from_numpy((1 + 0.02 * rs.randn(head_dim)).astype(np.float32))
        t[p + "adaln_proj.linear.weight"] = torch.from_numpy((rs.randn(18 * dim, t_dim) * 0.05).astype(np.float32))
        t[p + "adaln_proj.linear.bias"] = torch.zeros(18 * dim)
    t[prefix + "video_patch_proj.weight"] = torch.zeros(4, 4)       # a non-block tensor, as real checkpoints have
    save_file(t, str(path))
    return model
