"""Reading ComfyUI-layout MiniMax H3 checkpoints on the CPU (tfvideo/source.py): the ConvRot matrix, int8 + ConvRot
linears back in the model's basis, float linears, the block's small tensors and the implied engine config."""

from __future__ import annotations

import numpy as np
import torch

import ckpt_fixture as F


def test_hadamard_is_the_normalised_kronecker_power_and_its_own_inverse():
    from tfvideo.source import hadamard

    h = hadamard(256).double()
    assert np.allclose(h.numpy(), F.hadamard64(256), atol=1e-7)
    assert torch.allclose(h, h.T)
    assert torch.allclose(h @ h, torch.eye(256, dtype=torch.float64), atol=1e-6)


def test_checkpoint_linears_config_and_small_tensors(tmp_path):
    from tfvideo.source import Checkpoint

    path = tmp_path / "h3.safetensors"
    model = F.write(path, layers=2, act="swiglu", ffn=512)
    ck = Checkpoint(path)
    assert ck.layers == 2 and ck.prefix == "model.diffusion_model."
    cfg = ck.config()
    assert (cfg.layers, cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn, cfg.act, cfg.t_dim) == (2, 512, 4, 128, 512,
                                                                                             "swiglu", 8)
    for name, want in model.items():
        got = ck.linear(name, device="cpu").double().numpy()
        assert got.shape == want.shape
        assert np.abs(got - want).max() <= 1e-6 * np.abs(want).max() + 1e-7, name
    assert ck.quant_conf("blocks.0.mlp.fc2") is None                  # the float linear
    assert ck.quant_conf("blocks.1.mlp.fc2")["convrot"]
    small = ck.small(1, device="cpu")
    assert set(small) == {"norm1", "norm2", "q_norm", "k_norm", "ada_w", "ada_b"}
    assert small["ada_w"].shape == (18 * 512, 8) and small["ada_w"].dtype == torch.float32
