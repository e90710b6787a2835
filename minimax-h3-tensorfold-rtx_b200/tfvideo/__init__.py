"""MiniMax H3 DiT blocks on B200 (sm_100a): NVFP4 tcgen05 GEMMs, FP8 flash attention, fused elementwise kernels.

A drop-in for the reference package's block hot path (jayleaton/minimax-h3-tensorfold-rtx, ``tfvideo``): the same
module names (``linear``, ``attention``, ``kernels``, ``minimax_h3``, ``comfy_nodes``) over one C-ABI library,
``_native/libh3b200.so`` (include/h3b200.h), loaded through ``tfvideo.native``.
"""

__version__ = "0.1.0"
