"""CPU oracle for the MiniMax H3 DiT block hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy / torch-CPU, the arithmetic of the reference path
(jayleaton/minimax-h3-tensorfold-rtx, ``tfvideo/``) so that the CUDA kernels of
``libh3b200.so`` can be checked against it.  It is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``tfvideo`` in ``minimax-h3-tensorfold-rtx_b200/``) never imports this package
and fails loudly when its CUDA library is missing.

Modules
  nvfp4   e2m1 / e4m3 / bf16 rounding and the two-level NVFP4 quantiser
          (tfvideo/fp4attn.py:52-78 under the linear path's per-tensor scale,
          tfvideo/linear.py:30-38,141-151), the scale-factor tile layout, and
          the delayed-scale policy (tfvideo/linear.py:189-216).
  ops     norm_mod / gate_add / swiglu / gelu (tfvideo/kernels.py:15-84),
          QK-RMSNorm + split-half RoPE (call tfvideo/minimax_h3.py:296-298),
          modulation and row index (tfvideo/minimax_h3.py:252-269),
          NVFP4 fake-quant linear, FP8 attention recipe
          (tfvideo/fp4attn.py:82-147,170-238) and fp32 SDPA.
  block   one DiT block forward in the order of tfvideo/minimax_h3.py:275-324.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Triton kernels
(``tfvideo/kernels.py``, ``tfvideo/fp4attn.py``) under ``TRITON_INTERPRET=1`` in
the build container and commits the outputs as fixtures; ``tests/test_oracle.py``
checks this package against them.  TensorFold's activation quantiser and
comfy-kitchen's RoPE are absent from the reference tree, so their exact bits are
pinned only through the in-tree arithmetic they are called with: the quantiser of
tfvideo/fp4attn.py:52-78 under the linear path's per-tensor scale, and the
split-half RoPE convention stated in ops.py.
"""
