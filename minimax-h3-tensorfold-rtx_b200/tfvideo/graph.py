"""CUDA-graph capture of a whole denoising step (all DiT blocks) of a MiniMaxH3Engine.

A step after the first forward of a sampling run uses delayed activation scales: the scale update runs on the
device (``h3_scales_begin``), every buffer is resident and nothing reads the device from the host, so the 13 kernels
per block can be recorded once and replayed.  The reference removes its per-call host syncs the same way, batching
the scale read-back into one sync per forward (tfvideo/minimax_h3.py:220-235, tfvideo/linear.py:189-216).  The graph
reads its inputs from its own static tensors: copy the step's latents into ``graph.x`` and its timestep embedding into
``graph.t_emb``, call ``replay()``, and read the result from ``graph.x`` (updated in place, as EngineBlock does).

Single-GPU engines only: the Ulysses path's collectives are not recorded here.
"""

from __future__ import annotations

import torch


class StepGraph:
    def __init__(self, engine, x: torch.Tensor, t_emb: torch.Tensor, mod_segments, rope_freqs: torch.Tensor):
        if engine.sp is not None:
            raise ValueError("StepGraph: sequence-parallel engines are not captured")
        if not engine.delayed_scales:
            raise ValueError("StepGraph: needs delayed activation scales (TFVIDEO_DELAYED_SCALES != 0)")
        self.engine = engine
        self.x = x.detach().clone()
        self.t_emb = t_emb.detach().to(device=x.device, dtype=torch.float32).clone()
        self.rope = rope_freqs.detach().to(device=x.device, dtype=torch.float32).contiguous()
        self.mod_segments = mod_segments
        # one eager forward on a scratch copy when the run has none yet, so the captured forward is a delayed-scale
        # one; it also fills the engine's buffers and its row-index cache (nothing is allocated during capture)
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            if engine._forwards == 0:
                engine.forward(self.x.clone(), self.t_emb, mod_segments, self.rope)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            engine.forward(self.x, self.t_emb, self.mod_segments, self.rope)
        # capture recorded the forward without running it: the run's forward count moved on by one, which the first
        # replay makes true

    def replay(self) -> torch.Tensor:
        self.engine._forwards += 1   # each replay is one more delayed-scale forward of the run
        self.graph.replay()
        return self.x
