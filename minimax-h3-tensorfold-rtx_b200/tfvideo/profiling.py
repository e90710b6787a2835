"""Per-stage CUDA-event timing of engine blocks (the B200 counterpart of tools/profile_block.py:75-82).

``StageTimer`` records a start / end event pair on the current stream around each named stage; ``summary()``
synchronises once and returns total milliseconds and call counts per stage.
"""

from __future__ import annotations

import contextlib
from collections import defaultdict

import torch


class StageTimer:
    def __init__(self):
        self.spans = defaultdict(list)
        self.enabled = True

    @contextlib.contextmanager
    def span(self, name: str):
        if not self.enabled:
            yield
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            self.spans[name].append((a, b))

    def clear(self):
        self.spans.clear()

    def summary(self) -> dict:
        torch.cuda.synchronize()
        return {k: {"ms": sum(a.elapsed_time(b) for a, b in v), "calls": len(v)} for k, v in self.spans.items()}


def maybe(timer: StageTimer | None, name: str):
    return contextlib.nullcontext() if timer is None else timer.span(name)
