"""Per-phase timing of one training step (verifier, draft forward, head, backward, optimizer).

``train(..., phases=PhaseTimer(device))`` marks the phase boundaries as it runs. On
CUDA the marks are events on the launching stream, so the durations are device time
and marking never waits. On CPU they are wall-clock stamps. ``summary()`` synchronises
once and returns ``{phase: ms}``; a phase that did not run (no verifier, no optimizer)
is absent.
"""

from __future__ import annotations

import time

import torch


class PhaseTimer:
    def __init__(self, device=None):
        self.cuda = device is not None and torch.device(device).type == "cuda"
        self.marks = []  # (name, event or seconds)
        self.mark("start")

    def mark(self, name):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))
        else:
            self.marks.append((name, time.perf_counter()))

    def summary(self) -> dict:
        if self.cuda:
            self.marks[-1][1].synchronize()
        out = {}
        for (_, a), (name, b) in zip(self.marks, self.marks[1:]):
            ms = a.elapsed_time(b) if self.cuda else (b - a) * 1000.0
            out[name] = out.get(name, 0.0) + ms
        return out
