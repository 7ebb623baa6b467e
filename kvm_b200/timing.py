"""Per-launch timing of a layer call with CUDA events.

A layer that takes a `probe` calls probe.mark(name) on its launching stream
before its first launch ("start") and after each launch (the launch's name),
so the interval between two consecutive marks is the device time of the
launch between them. Events are created up front, one set per call, so the
timed calls only record them.
"""
from __future__ import annotations

import statistics

import torch


class PhaseProbe:
    """Events for `calls` layer calls, each marking the names in `phases`
    (the first must be "start") in order."""

    def __init__(self, calls: int, phases: list[str]):
        if not phases or phases[0] != "start":
            raise ValueError("the first phase mark must be 'start'")
        self.phases = list(phases)
        self.ev = [[torch.cuda.Event(enable_timing=True) for _ in phases]
                   for _ in range(calls)]
        self.call = -1
        self.j = 0

    def next_call(self) -> "PhaseProbe":
        self.call += 1
        self.j = 0
        return self

    def mark(self, name: str) -> None:
        if self.phases[self.j] != name:
            raise RuntimeError(f"phase mark {name!r} out of order (expected "
                               f"{self.phases[self.j]!r})")
        self.ev[self.call][self.j].record()
        self.j += 1

    def mean_ms(self) -> dict[str, float]:
        """Mean device time of each launch (phase names after "start") over
        the recorded calls; call after a synchronize."""
        n = self.call + 1
        out = {}
        for j in range(1, len(self.phases)):
            out[self.phases[j]] = statistics.mean(
                self.ev[i][j - 1].elapsed_time(self.ev[i][j]) for i in range(n))
        return out
