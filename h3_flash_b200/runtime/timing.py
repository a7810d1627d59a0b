"""Opt-in CUDA-event timing of the block's sections (attention, all-to-all, elementwise, GEMM).

Disabled by default (one attribute check per section). When enabled, each
section records a start/end event pair on the current stream of its device, so
the measured time is the device time of the kernels that section launched.
"""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch


class SectionTimer:
    def __init__(self) -> None:
        self.enabled = False
        self.records: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = defaultdict(list)

    def reset(self) -> None:
        self.records = defaultdict(list)

    @contextmanager
    def section(self, name: str):
        if not self.enabled:
            yield
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self.records[name].append((start, end))

    def milliseconds(self) -> dict[str, list[float]]:
        """Per-section list of durations (ms). Synchronises on the recorded events."""

        result: dict[str, list[float]] = {}
        for name, pairs in self.records.items():
            values = []
            for start, end in pairs:
                end.synchronize()
                values.append(start.elapsed_time(end))
            result[name] = values
        return result


TIMER = SectionTimer()
