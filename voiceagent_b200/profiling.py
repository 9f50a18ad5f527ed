"""Stage timing with CUDA events, off unless enabled (profiling.py of the reference).

Events are recorded in the stream and read only in ``collect``, so timing the
device never serialises the host against it mid-run.
"""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch


class StageTimer:
    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self._totals: dict[str, float] = defaultdict(float)
        self._counts: dict[str, int] = defaultdict(int)

    @contextmanager
    def phase(self, name: str):
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
            self._pending.append((name, start, end))

    def collect(self) -> None:
        if not self._pending:
            return
        torch.cuda.synchronize()
        for name, start, end in self._pending:
            self._totals[name] += start.elapsed_time(end) / 1000.0
            self._counts[name] += 1
        self._pending.clear()

    @property
    def totals(self) -> dict[str, float]:
        self.collect()
        return dict(self._totals)

    @property
    def counts(self) -> dict[str, int]:
        self.collect()
        return dict(self._counts)

    def reset(self) -> None:
        self._pending.clear()
        self._totals.clear()
        self._counts.clear()


NULL_TIMER = StageTimer(enabled=False)

# Bytes the engine moves between host and device (batch descriptors, mel features,
# token ids); read by benchmarks to report per-step transfer volume.
TRANSFERS = {"h2d": 0, "d2h": 0}
