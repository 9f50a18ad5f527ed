"""Device-time accounting per engine phase, and host<->device transfer counters.

``StageTimer`` brackets named phases (audio encode, prefill, decode, ...) with CUDA
events recorded on the current stream. Reading an event's time needs the GPU to have
passed it, so nothing is read while the engine runs: finished brackets queue up and are
resolved together when a total is asked for (one device synchronisation then). A
disabled timer records nothing, so leaving the brackets in the hot path costs nothing
beyond a branch. (The reference engine has a timer for the same purpose,
qwen_asr_vllm/profiling.py.)
"""

from __future__ import annotations

from contextlib import contextmanager

import torch


class StageTimer:
    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self._open: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self._seconds: dict[str, float] = {}
        self._calls: dict[str, int] = {}

    @contextmanager
    def phase(self, name: str):
        """Time the device work issued inside the block under ``name``."""
        if not self.enabled:
            yield
            return
        marks = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        marks[0].record()
        try:
            yield
        finally:
            marks[1].record()
            self._open.append((name, *marks))

    def collect(self) -> None:
        """Resolve every queued bracket into the totals (synchronises the device once)."""
        if not self._open:
            return
        torch.cuda.synchronize()
        for name, begin, end in self._open:
            self._seconds[name] = self._seconds.get(name, 0.0) + begin.elapsed_time(end) / 1e3
            self._calls[name] = self._calls.get(name, 0) + 1
        self._open = []

    @property
    def totals(self) -> dict[str, float]:
        """Seconds of device time per phase."""
        self.collect()
        return dict(self._seconds)

    @property
    def counts(self) -> dict[str, int]:
        """Brackets recorded per phase."""
        self.collect()
        return dict(self._calls)

    def reset(self) -> None:
        self._open, self._seconds, self._calls = [], {}, {}


# Shared by every component that takes a timer but was given none.
NULL_TIMER = StageTimer(enabled=False)

# Bytes the engine moves between host and device (batch descriptors, waveforms and mel
# features, sampled token ids), accumulated by the components that issue the copies;
# benchmarks read the difference over a timed region.
TRANSFERS = {"h2d": 0, "d2h": 0}
