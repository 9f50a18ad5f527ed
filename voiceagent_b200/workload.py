"""Seeded synthetic workloads of the benchmark configurations.

No dataset is available offline; these stand in for LibriSpeech-like short clips with
the shapes the benchmark configurations name: 16 kHz mono waveforms of Gaussian noise
(sigma 0.05) plus three sines with frequencies uniform in 200-3000 Hz, amplitude 0.2.
"""

from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000


def synthetic_waveform(seconds: float, rng: np.random.Generator) -> np.ndarray:
    n = int(round(seconds * SAMPLE_RATE))
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    wave = rng.normal(0.0, 0.05, size=n)
    for f in rng.uniform(200.0, 3000.0, size=3):
        wave += 0.2 * np.sin(2.0 * np.pi * f * t)
    return wave.astype(np.float32)


def config0_clip(seed: int = 0) -> np.ndarray:
    """Config 0: one 4.0 s clip from ``default_rng(seed)``."""
    return synthetic_waveform(4.0, np.random.default_rng(seed))


def lognormal_durations(count: int, seed: int = 0, median: float = 7.0, sigma: float = 0.6,
                        lo: float = 1.0, hi: float = 35.0) -> np.ndarray:
    """Config 3/4 durations: lognormal(ln median, sigma) clipped to [lo, hi] seconds."""
    rng = np.random.default_rng(seed)
    return np.clip(rng.lognormal(np.log(median), sigma, size=count), lo, hi)


def config3_clips(count: int = 512, seed: int = 0) -> list[np.ndarray]:
    durations = lognormal_durations(count, seed)
    rng = np.random.default_rng(seed + 1)
    return [synthetic_waveform(float(d), rng) for d in durations]


# ------------------------------------------------------------ routed (shared) jobs
#
# A multi-GPU job is ONE list of requests that the host router splits over the
# replicas (voiceagent_b200.replicas.route_by_duration). Every request's waveform comes
# from its own seeded generator, so a rank synthesises only the requests routed to it
# and the same index always yields the same samples whatever the world size.

LONG_FILE_SECONDS = 1200.0  # config 4: one 20-minute recording ...
LONG_CHUNK_SECONDS = 30.0   # ... submitted as 40 chunks of 30 s together


class Job:
    """A benchmark job: request durations plus the recipe for each request's waveform.

    ``kind`` "config3": ``count`` lognormal clips (median 7 s, sigma 0.6, in [1, 35] s).
    ``kind`` "config4": 4096 such clips plus one 20-minute synthetic recording cut into
    30 s chunks (requests 4096..4135), all submitted together.
    """

    def __init__(self, kind: str, count: int = 512, seed: int = 0):
        if kind not in ("config3", "config4"):
            raise ValueError(f"unknown job kind {kind!r}")
        self.kind, self.seed = kind, seed
        n_clips = count if kind == "config3" else 4096
        durations = list(lognormal_durations(n_clips, seed))
        self.n_clips = n_clips
        if kind == "config4":
            n_chunks = int(LONG_FILE_SECONDS // LONG_CHUNK_SECONDS)
            durations += [LONG_CHUNK_SECONDS] * n_chunks
        self.durations = np.asarray(durations, dtype=np.float64)
        self._long: np.ndarray | None = None

    def __len__(self) -> int:
        return len(self.durations)

    def _long_file(self) -> np.ndarray:
        if self._long is None:
            self._long = synthetic_waveform(LONG_FILE_SECONDS,
                                            np.random.default_rng([self.seed, 1 << 20]))
        return self._long

    def waveform(self, index: int) -> np.ndarray:
        if index < self.n_clips:
            return synthetic_waveform(float(self.durations[index]),
                                      np.random.default_rng([self.seed, index]))
        n = int(round(LONG_CHUNK_SECONDS * SAMPLE_RATE))
        start = (index - self.n_clips) * n
        return self._long_file()[start:start + n].copy()

    def waveforms(self, indices) -> list[np.ndarray]:
        return [self.waveform(int(i)) for i in indices]
