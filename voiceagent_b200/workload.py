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
