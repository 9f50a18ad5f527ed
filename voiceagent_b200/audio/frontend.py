"""Waveform -> log-mel features on the host (audio/frontend.py of the reference).

Qwen3-ASR uses a stock Whisper extractor (128 bins, hop 160, n_fft 400, 16 kHz).
Features are computed one request at a time so a request's frame count never
depends on what it was batched with.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from voiceagent_b200.audio.tokens import num_audio_tokens

TARGET_SAMPLE_RATE = 16000


@dataclass
class AudioFeatures:
    mel: torch.Tensor  # (num_mel_bins, mel_frames), unpadded
    mel_frames: int
    num_audio_tokens: int
    audio_seconds: float


class AudioFrontend:
    def __init__(self, model_path: str | None = None, dtype: torch.dtype = torch.float32):
        from transformers import WhisperFeatureExtractor

        cfg = os.path.join(model_path, "preprocessor_config.json") if model_path else None
        if cfg and os.path.isfile(cfg):
            self.extractor = WhisperFeatureExtractor.from_pretrained(model_path)
        else:
            self.extractor = WhisperFeatureExtractor(feature_size=128, sampling_rate=16000,
                                                     hop_length=160, n_fft=400)
        if self.extractor.sampling_rate != TARGET_SAMPLE_RATE:
            raise ValueError(f"expected a {TARGET_SAMPLE_RATE} Hz extractor")
        self.dtype = dtype

    @property
    def num_mel_bins(self) -> int:
        return self.extractor.feature_size

    @property
    def hop_length(self) -> int:
        return self.extractor.hop_length

    def __call__(self, waveform: np.ndarray, sample_rate: int = TARGET_SAMPLE_RATE) -> AudioFeatures:
        audio = np.asarray(waveform)
        if audio.ndim > 1:
            audio = audio.mean(axis=-1)
        audio = audio.astype(np.float32, copy=False)
        if sample_rate != TARGET_SAMPLE_RATE:
            raise ValueError(f"resample to {TARGET_SAMPLE_RATE} Hz first (got {sample_rate})")
        if audio.size < self.hop_length:
            raise ValueError(f"audio is too short to produce a mel frame ({audio.size} samples)")
        feats = self.extractor([audio], sampling_rate=TARGET_SAMPLE_RATE, padding=False,
                               truncation=False, return_attention_mask=True, return_tensors="pt")
        frames = int(feats["attention_mask"][0].sum())
        mel = feats["input_features"][0][:, :frames].to(self.dtype).contiguous()
        return AudioFeatures(mel=mel, mel_frames=frames, num_audio_tokens=num_audio_tokens(frames),
                             audio_seconds=audio.size / TARGET_SAMPLE_RATE)
