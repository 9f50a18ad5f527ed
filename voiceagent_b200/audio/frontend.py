"""Waveform -> log-mel features (audio/frontend.py of the reference).

Qwen3-ASR uses a stock Whisper extractor (128 bins, hop 160, n_fft 400, 16 kHz).
Features are computed one request at a time so a request's frame count never
depends on what it was batched with.

``AudioFrontend`` runs that extractor on the host, as the reference does.
``GpuMelFrontend`` defers the work: a request keeps its waveform (its frame and
token counts are closed-form in the sample count) until its encode batch, where the
batch's clips cross to the GPU in one pinned copy and ``b200asr_log_mel`` writes the
bf16 features straight into the encoder's packed input. A clip can be staged into
pinned memory earlier (``GpuMelFrontend.stage``, which the engine calls while the GPU
runs a decoder step); its encode batch then copies it to the device directly.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np
import torch

from voiceagent_b200.audio.tokens import num_audio_tokens

TARGET_SAMPLE_RATE = 16000


@dataclass
class AudioFeatures:
    mel: torch.Tensor | None  # (num_mel_bins, mel_frames), unpadded; None until rendered
    mel_frames: int
    num_audio_tokens: int
    audio_seconds: float
    waveform: np.ndarray | None = None  # 16 kHz float32 samples awaiting the GPU frontend
    # the samples copied into pinned host memory ahead of the encode batch
    # (GpuMelFrontend.stage), so that batch crosses to the GPU without a host copy
    staged: torch.Tensor | None = field(default=None, repr=False, compare=False)


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


class GpuMelFrontend:
    """Deferred Whisper log-mel: ``__call__`` only validates the clip and counts its
    frames (``n // 160``); ``render`` computes the features of an encode batch on the GPU.

    The extractor's filterbank (``[201, 128]``, cast to fp32 exactly as its torch path
    does), the periodic Hann window and a 400-entry cos/sin table are uploaded once.
    """

    N_FFT, HOP, BINS = 400, 160, 128

    def __init__(self, model_path: str | None = None, device="cuda"):
        host = AudioFrontend(model_path)
        ext = host.extractor
        if (ext.n_fft, ext.hop_length, ext.feature_size) != (self.N_FFT, self.HOP, self.BINS):
            raise ValueError("the GPU frontend implements n_fft 400, hop 160, 128 mel bins")
        self.extractor = ext
        self.device = torch.device(device)
        filters = np.asarray(ext.mel_filters, dtype=np.float64).astype(np.float32)  # [201, 128]
        nonzero = filters != 0
        first = nonzero.argmax(axis=0)
        count = nonzero.sum(axis=0)
        for m in range(filters.shape[1]):  # each filter is one contiguous run of bins
            if count[m] and not nonzero[first[m]:first[m] + count[m], m].all():
                raise ValueError(f"mel filter {m} is not a contiguous band")
        ranges = np.stack([first, count], axis=1).astype(np.int32)
        angle = 2.0 * np.pi * np.arange(self.N_FFT, dtype=np.float64) / self.N_FFT
        window = torch.hann_window(self.N_FFT, dtype=torch.float32).numpy()
        tables = np.concatenate([window, np.cos(angle).astype(np.float32),
                                 np.sin(angle).astype(np.float32)])
        self.tables = torch.from_numpy(tables).to(self.device)
        self.filters = torch.from_numpy(np.ascontiguousarray(filters)).to(self.device)
        self.filter_range = torch.from_numpy(ranges).to(self.device)
        self.dtype = torch.bfloat16

    @property
    def num_mel_bins(self) -> int:
        return self.BINS

    @property
    def hop_length(self) -> int:
        return self.HOP

    def __call__(self, waveform: np.ndarray, sample_rate: int = TARGET_SAMPLE_RATE) -> AudioFeatures:
        audio = np.asarray(waveform)
        if audio.ndim > 1:
            audio = audio.mean(axis=-1)
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        if sample_rate != TARGET_SAMPLE_RATE:
            raise ValueError(f"resample to {TARGET_SAMPLE_RATE} Hz first (got {sample_rate})")
        if audio.size <= self.N_FFT // 2:
            raise ValueError(f"audio is too short for the centred STFT ({audio.size} samples; "
                             f"needs more than {self.N_FFT // 2})")
        frames = audio.size // self.HOP
        return AudioFeatures(mel=None, mel_frames=frames, num_audio_tokens=num_audio_tokens(frames),
                             audio_seconds=audio.size / TARGET_SAMPLE_RATE, waveform=audio)

    def stage(self, features: AudioFeatures) -> bool:
        """Copy a deferred clip's samples into pinned host memory now, ahead of its encode
        batch. Returns whether it copied (False: not deferred, already staged, or no GPU)."""
        if (self.device.type != "cuda" or features.waveform is None or features.mel is not None
                or features.staged is not None):
            return False
        staged = torch.empty(features.waveform.size, dtype=torch.float32, pin_memory=True)
        staged.copy_(torch.from_numpy(features.waveform))
        features.staged = staged
        return True

    def render(self, features: list[AudioFeatures], out: torch.Tensor, columns: list[int],
               error_flag: torch.Tensor | None = None) -> int:
        """Write the log-mel of every deferred clip into ``out[:, columns[i]:...]``
        (bf16 ``[128, cols]`` on the GPU). Returns the host-to-device bytes copied."""
        from voiceagent_b200 import kernels as kx

        if not features:
            return 0
        lens = np.asarray([f.waveform.size for f in features], dtype=np.int64)
        frames = lens // self.HOP
        total = int(frames.sum())
        n = int(lens.sum())
        b = len(features)
        # one pinned staging buffer: int64 cu_samples, int32 frame starts + columns, then
        # the samples at a 16-byte boundary
        meta_i64 = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        meta_i32 = np.concatenate([np.concatenate([[0], np.cumsum(frames)]),
                                   np.asarray(columns, dtype=np.int64)]).astype(np.int32)
        wave_at = (meta_i64.nbytes + meta_i32.nbytes + 15) // 16 * 16
        host = torch.empty(wave_at + n * 4, dtype=torch.uint8, pin_memory=self.device.type == "cuda")
        hv = host.numpy()
        hv[:meta_i64.nbytes] = meta_i64.view(np.uint8)
        hv[meta_i64.nbytes:meta_i64.nbytes + meta_i32.nbytes] = meta_i32.view(np.uint8)
        # the samples: one torch.cat on the intra-op threads (a 32-clip batch is ~14 MB; a
        # single-threaded numpy copy cost ~2.5 ms of host time per batch, one torch copy
        # per clip ~2 ms), unless clips were staged ahead: those copy from their own
        # pinned buffers, the others through this one
        wave_host = host[wave_at:].view(torch.float32)
        if all(f.staged is None for f in features):
            torch.cat([torch.from_numpy(f.waveform) for f in features], out=wave_host)
            dev = host.to(self.device, non_blocking=True)
        else:
            dev = torch.empty_like(host, device=self.device)
            dev[:wave_at].copy_(host[:wave_at], non_blocking=True)
            wave_dev = dev[wave_at:].view(torch.float32)
            starts = meta_i64.tolist()
            run = None  # [first, end) of clips not staged, copied as one range
            for i, f in enumerate(features + [None]):
                if f is not None and f.staged is None:
                    lo, hi = starts[i], starts[i + 1]
                    wave_host[lo:hi].copy_(torch.from_numpy(f.waveform))
                    run = (run[0] if run else lo, hi)
                    continue
                if run:
                    wave_dev[run[0]:run[1]].copy_(wave_host[run[0]:run[1]], non_blocking=True)
                    run = None
                if f is not None:
                    wave_dev[starts[i]:starts[i + 1]].copy_(f.staged, non_blocking=True)
                    f.staged = None  # the copy holds the pinned block until it has run
        cu_samples = dev[:meta_i64.nbytes].view(torch.int64)
        i32 = dev[meta_i64.nbytes:meta_i64.nbytes + meta_i32.nbytes].view(torch.int32)
        frame_start, out_col = i32[:b + 1], i32[b + 1:]
        wave = dev[wave_at:].view(torch.float32)
        ws = torch.empty(kx.log_mel_workspace_size(b, total), dtype=torch.uint8, device=self.device)
        kx.log_mel(wave, cu_samples, frame_start, total_frames=total, tables=self.tables,
                   mel_filters=self.filters, filter_range=self.filter_range, out=out,
                   out_col=out_col, workspace=ws, error_flag=error_flag)
        return int(host.numel())
