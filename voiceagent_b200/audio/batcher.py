"""Cross-request packing for the audio encoder (audio/batcher.py of the reference).

The host computes only scalars from the closed-form accounting (chunk, window and
token counts); per-chunk lengths, chunk starts, valid lengths and the window
``cu_seqlens`` are built on the GPU by the ``pack_audio`` kernel from one int32 per
request. As in the reference, chunks are always padded to ``chunk_frames`` and the
window is ``TOKENS_PER_FULL_CHUNK * (n_window_infer // chunk_frames)`` tokens, so the
encoder output does not depend on how requests were grouped.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from voiceagent_b200 import kernels as kx
from voiceagent_b200.profiling import TRANSFERS
from voiceagent_b200.audio.tokens import (CHUNK_FRAMES, TOKENS_PER_FULL_CHUNK, after_cnn_len,
                                          attention_window_tokens, num_audio_tokens, num_chunks,
                                          num_windows)


@dataclass
class PackedAudioBatch:
    mel: torch.Tensor               # (num_mel_bins, sum(frames)) bf16, device
    chunk_lengths: torch.Tensor     # i64 [C]
    chunk_valid_lens: torch.Tensor  # i64 [C]
    chunk_start: torch.Tensor       # i32 [C] first frame of each chunk in `mel`
    cu_seqlens: torch.Tensor        # i32 [W + 1] attention windows over packed tokens
    token_index: torch.Tensor       # i64 [T] rows of the (C * 13)-row conv output kept
    audio_token_lens: list[int]
    window_tokens: int
    max_seqlen: int
    num_chunks: int

    @property
    def total_tokens(self) -> int:
        return sum(self.audio_token_lens)

    def split_outputs(self, packed: torch.Tensor) -> list[torch.Tensor]:
        if packed.size(0) != self.total_tokens:
            raise ValueError(f"encoder returned {packed.size(0)} tokens, expected {self.total_tokens}")
        return list(torch.split(packed, self.audio_token_lens, dim=0))


def pack_audio_batch(items: list, n_window_infer: int, device, chunk_frames: int = CHUNK_FRAMES,
                     renderer=None, error_flag: torch.Tensor | None = None) -> PackedAudioBatch:
    """Pack per-request features into one encoder batch.

    Each item is a mel tensor ``(bins, frames)`` or an ``AudioFeatures``; features whose
    mel is still deferred (``mel is None``, waveform attached) are rendered on the GPU by
    ``renderer`` (a ``GpuMelFrontend``) straight into the packed bf16 input.
    """
    if not items:
        raise ValueError("pack_audio_batch requires at least one request")
    mels = [it if isinstance(it, torch.Tensor) else it.mel for it in items]
    frames = [int(it.shape[-1]) if isinstance(it, torch.Tensor) else int(it.mel_frames)
              for it in items]
    window = attention_window_tokens(n_window_infer, chunk_frames)
    tokens = [num_audio_tokens(f, chunk_frames) for f in frames]
    n_chunks = sum(num_chunks(f, chunk_frames) for f in frames)
    n_windows = sum(num_windows(t, window) for t in tokens)
    max_seqlen = max(min(t, window) for t in tokens)

    # Valid rows of the padded conv output, chunk by chunk (13 rows per chunk).
    valid = []
    for f in frames:
        full, tail = divmod(f, chunk_frames)
        valid.extend([TOKENS_PER_FULL_CHUNK] * full)
        if tail:
            valid.append(after_cnn_len(tail))
    valid_np = np.asarray(valid, dtype=np.int64)
    base = np.repeat(np.arange(len(valid_np), dtype=np.int64) * TOKENS_PER_FULL_CHUNK, valid_np)
    offs = np.arange(base.size, dtype=np.int64) - np.repeat(np.cumsum(valid_np) - valid_np, valid_np)
    token_index = torch.from_numpy(base + offs).pin_memory().to(device, non_blocking=True)
    TRANSFERS["h2d"] += 8 * int(token_index.numel()) + 4 * len(frames) + sum(
        m.numel() * m.element_size() for m in mels if m is not None and not m.is_cuda)

    if all(m is not None for m in mels):
        mel = torch.cat([m.to(device, non_blocking=True) for m in mels], dim=-1)
        if mel.dtype != torch.bfloat16:
            mel = mel.to(torch.bfloat16)
        mel = mel.contiguous()
    else:
        if renderer is None:
            raise ValueError("deferred mel features need a GPU frontend to render them")
        bins = next((int(m.shape[0]) for m in mels if m is not None), renderer.num_mel_bins)
        cols = np.concatenate([[0], np.cumsum(frames)]).astype(np.int64)
        mel = torch.empty(bins, int(cols[-1]), dtype=torch.bfloat16, device=device)
        deferred, where = [], []
        for i, m in enumerate(mels):
            if m is None:
                deferred.append(items[i])
                where.append(int(cols[i]))
            else:
                mel[:, cols[i]:cols[i + 1]].copy_(m.to(device, non_blocking=True))
        TRANSFERS["h2d"] += renderer.render(deferred, mel, where, error_flag)
    mel_frames = torch.tensor(frames, dtype=torch.int32).pin_memory().to(device, non_blocking=True)
    out = {
        "chunk_lengths": torch.empty(n_chunks, dtype=torch.int64, device=device),
        "chunk_valid_lens": torch.empty(n_chunks, dtype=torch.int64, device=device),
        "chunk_start": torch.empty(n_chunks, dtype=torch.int32, device=device),
        "audio_token_lens": torch.empty(len(frames), dtype=torch.int32, device=device),
        "cu_seqlens": torch.empty(n_windows + 1, dtype=torch.int32, device=device),
        "counts": torch.empty(3, dtype=torch.int32, device=device),
    }
    kx.pack_audio(mel_frames, chunk_frames=chunk_frames, window_tokens=window,
                  max_chunks=n_chunks, max_windows=n_windows, out=out)
    return PackedAudioBatch(
        mel=mel, chunk_lengths=out["chunk_lengths"], chunk_valid_lens=out["chunk_valid_lens"],
        chunk_start=out["chunk_start"], cu_seqlens=out["cu_seqlens"], token_index=token_index,
        audio_token_lens=tokens, window_tokens=window, max_seqlen=max_seqlen,
        num_chunks=n_chunks)
