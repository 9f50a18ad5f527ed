"""Closed-form audio token accounting (audio/tokens.py of the reference).

The audio token count of a request is a function of its mel frame count alone, so
the scheduler can size KV blocks before the encoder runs: 100-frame chunks, three
stride-2 convolutions, 13 tokens per full chunk.
"""

from __future__ import annotations

CHUNK_FRAMES = 100


def conv_output_len(length: int) -> int:
    """Output length of one Conv2d(kernel 3, stride 2, padding 1)."""
    return (length - 1) // 2 + 1


def after_cnn_len(frames: int) -> int:
    return conv_output_len(conv_output_len(conv_output_len(frames)))


TOKENS_PER_FULL_CHUNK = after_cnn_len(CHUNK_FRAMES)  # 13


def num_audio_tokens(mel_frames: int, chunk_frames: int = CHUNK_FRAMES) -> int:
    full, tail = divmod(mel_frames, chunk_frames)
    return full * after_cnn_len(chunk_frames) + (after_cnn_len(tail) if tail else 0)


def num_chunks(mel_frames: int, chunk_frames: int = CHUNK_FRAMES) -> int:
    if mel_frames <= 0:
        raise ValueError(f"mel_frames must be positive, got {mel_frames}")
    return -(-mel_frames // chunk_frames)


def chunk_lengths_for(mel_frames: int, chunk_frames: int = CHUNK_FRAMES) -> list[int]:
    if mel_frames <= 0:
        raise ValueError(f"mel_frames must be positive, got {mel_frames}")
    full, tail = divmod(mel_frames, chunk_frames)
    return [chunk_frames] * full + ([tail] if tail else [])


def attention_window_tokens(n_window_infer: int, chunk_frames: int = CHUNK_FRAMES) -> int:
    return TOKENS_PER_FULL_CHUNK * (n_window_infer // chunk_frames)


def num_windows(audio_tokens: int, window_tokens: int) -> int:
    return -(-audio_tokens // window_tokens)
