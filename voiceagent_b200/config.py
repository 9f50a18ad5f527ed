"""Engine and model configuration, read straight from a Qwen3-ASR checkpoint directory.

Mirrors ``qwen_asr_vllm/config.py``: ``config.json`` (``thinker_config`` with
``audio_config`` / ``text_config``) and ``generation_config.json`` (stop ids) are
parsed directly, without requiring the model type to be registered in transformers.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, fields
from typing import Any

import torch


def resolve_dtype(value) -> torch.dtype:
    if isinstance(value, torch.dtype):
        return value
    if value is None:
        return torch.bfloat16
    dtype = getattr(torch, str(value), None)
    if not isinstance(dtype, torch.dtype):
        raise ValueError(f"unsupported dtype: {value!r}")
    return dtype


def _known(cls, raw: dict[str, Any]) -> dict[str, Any]:
    names = {f.name for f in fields(cls)}
    return {k: v for k, v in raw.items() if k in names}


@dataclass
class AudioEncoderConfig:
    num_mel_bins: int = 128
    d_model: int = 896
    encoder_layers: int = 18
    encoder_attention_heads: int = 14
    encoder_ffn_dim: int = 3584
    downsample_hidden_size: int = 480
    output_dim: int = 1024
    n_window: int = 50
    n_window_infer: int = 800
    conv_chunksize: int = 500
    max_source_positions: int = 1500
    activation_function: str = "gelu"

    @property
    def head_dim(self) -> int:
        return self.d_model // self.encoder_attention_heads

    @property
    def chunk_frames(self) -> int:
        return self.n_window * 2

    @classmethod
    def from_dict(cls, raw: dict[str, Any]) -> "AudioEncoderConfig":
        return cls(**_known(cls, raw))


@dataclass
class TextConfig:
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 65536
    tie_word_embeddings: bool = True
    attention_bias: bool = False
    hidden_act: str = "silu"

    @classmethod
    def from_dict(cls, raw: dict[str, Any]) -> "TextConfig":
        return cls(**_known(cls, raw))


@dataclass
class Qwen3ASRConfig:
    audio: AudioEncoderConfig
    text: TextConfig
    audio_token_id: int = 151676
    audio_start_token_id: int = 151669
    audio_end_token_id: int = 151670
    dtype: torch.dtype = torch.bfloat16
    support_languages: list[str] = field(default_factory=list)
    stop_token_ids: list[int] = field(default_factory=list)

    @classmethod
    def from_pretrained(cls, model_path: str) -> "Qwen3ASRConfig":
        path = os.path.join(model_path, "config.json")
        if not os.path.isfile(path):
            raise FileNotFoundError(f"config.json not found under {model_path}")
        with open(path, encoding="utf-8") as handle:
            raw = json.load(handle)
        thinker = raw.get("thinker_config", raw)
        stop: list[int] = []
        gen_path = os.path.join(model_path, "generation_config.json")
        if os.path.isfile(gen_path):
            with open(gen_path, encoding="utf-8") as handle:
                eos = json.load(handle).get("eos_token_id")
            if eos is not None:
                stop = [int(eos)] if isinstance(eos, int) else [int(e) for e in eos]
        return cls(
            audio=AudioEncoderConfig.from_dict(thinker["audio_config"]),
            text=TextConfig.from_dict(thinker["text_config"]),
            audio_token_id=int(thinker["audio_token_id"]),
            audio_start_token_id=int(thinker["audio_start_token_id"]),
            audio_end_token_id=int(thinker["audio_end_token_id"]),
            dtype=resolve_dtype(thinker.get("dtype") or raw.get("dtype")),
            support_languages=list(raw.get("support_languages", [])),
            stop_token_ids=stop,
        )


@dataclass
class EngineConfig:
    """Runtime knobs of :class:`voiceagent_b200.engine.AsrEngine` (same names and
    defaults as the reference's ``EngineConfig``, config.py:126-204)."""

    model: str
    max_model_len: int = 4096
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 8192
    max_audio_batch_frames: int = 48000
    max_audio_batch_size: int = 32
    gpu_memory_utilization: float = 0.85
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    enable_prefix_cache: bool = True
    enforce_eager: bool = False
    frontend_threads: int = 8
    # "gpu": log-mel on the GPU at encode time (b200asr_log_mel); "cpu": the host
    # Whisper extractor per request, as the reference does.
    frontend: str = "gpu"
    # Programmatic dependent launch between the decode-path kernels (overlaps each
    # kernel's launch and prologue with its predecessor, also inside CUDA graphs).
    pdl: bool = True
    # Decode steps per CUDA-graph call when every running request can take them: the
    # graph is replayed back to back with the sampled tokens fed back on the device and
    # the host syncs once per call (1 = one host round trip per token).
    decode_steps: int = 4
    # Decode-sized batches (<= 64 rows) on the fused projections: each RMSNorm split
    # across the projections around it, q/k norm + RoPE + KV store in qkv_proj's
    # epilogue (five launches per decoder layer instead of eight).
    fused_decode: bool = True
    # Fused decode steps: each layer's gate_up kernel requests the next layer's cached
    # K/V and its qkv / o_proj weights into L2 (the block tables are fixed for the step),
    # to move that HBM traffic out of the attention window into the MLP's. Off: measured
    # 983 vs 952 us per 32-row 0.6B step (weights alone 953, K/V alone 975).
    l2_prefetch: bool = False
    device: str = "cuda"
    dtype: Any = None
    model_config: Qwen3ASRConfig | None = None

    def __post_init__(self):
        if self.decode_steps < 1:
            raise ValueError("decode_steps must be >= 1")
        if self.frontend not in ("gpu", "cpu"):
            raise ValueError(f"frontend must be 'gpu' or 'cpu', got {self.frontend!r}")
        if self.num_kvcache_blocks == 0 or self.num_kvcache_blocks < -1:
            raise ValueError("num_kvcache_blocks must be -1 or positive")
        if self.model_config is None:
            if not os.path.isdir(self.model):
                raise NotADirectoryError(f"model path is not a directory: {self.model}")
            self.model_config = Qwen3ASRConfig.from_pretrained(self.model)
        if self.kvcache_block_size % 256 != 0:
            raise ValueError("kvcache_block_size must be a multiple of 256")
        self.dtype = resolve_dtype(self.dtype or self.model_config.dtype)
        if self.dtype != torch.bfloat16:
            raise ValueError("the b200asr kernels compute in bf16; dtype must be bfloat16")
        self.max_model_len = min(self.max_model_len,
                                 self.model_config.text.max_position_embeddings)
        if self.max_num_batched_tokens < self.max_model_len:
            raise ValueError("max_num_batched_tokens must be >= max_model_len so that a single "
                             "request can always be prefilled")
