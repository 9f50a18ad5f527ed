"""Qwen3-ASR audio tower, batched across requests (models/audio_encoder.py).

Differences from the reference, all numerically neutral: the chunk padding is the
``audio_chunk_pad`` kernel instead of a Python loop, q/k/v are one fused projection
(``qkv_proj`` = [q | k | v] rows, loaded from the checkpoint's three tensors), the
valid-token gather uses host-known indices instead of a boolean mask (no device
sync), and window attention is the tcgen05 ``varlen_attention`` kernel.

The convolutional downsampler runs on groups of a few fixed sizes (8, 16, 32 or 64
chunks, the last group zero-padded) in channels-last layout. Every encode batch has a
different chunk count, and cuDNN builds an execution plan per new input shape -- tens
of milliseconds of host time that dwarfed the few milliseconds of GPU work; with fixed
group shapes the plans are built once. Chunks are independent through the convolutions
(padding only ever adds whole zero chunks), so the grouping does not change results.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from voiceagent_b200 import kernels as kx
from voiceagent_b200.audio.batcher import PackedAudioBatch
from voiceagent_b200.config import AudioEncoderConfig
from voiceagent_b200.layers.attention import VarlenSelfAttention
from voiceagent_b200.shapes import padded_rows


def sinusoid_table(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    """Whisper-style fixed positions (audio_encoder.py:20-37)."""
    if channels % 2:
        raise ValueError("sinusoid positions need an even channel count")
    inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2, dtype=torch.float32))
    scaled = torch.arange(length, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([torch.sin(scaled), torch.cos(scaled)], dim=1)


class AudioAttention(nn.Module):
    def __init__(self, config: AudioEncoderConfig):
        super().__init__()
        self.embed_dim = config.d_model
        self.num_heads = config.encoder_attention_heads
        self.head_dim = config.head_dim
        self.qkv_proj = nn.Linear(self.embed_dim, 3 * self.embed_dim, bias=True)
        self.out_proj = nn.Linear(self.embed_dim, self.embed_dim, bias=True)
        self.attn = VarlenSelfAttention(self.num_heads, self.head_dim, self.head_dim ** -0.5)

    def forward(self, hidden, cu_seqlens, max_seqlen: int) -> torch.Tensor:
        t = hidden.shape[0]
        qkv = self.qkv_proj(hidden)  # [T, 3 * d]
        d = self.embed_dim
        heads = (self.num_heads, self.head_dim)
        # Strided views into the fused projection: row stride 3 * d, no copies.
        q, k, v = (qkv[:, i * d : (i + 1) * d].unflatten(1, heads) for i in range(3))
        out = self.attn(q, k, v, cu_seqlens, max_seqlen)
        return self.out_proj(out.view(t, d))


class AudioEncoderLayer(nn.Module):
    def __init__(self, config: AudioEncoderConfig):
        super().__init__()
        if config.activation_function != "gelu":
            raise ValueError(f"unsupported audio activation: {config.activation_function}")
        self.self_attn = AudioAttention(config)
        self.self_attn_layer_norm = nn.LayerNorm(config.d_model)
        self.fc1 = nn.Linear(config.d_model, config.encoder_ffn_dim)
        self.fc2 = nn.Linear(config.encoder_ffn_dim, config.d_model)
        self.final_layer_norm = nn.LayerNorm(config.d_model)

    def forward(self, hidden, cu_seqlens, max_seqlen):
        residual = hidden
        hidden = residual + self.self_attn(self.self_attn_layer_norm(hidden), cu_seqlens, max_seqlen)
        residual = hidden
        return residual + self.fc2(F.gelu(self.fc1(self.final_layer_norm(hidden))))


class AudioEncoder(nn.Module):
    def __init__(self, config: AudioEncoderConfig):
        super().__init__()
        self.config = config
        self.chunk_frames = config.chunk_frames
        c = config.downsample_hidden_size
        self.register_buffer("positional_embedding",
                             sinusoid_table(config.max_source_positions, config.d_model),
                             persistent=False)
        self.conv2d1 = nn.Conv2d(1, c, 3, 2, padding=1)
        self.conv2d2 = nn.Conv2d(c, c, 3, 2, padding=1)
        self.conv2d3 = nn.Conv2d(c, c, 3, 2, padding=1)
        freq = (((config.num_mel_bins + 1) // 2 + 1) // 2 + 1) // 2
        self.conv_out = nn.Linear(c * freq, config.d_model, bias=False)
        self.layers = nn.ModuleList([AudioEncoderLayer(config) for _ in range(config.encoder_layers)])
        self.ln_post = nn.LayerNorm(config.d_model)
        self.proj1 = nn.Linear(config.d_model, config.d_model)
        self.proj2 = nn.Linear(config.d_model, config.output_dim)

    CONV_GROUPS = (8, 16, 32, 64)  # chunk counts of the conv launches (shape-stable)

    @classmethod
    def conv_rows(cls, num_chunks: int) -> int:
        """Rows to allocate for ``num_chunks`` chunks: whole fixed-size groups."""
        g = cls.conv_group(num_chunks)
        return -(-num_chunks // g) * g

    @classmethod
    def conv_group(cls, num_chunks: int) -> int:
        return next((g for g in cls.CONV_GROUPS if g >= num_chunks), cls.CONV_GROUPS[-1])

    def _downsample(self, padded: torch.Tensor, num_chunks: int) -> torch.Tensor:
        g = self.conv_group(num_chunks)
        outs = []
        for part in padded.split(g, dim=0):
            h = F.gelu(self.conv2d1(part.contiguous(memory_format=torch.channels_last)))
            h = F.gelu(self.conv2d2(h))
            outs.append(F.gelu(self.conv2d3(h)))
        x = torch.cat(outs, dim=0) if len(outs) > 1 else outs[0]
        x = x[:num_chunks]
        n, c, f, t = x.shape
        return self.conv_out(x.permute(0, 3, 1, 2).reshape(n, t, c * f))

    @torch.inference_mode()
    def warm_up(self) -> None:
        """Build the cuDNN plans of every conv group shape once, at engine start."""
        p = next(self.parameters())
        for g in self.CONV_GROUPS:
            self._downsample(torch.zeros(g, 1, self.config.num_mel_bins, self.chunk_frames,
                                         dtype=p.dtype, device=p.device), g)

    @torch.inference_mode()
    def forward(self, batch: PackedAudioBatch) -> torch.Tensor:
        """Encode a packed batch into (total audio tokens, output_dim)."""
        rows = self.conv_rows(batch.num_chunks)
        padded = torch.empty(rows, self.config.num_mel_bins, self.chunk_frames,
                             dtype=batch.mel.dtype, device=batch.mel.device)
        if rows > batch.num_chunks:
            padded[batch.num_chunks:].zero_()
        kx.audio_chunk_pad(batch.mel, batch.chunk_start, batch.chunk_lengths, batch.num_chunks,
                           self.chunk_frames, padded)
        embed = self._downsample(padded.unsqueeze(1), batch.num_chunks)
        embed = embed + self.positional_embedding[: embed.shape[1]].unsqueeze(0).to(embed.dtype)
        flat = embed.reshape(-1, embed.shape[-1])
        t = batch.token_index.numel()
        # bucketed row count (shape-stable GEMMs); rows t.. are zeros that attention never
        # reads (cu_seqlens covers the first t) and that are dropped at the end
        hidden = flat.new_zeros(padded_rows(t), flat.shape[-1])
        torch.index_select(flat, 0, batch.token_index, out=hidden[:t])
        for layer in self.layers:
            hidden = layer(hidden, batch.cu_seqlens, batch.max_seqlen)
        hidden = self.ln_post(hidden[:t])
        return self.proj2(F.gelu(self.proj1(hidden)))
