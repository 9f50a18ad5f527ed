"""Qwen3-ASR audio tower, batched across requests (models/audio_encoder.py).

Differences from the reference, all numerically neutral: the chunk padding is the
``audio_chunk_pad`` kernel instead of a Python loop, q/k/v are one fused projection
(``qkv_proj`` = [q | k | v] rows, loaded from the checkpoint's three tensors), the
valid-token gather uses host-known indices instead of a boolean mask (no device
sync), and window attention is the tcgen05 ``varlen_attention`` kernel.
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

    def _downsample(self, padded: torch.Tensor) -> torch.Tensor:
        outs = []
        for part in padded.split(self.config.conv_chunksize, dim=0):
            h = F.gelu(self.conv2d1(part))
            h = F.gelu(self.conv2d2(h))
            outs.append(F.gelu(self.conv2d3(h)))
        x = torch.cat(outs, dim=0) if len(outs) > 1 else outs[0]
        n, c, f, t = x.shape
        return self.conv_out(x.permute(0, 3, 1, 2).reshape(n, t, c * f))

    @torch.inference_mode()
    def forward(self, batch: PackedAudioBatch) -> torch.Tensor:
        """Encode a packed batch into (total audio tokens, output_dim)."""
        padded = torch.empty(batch.num_chunks, self.config.num_mel_bins, self.chunk_frames,
                             dtype=batch.mel.dtype, device=batch.mel.device)
        kx.audio_chunk_pad(batch.mel, batch.chunk_start, batch.chunk_lengths, batch.num_chunks,
                           self.chunk_frames, padded)
        embed = self._downsample(padded.unsqueeze(1))
        embed = embed + self.positional_embedding[: embed.shape[1]].unsqueeze(0).to(embed.dtype)
        hidden = embed.reshape(-1, embed.shape[-1]).index_select(0, batch.token_index)
        for layer in self.layers:
            hidden = layer(hidden, batch.cu_seqlens, batch.max_seqlen)
        hidden = self.ln_post(hidden)
        return self.proj2(F.gelu(self.proj1(hidden)))
