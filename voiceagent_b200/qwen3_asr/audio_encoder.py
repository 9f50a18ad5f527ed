"""Qwen3-ASR audio tower, batched across requests (models/audio_encoder.py).

Differences from the reference, all numerically neutral: the chunk padding is the
``audio_chunk_pad`` kernel instead of a Python loop, q/k/v are one fused projection
(``qkv_proj`` = [q | k | v] rows, loaded from the checkpoint's three tensors), the
positional add and the valid-token gather are one ``audio_gather_pos`` kernel over
host-known indices instead of a boolean mask (no device sync), and window attention is
the tcgen05 ``varlen_attention`` kernel.

The convolutional downsampler runs on this library's kernels (csrc/conv.cu): conv2d1
(one input channel) as a direct stencil, conv2d2 and conv2d3 as tcgen05 implicit GEMMs,
each with its bias and GELU fused and the reference's roundings, on channels-last
activations over all chunks of the batch at once. conv2d3 writes its pixels in the
order conv_out reads them (per chunk, time-major rows of (frequency, channel)), so
conv_out multiplies by its weight with the columns permuted to match -- no transpose
copy. The modules keep the checkpoint's parameters; ``prepare_kernels`` repacks them.
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

    @torch.inference_mode()
    def prepare_kernels(self) -> None:
        """Repack the convolution weights for csrc/conv.cu and permute conv_out's columns
        from the reference's (channel, frequency) order to the (frequency, channel) order
        conv2d3 writes. Call after the weights are loaded."""
        self._conv_packed = [kx.conv_pack_weight(c.weight.detach().contiguous())
                             for c in (self.conv2d1, self.conv2d2, self.conv2d3)]
        w = self.conv_out.weight.detach()
        c = self.config.downsample_hidden_size
        freq = w.shape[1] // c
        self._conv_out_fc = w.view(w.shape[0], c, freq).transpose(1, 2).reshape(w.shape[0], -1) \
            .contiguous()

    def _downsample(self, padded: torch.Tensor, num_chunks: int) -> torch.Tensor:
        """[chunks, mel bins, frames] -> conv_out embeddings [chunks, tokens, d_model]."""
        if getattr(self, "_conv_packed", None) is None:
            self.prepare_kernels()
        c = self.config.downsample_hidden_size
        convs = (self.conv2d1, self.conv2d2, self.conv2d3)
        x = padded.unsqueeze(-1)  # channels-last with one channel
        for i, (conv, packed) in enumerate(zip(convs, self._conv_packed)):
            x = kx.conv3x3s2_gelu(x, packed, conv.bias.detach(), c_out=c,
                                  out_order="nxyc" if i == 2 else "nyxc")
        n, t, f, _ = x.shape
        return x.view(n, t, f * c) @ self._conv_out_fc.T

    @torch.inference_mode()
    def warm_up(self) -> None:
        """Repack the convolution weights and run the front once, at engine start."""
        self.prepare_kernels()
        p = next(self.parameters())
        self._downsample(torch.zeros(1, self.config.num_mel_bins, self.chunk_frames,
                                     dtype=p.dtype, device=p.device), 1)

    @torch.inference_mode()
    def forward(self, batch: PackedAudioBatch) -> torch.Tensor:
        """Encode a packed batch into (total audio tokens, output_dim)."""
        padded = torch.empty(batch.num_chunks, self.config.num_mel_bins, self.chunk_frames,
                             dtype=batch.mel.dtype, device=batch.mel.device)
        kx.audio_chunk_pad(batch.mel, batch.chunk_start, batch.chunk_lengths, batch.num_chunks,
                           self.chunk_frames, padded)
        embed = self._downsample(padded, batch.num_chunks)
        t = batch.token_index.numel()
        # positional add + valid-token gather in one kernel, into a bucketed row count
        # (shape-stable GEMMs); rows t.. are zeros that attention never reads (cu_seqlens
        # covers the first t) and that are dropped at the end
        pos = self.positional_embedding[: embed.shape[1]].to(embed.dtype).contiguous()
        hidden = kx.audio_gather_pos(embed, pos, batch.token_index, padded_rows(t))
        for layer in self.layers:
            hidden = layer(hidden, batch.cu_seqlens, batch.max_seqlen)
        hidden = self.ln_post(hidden[:t])
        return self.proj2(F.gelu(self.proj1(hidden)))
