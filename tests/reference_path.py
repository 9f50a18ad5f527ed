"""A bf16 GPU restatement of the reference engine's forward, for token parity tests.

Test infrastructure only. It follows qwen-asr-vllm's modules operation by operation
in torch eager -- RMSNorm with its two bf16 roundings (layers/layernorm.py:19-36),
half-split RoPE in fp32 (layers/rotary_embedding.py:9-32), F.silu(gate) * up
(layers/activation.py:11-14), the chunk/pad/conv/windowed-attention encoder
(models/audio_encoder.py:130-189) -- and calls ``flash_attn_varlen_func`` exactly
as layers/attention.py does (no other attention backend: if flash-attn cannot run,
the tests that use this path fail). Weights are read from the
engine's own modules, so engine and reference path see identical parameters.

The decoder is run teacher-forced over a whole sequence in one causal varlen pass
(what the reference computes for a prefill), giving its greedy prediction at every
position in one forward.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

ATTENTION_BACKEND = {"name": None}


def _varlen(q, k, v, cu, max_len, scale, causal):
    """``flash_attn_varlen_func`` exactly as layers/attention.py calls it. There is no
    fallback: if flash-attn cannot run here the parity tests fail and say why, rather
    than comparing against a different attention implementation."""
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:
        raise RuntimeError(f"reference path needs flash-attn: {type(exc).__name__}: {exc}") from exc
    out = flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max_len,
                                 max_seqlen_k=max_len, softmax_scale=scale, causal=causal)
    ATTENTION_BACKEND["name"] = "flash_attn"
    return out


def _rms(x, w, eps):
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf.to(x.dtype) * w


def _add_rms(x, residual, w, eps):
    xf = x.float() + residual.float()
    res = xf.to(x.dtype)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf.to(x.dtype) * w, res


def _rope(x, cos, sin):
    first, second = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((first * cos - second * sin, second * cos + first * sin), -1).to(x.dtype)


@torch.inference_mode()
def encode_audio(model, mel: torch.Tensor) -> torch.Tensor:
    """One request's mel (bins, frames) -> audio embeddings, reference operations."""
    enc = model.audio_tower
    cfg = enc.config
    mel = mel.to(device=enc.conv2d1.weight.device, dtype=torch.bfloat16)
    frames = mel.shape[1]
    lens = [100] * (frames // 100) + ([frames % 100] if frames % 100 else [])
    padded = mel.new_zeros(len(lens), 100, cfg.num_mel_bins)
    start = 0
    for i, n in enumerate(lens):
        padded[i, :n] = mel[:, start:start + n].T
        start += n
    x = padded.transpose(1, 2).unsqueeze(1)
    x = F.gelu(enc.conv2d1(x))
    x = F.gelu(enc.conv2d2(x))
    x = F.gelu(enc.conv2d3(x))
    n, c, f, t = x.shape
    x = enc.conv_out(x.permute(0, 3, 1, 2).contiguous().view(n, t, c * f))
    x = x + enc.positional_embedding[:t].unsqueeze(0).to(x.dtype)
    valid = [(((m - 1) // 2 + 1 - 1) // 2 + 1 - 1) // 2 + 1 for m in lens]
    mask = torch.arange(13, device=x.device)[None, :] < torch.tensor(valid, device=x.device)[:, None]
    h = x[mask]
    total = h.shape[0]
    bounds = [0]
    while bounds[-1] < total:
        bounds.append(min(bounds[-1] + 104, total))
    cu = torch.tensor(bounds, dtype=torch.int32, device=x.device)
    heads, d = cfg.encoder_attention_heads, cfg.d_model
    hd = d // heads
    for layer in enc.layers:
        r = h
        y = layer.self_attn_layer_norm(h)
        w, b = layer.self_attn.qkv_proj.weight, layer.self_attn.qkv_proj.bias
        q = F.linear(y, w[:d], b[:d]).view(total, heads, hd)
        k = F.linear(y, w[d:2 * d], b[d:2 * d]).view(total, heads, hd)
        v = F.linear(y, w[2 * d:], b[2 * d:]).view(total, heads, hd)
        o = _varlen(q, k, v, cu, int(max(b - a for a, b in zip(bounds[:-1], bounds[1:]))),
                    hd ** -0.5, False)
        h = r + layer.self_attn.out_proj(o.reshape(total, d))
        r = h
        h = r + layer.fc2(F.gelu(layer.fc1(layer.final_layer_norm(h))))
    h = enc.ln_post(h)
    return enc.proj2(F.gelu(enc.proj1(h)))


@torch.inference_mode()
def greedy_logits(model, token_ids: list[int], audio_embeds: torch.Tensor,
                  audio_offset: int) -> torch.Tensor:
    """Logits (fp32 view of the bf16 lm_head output) at every position of ``token_ids``,
    teacher forced, reference ops."""
    dec = model.model
    dev = dec.embed_tokens.weight.device
    ids = torch.tensor(token_ids, dtype=torch.long, device=dev)
    h = dec.embed_tokens(ids)
    h[audio_offset:audio_offset + audio_embeds.shape[0]] = audio_embeds.to(h.dtype)
    n = ids.shape[0]
    pos = torch.arange(n, device=dev)
    table = dec.rope.table
    cos, sin = table[pos].chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
    residual = None
    for layer in dec.layers:
        attn = layer.self_attn
        eps = attn.eps
        if residual is None:
            residual, h = h, _rms(h, layer.input_layernorm.weight, eps)
        else:
            h, residual = _add_rms(h, residual, layer.input_layernorm.weight, eps)
        qkv = F.linear(h, attn.qkv_proj.weight)
        q, k, v = qkv.split([attn.q_size, attn.kv_size, attn.kv_size], dim=-1)
        q = _rms(q.reshape(n, attn.num_heads, attn.head_dim), attn.q_norm.weight, eps)
        k = _rms(k.reshape(n, attn.num_kv_heads, attn.head_dim), attn.k_norm.weight, eps)
        v = v.reshape(n, attn.num_kv_heads, attn.head_dim)
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        o = _varlen(q, k.contiguous(), v.contiguous(), cu, n, attn.head_dim ** -0.5, True)
        h = attn.o_proj(o.reshape(n, attn.q_size))
        h, residual = _add_rms(h, residual, layer.post_attention_layernorm.weight, eps)
        gate, up = layer.mlp.gate_up_proj(h).chunk(2, dim=-1)
        h = layer.mlp.down_proj(F.silu(gate) * up)
    h, _ = _add_rms(h, residual, dec.norm.weight, dec.norm.eps)
    return model.compute_logits(h).float()


def greedy_predictions(model, token_ids: list[int], audio_embeds: torch.Tensor,
                       audio_offset: int) -> torch.Tensor:
    """Argmax at every position of ``token_ids`` (teacher forced), reference ops."""
    return greedy_logits(model, token_ids, audio_embeds, audio_offset).argmax(-1)
