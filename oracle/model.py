"""CPU fp32 restatement of the upstream Qwen3-ASR thinker (test infrastructure).

Follows ``reference/modeling_qwen3_asr.py`` of the qwen-asr-vllm project:

* audio tower   -- ``Qwen3ASRAudioEncoder.forward`` (modeling_qwen3_asr.py:669-740):
  100-frame chunks padded to the longest chunk, 3x Conv2d(s2)+GELU, ``conv_out``,
  sinusoid positions, windowed bidirectional attention (``cu_seqlens``), ``ln_post``,
  ``proj1``/GELU/``proj2``;
* text decoder  -- ``Qwen3ASRThinkerTextModel`` (961-1059) with
  ``Qwen3ASRThinkerTextAttention`` (877-953): per-head q/k RMSNorm, half-split RoPE
  (the interleaved MRoPE of 794-830 reduces to 1-D RoPE because all three position
  rows are equal, see ``get_rope_index`` 414-448), causal GQA, SwiGLU MLP;
* greedy loop   -- a fixed number of argmax steps over a KV cache, the way the
  reference's ``ReferenceTranscriber`` drives ``generate`` with EOS ignored.

It is the oracle for end-to-end parity and the timed CPU baseline of ``bench.py``.
Weights come from :func:`init_weights` (seeded, HF initializer_range 0.02), keyed by
the checkpoint names without the ``thinker.`` prefix.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

from oracle.kernels import chunk_lengths_for, num_audio_tokens  # noqa: F401  (re-export)

# ------------------------------------------------------------------------ config


@dataclass
class AudioCfg:
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


@dataclass
class TextCfg:
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


@dataclass
class ThinkerCfg:
    audio: AudioCfg = field(default_factory=AudioCfg)
    text: TextCfg = field(default_factory=TextCfg)
    audio_token_id: int = 151676
    audio_start_token_id: int = 151669
    audio_end_token_id: int = 151670

    @classmethod
    def from_dict(cls, raw: dict) -> "ThinkerCfg":
        return cls(
            audio=AudioCfg(**{k: v for k, v in raw.get("audio", {}).items()
                              if k in AudioCfg.__dataclass_fields__}),
            text=TextCfg(**{k: v for k, v in raw.get("text", {}).items()
                            if k in TextCfg.__dataclass_fields__}),
            audio_token_id=raw.get("audio_token_id", 151676),
            audio_start_token_id=raw.get("audio_start_token_id", 151669),
            audio_end_token_id=raw.get("audio_end_token_id", 151670),
        )


def _as_cfg(cfg) -> ThinkerCfg:
    return cfg if isinstance(cfg, ThinkerCfg) else ThinkerCfg.from_dict(cfg)


# ----------------------------------------------------------------------- weights


def weight_shapes(cfg) -> dict[str, tuple[tuple[int, ...], str]]:
    """Checkpoint tensor names (no ``thinker.`` prefix) -> (shape, init kind)."""
    cfg = _as_cfg(cfg)
    a, t = cfg.audio, cfg.text
    shapes: dict[str, tuple[tuple[int, ...], str]] = {}
    c = a.downsample_hidden_size
    shapes["audio_tower.conv2d1.weight"] = ((c, 1, 3, 3), "normal")
    shapes["audio_tower.conv2d1.bias"] = ((c,), "zeros")
    for n in ("conv2d2", "conv2d3"):
        shapes[f"audio_tower.{n}.weight"] = ((c, c, 3, 3), "normal")
        shapes[f"audio_tower.{n}.bias"] = ((c,), "zeros")
    freq = (((a.num_mel_bins + 1) // 2 + 1) // 2 + 1) // 2
    shapes["audio_tower.conv_out.weight"] = ((a.d_model, c * freq), "normal")
    for i in range(a.encoder_layers):
        p = f"audio_tower.layers.{i}."
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            shapes[p + f"self_attn.{proj}.weight"] = ((a.d_model, a.d_model), "normal")
            shapes[p + f"self_attn.{proj}.bias"] = ((a.d_model,), "zeros")
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            shapes[p + f"{ln}.weight"] = ((a.d_model,), "ones")
            shapes[p + f"{ln}.bias"] = ((a.d_model,), "zeros")
        shapes[p + "fc1.weight"] = ((a.encoder_ffn_dim, a.d_model), "normal")
        shapes[p + "fc1.bias"] = ((a.encoder_ffn_dim,), "zeros")
        shapes[p + "fc2.weight"] = ((a.d_model, a.encoder_ffn_dim), "normal")
        shapes[p + "fc2.bias"] = ((a.d_model,), "zeros")
    shapes["audio_tower.ln_post.weight"] = ((a.d_model,), "ones")
    shapes["audio_tower.ln_post.bias"] = ((a.d_model,), "zeros")
    shapes["audio_tower.proj1.weight"] = ((a.d_model, a.d_model), "normal")
    shapes["audio_tower.proj1.bias"] = ((a.d_model,), "zeros")
    shapes["audio_tower.proj2.weight"] = ((a.output_dim, a.d_model), "normal")
    shapes["audio_tower.proj2.bias"] = ((a.output_dim,), "zeros")

    h, d = t.hidden_size, t.head_dim
    shapes["model.embed_tokens.weight"] = ((t.vocab_size, h), "normal")
    for i in range(t.num_hidden_layers):
        p = f"model.layers.{i}."
        shapes[p + "self_attn.q_proj.weight"] = ((t.num_attention_heads * d, h), "normal")
        shapes[p + "self_attn.k_proj.weight"] = ((t.num_key_value_heads * d, h), "normal")
        shapes[p + "self_attn.v_proj.weight"] = ((t.num_key_value_heads * d, h), "normal")
        shapes[p + "self_attn.o_proj.weight"] = ((h, t.num_attention_heads * d), "normal")
        shapes[p + "self_attn.q_norm.weight"] = ((d,), "ones")
        shapes[p + "self_attn.k_norm.weight"] = ((d,), "ones")
        shapes[p + "mlp.gate_proj.weight"] = ((t.intermediate_size, h), "normal")
        shapes[p + "mlp.up_proj.weight"] = ((t.intermediate_size, h), "normal")
        shapes[p + "mlp.down_proj.weight"] = ((h, t.intermediate_size), "normal")
        shapes[p + "input_layernorm.weight"] = ((h,), "ones")
        shapes[p + "post_attention_layernorm.weight"] = ((h,), "ones")
    shapes["model.norm.weight"] = ((h,), "ones")
    if not t.tie_word_embeddings:
        shapes["lm_head.weight"] = ((t.vocab_size, h), "normal")
    return shapes


def init_weights(cfg, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded random init in fp32: N(0, std) weights, zero biases, unit norms.

    Deterministic across machines: one CPU generator, names in sorted order.
    With tied embeddings, ``lm_head.weight`` is the embedding tensor itself.
    """
    gen = torch.Generator().manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, (shape, kind) in sorted(weight_shapes(cfg).items()):
        if kind == "normal":
            out[name] = torch.randn(shape, generator=gen) * std
        elif kind == "zeros":
            out[name] = torch.zeros(shape)
        else:
            out[name] = torch.ones(shape)
    if _as_cfg(cfg).text.tie_word_embeddings:
        out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out


# ------------------------------------------------------------------ audio tower


def sinusoid_table(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    """``SinusoidsPositionEmbedding`` (modeling_qwen3_asr.py:575-590)."""
    inc = np.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2).float())
    scaled = torch.arange(length)[:, None] * inv[None, :]
    return torch.cat([torch.sin(scaled), torch.cos(scaled)], dim=1)


class OracleThinker:
    """fp32 CPU thinker: ``encode_audio`` + KV-cached decoder + greedy loop."""

    def __init__(self, cfg, weights: dict[str, torch.Tensor]):
        self.cfg = _as_cfg(cfg)
        self.w = {k: v.float() for k, v in weights.items()}
        a = self.cfg.audio
        self.pos = sinusoid_table(a.max_source_positions, a.d_model)
        t = self.cfg.text
        inv = 1.0 / (t.rope_theta ** (torch.arange(0, t.head_dim, 2, dtype=torch.int64).float()
                                      / t.head_dim))
        self.inv_freq = inv

    # audio -----------------------------------------------------------------

    def conv_front(self, chunks: torch.Tensor) -> torch.Tensor:
        """Chunks (n, bins, frames) -> conv_out output (n, tokens, d_model): three
        Conv2d(3, stride 2, pad 1) + GELU and the (channel, frequency)-flattened conv_out
        projection, modeling_qwen3_asr.py:700-710, in fp32."""
        w = self.w
        x = chunks.unsqueeze(1)
        for n in ("conv2d1", "conv2d2", "conv2d3"):
            x = F.gelu(F.conv2d(x, w[f"audio_tower.{n}.weight"], w[f"audio_tower.{n}.bias"],
                                stride=2, padding=1))
        b, c, f, t = x.shape
        return x.permute(0, 3, 1, 2).reshape(b, t, c * f) @ w["audio_tower.conv_out.weight"].T

    def encode_audio(self, mel: torch.Tensor) -> torch.Tensor:
        """One request's mel (bins, frames) -> (audio tokens, output_dim).

        modeling_qwen3_asr.py:669-740 for a single request, with ``eager``
        attention restricted to the ``cu_seqlens`` windows (the block-diagonal mask
        of ``_prepare_attention_mask`` 649-666).
        """
        a, w = self.cfg.audio, self.w
        frames = mel.shape[1]
        lens = chunk_lengths_for(frames, a.n_window * 2)
        max_len = max(lens)
        chunks = torch.zeros(len(lens), a.num_mel_bins, max_len)
        s = 0
        for i, n in enumerate(lens):
            chunks[i, :, :n] = mel[:, s : s + n]
            s += n
        x = self.conv_front(chunks)
        t = x.shape[1]
        x = x + self.pos[:t].unsqueeze(0)
        valid = [(((n - 1) // 2 + 1 - 1) // 2 + 1 - 1) // 2 + 1 for n in lens]
        h = torch.cat([x[i, :v] for i, v in enumerate(valid)], dim=0)

        window = t * (a.n_window_infer // (a.n_window * 2))
        total = h.shape[0]
        bounds = [0]
        full, rem = divmod(total, window)
        bounds += [window] * full + ([rem] if rem else [])
        cu = np.cumsum(bounds)

        heads, hd = a.encoder_attention_heads, a.d_model // a.encoder_attention_heads
        for i in range(a.encoder_layers):
            p = f"audio_tower.layers.{i}."
            r = h
            y = F.layer_norm(h, (a.d_model,), w[p + "self_attn_layer_norm.weight"],
                             w[p + "self_attn_layer_norm.bias"])
            q = (y @ w[p + "self_attn.q_proj.weight"].T + w[p + "self_attn.q_proj.bias"])
            k = (y @ w[p + "self_attn.k_proj.weight"].T + w[p + "self_attn.k_proj.bias"])
            v = (y @ w[p + "self_attn.v_proj.weight"].T + w[p + "self_attn.v_proj.bias"])
            q, k, v = (z.view(total, heads, hd).transpose(0, 1) for z in (q, k, v))
            o = torch.empty_like(q)
            for s0, s1 in zip(cu[:-1], cu[1:]):
                sc = (q[:, s0:s1] @ k[:, s0:s1].transpose(1, 2)) * hd**-0.5
                o[:, s0:s1] = torch.softmax(sc, dim=-1) @ v[:, s0:s1]
            o = o.transpose(0, 1).reshape(total, a.d_model)
            h = r + (o @ w[p + "self_attn.out_proj.weight"].T + w[p + "self_attn.out_proj.bias"])
            r = h
            y = F.layer_norm(h, (a.d_model,), w[p + "final_layer_norm.weight"],
                             w[p + "final_layer_norm.bias"])
            y = F.gelu(y @ w[p + "fc1.weight"].T + w[p + "fc1.bias"])
            h = r + (y @ w[p + "fc2.weight"].T + w[p + "fc2.bias"])
        h = F.layer_norm(h, (a.d_model,), w["audio_tower.ln_post.weight"], w["audio_tower.ln_post.bias"])
        h = F.gelu(h @ w["audio_tower.proj1.weight"].T + w["audio_tower.proj1.bias"])
        return h @ w["audio_tower.proj2.weight"].T + w["audio_tower.proj2.bias"]

    # text ------------------------------------------------------------------

    def _rms(self, x, weight):
        t = self.cfg.text
        return weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + t.rms_norm_eps))

    def _rope(self, x, positions):
        freqs = positions.float()[:, None] * self.inv_freq[None, :]
        emb = torch.cat([freqs, freqs], dim=-1)
        cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]
        d2 = x.shape[-1] // 2
        rot = torch.cat([-x[..., d2:], x[..., :d2]], dim=-1)
        return x * cos + rot * sin

    def new_cache(self):
        return [[None, None] for _ in range(self.cfg.text.num_hidden_layers)]

    def forward_text(self, embeds: torch.Tensor, positions: torch.Tensor, cache) -> torch.Tensor:
        """Decoder over new tokens ``embeds`` (T, hidden) appended to ``cache``."""
        t, w = self.cfg.text, self.w
        hq, hk, d = t.num_attention_heads, t.num_key_value_heads, t.head_dim
        n = embeds.shape[0]
        h = embeds
        for i in range(t.num_hidden_layers):
            p = f"model.layers.{i}."
            r = h
            y = self._rms(h, w[p + "input_layernorm.weight"])
            q = (y @ w[p + "self_attn.q_proj.weight"].T).view(n, hq, d)
            k = (y @ w[p + "self_attn.k_proj.weight"].T).view(n, hk, d)
            v = (y @ w[p + "self_attn.v_proj.weight"].T).view(n, hk, d)
            q = self._rope(self._rms(q, w[p + "self_attn.q_norm.weight"]), positions)
            k = self._rope(self._rms(k, w[p + "self_attn.k_norm.weight"]), positions)
            kc, vc = cache[i]
            kc = k if kc is None else torch.cat([kc, k], 0)
            vc = v if vc is None else torch.cat([vc, v], 0)
            cache[i] = [kc, vc]
            total = kc.shape[0]
            qi = torch.arange(n)[:, None] + (total - n)
            mask = torch.arange(total)[None, :] <= qi
            kk = kc.repeat_interleave(hq // hk, dim=1).transpose(0, 1)
            vv = vc.repeat_interleave(hq // hk, dim=1).transpose(0, 1)
            sc = (q.transpose(0, 1) @ kk.transpose(1, 2)) * d**-0.5
            sc = sc.masked_fill(~mask, float("-inf"))
            o = (torch.softmax(sc, dim=-1) @ vv).transpose(0, 1).reshape(n, hq * d)
            h = r + o @ w[p + "self_attn.o_proj.weight"].T
            r = h
            y = self._rms(h, w[p + "post_attention_layernorm.weight"])
            y = F.silu(y @ w[p + "mlp.gate_proj.weight"].T) * (y @ w[p + "mlp.up_proj.weight"].T)
            h = r + y @ w[p + "mlp.down_proj.weight"].T
        return self._rms(h, w["model.norm.weight"])

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return hidden @ self.w["lm_head.weight"].T

    def embed(self, ids) -> torch.Tensor:
        return self.w["model.embed_tokens.weight"][torch.as_tensor(ids, dtype=torch.long)]

    @torch.no_grad()
    def greedy(self, prompt_ids, audio_embeds: torch.Tensor, steps: int,
               forced: list[int] | None = None):
        """Fixed-length greedy decode (EOS ignored).

        Returns (generated ids, per-step argmax ids). With ``forced`` the loop feeds
        those ids instead of its own argmax (teacher forcing), so per-position
        agreement with another decoder can be measured without error cascades.
        """
        ids = list(prompt_ids)
        emb = self.embed(ids)
        off = ids.index(self.cfg.audio_token_id)
        emb[off : off + audio_embeds.shape[0]] = audio_embeds
        cache = self.new_cache()
        hidden = self.forward_text(emb, torch.arange(len(ids)), cache)
        out, argmaxes = [], []
        nxt = int(torch.argmax(self.logits(hidden[-1:])[0]))
        for step in range(steps):
            argmaxes.append(nxt)
            tok = forced[step] if forced is not None else nxt
            out.append(tok)
            if step == steps - 1:
                break
            hidden = self.forward_text(self.embed([tok]), torch.tensor([len(ids) + step]), cache)
            nxt = int(torch.argmax(self.logits(hidden[-1:])[0]))
        return out, argmaxes

    @torch.no_grad()
    def transcribe(self, mel: torch.Tensor, prompt_ids, steps: int):
        """Encode one clip and greedily decode ``steps`` tokens."""
        audio = self.encode_audio(mel)
        return self.greedy(prompt_ids, audio, steps)[0]
