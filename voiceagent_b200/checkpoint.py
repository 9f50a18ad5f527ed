"""Seeded random-init Qwen3-ASR checkpoints in the upstream on-disk format.

No real weights are available offline, so benchmarks and tests run on random-init
models of the released architectures. ``write_checkpoint`` produces a directory the
reference engine's loader would also accept (loader.py:22-34,87-150): ``config.json``
with a ``thinker_config``, ``generation_config.json`` (stop ids), a Whisper
``preprocessor_config.json`` and ``model.safetensors`` with ``thinker.*`` tensors in
per-projection layout. Initialisation: N(0, 0.02) weights, zero biases, unit norm
scales, one seeded CPU generator over names in sorted order (bit-reproducible).
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import torch

STOP_TOKEN_IDS = [151643, 151645]

PRESETS: dict[str, dict] = {
    "0.6b": {
        "audio": dict(num_mel_bins=128, d_model=896, encoder_layers=18, encoder_attention_heads=14,
                      encoder_ffn_dim=3584, downsample_hidden_size=480, output_dim=1024,
                      n_window=50, n_window_infer=800, conv_chunksize=500,
                      max_source_positions=1500),
        "text": dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                     num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                     head_dim=128, rms_norm_eps=1e-6, rope_theta=1_000_000.0,
                     max_position_embeddings=65536, tie_word_embeddings=True),
    },
    # Encoder dims of the 1.7B release are not available offline; the 0.6B encoder
    # defaults are used with output_dim = decoder hidden (needed by the audio scatter).
    "1.7b": {
        "audio": dict(num_mel_bins=128, d_model=896, encoder_layers=18, encoder_attention_heads=14,
                      encoder_ffn_dim=3584, downsample_hidden_size=480, output_dim=2048,
                      n_window=50, n_window_infer=800, conv_chunksize=500,
                      max_source_positions=1500),
        "text": dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                     num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                     head_dim=128, rms_norm_eps=1e-6, rope_theta=1_000_000.0,
                     max_position_embeddings=65536, tie_word_embeddings=True),
    },
    # A structurally faithful miniature for fast tests (GQA 2, head_dim 128, 3 convs).
    "tiny": {
        "audio": dict(num_mel_bins=128, d_model=128, encoder_layers=2, encoder_attention_heads=2,
                      encoder_ffn_dim=256, downsample_hidden_size=32, output_dim=256,
                      n_window=50, n_window_infer=800, conv_chunksize=500,
                      max_source_positions=1500),
        "text": dict(vocab_size=152064, hidden_size=256, intermediate_size=512,
                     num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                     head_dim=128, rms_norm_eps=1e-6, rope_theta=1_000_000.0,
                     max_position_embeddings=65536, tie_word_embeddings=True),
    },
}

TOKEN_IDS = dict(audio_token_id=151676, audio_start_token_id=151669, audio_end_token_id=151670)


def _shapes(audio: dict, text: dict) -> dict[str, tuple[tuple[int, ...], str]]:
    s: dict[str, tuple[tuple[int, ...], str]] = {}
    c, dm = audio["downsample_hidden_size"], audio["d_model"]
    s["audio_tower.conv2d1.weight"] = ((c, 1, 3, 3), "normal")
    s["audio_tower.conv2d1.bias"] = ((c,), "zeros")
    for n in ("conv2d2", "conv2d3"):
        s[f"audio_tower.{n}.weight"] = ((c, c, 3, 3), "normal")
        s[f"audio_tower.{n}.bias"] = ((c,), "zeros")
    freq = (((audio["num_mel_bins"] + 1) // 2 + 1) // 2 + 1) // 2
    s["audio_tower.conv_out.weight"] = ((dm, c * freq), "normal")
    for i in range(audio["encoder_layers"]):
        p = f"audio_tower.layers.{i}."
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            s[p + f"self_attn.{proj}.weight"] = ((dm, dm), "normal")
            s[p + f"self_attn.{proj}.bias"] = ((dm,), "zeros")
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            s[p + f"{ln}.weight"] = ((dm,), "ones")
            s[p + f"{ln}.bias"] = ((dm,), "zeros")
        s[p + "fc1.weight"] = ((audio["encoder_ffn_dim"], dm), "normal")
        s[p + "fc1.bias"] = ((audio["encoder_ffn_dim"],), "zeros")
        s[p + "fc2.weight"] = ((dm, audio["encoder_ffn_dim"]), "normal")
        s[p + "fc2.bias"] = ((dm,), "zeros")
    s["audio_tower.ln_post.weight"] = ((dm,), "ones")
    s["audio_tower.ln_post.bias"] = ((dm,), "zeros")
    s["audio_tower.proj1.weight"] = ((dm, dm), "normal")
    s["audio_tower.proj1.bias"] = ((dm,), "zeros")
    s["audio_tower.proj2.weight"] = ((audio["output_dim"], dm), "normal")
    s["audio_tower.proj2.bias"] = ((audio["output_dim"],), "zeros")
    h, d = text["hidden_size"], text["head_dim"]
    s["model.embed_tokens.weight"] = ((text["vocab_size"], h), "normal")
    for i in range(text["num_hidden_layers"]):
        p = f"model.layers.{i}."
        s[p + "self_attn.q_proj.weight"] = ((text["num_attention_heads"] * d, h), "normal")
        s[p + "self_attn.k_proj.weight"] = ((text["num_key_value_heads"] * d, h), "normal")
        s[p + "self_attn.v_proj.weight"] = ((text["num_key_value_heads"] * d, h), "normal")
        s[p + "self_attn.o_proj.weight"] = ((h, text["num_attention_heads"] * d), "normal")
        s[p + "self_attn.q_norm.weight"] = ((d,), "ones")
        s[p + "self_attn.k_norm.weight"] = ((d,), "ones")
        s[p + "mlp.gate_proj.weight"] = ((text["intermediate_size"], h), "normal")
        s[p + "mlp.up_proj.weight"] = ((text["intermediate_size"], h), "normal")
        s[p + "mlp.down_proj.weight"] = ((h, text["intermediate_size"]), "normal")
        s[p + "input_layernorm.weight"] = ((h,), "ones")
        s[p + "post_attention_layernorm.weight"] = ((h,), "ones")
    s["model.norm.weight"] = ((h,), "ones")
    if not text.get("tie_word_embeddings", True):
        s["lm_head.weight"] = ((text["vocab_size"], h), "normal")
    return s


def random_state_dict(preset: str | dict = "0.6b", seed: int = 0, std: float = 0.02,
                      dtype: torch.dtype = torch.bfloat16) -> dict[str, torch.Tensor]:
    """Checkpoint tensors (no ``thinker.`` prefix) for a preset or a config dict."""
    cfg = PRESETS[preset] if isinstance(preset, str) else preset
    gen = torch.Generator().manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, (shape, kind) in sorted(_shapes(cfg["audio"], cfg["text"]).items()):
        if kind == "normal":
            t = torch.randn(shape, generator=gen) * std
        elif kind == "zeros":
            t = torch.zeros(shape)
        else:
            t = torch.ones(shape)
        out[name] = t.to(dtype)
    return out


def config_json(preset: str | dict = "0.6b") -> dict:
    cfg = PRESETS[preset] if isinstance(preset, str) else preset
    return {
        "architectures": ["Qwen3ASRForConditionalGeneration"],
        "model_type": "qwen3_asr",
        "thinker_config": {"audio_config": dict(cfg["audio"]), "text_config": dict(cfg["text"]),
                           "dtype": "bfloat16", **TOKEN_IDS},
        "support_languages": ["English", "Chinese"],
    }


def write_checkpoint(path: str | os.PathLike, preset: str | dict = "0.6b", seed: int = 0,
                     weights: bool = True) -> Path:
    """Write a loadable checkpoint directory; returns its path."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(config_json(preset), indent=1))
    (path / "generation_config.json").write_text(json.dumps({"eos_token_id": STOP_TOKEN_IDS}))
    (path / "preprocessor_config.json").write_text(json.dumps({
        "feature_extractor_type": "WhisperFeatureExtractor", "feature_size": 128,
        "hop_length": 160, "n_fft": 400, "sampling_rate": 16000, "chunk_length": 30,
        "padding_value": 0.0, "return_attention_mask": True}))
    if weights:
        tensors = {"thinker." + k: v.contiguous() for k, v in random_state_dict(preset, seed).items()}
        save_file(tensors, str(path / "model.safetensors"))
    return path
