"""Checkpoint loading into fused parameters.

Same contract as the reference's ``load_weights`` (loader.py:87-150): tensors are
stored under ``thinker.`` with per-projection names; the decoder holds q/k/v and
gate/up fused, and a checkpoint tensor with no destination or a parameter never
written is an error. This engine additionally fuses the audio encoder's q/k/v (and
their biases) into one projection so the encoder runs one GEMM per layer.
"""

from __future__ import annotations

import glob
import json
import os
from collections.abc import Iterable, Iterator

import torch
from torch import nn

PREFIX = "thinker."

_DECODER_SHARDS = {
    "self_attn.q_proj.": ("self_attn.qkv_proj.", "q"),
    "self_attn.k_proj.": ("self_attn.qkv_proj.", "k"),
    "self_attn.v_proj.": ("self_attn.qkv_proj.", "v"),
    "mlp.gate_proj.": ("mlp.gate_up_proj.", "gate"),
    "mlp.up_proj.": ("mlp.gate_up_proj.", "up"),
}
_ENCODER_SHARDS = {
    "self_attn.q_proj.": ("self_attn.qkv_proj.", "eq"),
    "self_attn.k_proj.": ("self_attn.qkv_proj.", "ek"),
    "self_attn.v_proj.": ("self_attn.qkv_proj.", "ev"),
}
_GROUPS = {"self_attn.qkv_proj.": ({"q", "k", "v"}, {"eq", "ek", "ev"}),
           "mlp.gate_up_proj.": ({"gate", "up"},)}


def iter_checkpoint(model_path: str) -> Iterator[tuple[str, torch.Tensor]]:
    from safetensors import safe_open

    index = os.path.join(model_path, "model.safetensors.index.json")
    if os.path.isfile(index):
        with open(index, encoding="utf-8") as handle:
            files = [os.path.join(model_path, f)
                     for f in sorted(set(json.load(handle)["weight_map"].values()))]
    else:
        files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors found under {model_path}")
    for path in files:
        with safe_open(path, framework="pt", device="cpu") as reader:
            for name in reader.keys():
                yield name, reader.get_tensor(name)


def _resolve(name: str) -> tuple[str, str | None]:
    if name.startswith("model.layers."):
        table = _DECODER_SHARDS
    elif name.startswith("audio_tower.layers."):
        table = _ENCODER_SHARDS
    else:
        return name, None
    for marker, (fused, shard) in table.items():
        if marker in name:
            return name.replace(marker, fused), shard
    return name, None


def load_tensors(model: nn.Module, tensors: Iterable[tuple[str, torch.Tensor]],
                 prefixed: bool = True) -> None:
    """Copy checkpoint tensors into ``model``'s (fused) parameters."""
    text = model.config.text
    audio = model.config.audio
    hd = text.head_dim or text.hidden_size // text.num_attention_heads
    q, kv, inter, dm = (text.num_attention_heads * hd, text.num_key_value_heads * hd,
                        text.intermediate_size, audio.d_model)
    offsets = {"q": (0, q), "k": (q, kv), "v": (q + kv, kv), "gate": (0, inter),
               "up": (inter, inter), "eq": (0, dm), "ek": (dm, dm), "ev": (2 * dm, dm)}

    params = dict(model.named_parameters())
    aliases = {}
    if "lm_head.weight" not in params:
        aliases["lm_head.weight"] = "model.embed_tokens.weight"
    written: dict[str, set] = {}
    orphans: list[str] = []
    for raw, tensor in tensors:
        if prefixed:
            if not raw.startswith(PREFIX):
                orphans.append(raw)
                continue
            raw_name = raw[len(PREFIX):]
        else:
            raw_name = raw
        target, shard = _resolve(raw_name)
        target = aliases.get(target, target)
        param = params.get(target)
        if param is None:
            orphans.append(raw)
            continue
        with torch.no_grad():
            if shard is None:
                if tuple(param.shape) != tuple(tensor.shape):
                    raise ValueError(f"shape mismatch for {target}: checkpoint {tuple(tensor.shape)} "
                                     f"vs model {tuple(param.shape)}")
                param.copy_(tensor)
            else:
                off, n = offsets[shard]
                if tensor.size(0) != n:
                    raise ValueError(f"shard {shard} of {raw} has {tensor.size(0)} rows, expected {n}")
                param.narrow(0, off, n).copy_(tensor)
        written.setdefault(target, set()).add(shard)
    if orphans:
        raise RuntimeError(f"{len(orphans)} checkpoint tensors had no destination, "
                           f"e.g. {sorted(orphans)[:5]}")
    missing = sorted(set(params) - set(written))
    if missing:
        raise RuntimeError(f"{len(missing)} parameters were never loaded, e.g. {missing[:5]}")
    for target, shards in written.items():
        for marker, options in _GROUPS.items():
            if marker in target and shards not in options:
                raise RuntimeError(f"{target} is missing fused shards (got {sorted(map(str, shards))})")


def load_weights(model: nn.Module, model_path: str) -> None:
    load_tensors(model, iter_checkpoint(model_path))
