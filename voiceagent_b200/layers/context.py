"""Per-forward attention metadata, shared with the layers through a module value.

Same bridge as the reference (layers/context.py:19-51): the runner builds the batch
metadata and attention reads it deep in the layer stack. All tensors are device
tensors produced by the on-GPU packer; the two extra fields carry the split-K
decode workspace and the device error word.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class AttentionContext:
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    # True when every row has exactly one query token (the CUDA-graph decode).
    decode_only: bool = False
    decode_workspace: torch.Tensor | None = None
    error_flag: torch.Tensor | None = None


_CONTEXT = AttentionContext()


def get_attention_context() -> AttentionContext:
    return _CONTEXT


def set_attention_context(context: AttentionContext) -> None:
    global _CONTEXT
    _CONTEXT = context


@contextmanager
def attention_context(context: AttentionContext):
    previous = get_attention_context()
    set_attention_context(context)
    try:
        yield
    finally:
        set_attention_context(previous)
