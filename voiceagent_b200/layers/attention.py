"""Paged decoder attention and encoder window attention on the b200asr kernels.

``PagedAttention`` keeps the reference's contract (layers/attention.py:70-107): one
call serves prefill rows, decode rows and mixed batches, with the causal mask aligned
bottom-right; metadata comes from the attention context. Decode-only batches (every
row one query token, the CUDA-graph path) run the split-K HBM-bound decode kernel;
anything else runs the tcgen05 varlen kernel over the paged cache.
"""

from __future__ import annotations

import torch
from torch import nn

from voiceagent_b200 import kernels as kx
from voiceagent_b200.layers.context import get_attention_context


def store_kvcache(key, value, k_cache, v_cache, slot_mapping, error_flag=None) -> None:
    """Scatter K/V rows into paged slots (layers/attention.py:52-67); -1 skips.
    Caches are one layer's [num_blocks, block_size, num_kv_heads, head_dim] views."""
    kx.store_kvcache(key, value, k_cache, v_cache, slot_mapping, error_flag)


class PagedAttention(nn.Module):
    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        # Bound to slices of the engine-owned cache by the model runner.
        self.k_cache = torch.tensor([])
        self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor | None = None,
                v: torch.Tensor | None = None) -> torch.Tensor:
        """q [T, H, D]; with k/v given they are first stored at the context's slots
        (the reference's store-then-attend). The decoder layer normally stores K/V
        inside the fused norm+RoPE kernel and calls this with q only."""
        ctx = get_attention_context()
        if k is not None:
            store_kvcache(k, v, self.k_cache, self.v_cache, ctx.slot_mapping, ctx.error_flag)
        out = torch.empty_like(q)
        if ctx.decode_only:
            return kx.paged_decode(q, self.k_cache, self.v_cache, ctx.cu_seqlens_k,
                                   ctx.block_tables, max_seqlen_k=ctx.max_seqlen_k,
                                   scale=self.scale, out=out, workspace=ctx.decode_workspace,
                                   error_flag=ctx.error_flag)
        return kx.paged_prefill(q, self.k_cache, self.v_cache, ctx.cu_seqlens_q,
                                ctx.cu_seqlens_k, ctx.block_tables,
                                max_seqlen_q=ctx.max_seqlen_q, scale=self.scale, out=out,
                                error_flag=ctx.error_flag)


class VarlenSelfAttention(nn.Module):
    """Non-causal varlen attention for the audio encoder (layers/attention.py:110-139)."""

    def __init__(self, num_heads: int, head_dim: int, scale: float):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale

    def forward(self, q, k, v, cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
        return kx.varlen_attention(q, k, v, cu_seqlens, max_seqlen, self.scale)
