"""TTS talker decode attention over request-owned KV pages, on the b200asr kernel.

Drop-in for ``paged_attention_decode`` of ``agent/qwen_tts_paged_attention.py``
(383-516), the call ``QwenPagedCache.paged_attention_decode`` makes once per layer and
decode step (agent/qwen_tts_outer_varlen.py:392-436): same arguments, same validation
messages and exception class, same result -- one-token GQA attention of
``query [B, H, 1, D]`` over the pools ``[pages, H_kv, page_size, D]`` through an int64
page table, with the current token's key/value written into its page by the same launch.

Differences, by design:

* every call runs the CUDA kernel (``b200asr_pool_paged_decode``); there is no torch or
  CPU path, so ``use_triton=False`` and CPU tensors raise ``PagedAttentionKernelError``;
* ``block_n`` only rounds the default ``kernel_seq_len`` (as in the reference) and
  ``num_warps`` is checked and otherwise unused: the kernel picks its own launch shape;
* a narrow page table is not copied out to ``kernel_page_count`` columns of zeros:
  logical pages past its width are outside the table, and with ``validate=False`` a row
  that reaches them has those positions skipped (``B200ASR_DEVERR_BLOCK``) instead of
  reading physical page 0.
"""

from __future__ import annotations

import math

import torch

from voiceagent_b200 import kernels as kx

HAS_KERNEL = True


class PagedAttentionKernelError(RuntimeError):
    """Raised when the paged decode attention contract is invalid."""


def _validate_inputs(query, key_pool, value_pool, page_table, seq_lens, key_valid_mask):
    """The reference's input contract (agent/qwen_tts_paged_attention.py:290-350)."""
    tensors = (query, key_pool, value_pool, page_table, seq_lens)
    if not all(torch.is_tensor(t) for t in tensors):
        raise PagedAttentionKernelError("paged attention inputs must be tensors")
    if query.ndim != 4 or query.shape[2] != 1:
        raise PagedAttentionKernelError("query must have shape [batch, heads, 1, head_dim]")
    if key_pool.ndim != 4 or value_pool.shape != key_pool.shape:
        raise PagedAttentionKernelError(
            "KV pool must have shape [pages, kv_heads, page_size, head_dim]")
    if page_table.ndim != 2 or seq_lens.ndim != 1 or page_table.shape[0] != query.shape[0]:
        raise PagedAttentionKernelError("page table and sequence lengths must match query batch")
    if seq_lens.shape[0] != query.shape[0] or seq_lens.dtype != torch.long:
        raise PagedAttentionKernelError("seq_lens must be a torch.long vector")
    if page_table.dtype != torch.long:
        raise PagedAttentionKernelError("page_table must be a torch.long matrix")
    if any(t.device != query.device for t in tensors):
        raise PagedAttentionKernelError("paged attention inputs must share a device")
    if key_pool.dtype != query.dtype or value_pool.dtype != query.dtype:
        raise PagedAttentionKernelError("query and KV pool must share a dtype")
    if key_pool.shape[3] != query.shape[3]:
        raise PagedAttentionKernelError("query and KV pool head dimensions must match")
    if query.shape[1] % key_pool.shape[1] != 0:
        raise PagedAttentionKernelError("query heads must be divisible by KV heads")
    if key_valid_mask is not None and (
            key_valid_mask.ndim != 2 or key_valid_mask.shape[0] != query.shape[0]
            or key_valid_mask.dtype != torch.bool or key_valid_mask.device != query.device):
        raise PagedAttentionKernelError("key_valid_mask must be [batch, max_seq] bool on device")
    if bool((seq_lens <= 0).any()):
        raise PagedAttentionKernelError("sequence lengths must be positive")
    page_size = key_pool.shape[2]
    if bool((seq_lens > page_table.shape[1] * page_size).any()):
        raise PagedAttentionKernelError("sequence length exceeds page table capacity")
    # Every page a row uses must lie in the pool (one vectorised check for all rows).
    used = torch.arange(page_table.shape[1], device=page_table.device)[None, :] < (
        (seq_lens + page_size - 1) // page_size)[:, None]
    if bool((used & ((page_table < 0) | (page_table >= key_pool.shape[0]))).any()):
        raise PagedAttentionKernelError("page table contains an invalid page table entry")
    if key_valid_mask is not None and key_valid_mask.shape[1] < int(seq_lens.max()):
        raise PagedAttentionKernelError("key_valid_mask is shorter than sequence length")


def paged_attention_decode(query, key_pool, value_pool, page_table, seq_lens,
                           key_valid_mask=None, *, new_key=None, new_value=None,
                           kernel_seq_len=None, kernel_page_count=None, block_n: int = 128,
                           num_warps: int = 4, scale=None, use_triton: bool = True,
                           validate: bool = True) -> torch.Tensor:
    """One-token GQA attention directly from a physical page pool.

    ``page_table`` maps each request's logical page to a physical page of the pool; no
    dense K/V tensor is built. ``key_valid_mask`` (bool ``[B, >= max seq]``) drops
    left-padded prompt positions. With ``new_key``/``new_value`` (``[B, H_kv, 1, D]``)
    the current token is stored at position ``seq_lens[b] - 1`` and attended in the
    same launch. Returns ``[B, H, 1, D]`` in the query's dtype.
    """
    if validate:
        _validate_inputs(query, key_pool, value_pool, page_table, seq_lens, key_valid_mask)
    num_kv_heads = int(key_pool.shape[1])
    scale = float(scale if scale is not None else 1.0 / math.sqrt(query.shape[-1]))
    if (new_key is None) != (new_value is None):
        raise PagedAttentionKernelError("new_key and new_value must be provided together")
    if new_key is not None:
        expected = (query.shape[0], num_kv_heads, 1, query.shape[-1])
        if (tuple(new_key.shape) != expected or tuple(new_value.shape) != expected
                or new_key.dtype != query.dtype or new_value.dtype != query.dtype
                or new_key.device != query.device or new_value.device != query.device):
            raise PagedAttentionKernelError(
                "new KV must have shape [batch, kv_heads, 1, head_dim] and match query")
    if not use_triton or query.device.type != "cuda":
        raise PagedAttentionKernelError(
            "paged attention runs only on the CUDA kernel (CUDA tensors, use_triton=True)")
    block_n = int(block_n)
    if block_n <= 0 or block_n & (block_n - 1):
        raise PagedAttentionKernelError("block_n must be a positive power of two")
    if int(num_warps) <= 0:
        raise PagedAttentionKernelError("num_warps must be positive")
    if kernel_seq_len is None:
        kernel_seq_len = int(math.ceil(int(seq_lens.max()) / block_n) * block_n)
    kernel_seq_len = int(kernel_seq_len)
    if kernel_page_count is not None and int(kernel_page_count) <= 0:
        raise PagedAttentionKernelError("kernel metadata dimensions must be positive")
    if kernel_seq_len <= 0:
        raise PagedAttentionKernelError("kernel metadata dimensions must be positive")
    if new_key is not None:
        # the kernel reads both with one set of strides (as the reference's kernel does)
        if new_key.stride() != new_value.stride() or new_key.stride(-1) != 1:
            new_key, new_value = new_key.contiguous(), new_value.contiguous()
    if query.stride(-1) != 1:
        query = query.contiguous()
    if key_pool.stride(-1) != 1 or key_pool.stride() != value_pool.stride():
        raise PagedAttentionKernelError("KV pools must share strides with a unit head_dim stride")
    mask = None
    if key_valid_mask is not None:
        mask = key_valid_mask if key_valid_mask.stride(-1) == 1 else key_valid_mask.contiguous()
    try:
        return kx.pool_paged_decode(query, key_pool, value_pool, page_table, seq_lens,
                                    max_seq_len=kernel_seq_len, scale=scale,
                                    key_valid_mask=mask, new_key=new_key, new_value=new_value)
    except (ValueError, RuntimeError) as exc:
        raise PagedAttentionKernelError(str(exc)) from exc
