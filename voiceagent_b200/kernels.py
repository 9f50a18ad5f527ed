"""Torch-facing wrappers over the b200asr C ABI.

Each wrapper checks dtypes, devices, shapes and strides on the host (the way the
reference's asserts do, e.g. layers/attention.py:59-64), then launches on the current
CUDA stream. Nothing here allocates inside a captured region when the caller passes
``out=`` / workspace tensors, so the calls are CUDA-graph capturable.
"""

from __future__ import annotations

import ctypes

import torch

from voiceagent_b200._lib import check, lib

BF16 = torch.bfloat16

# Kernel launches issued through these wrappers (eager calls and calls recorded
# while capturing a CUDA graph alike); the graph runner adds its per-replay count.
LAUNCHES = {"count": 0}


def _count(n: int = 1) -> None:
    LAUNCHES["count"] += n


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


if hasattr(torch._C, "_cuda_getCurrentRawStream") and hasattr(torch._C, "_cuda_getDevice"):
    def _stream():
        """The current CUDA stream as a raw handle (the capture stream inside a graph
        capture). The direct query: ``torch.cuda.current_stream()`` resolves the device in
        Python and cost ~15 us per kernel call, which added up on the eager prefill and
        encode paths."""
        return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())
else:  # pragma: no cover - older torch
    def _stream():
        return torch.cuda.current_stream().cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None:
            _need(t.is_cuda, "b200asr kernels need CUDA tensors")


# --------------------------------------------------------------------- packers


def pack_decoder(req_start, req_end, table_off, table_len, tables, query_tokens, *,
                 total_tokens: int, width: int, block_size: int, out: dict) -> None:
    """``ModelRunner._prepare`` (engine/model_runner.py:183-233) on the GPU.

    Inputs are int32 device tensors; ``out`` holds preallocated device tensors
    ``input_ids``/``positions`` (i64), ``slot_mapping`` (i32), ``cu_seqlens_q``/
    ``cu_seqlens_k`` (i32), ``max_seqlen`` (i32[2]), ``block_tables`` (i32 [B, width])
    and ``last_token_index`` (i64).
    """
    batch = req_start.numel()
    _cuda(req_start, req_end, table_off, table_len, tables, query_tokens)
    for t in (req_start, req_end, table_off, table_len, tables, query_tokens):
        _need(t.dtype == torch.int32, "pack_decoder inputs are int32")
    _count()
    check(lib.b200asr_pack_decoder(
        _p(req_start), _p(req_end), _p(table_off), _p(table_len), _p(tables), _p(query_tokens),
        batch, total_tokens, width, block_size, _p(out["input_ids"]), _p(out["positions"]),
        _p(out["slot_mapping"]), _p(out["cu_seqlens_q"]), _p(out["cu_seqlens_k"]),
        _p(out["max_seqlen"]), _p(out["block_tables"]), _p(out["last_token_index"]), _stream()),
        "pack_decoder")


def pack_decode_bucket(lens, last_ids, table_off, table_len, tables, *, batch: int, bucket: int,
                       max_blocks: int, block_size: int, input_ids, positions, slot_mapping,
                       cu_seqlens_k, block_tables) -> None:
    """``GraphRunner.run`` staging (engine/graph_runner.py:149-191) on the GPU."""
    _count()
    check(lib.b200asr_pack_decode_bucket(
        _p(lens), _p(last_ids), _p(table_off), _p(table_len), _p(tables), batch, bucket,
        max_blocks, block_size, _p(input_ids), _p(positions), _p(slot_mapping), _p(cu_seqlens_k),
        _p(block_tables), _stream()), "pack_decode_bucket")


def advance_decode_bucket(lens, last_ids, table_len, sampled, *, bucket: int) -> None:
    """One generated token onto a decode-bucket descriptor, on the device."""
    _count()
    check(lib.b200asr_advance_decode_bucket(_p(lens), _p(last_ids), _p(table_len), _p(sampled),
                                            bucket, _stream()), "advance_decode_bucket")


def pack_audio(mel_frames, *, chunk_frames: int, window_tokens: int, max_chunks: int,
               max_windows: int, out: dict, error_flag=None) -> None:
    """Metadata of ``pack_audio_batch`` (audio/batcher.py:101-141) on the GPU."""
    _need(mel_frames.dtype == torch.int32, "mel_frames is int32")
    _count()
    check(lib.b200asr_pack_audio(
        _p(mel_frames), mel_frames.numel(), chunk_frames, window_tokens, max_chunks, max_windows,
        _p(out["chunk_lengths"]), _p(out["chunk_valid_lens"]), _p(out["chunk_start"]),
        _p(out["audio_token_lens"]), _p(out["cu_seqlens"]), _p(out["counts"]), _p(error_flag),
        _stream()), "pack_audio")


def audio_chunk_pad(mel, chunk_start, chunk_lengths, num_chunks: int, chunk_frames: int,
                    out: torch.Tensor) -> torch.Tensor:
    """``AudioEncoder._chunk_and_pad`` (models/audio_encoder.py:130-143): mel [bins, F]
    -> out [num_chunks, bins, chunk_frames] bf16, zero past each chunk's length."""
    _need(mel.dtype == BF16 and mel.is_contiguous() and out.dtype == BF16, "bf16 contiguous mel")
    _count()
    check(lib.b200asr_audio_chunk_pad(
        _p(mel), mel.shape[0], mel.shape[1], _p(chunk_start), _p(chunk_lengths), num_chunks,
        chunk_frames, _p(out), _stream()), "audio_chunk_pad")
    return out


def audio_gather_pos(embed, pos, token_index, rows_out: int, error_flag=None) -> torch.Tensor:
    """Positional add + valid-token selection of the conv front ("conv.gather" in
    AudioEncoder.forward, models/audio_encoder.py:169-173): embed bf16 [chunks, P, d],
    pos bf16 [P, d] -> [rows_out, d] whose first token_index.numel() rows are
    embed[i] + pos[i % P] for i in token_index (flat rows) and the rest zero."""
    _cuda(embed, pos, token_index)
    _need(embed.dtype == BF16 and pos.dtype == BF16 and embed.is_contiguous() and pos.is_contiguous(),
          "audio_gather_pos: contiguous bf16 embed and pos")
    _need(token_index.dtype == torch.int64 and token_index.is_contiguous(),
          "audio_gather_pos: int64 token_index")
    d = embed.shape[-1]
    per_chunk = pos.shape[0]
    _need(embed.dim() == 3 and embed.shape[1] == per_chunk and pos.shape[1] == d,
          "audio_gather_pos: embed [chunks, P, d] and pos [P, d]")
    tokens = token_index.numel()
    _need(rows_out >= tokens, "audio_gather_pos: rows_out below the token count")
    out = torch.empty(rows_out, d, dtype=BF16, device=embed.device)
    _count()
    check(lib.b200asr_audio_gather_pos(_p(embed), embed.shape[0] * per_chunk, _p(pos), per_chunk,
                                       _p(token_index), tokens, rows_out, d, _p(out),
                                       _p(error_flag), _stream()), "audio_gather_pos")
    return out


# -------------------------------------------------------------------- KV store


def store_kvcache(key, value, k_cache, v_cache, slot_mapping, error_flag=None) -> None:
    """``store_kvcache`` (layers/attention.py:52-67): same arguments and checks."""
    num_tokens, num_heads, head_dim = key.shape
    hidden = num_heads * head_dim
    _cuda(key, value, k_cache, v_cache, slot_mapping)
    _need(key.dtype == BF16 and value.dtype == BF16 and k_cache.dtype == BF16, "bf16 K/V")
    _need(key.stride(-1) == 1 and value.stride(-1) == 1, "key/value rows must be contiguous")
    _need(key.stride(1) == head_dim and value.stride(1) == head_dim, "head stride == head_dim")
    _need(k_cache.stride(1) == hidden and v_cache.stride(1) == hidden, "cache slot stride")
    _need(slot_mapping.numel() == num_tokens and slot_mapping.dtype == torch.int32, "slots")
    num_slots = k_cache.numel() // hidden
    _count()
    check(lib.b200asr_store_kvcache(
        _p(key), key.stride(0), _p(value), value.stride(0), _p(k_cache), _p(v_cache),
        _p(slot_mapping), num_tokens, num_heads, head_dim, num_slots, _p(error_flag), _stream()),
        "store_kvcache")


# ------------------------------------------------------- norms, rope, activation


def qk_norm_rope_store(qkv, positions, *, num_heads: int, num_kv_heads: int, head_dim: int,
                       q_weight, k_weight, eps: float, cos_sin_cache, q_out, k_cache=None,
                       v_cache=None, slot_mapping=None, k_out=None, error_flag=None) -> torch.Tensor:
    """Qwen3Attention q/k RMSNorm + RoPE (models/qwen3.py:43-48) fused with the KV store.

    ``cos_sin_cache`` is fp32 [max_position, head_dim]; returns ``q_out``.
    """
    _cuda(qkv, positions, q_weight, k_weight, cos_sin_cache, q_out)
    _need(qkv.dtype == BF16 and qkv.stride(-1) == 1, "qkv bf16 with contiguous rows")
    _need(positions.dtype == torch.int64, "positions int64")
    _need(cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous(), "fp32 rope table")
    num_slots = 0
    if slot_mapping is not None:
        _need(slot_mapping.dtype == torch.int32, "slot_mapping int32")
        num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    _count()
    check(lib.b200asr_qk_norm_rope_store(
        _p(qkv), qkv.stride(0), _p(positions), qkv.shape[0], num_heads, num_kv_heads, head_dim,
        _p(q_weight), _p(k_weight), float(eps), _p(cos_sin_cache), cos_sin_cache.shape[0],
        _p(q_out), q_out.stride(0), _p(k_out), _p(k_cache), _p(v_cache), _p(slot_mapping),
        num_slots, _p(error_flag), _stream()), "qk_norm_rope_store")
    return q_out


def rmsnorm(x, weight, eps: float, residual=None, out=None) -> torch.Tensor:
    """``RMSNorm`` (layers/layernorm.py:19-36). With ``residual`` it is updated in place
    to ``x + residual`` (bf16) and the norm is taken of that sum."""
    _need(x.dtype == BF16 and x.is_contiguous(), "x bf16 contiguous")
    rows, hidden = x.numel() // x.shape[-1], x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _count()
    check(lib.b200asr_rmsnorm(_p(x), _p(residual), _p(weight), float(eps), rows, hidden, _p(out),
                              _stream()), "rmsnorm")
    return out


def silu_mul(x, out=None) -> torch.Tensor:
    """``SiluAndMul`` (layers/activation.py:11-14)."""
    _need(x.dtype == BF16 and x.is_contiguous(), "x bf16 contiguous")
    inner = x.shape[-1] // 2
    rows = x.numel() // x.shape[-1]
    if out is None:
        out = torch.empty(*x.shape[:-1], inner, dtype=x.dtype, device=x.device)
    _count()
    check(lib.b200asr_silu_mul(_p(x), rows, inner, _p(out), _stream()), "silu_mul")
    return out


# ------------------------------------------------------------------- attention


def paged_decode_workspace_size(batch: int, max_seqlen_k: int, num_heads: int,
                                head_dim: int = 128) -> int:
    return int(lib.b200asr_paged_decode_workspace_size(batch, max_seqlen_k, num_heads, head_dim))


# max_seqlen_k at or below this selects the short-context decode kernel (one CTA per
# sequence and KV head, no split-K); must match kShortMaxCtx in csrc/paged_decode.cu.
DECODE_SHORT_CTX = 512


def paged_decode(q, k_cache, v_cache, cu_seqlens_k, block_tables, *, max_seqlen_k: int,
                 scale: float, out, workspace, error_flag=None) -> torch.Tensor:
    """One-token paged decode (split-K). q/out: [>= B, H, D] (rows past B, e.g. bucket
    padding, are left alone); B = cu_seqlens_k.numel() - 1; caches [N, bs, Hkv, D]."""
    _cuda(q, k_cache, v_cache, cu_seqlens_k, block_tables, out, workspace)
    rows, num_heads, head_dim = q.shape
    batch = cu_seqlens_k.numel() - 1
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    _need(block_tables.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32, "int32 metadata")
    _need(batch <= rows and batch <= block_tables.shape[0], "cu_seqlens_k longer than the batch")
    _count()  # one stream-K launch; the merge is fused into it
    check(lib.b200asr_paged_decode(
        _p(q), q.stride(0), _p(k_cache), _p(v_cache), num_blocks, block_size, num_heads,
        num_kv_heads, head_dim, _p(cu_seqlens_k), _p(block_tables), block_tables.stride(0), batch,
        max_seqlen_k, float(scale), _p(out), out.stride(0), _p(workspace),
        workspace.numel() * workspace.element_size(), _p(error_flag), _stream()), "paged_decode")
    return out


_POOL_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
_POOL_WORKSPACE: dict[int, list[torch.Tensor]] = {}


def pool_decode_workspace(batch: int, num_heads: int, head_dim: int, max_seq_len: int,
                          device) -> torch.Tensor:
    """A zero-filled workspace for :func:`pool_paged_decode`, cached per device and grown
    on demand. Growing allocates a new, larger buffer but keeps every buffer handed out
    before alive for the life of the process, so a CUDA graph captured earlier with a
    smaller one still replays into memory it owns (allocate before capturing)."""
    need = lib.b200asr_pool_paged_decode_workspace_size(batch, num_heads, head_dim, max_seq_len)
    device = torch.device(device)
    dev = device.index if device.index is not None else torch.cuda.current_device()
    held = _POOL_WORKSPACE.setdefault(dev, [])
    if not held or held[-1].numel() < need:
        held.append(torch.zeros(max(need, 1 << 20), dtype=torch.uint8,
                                device=torch.device("cuda", dev)))
    return held[-1]


def pool_paged_decode(query, key_pool, value_pool, page_table, seq_lens, *, max_seq_len: int,
                      scale: float, out=None, key_valid_mask=None, new_key=None, new_value=None,
                      tokens_per_cta: int = 0, workspace=None, error_flag=None) -> torch.Tensor:
    """One-token decode over a page pool ``[pages, H_kv, page_size, D]`` with the fused
    current-token write (agent/qwen_tts_paged_attention.py:130-287, 383-532).

    query/out ``[B, H, 1, D]`` (any strides with a unit last one), page_table/seq_lens
    int64, key_valid_mask bool ``[B, >= 0]``, new_key/new_value ``[B, H_kv, 1, D]`` or
    None. The pools are updated in place when new K/V are given."""
    _cuda(query, key_pool, value_pool, page_table, seq_lens, key_valid_mask, new_key, new_value)
    batch, num_heads, _, head_dim = query.shape
    num_pages, num_kv_heads, page_size, _ = key_pool.shape
    dtype = _POOL_DTYPES.get(query.dtype)
    _need(dtype is not None, "pool_paged_decode: bf16, fp16 or fp32 tensors")
    _need(key_pool.dtype == query.dtype and value_pool.dtype == query.dtype,
          "pool_paged_decode: query and pools must share a dtype")
    _need(key_pool.stride() == value_pool.stride(), "pool_paged_decode: pools must share strides")
    _need(query.stride(-1) == 1 and key_pool.stride(-1) == 1, "pool_paged_decode: unit head_dim stride")
    _need(page_table.dtype == torch.int64 and seq_lens.dtype == torch.int64,
          "pool_paged_decode: int64 page table and lengths")
    if page_table.stride(-1) != 1:
        page_table = page_table.contiguous()
    if seq_lens.stride(0) != 1:  # the kernel reads lengths as a dense vector
        seq_lens = seq_lens.contiguous()
    if out is None:
        out = torch.empty_like(query)
    valid_stride = valid_len = 0
    if key_valid_mask is not None:
        _need(key_valid_mask.dtype in (torch.bool, torch.uint8) and key_valid_mask.dim() == 2,
              "pool_paged_decode: key_valid_mask [B, L] bool")
        if key_valid_mask.stride(-1) != 1:
            key_valid_mask = key_valid_mask.contiguous()
        valid_stride, valid_len = key_valid_mask.stride(0), key_valid_mask.shape[1]
    new_sb = new_sh = 0
    if new_key is not None:
        _need(new_value is not None and new_key.stride() == new_value.stride()
              and new_key.dtype == query.dtype and new_key.stride(-1) == 1,
              "pool_paged_decode: new_key/new_value must match (dtype, strides)")
        new_sb, new_sh = new_key.stride(0), new_key.stride(1)
    if workspace is None:
        workspace = pool_decode_workspace(batch, num_heads, head_dim, max_seq_len, query.device)
    _count()
    check(lib.b200asr_pool_paged_decode(
        dtype, batch, num_heads, num_kv_heads, head_dim, _p(query), query.stride(0),
        query.stride(1), _p(key_pool), _p(value_pool), num_pages, page_size, key_pool.stride(0),
        key_pool.stride(1), key_pool.stride(2), _p(page_table), page_table.stride(0),
        page_table.shape[1], _p(seq_lens), _p(key_valid_mask), valid_stride, valid_len,
        _p(new_key), _p(new_value), new_sb, new_sh, _p(out), out.stride(0), out.stride(1),
        int(max_seq_len), int(tokens_per_cta), float(scale), _p(workspace),
        workspace.numel() * workspace.element_size(), _p(error_flag), _stream()),
        "pool_paged_decode")
    return out


def paged_prefill(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_tables, *,
                  max_seqlen_q: int, scale: float, out, error_flag=None) -> torch.Tensor:
    """Varlen causal GQA over the paged cache on tcgen05 (layers/attention.py:96-107)."""
    _cuda(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_tables, out)
    total_q, num_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    batch = cu_seqlens_q.numel() - 1
    _count()
    check(lib.b200asr_paged_prefill(
        _p(q), q.stride(0), _p(k_cache), _p(v_cache), num_blocks, block_size, num_heads,
        num_kv_heads, head_dim, _p(cu_seqlens_q), _p(cu_seqlens_k), _p(block_tables),
        block_tables.stride(0), batch, total_q, max_seqlen_q, float(scale), _p(out), out.stride(0),
        _p(error_flag), _stream()), "paged_prefill")
    return out


def varlen_attention(q, k, v, cu_seqlens, max_seqlen: int, scale: float, out=None,
                     error_flag=None) -> torch.Tensor:
    """``VarlenSelfAttention.forward`` (layers/attention.py:121-139), causal=False."""
    _cuda(q, k, v, cu_seqlens)
    total, num_heads, head_dim = q.shape
    for t in (q, k, v):
        _need(t.dtype == BF16 and t.stride(-1) == 1 and t.stride(1) == head_dim, "q/k/v layout")
    if out is None:
        out = torch.empty(total, num_heads, head_dim, dtype=q.dtype, device=q.device)
    _count()
    check(lib.b200asr_varlen_attention(
        _p(q), q.stride(0), _p(k), k.stride(0), _p(v), v.stride(0), _p(cu_seqlens),
        cu_seqlens.numel() - 1, total, int(max_seqlen), num_heads, head_dim, float(scale), _p(out),
        out.stride(0), _p(error_flag), _stream()), "varlen_attention")
    return out


# --------------------------------------------------------------------- sampler


def greedy_argmax(logits, out=None) -> torch.Tensor:
    """Greedy branch of ``Sampler`` (layers/sampler.py:16-20): first-max index per row."""
    _cuda(logits)
    _need(logits.dtype == BF16 and logits.stride(-1) == 1, "bf16 logits with contiguous rows")
    batch, vocab = logits.shape
    if out is None:
        out = torch.empty(batch, dtype=torch.int64, device=logits.device)
    _count()
    check(lib.b200asr_greedy_argmax(_p(logits), logits.stride(0), batch, vocab, _p(out),
                                    _stream()), "greedy_argmax")
    return out


# ------------------------------------------------------------------ frontend


def log_mel_workspace_size(batch: int, total_frames: int) -> int:
    return int(lib.b200asr_log_mel_workspace_size(batch, total_frames))


def log_mel(waveform, cu_samples, frame_start, *, total_frames: int, tables, mel_filters,
            filter_range, out, out_col, workspace, error_flag=None) -> None:
    """Whisper log-mel of every clip into bf16 ``out[128, cols]`` (audio/frontend.py:71-94).

    waveform f32 [S]; cu_samples i64 [B+1]; frame_start i32 [B+1]; out_col i32 [B]."""
    _cuda(waveform, cu_samples, frame_start, tables, mel_filters, filter_range, out, out_col,
          workspace)
    _need(waveform.dtype == torch.float32 and waveform.is_contiguous(), "f32 contiguous waveform")
    _need(cu_samples.dtype == torch.int64 and frame_start.dtype == torch.int32
          and out_col.dtype == torch.int32 and filter_range.dtype == torch.int32,
          "int64 cu_samples, int32 frame_start/out_col/filter_range")
    _need(out.dtype == BF16 and out.dim() == 2 and out.shape[0] == 128 and out.stride(1) == 1,
          "bf16 [128, cols] output with contiguous rows")
    batch = cu_samples.numel() - 1
    _count(2)  # log-mel + finish (plus a memset of the per-clip maxima)
    check(lib.b200asr_log_mel(
        _p(waveform), _p(cu_samples), _p(frame_start), batch, int(total_frames), _p(tables),
        _p(mel_filters), _p(filter_range), _p(workspace),
        workspace.numel() * workspace.element_size(), _p(out), out.stride(0), _p(out_col),
        _p(error_flag), _stream()), "log_mel")


# ------------------------------------------------------------------- linears

LINEAR_SMALL_MAX_ROWS = 64


def linear_small_ok(x, weight, silu: bool = False) -> bool:
    """Whether ``linear_small`` takes this projection (decode batch sizes, aligned dims)."""
    if x.dim() != 2 or x.dtype != BF16 or weight.dtype != BF16 or not weight.is_contiguous():
        return False
    m, k = x.shape
    n = weight.shape[0]
    if not (1 <= m <= LINEAR_SMALL_MAX_ROWS and k % 64 == 0 and weight.shape[1] == k
            and x.stride(1) == 1 and x.stride(0) % 8 == 0):
        return False
    return (n % 2 == 0 and (n // 2) % 64 == 0) if silu else n % 128 == 0


def linear_small(x, weight, *, silu: bool = False, out=None, error_flag=None) -> torch.Tensor:
    """``x @ weight.T`` for 1..64 rows on tcgen05 (fused SiLU*mul when ``silu``)."""
    _cuda(x, weight)
    _need(linear_small_ok(x, weight, silu), "linear_small: unsupported shape/layout")
    m, k = x.shape
    n = weight.shape[0]
    cols = n // 2 if silu else n
    if out is None:
        out = torch.empty(m, cols, dtype=BF16, device=x.device)
    _count()
    check(lib.b200asr_linear_small(_p(x), x.stride(0), m, k, _p(weight), n, cols if silu else 0,
                                   _p(out), out.stride(0), _p(error_flag), _stream()),
          "linear_small")
    return out


# ---------------------------------------------------------------- decode-step fusions
# A decoder row between the projections of a decode step is carried as ``h`` (fp32
# [m, hidden], the pre-norm residual sum) and ``ss`` (fp32 [m, hidden / 128], per
# 128-column partial sums of h^2); the RMSNorm is applied by the next projection.


def l2_prefetch(kv=None, ranges=()):
    """A ``b200asr_l2_prefetch`` for the fused projections: ``kv = (cu_seqlens_k,
    block_tables, k_cache, v_cache)`` of one layer (4-D caches) and up to two tensors
    whose bytes to request (e.g. the next layer's weights). None when empty."""
    from voiceagent_b200._lib import L2Prefetch

    if kv is None and not ranges:
        return None
    p = L2Prefetch()
    if kv is not None:
        cu, tables, kc, vc = kv
        _cuda(cu, tables, kc, vc)
        _need(cu.dtype == torch.int32 and tables.dtype == torch.int32 and tables.dim() == 2
              and tables.stride(1) == 1 and kc.dim() == 4 and kc.is_contiguous()
              and vc.is_contiguous(), "l2_prefetch: int32 metadata, 4-D contiguous caches")
        p.cu_seqlens_k, p.block_tables = cu.data_ptr(), tables.data_ptr()
        p.bt_stride, p.batch = tables.stride(0), tables.shape[0]
        p.block_size, p.num_kv_heads, p.head_dim = kc.shape[1], kc.shape[2], kc.shape[3]
        p.k_cache, p.v_cache = kc.data_ptr(), vc.data_ptr()
        p.num_slots = kc.shape[0] * kc.shape[1]
    _need(len(ranges) <= 2, "l2_prefetch: at most two ranges")
    for i, t in enumerate(ranges):
        _cuda(t)
        _need(t.is_contiguous(), "l2_prefetch: contiguous ranges")
        p.range[i] = t.data_ptr()
        p.range_bytes[i] = t.numel() * t.element_size()
    return p


def _pf(p):
    return None if p is None else ctypes.byref(p)


class NormState:
    """``h`` and ``ss`` buffers of a decode step (rows <= 64)."""

    def __init__(self, rows: int, hidden: int, device):
        self.rows, self.hidden = rows, hidden
        self.h = torch.empty(rows, hidden, dtype=torch.float32, device=device)
        self.ss = torch.empty(rows, hidden // 128, dtype=torch.float32, device=device)

    @property
    def tiles(self) -> int:
        return self.hidden // 128


def fused_decode_ok(m: int, hidden: int, intermediate: int, num_heads: int, num_kv_heads: int,
                    head_dim: int) -> bool:
    """Whether the fused decode-step projections take a batch of ``m`` rows."""
    # The RMSNorm prologue needs a CTA's whole K slice (the hidden size / the split) in its
    # 4-stage ring. Up to hidden 1024 a 4-way split does that; at 2048 (1.7B) it takes an
    # 8-way split -- 768 gate_up CTAs, 2.6 waves -- and the fused 1.7B step measured
    # 3487 us against 2286 us for the unfused kernels at 64 rows, so wider models take the
    # unfused path. The MLP width only sets gate_up's tile count and down_proj's K.
    return (1 <= m <= LINEAR_SMALL_MAX_ROWS and head_dim == 128 and hidden % 512 == 0
            and hidden <= 1024 and intermediate % 64 == 0 and intermediate <= 16384
            and (num_heads * head_dim) % 64 == 0 and num_heads % num_kv_heads == 0)


def rms_stats(x, state: NormState, residual=None) -> NormState:
    """h = x (+ residual, updated in place to bf16(x + residual)) and its tile sums."""
    _cuda(x, residual)
    _need(x.dtype == BF16 and x.is_contiguous() and x.shape == state.h.shape, "x bf16 [m, hidden]")
    _count()
    check(lib.b200asr_rms_stats(_p(x), _p(residual), x.shape[0], x.shape[1], _p(state.h),
                                _p(state.ss), _stream()), "rms_stats")
    return state


def norm_apply(state: NormState, weight, eps: float, out=None) -> torch.Tensor:
    """RMSNorm (layers/layernorm.py:19-25) of rows held as (h, ss)."""
    if out is None:
        out = torch.empty(state.rows, state.hidden, dtype=BF16, device=state.h.device)
    _count()
    check(lib.b200asr_norm_apply(_p(state.h), _p(state.ss), _p(weight), float(eps), state.rows,
                                 state.hidden, _p(out), _stream()), "norm_apply")
    return out


def linear_small_add(x, weight, residual, state: NormState, prefetch=None,
                     error_flag=None) -> NormState:
    """``x @ weight.T`` + the residual add of the following RMSNorm: residual <- bf16(h),
    state <- (h, tile sums of h^2)."""
    _cuda(x, weight, residual)
    _need(linear_small_ok(x, weight), "linear_small_add: unsupported shape/layout")
    m, k = x.shape
    n = weight.shape[0]
    _need(residual.dtype == BF16 and residual.shape == (m, n) and residual.stride(1) == 1
          and state.h.shape == (m, n), "linear_small_add: residual / state shape")
    _count()
    check(lib.b200asr_linear_small_add(_p(x), x.stride(0), m, k, _p(weight), n, _p(residual),
                                       residual.stride(0), _p(state.h), state.h.stride(0),
                                       _p(state.ss), _pf(prefetch), _p(error_flag), _stream()),
          "linear_small_add")
    return state


def linear_small_norm(state: NormState, norm_weight, eps: float, weight, *, silu: bool = False,
                      out=None, prefetch=None, error_flag=None) -> torch.Tensor:
    """``RMSNorm(h) @ weight.T`` (fused SiLU*mul when ``silu``)."""
    _cuda(norm_weight, weight)
    m, k = state.rows, state.hidden
    n = weight.shape[0]
    _need(weight.dtype == BF16 and weight.is_contiguous() and weight.shape[1] == k,
          "linear_small_norm: weight [n, hidden] bf16")
    cols = n // 2 if silu else n
    if out is None:
        out = torch.empty(m, cols, dtype=BF16, device=weight.device)
    _count()
    check(lib.b200asr_linear_small_norm(_p(state.h), state.h.stride(0), _p(state.ss), state.tiles,
                                        _p(norm_weight), float(eps), m, k, _p(weight), n,
                                        cols if silu else 0, _p(out), out.stride(0),
                                        _pf(prefetch), _p(error_flag), _stream()),
          "linear_small_norm")
    return out


def linear_small_norm_qk_rope(state: NormState, norm_weight, eps: float, weight, positions, *,
                              num_heads: int, num_kv_heads: int, head_dim: int, q_weight,
                              k_weight, qk_eps: float, cos_sin_cache, q_out, k_cache, v_cache,
                              slot_mapping, prefetch=None, error_flag=None) -> torch.Tensor:
    """qkv_proj of RMSNorm(h), then q/k RMSNorm + RoPE and the K/V cache store per head
    (``prefetch``: an ``l2_prefetch`` hint or None)."""
    _cuda(norm_weight, weight, positions, q_weight, k_weight, cos_sin_cache, q_out, k_cache,
          v_cache, slot_mapping)
    _need(positions.dtype == torch.int64 and slot_mapping.dtype == torch.int32,
          "positions int64, slot_mapping int32")
    _need(cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous(), "fp32 rope table")
    _need(weight.dtype == BF16 and weight.is_contiguous() and weight.shape[1] == state.hidden,
          "qkv weight [n, hidden] bf16")
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    _count()
    check(lib.b200asr_linear_small_norm_qk_rope(
        _p(state.h), state.h.stride(0), _p(state.ss), state.tiles, _p(norm_weight), float(eps),
        state.rows, state.hidden, _p(weight), num_heads, num_kv_heads, head_dim, _p(q_weight),
        _p(k_weight), float(qk_eps), _p(positions), _p(cos_sin_cache), cos_sin_cache.shape[0],
        _p(q_out), q_out.stride(0), _p(k_cache), _p(v_cache), _p(slot_mapping), num_slots,
        _pf(prefetch), _p(error_flag), _stream()),
        "linear_small_norm_qk_rope")
    return q_out


def linear_small_qk_rope(x, weight, positions, *, num_heads: int, num_kv_heads: int,
                         head_dim: int, q_weight, k_weight, qk_eps: float, cos_sin_cache, q_out,
                         k_cache, v_cache, slot_mapping, error_flag=None) -> torch.Tensor:
    """qkv_proj of an already normalised x, then q/k RMSNorm + RoPE and the K/V cache
    store per head: :func:`linear_small` followed by :func:`qk_norm_rope_store` in one
    kernel."""
    _cuda(x, weight, positions, q_weight, k_weight, cos_sin_cache, q_out, k_cache, v_cache,
          slot_mapping)
    _need(x.dtype == BF16 and x.dim() == 2 and x.stride(1) == 1, "x bf16 [m, k], unit column stride")
    _need(positions.dtype == torch.int64 and slot_mapping.dtype == torch.int32,
          "positions int64, slot_mapping int32")
    _need(cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous(), "fp32 rope table")
    _need(weight.dtype == BF16 and weight.is_contiguous() and weight.shape[1] == x.shape[1],
          "qkv weight [n, k] bf16")
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    _count()
    check(lib.b200asr_linear_small_qk_rope(
        _p(x), x.stride(0), x.shape[0], x.shape[1], _p(weight), num_heads, num_kv_heads, head_dim,
        _p(q_weight), _p(k_weight), float(qk_eps), _p(positions), _p(cos_sin_cache),
        cos_sin_cache.shape[0], _p(q_out), q_out.stride(0), _p(k_cache), _p(v_cache),
        _p(slot_mapping), num_slots, _p(error_flag), _stream()), "linear_small_qk_rope")
    return q_out


# ----------------------------------------------------------------- encoder front


def conv_pack_weight(weight: torch.Tensor) -> torch.Tensor:
    """A Conv2d(3x3) weight [C_out, C_in, 3, 3] bf16 repacked for
    :func:`conv3x3s2_gelu` (call once, at load time)."""
    _cuda(weight)
    c_out, c_in = weight.shape[:2]
    _need(weight.dtype == BF16 and tuple(weight.shape[2:]) == (3, 3), "bf16 [C_out, C_in, 3, 3]")
    weight = weight.contiguous()
    packed = torch.empty(lib.b200asr_conv_weight_bytes(c_out, c_in) // 2, dtype=BF16,
                         device=weight.device)
    _count()
    check(lib.b200asr_conv_pack_weight(_p(weight), c_out, c_in, _p(packed), _stream()),
          "conv_pack_weight")
    return packed


def conv3x3s2_gelu(x: torch.Tensor, packed_weight: torch.Tensor, bias: torch.Tensor, *,
                   c_out: int, out: torch.Tensor | None = None, out_order: str = "nyxc",
                   error_flag=None) -> torch.Tensor:
    """GELU(Conv2d(x, kernel 3, stride 2, padding 1) + bias) on channels-last bf16
    x [N, H, W, C_in] (models/audio_encoder.py:145-175). The output is [N, Ho, Wo, C_out]
    (``out_order`` "nyxc") or [N, Wo, Ho, C_out] ("nxyc": per chunk, time-major rows of
    (frequency, channel) -- the layout conv_out reads)."""
    _cuda(x, packed_weight, bias, out)
    n, h, w, c_in = x.shape
    _need(x.dtype == BF16 and x.is_contiguous(), "conv3x3s2_gelu: contiguous bf16 channels-last x")
    _need(bias.dtype == BF16 and bias.numel() == c_out, "conv3x3s2_gelu: bf16 bias [C_out]")
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    shape = (n, ho, wo, c_out) if out_order == "nyxc" else (n, wo, ho, c_out)
    if out is None:
        out = torch.empty(shape, dtype=BF16, device=x.device)
    _need(tuple(out.shape) == shape and out.is_contiguous(), "conv3x3s2_gelu: output shape")
    sn = ho * wo * c_out
    sy, sx = (wo * c_out, c_out) if out_order == "nyxc" else (c_out, ho * c_out)
    _count()
    check(lib.b200asr_conv3x3s2_gelu(_p(x), n, h, w, c_in, _p(packed_weight), _p(bias), c_out,
                                     _p(out), sn, sy, sx, _p(error_flag), _stream()),
          "conv3x3s2_gelu")
    return out


def set_pdl(enable: bool) -> None:
    """Programmatic dependent launch for the decode-path kernels (process-wide)."""
    lib.b200asr_set_pdl(1 if enable else 0)


def pdl_enabled() -> bool:
    return bool(lib.b200asr_pdl_enabled())
