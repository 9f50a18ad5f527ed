"""Numpy restatements of the qwen_asr_vllm hot-path functions (test infrastructure).

Every function names the reference function it restates (path:line inside the
``qwen-asr-vllm`` project). Integer outputs are exact; floating-point outputs are
computed in float64 from inputs that hold bf16-representable values, and rounded
to bf16 only where the reference rounds.

bf16 tensors are represented as float32 numpy arrays whose values are exactly
representable in bf16 (see :func:`bf16_round`).
"""

from __future__ import annotations

import numpy as np

BLOCK_SIZE = 256
CHUNK_FRAMES = 100


# --------------------------------------------------------------------------- bf16


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (ties to even), as float32.

    Matches ``tensor.to(torch.bfloat16)`` for finite values and keeps NaN/Inf.
    """
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isfinite(x), r, x).astype(np.float32)


# -------------------------------------------------------------- audio accounting


def conv_output_len(length: int) -> int:
    """``audio/tokens.py:16-18``: one Conv2d(k=3, s=2, p=1) output length."""
    return (length - 1) // 2 + 1


def after_cnn_len(frames: int) -> int:
    """``audio/tokens.py:21-23``: frames left after three stride-2 convolutions."""
    return conv_output_len(conv_output_len(conv_output_len(frames)))


TOKENS_PER_FULL_CHUNK = after_cnn_len(CHUNK_FRAMES)


def num_audio_tokens(mel_frames: int, chunk_frames: int = CHUNK_FRAMES) -> int:
    """``audio/tokens.py:30-37``: closed-form audio token count."""
    full, tail = divmod(int(mel_frames), chunk_frames)
    return full * after_cnn_len(chunk_frames) + after_cnn_len(tail)


def chunk_lengths_for(mel_frames: int, chunk_frames: int = CHUNK_FRAMES) -> list[int]:
    """``audio/tokens.py:40-52``: split mel frames into convolution chunks."""
    if mel_frames <= 0:
        raise ValueError(f"mel_frames must be positive, got {mel_frames}")
    full, tail = divmod(int(mel_frames), chunk_frames)
    return [chunk_frames] * full + ([tail] if tail else [])


def attention_window_tokens(n_window_infer: int, chunk_frames: int = CHUNK_FRAMES) -> int:
    """``audio/batcher.py:75-77``."""
    return TOKENS_PER_FULL_CHUNK * (n_window_infer // chunk_frames)


def build_window_boundaries(audio_token_lens, window_tokens: int) -> list[int]:
    """``audio/batcher.py:80-98``: cumulative encoder window boundaries."""
    out = [0]
    for n in audio_token_lens:
        full, rem = divmod(int(n), window_tokens)
        for _ in range(full):
            out.append(out[-1] + window_tokens)
        if rem:
            out.append(out[-1] + rem)
    return out


def pack_audio_metadata(mel_frames, n_window_infer: int = 800) -> dict:
    """Metadata half of ``audio/batcher.py:101-141`` (``pack_audio_batch``)."""
    if len(mel_frames) == 0:
        raise ValueError("pack_audio_batch requires at least one request")
    chunk_lengths: list[int] = []
    token_lens: list[int] = []
    for f in mel_frames:
        chunk_lengths.extend(chunk_lengths_for(int(f)))
        token_lens.append(num_audio_tokens(int(f)))
    window = attention_window_tokens(n_window_infer)
    cu = build_window_boundaries(token_lens, window)
    max_seqlen = max((b - a for a, b in zip(cu[:-1], cu[1:])), default=cu[0])
    return {
        "chunk_lengths": np.asarray(chunk_lengths, dtype=np.int64),
        "chunk_valid_lens": np.asarray([after_cnn_len(c) for c in chunk_lengths], dtype=np.int64),
        "cu_seqlens": np.asarray(cu, dtype=np.int32),
        "audio_token_lens": np.asarray(token_lens, dtype=np.int32),
        "window_tokens": window,
        "max_seqlen": int(max_seqlen),
    }


def chunk_and_pad(mel: np.ndarray, chunk_lengths, chunk_frames: int = CHUNK_FRAMES) -> np.ndarray:
    """``models/audio_encoder.py:130-143``: packed mel -> (chunks, mel_bins, chunk_frames)."""
    bins = mel.shape[0]
    out = np.zeros((len(chunk_lengths), bins, chunk_frames), dtype=mel.dtype)
    start = 0
    for i, n in enumerate(chunk_lengths):
        out[i, :, :n] = mel[:, start : start + n]
        start += n
    return out


# ---------------------------------------------------------------- decoder packer


def pack_decoder(starts, ends, tables, token_ids, block_size: int = BLOCK_SIZE) -> dict:
    """``engine/model_runner.py:183-233`` (``ModelRunner._prepare``), metadata part.

    ``token_ids[i]`` is request i's full token list; the query span is
    ``token_ids[i][starts[i]:ends[i]]``. Block tables are padded with -1 to the
    widest table in the batch.
    """
    input_ids, positions, slots = [], [], []
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    for s, e, table, toks in zip(starts, ends, tables, token_ids):
        s, e = int(s), int(e)
        input_ids.extend(int(t) for t in toks[s:e])
        positions.extend(range(s, e))
        for p in range(s, e):
            slots.append(int(table[p // block_size]) * block_size + p % block_size)
        cu_q.append(cu_q[-1] + (e - s))
        cu_k.append(cu_k[-1] + e)
        max_q = max(max_q, e - s)
        max_k = max(max_k, e)
    width = max(len(t) for t in tables)
    bt = np.full((len(tables), width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = t
    cu_q_arr = np.asarray(cu_q, dtype=np.int32)
    return {
        "input_ids": np.asarray(input_ids, dtype=np.int64),
        "positions": np.asarray(positions, dtype=np.int64),
        "slot_mapping": np.asarray(slots, dtype=np.int32),
        "cu_seqlens_q": cu_q_arr,
        "cu_seqlens_k": np.asarray(cu_k, dtype=np.int32),
        "max_seqlen_q": max_q,
        "max_seqlen_k": max_k,
        "block_tables": bt,
        # model_runner.py:296 -- the row of each request's last query token
        "last_token_indices": cu_q_arr[1:].astype(np.int64) - 1,
    }


def pack_decode_bucket(
    lens, last_ids, tables, bucket: int, max_blocks: int, block_size: int = BLOCK_SIZE
) -> dict:
    """``engine/graph_runner.py:149-191`` (``GraphRunner.run``) host staging.

    Padding rows get slot -1, key length 1 and an all-zero block-table row.
    Padding rows of ``input_ids``/``positions`` are written as 0 here (the
    reference leaves stale values there; those rows are discarded either way).
    """
    b = len(lens)
    input_ids = np.zeros(bucket, dtype=np.int64)
    positions = np.zeros(bucket, dtype=np.int64)
    slots = np.full(bucket, -1, dtype=np.int32)
    cu_k = np.zeros(bucket + 1, dtype=np.int32)
    bt = np.zeros((bucket, max_blocks), dtype=np.int32)
    running = 0
    for i in range(b):
        pos = int(lens[i]) - 1
        table = tables[i]
        input_ids[i] = int(last_ids[i])
        positions[i] = pos
        slots[i] = int(table[pos // block_size]) * block_size + pos % block_size
        bt[i, : len(table)] = table
        running += int(lens[i])
        cu_k[i + 1] = running
    for i in range(b, bucket):
        running += 1
        cu_k[i + 1] = running
    return {
        "input_ids": input_ids,
        "positions": positions,
        "slot_mapping": slots,
        "cu_seqlens_k": cu_k,
        "block_tables": bt,
    }


# ---------------------------------------------------------------------- KV store


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """``layers/attention.py:31-67``: scatter K/V rows into slots; -1 skips.

    ``key``/``value``: (T, H_kv, D); caches: (N, block, H_kv, D). Updated in place.
    """
    kf = k_cache.reshape(-1, k_cache.shape[-2] * k_cache.shape[-1])
    vf = v_cache.reshape(-1, v_cache.shape[-2] * v_cache.shape[-1])
    for t, slot in enumerate(np.asarray(slot_mapping)):
        if int(slot) == -1:
            continue
        kf[int(slot)] = key[t].reshape(-1)
        vf[int(slot)] = value[t].reshape(-1)


# --------------------------------------------------------------------- attention


def _softmax_attend(q, keys, values, scale, mask=None):
    """q: (Lq, D), keys/values: (Lk, D) -> (Lq, D) in float64."""
    s = (q.astype(np.float64) @ keys.astype(np.float64).T) * scale
    if mask is not None:
        s = np.where(mask, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    return p @ values.astype(np.float64)


def gather_paged(cache, table, length: int, block_size: int = BLOCK_SIZE):
    """Logical rows 0..length-1 of one sequence from a paged cache (N, bs, H, D)."""
    pos = np.arange(length)
    blocks = np.asarray(table, dtype=np.int64)[pos // block_size]
    return cache[blocks, pos % block_size]  # (length, H, D)


def paged_attention(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_tables, scale,
                    block_size: int = BLOCK_SIZE) -> np.ndarray:
    """``layers/attention.py:87-107``: FlashAttention varlen over the paged cache.

    Causal with bottom-right alignment (attention.py:1-11): query i of a request
    with q_len queries and k_len keys attends keys ``0 .. k_len - q_len + i``.
    GQA: query head h reads KV head ``h // (H_q // H_kv)``.
    """
    hq = q.shape[1]
    hkv = k_cache.shape[2]
    group = hq // hkv
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(len(cu_seqlens_q) - 1):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        lk = int(cu_seqlens_k[b + 1]) - int(cu_seqlens_k[b])
        lq = q1 - q0
        if lq == 0:
            continue
        keys = gather_paged(k_cache, block_tables[b], lk, block_size)
        vals = gather_paged(v_cache, block_tables[b], lk, block_size)
        qi = np.arange(lq)[:, None] + (lk - lq)
        kj = np.arange(lk)[None, :]
        mask = kj <= qi
        for h in range(hq):
            out[q0:q1, h] = _softmax_attend(q[q0:q1, h], keys[:, h // group], vals[:, h // group],
                                            scale, mask)
    return out


def write_current_kv(key_pool, value_pool, page_table, seq_lens, new_key, new_value) -> None:
    """``agent/qwen_tts_paged_attention.py:519-532`` (``_write_current_kv``): row b's new
    key/value (``[B, H_kv, 1, D]``) land at position ``seq_lens[b] - 1`` of its pages in
    the pool ``[pages, H_kv, page_size, D]`` (in place)."""
    ps = key_pool.shape[2]
    for b in range(new_key.shape[0]):
        pos = int(seq_lens[b]) - 1
        page = int(page_table[b, pos // ps])
        key_pool[page, :, pos % ps, :] = new_key[b, :, 0, :]
        value_pool[page, :, pos % ps, :] = new_value[b, :, 0, :]


def pool_paged_attention(query, key_pool, value_pool, page_table, seq_lens, scale,
                         key_valid_mask=None, new_key=None, new_value=None,
                         kernel_seq_len=None) -> np.ndarray:
    """One-token GQA attention over a page pool in the TTS talker layout.

    Restates ``paged_attention_decode`` (agent/qwen_tts_paged_attention.py:383-516) with
    the semantics of its CUDA kernel (130-287) and torch path (353-380):

    * query ``[B, H, 1, D]``; pools ``[pages, H_kv, page_size, D]``; ``page_table``
      ``[B, W]`` maps logical page ``p // page_size`` of row b to a physical page;
    * with ``new_key``/``new_value`` the current token is written first
      (:func:`write_current_kv`, in place) and attended like any cached token;
    * row b attends positions ``0 .. min(seq_lens[b], kernel_seq_len) - 1`` (the kernel's
      loop bound, 226-232), minus those whose ``key_valid_mask[b, t]`` is False; mask
      columns beyond the mask's width count as valid (the launcher pads with True,
      466-475);
    * a row with no valid key returns zeros (the kernel's ``max(sum, 1e-20)`` guard with
      zero-filled masked values; the torch path would average the masked values instead).

    Float64 arithmetic; returns ``[B, H, 1, D]``.
    """
    if new_key is not None:
        write_current_kv(key_pool, value_pool, page_table, seq_lens, new_key, new_value)
    bsz, hq, _, d = query.shape
    hkv, ps = key_pool.shape[1], key_pool.shape[2]
    group = hq // hkv
    out = np.zeros((bsz, hq, 1, d), dtype=np.float64)
    for b in range(bsz):
        length = int(seq_lens[b])
        if kernel_seq_len is not None:
            length = min(length, int(kernel_seq_len))
        pos = np.arange(length)
        valid = np.ones(length, dtype=bool)
        if key_valid_mask is not None:
            w = min(length, key_valid_mask.shape[1])
            valid[:w] = key_valid_mask[b, :w]
        pos = pos[valid]
        if pos.size == 0:
            continue
        pages = np.asarray(page_table[b], dtype=np.int64)[pos // ps]
        keys = key_pool[pages, :, pos % ps, :]    # (n, H_kv, D)
        vals = value_pool[pages, :, pos % ps, :]
        for h in range(hq):
            out[b, h, 0] = _softmax_attend(query[b, h], keys[:, h // group], vals[:, h // group],
                                           scale)
    return out


def varlen_attention(q, k, v, cu_seqlens, scale) -> np.ndarray:
    """``layers/attention.py:121-139``: non-causal attention inside each segment."""
    out = np.zeros(q.shape, dtype=np.float64)
    for w in range(len(cu_seqlens) - 1):
        a, b = int(cu_seqlens[w]), int(cu_seqlens[w + 1])
        if b <= a:
            continue
        for h in range(q.shape[1]):
            out[a:b, h] = _softmax_attend(q[a:b, h], k[a:b, h], v[a:b, h], scale)
    return out


# ------------------------------------------------------- norms, rope, activation


def rms_norm(x, weight, eps: float = 1e-6) -> np.ndarray:
    """``layers/layernorm.py:19-25``: fp32 RMSNorm, cast to bf16, times bf16 weight."""
    xf = np.asarray(x, dtype=np.float32)
    var = np.mean(xf.astype(np.float64) ** 2, axis=-1, keepdims=True)
    y = bf16_round(xf * (1.0 / np.sqrt(var + eps)).astype(np.float32))
    return bf16_round(y * np.asarray(weight, dtype=np.float32))


def add_rms_norm(x, residual, weight, eps: float = 1e-6):
    """``layers/layernorm.py:27-36``: returns (normed bf16, new residual bf16)."""
    s = np.asarray(x, dtype=np.float32) + np.asarray(residual, dtype=np.float32)
    new_res = bf16_round(s)
    var = np.mean(s.astype(np.float64) ** 2, axis=-1, keepdims=True)
    y = bf16_round(s * (1.0 / np.sqrt(var + eps)).astype(np.float32))
    return bf16_round(y * np.asarray(weight, dtype=np.float32)), new_res


def rope_cache(head_dim: int, max_position: int, base: float) -> np.ndarray:
    """``layers/rotary_embedding.py:17-25``: (max_position, head_dim) fp32 [cos | sin].

    The angle is the fp32 product the reference forms; cos/sin of it are taken in
    float64 and rounded once. (torch's fp32 cos/sin carry up to ~2e-4 absolute
    error at angles near 4096 rad, so the table is an input of every kernel and
    test, never recomputed inside one.)
    """
    inv = (1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)
    freqs = (np.arange(max_position, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    f64 = freqs.astype(np.float64)
    return np.concatenate([np.cos(f64), np.sin(f64)], axis=-1).astype(np.float32)


def apply_rope(x, positions, cache) -> np.ndarray:
    """``layers/rotary_embedding.py:9-14,27-32``: half-split rotation in fp32 -> bf16.

    x: (T, H, D) bf16 values; cache rows are [cos(D/2) | sin(D/2)].
    """
    d2 = x.shape[-1] // 2
    cs = cache[np.asarray(positions, dtype=np.int64)]  # (T, D)
    cos = cs[:, None, :d2].astype(np.float32)
    sin = cs[:, None, d2:].astype(np.float32)
    first = np.asarray(x[..., :d2], dtype=np.float32)
    second = np.asarray(x[..., d2:], dtype=np.float32)
    a = (first * cos).astype(np.float32) - (second * sin).astype(np.float32)
    b = (second * cos).astype(np.float32) + (first * sin).astype(np.float32)
    return bf16_round(np.concatenate([a, b], axis=-1))


def qk_norm_rope(qkv, positions, q_weight, k_weight, cache, num_heads: int, num_kv_heads: int,
                 head_dim: int, eps: float = 1e-6):
    """``models/qwen3.py:42-48``: split fused qkv, per-head RMSNorm of q/k, then RoPE.

    Returns (q, k, v) as (T, H, D) arrays of bf16 values.
    """
    qs, ks = num_heads * head_dim, num_kv_heads * head_dim
    t = qkv.shape[0]
    q = qkv[:, :qs].reshape(t, num_heads, head_dim)
    k = qkv[:, qs : qs + ks].reshape(t, num_kv_heads, head_dim)
    v = qkv[:, qs + ks : qs + 2 * ks].reshape(t, num_kv_heads, head_dim)
    q = rms_norm(q, q_weight, eps)
    k = rms_norm(k, k_weight, eps)
    return apply_rope(q, positions, cache), apply_rope(k, positions, cache), np.array(v)


def silu_mul(x) -> np.ndarray:
    """``layers/activation.py:11-14``: silu(gate) * up over a fused [gate | up] row."""
    xf = np.asarray(x, dtype=np.float32)
    h = xf.shape[-1] // 2
    gate, up = xf[..., :h].astype(np.float64), xf[..., h:]
    silu = bf16_round((gate / (1.0 + np.exp(-gate))).astype(np.float32))
    return bf16_round(silu * up)


# ----------------------------------------------------------------------- sampler


def greedy_argmax(logits) -> np.ndarray:
    """``layers/sampler.py:16-20``: argmax of fp32 logits, first index on ties."""
    return np.argmax(np.asarray(logits, dtype=np.float32), axis=-1).astype(np.int64)


def log_mel(waveform, mel_filters, n_fft: int = 400, hop: int = 160) -> np.ndarray:
    """Whisper log-mel features ``[128, n // hop]`` of one clip, in float64.

    Follows AudioFrontend.__call__ (audio/frontend.py:71-94), which calls the stock
    transformers WhisperFeatureExtractor (transformers 5.5.0 here; the reference pins
    4.57.6, same algorithm): centred STFT with reflect padding ``n_fft // 2``, periodic
    Hann window, power spectrum of the ``n_fft // 2 + 1`` bins, the last STFT frame
    dropped, ``mel_filters^T power``, ``log10(max(mel, 1e-10))``, then per clip
    ``max(x, max(x) - 8)`` and ``(x + 4) / 4``. ``mel_filters`` is the extractor's
    ``[201, 128]`` filterbank.
    """
    x = np.asarray(waveform, dtype=np.float64).reshape(-1)
    if x.size <= n_fft // 2:
        raise ValueError(f"clip of {x.size} samples is too short for reflect padding")
    padded = np.pad(x, n_fft // 2, mode="reflect")
    frames = x.size // hop
    idx = np.arange(frames)[:, None] * hop + np.arange(n_fft)[None, :]
    window = 0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(n_fft) / n_fft)
    spec = np.fft.rfft(padded[idx] * window, axis=1)
    power = spec.real ** 2 + spec.imag ** 2
    mel = power @ np.asarray(mel_filters, dtype=np.float64)
    logm = np.log10(np.maximum(mel, 1e-10))
    logm = np.maximum(logm, logm.max() - 8.0)
    return ((logm + 4.0) / 4.0).T
