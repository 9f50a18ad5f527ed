"""Per-kernel microbenchmarks of the hot path on one B200.

    python -m voiceagent_b200.microbench [--only decode prefill ...]

prints one JSON line per kernel configuration: device time per launch, algorithmic
bytes (and FLOPs for the attention contractions), achieved GB/s (TFLOP/s) and the
fraction of the measured peaks in MEASURED_PEAKS.json (copy bandwidth; cuBLAS bf16
GEMM burst throughput). Timing: the launches are captured back to back in a CUDA
graph and timed with CUDA events around a replay (no host gaps); kernels that stream
HBM rotate over input sets that together exceed the 126 MB L2, so no launch finds
its inputs cached. Latency-bound kernels (packers, decode-size rows) are reported
the same way and labelled ``latency``.

Workloads follow the reference's benchmark configurations: config 1 (paged decode,
B = 32, ctx ~ U[64, 1024], 4096-block pool), config 2 (32 clips of U(2, 30) s: the
decoder prefill over L = 13 s + 24 tokens each and the encoder's 104-token windows),
and the config-3 decode step shapes (32 rows, Qwen3-ASR-0.6B projections).
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np
import torch

from voiceagent_b200 import kernels as kx
from voiceagent_b200.audio.tokens import attention_window_tokens, num_audio_tokens

REPO = Path(__file__).resolve().parents[1]
L2_BYTES = 126 * 2**20


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def graph_time_us(launches, reps: int = 3) -> float:
    """Mean device time per callable when ``launches`` replay back to back in a graph."""
    for f in launches:
        f()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in launches:
            f()
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        graph.replay()
    e.record()
    e.synchronize()
    del graph
    return s.elapsed_time(e) * 1000.0 / reps / len(launches)


def _line(kernel, config, us, nbytes, flops=None, bound="hbm", **extra) -> dict:
    peaks = measured_peaks()
    out = {"kernel": kernel, "config": config, "us": round(us, 3), "algo_bytes": int(nbytes),
           "gbs": round(nbytes / us / 1e3, 1), "frac_hbm": round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4),
           "bound": bound, "peak_source": peaks["source"]}
    if flops is not None:
        tf = flops / us / 1e6
        out.update(flops=int(flops), tflops=round(tf, 1), frac_tensor=round(tf / peaks["bf16_tflops"], 4))
    out.update(extra)
    return out


def _sets(per_set_bytes: int) -> int:
    return max(2, -(-2 * L2_BYTES // max(per_set_bytes, 1)))


# ------------------------------------------------------------------ config 1


def decode_config1(iters: int = 64, sets: int = 4, lo: int = 64, hi: int = 1024,
                   label: str = "config1 B=32 ctx~U[64,1024] Hq16/Hkv8 d128",
                   max_seqlen_k: int = 4096, pdl: bool = False, batch: int = 32) -> dict:
    """Paged decode, config 1: B = 32, ctx ~ U[lo, hi] (64-1024), 4096-block pool (2 GiB per
    K/V), block tables = slices of a random permutation; ``sets`` disjoint table sets rotate.
    ``batch`` = 64 gives the decode-step shape of configuration 4."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)
    b, h, hkv, d, nb = batch, 16, 8, 128, 4096
    lens = rng.integers(lo, hi + 1, size=b)
    need = int(sum((lens + 255) // 256))
    gen = torch.Generator(device=dev).manual_seed(0)
    kc = (torch.randn(nb, 256, hkv, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    vc = (torch.randn(nb, 256, hkv, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    q = (torch.randn(b, h, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    perm = rng.permutation(nb)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).to(dev)
    tables = []
    for k in range(sets):
        t = np.zeros((b, 16), np.int32)
        c = k * need
        for i, n in enumerate(lens):
            m = (int(n) + 255) // 256
            t[i, :m] = perm[c:c + m]
            c += m
        tables.append(torch.from_numpy(t).to(dev))
    out = torch.empty_like(q)
    ws = torch.zeros(kx.paged_decode_workspace_size(b, 4096, h) // 4 + 64, dtype=torch.float32,
                     device=dev)

    def op(i):
        return lambda: kx.paged_decode(q, kc, vc, cu, tables[i % sets], max_seqlen_k=max_seqlen_k,
                                       scale=d ** -0.5, out=out, workspace=ws)

    was = kx.pdl_enabled()
    kx.set_pdl(pdl)  # PDL: each launch's metadata reads and first ring overlap the last
    try:
        us = graph_time_us([op(i) for i in range(iters)])
    finally:
        kx.set_pdl(was)
    sumctx = int(lens.sum())
    algo = sumctx * hkv * d * 2 * 2 + 2 * b * h * d * 2 + 4 * need + 4 * b
    del kc, vc
    torch.cuda.empty_cache()
    return _line("paged_decode", label + (", PDL chain" if pdl else ""), us, algo,
                 sum_ctx=sumctx, timing=f"graph of {iters} launches over {sets} rotating KV sets "
                                           f"of {algo / 1e6:.0f} MB each (together > L2)"
                                           + (", programmatic dependent launch between them"
                                              if pdl else ""))


def tts_pool_decode_variants(iters: int = 64) -> list[dict]:
    """The talker's pool decode (the same geometry as ``tts_pool_decode``) through the
    public wrapper with and without its optional inputs -- the key-valid mask and the
    current token's K/V -- and on the chunked CUDA-core kernel (``tokens_per_cta``), to
    show what each part of the call costs."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)
    b, h, hkv, d, page = 32, 16, 8, 128, 16
    pages = (1 << 21) // page
    lens = rng.integers(64, 1025, size=b)
    need = (lens + page - 1) // page
    gen = torch.Generator(device=dev).manual_seed(0)
    kp = (torch.randn(pages, hkv, page, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    vp = kp.clone()
    q = (torch.randn(b, h, 1, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    nk = (torch.randn(b, hkv, 1, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    nv = nk.clone()
    perm = rng.permutation(pages)
    tables = []
    for k in range(4):
        t = np.full((b, 64), -1, np.int64)
        c = k * int(need.sum())
        for i, n in enumerate(need):
            t[i, :n] = perm[c:c + n]
            c += int(n)
        tables.append(torch.from_numpy(t).to(dev))
    seq = torch.from_numpy(lens.astype(np.int64)).to(dev)
    valid = torch.ones(b, 1024, dtype=torch.bool, device=dev)
    out = torch.empty_like(q)
    ws = kx.pool_decode_workspace(b, h, d, 1024, dev)
    algo = int(lens.sum()) * hkv * d * 2 * 2 + 2 * b * h * d * 2
    lines = []
    for name, kw in (("mask + current token", dict(key_valid_mask=valid, new_key=nk, new_value=nv)),
                     ("current token only", dict(new_key=nk, new_value=nv)),
                     ("mask only", dict(key_valid_mask=valid)),
                     ("neither", {}),
                     ("mask + current token, chunked kernel (tokens_per_cta 256)",
                      dict(key_valid_mask=valid, new_key=nk, new_value=nv, tokens_per_cta=256))):
        ops = [lambda i=i, kw=kw: kx.pool_paged_decode(q, kp, vp, tables[i % 4], seq,
                                                        max_seq_len=1024, scale=d ** -0.5,
                                                        out=out, workspace=ws, **kw)
               for i in range(iters)]
        lines.append(_line("pool_paged_decode", f"talker B=32 ctx~U[64,1024], {name}",
                           graph_time_us(ops), algo, timing=f"graph of {iters} launches"))
    del kp, vp
    torch.cuda.empty_cache()
    return lines


def _reference_tts_module():
    """The reference's TTS paged attention module from its installed copy (baseline/_ref),
    or None when it or Triton is unavailable."""
    import sys

    ref = REPO / "baseline" / "_ref"
    if not (ref / "qwen_asr_vllm").is_dir():
        return None
    sys.path.insert(0, str(ref))
    try:
        from qwen_asr_vllm.agent import qwen_tts_paged_attention as m
    except Exception:  # noqa: BLE001 - the comparison arm is optional
        return None
    finally:
        sys.path.remove(str(ref))
    return m if getattr(m, "HAS_TRITON", False) else None


def tts_pool_decode(iters: int = 64, sets: int = 4, lo: int = 64, hi: int = 1024,
                    page: int = 16, pool_tokens: int = 4096 * 256,
                    reference: bool = True) -> list[dict]:
    """TTS talker decode over a page pool [pages, H_kv, page, D] (the reference's default
    page of 16 tokens), config-1 geometry and lengths: B = 32, H 16 / H_kv 8, d 128, ctx ~
    U[64, 1024], a 2 GiB pool per K/V, page tables slices of a random permutation, with
    the fused current-token write and an all-true key-valid mask as QwenPagedCache passes
    them (agent/qwen_tts_outer_varlen.py:392-436). Both this library's kernel and, when
    its installed copy imports, the reference's Triton kernel on the same inputs."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)
    b, h, hkv, d = 32, 16, 8, 128
    pages = pool_tokens // page
    lens = rng.integers(lo, hi + 1, size=b)
    need = (lens + page - 1) // page
    gen = torch.Generator(device=dev).manual_seed(0)
    kp = (torch.randn(pages, hkv, page, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    vp = (torch.randn(pages, hkv, page, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    q = (torch.randn(b, h, 1, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    nk = (torch.randn(b, hkv, 1, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    nv = (torch.randn(b, hkv, 1, d, device=dev, generator=gen) / d ** 0.5).bfloat16()
    perm = rng.permutation(pages)
    width = -(-hi // page)
    tables = []
    for k in range(sets):
        t = np.full((b, width), -1, np.int64)
        c = k * int(need.sum())
        for i, n in enumerate(need):
            t[i, :n] = perm[c:c + n]
            c += int(n)
        tables.append(torch.from_numpy(t).to(dev))
    seq = torch.from_numpy(lens.astype(np.int64)).to(dev)
    max_len = -(-hi // 128) * 128
    valid = torch.ones(b, max_len, dtype=torch.bool, device=dev)
    out = torch.empty_like(q)
    ws = kx.pool_decode_workspace(b, h, d, max_len, dev)
    sumctx = int(lens.sum())
    algo = (sumctx * hkv * d * 2 * 2 + 2 * b * h * d * 2 + 2 * b * hkv * d * 2
            + 8 * int(need.sum()) + 8 * b + b * max_len)
    cfg = f"talker B=32 ctx~U[{lo},{hi}] Hq16/Hkv8 d128 page {page} (+ current-token write)"
    timing = (f"graph of {iters} launches over {sets} rotating page-table sets of "
              f"{algo / 1e6:.0f} MB each (together > L2)")

    def mine(i):
        return lambda: kx.pool_paged_decode(q, kp, vp, tables[i % sets], seq, max_seq_len=max_len,
                                            scale=d ** -0.5, out=out, key_valid_mask=valid,
                                            new_key=nk, new_value=nv, workspace=ws)

    lines = [_line("pool_paged_decode", cfg, graph_time_us([mine(i) for i in range(iters)]), algo,
                   sum_ctx=sumctx, timing=timing)]
    m = _reference_tts_module() if reference else None
    if m is not None:
        def theirs(i):
            return lambda: m.paged_attention_decode(
                q, kp, vp, tables[i % sets], seq, valid, new_key=nk, new_value=nv,
                kernel_seq_len=max_len, kernel_page_count=width, scale=d ** -0.5,
                use_triton=True, validate=False)

        lines.append(_line("reference _paged_decode_attention_kernel (Triton)", cfg,
                           graph_time_us([theirs(i) for i in range(iters)]), algo,
                           sum_ctx=sumctx, timing=timing + "; block_n 128, num_warps 4 "
                                                           "(QwenPagedCache defaults)"))
    del kp, vp
    torch.cuda.empty_cache()
    return lines


# ------------------------------------------------------------------ config 2


def _config2_lengths():
    rng = np.random.default_rng(0)
    secs = rng.uniform(2.0, 30.0, size=32)
    dec = [num_audio_tokens(int(100 * s)) + 24 for s in secs]
    enc = [num_audio_tokens(int(100 * s)) for s in secs]
    return dec, enc


def prefill_config2() -> dict:
    """Varlen causal GQA prefill over the paged cache, config 2 decoder lengths."""
    dev = torch.device("cuda")
    lens, _ = _config2_lengths()
    t = sum(lens)
    nblk = [(n + 255) // 256 for n in lens]
    per_set = t * (16 + 8 + 8 + 16) * 128 * 2
    sets = _sets(per_set)
    gen = torch.Generator(device=dev).manual_seed(1)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).to(dev)
    runs = []
    for k in range(sets):
        q = torch.randn(t, 16, 128, device=dev, generator=gen).bfloat16()
        kc = torch.randn(sum(nblk) + 1, 256, 8, 128, device=dev, generator=gen).bfloat16()
        vc = torch.randn_like(kc)
        tb = np.zeros((32, max(nblk)), np.int32)
        c = 0
        for i, n in enumerate(nblk):
            tb[i, :n] = np.arange(c, c + n)
            c += n
        out = torch.empty_like(q)
        runs.append((q, kc, vc, torch.from_numpy(tb).to(dev), out))

    def op(r):
        q, kc, vc, tb, out = r
        return lambda: kx.paged_prefill(q, kc, vc, cu, cu, tb, max_seqlen_q=max(lens),
                                        scale=128 ** -0.5, out=out)

    us = graph_time_us([op(runs[i % sets]) for i in range(4 * sets)])
    flops = sum(4096 * n * (n + 1) for n in lens)  # causal QK^T + PV, 16 heads, d 128
    return _line("paged_prefill", "config2 decoder 32 prompts L=13s+24, s~U(2,30), Hq16/Hkv8 d128",
                 us, per_set, flops=flops, bound="hbm (below the bf16 ridge)", tokens=t,
                 timing=f"graph over {sets} rotating input sets of {per_set / 1e6:.0f} MB")


def _window_bounds(tokens, window: int) -> np.ndarray:
    """cu_seqlens of the encoder's attention windows: each clip cut into ``window``-token
    segments, the last one ragged (audio/batcher.py build_window_boundaries)."""
    cu = [0]
    for t in tokens:
        full, rem = divmod(int(t), window)
        base = cu[-1]
        cu.extend(base + window * (i + 1) for i in range(full))
        if rem:
            cu.append(cu[-1] + rem)
    return np.asarray(cu, np.int32)


def window_config2() -> dict:
    """Encoder windowed bidirectional attention, config 2 clips (104-token windows)."""
    dev = torch.device("cuda")
    _, toks = _config2_lengths()
    cuw = _window_bounds(toks, attention_window_tokens(800))
    t = int(cuw[-1])
    per_set = t * 4 * 896 * 2
    sets = _sets(per_set)
    gen = torch.Generator(device=dev).manual_seed(2)
    cu = torch.from_numpy(cuw).to(dev)
    runs = []
    for _ in range(sets):
        qkv = torch.randn(t, 3 * 896, device=dev, generator=gen).bfloat16()
        views = [qkv[:, i * 896:(i + 1) * 896].unflatten(1, (14, 64)) for i in range(3)]
        runs.append((views, torch.empty(t, 14, 64, device=dev, dtype=torch.bfloat16)))

    def op(r):
        (q, k, v), out = r
        return lambda: kx.varlen_attention(q, k, v, cu, int(np.diff(cuw).max()), 64 ** -0.5, out=out)

    us = graph_time_us([op(runs[i % sets]) for i in range(4 * sets)])
    flops = sum(4 * int(w) * int(w) * 64 * 14 for w in np.diff(cuw))
    return _line("varlen_window", "config2 encoder windows (104 tokens), 14 heads d64", us, per_set,
                 flops=flops, bound="hbm", tokens=t, windows=len(cuw) - 1,
                 timing=f"graph over {sets} rotating input sets of {per_set / 1e6:.0f} MB")


def encoder_conv(chunks: int = 512) -> list[dict]:
    """The audio encoder's convolutional front (models/audio_encoder.py:145-175), 0.6B
    dims (1 -> 480 -> 480 -> 480 channels over 128 mel x 100 frames per chunk): three
    Conv2d(3x3, stride 2, pad 1) + GELU on cuDNN in channels-last bf16 (the comparison),
    then this library's conv3x3s2_gelu kernels on the same inputs, then conv_out
    (7680 -> 896) on cuBLAS; one line per stage."""
    import torch.nn.functional as F

    dev = torch.device("cuda")
    c, d = 480, 896
    torch.manual_seed(0)
    convs = [torch.nn.Conv2d(1 if i == 0 else c, c, 3, 2, padding=1).to(dev, torch.bfloat16)
             .to(memory_format=torch.channels_last) for i in range(3)]
    out_w = (torch.randn(d, c * 16, device=dev) * 0.02).bfloat16()
    x0 = torch.randn(chunks, 1, 128, 100, device=dev).bfloat16().contiguous(
        memory_format=torch.channels_last)
    acts = [x0]
    with torch.inference_mode():
        for conv in convs:
            acts.append(F.gelu(conv(acts[-1])))
    lines = []
    shapes = [(64, 50), (32, 25), (16, 13)]
    for i, conv in enumerate(convs):
        cin = 1 if i == 0 else c
        ho, wo = shapes[i]
        flops = 2 * chunks * ho * wo * c * cin * 9
        nbytes = acts[i].numel() * 2 + acts[i + 1].numel() * 2 + conv.weight.numel() * 2

        def op(conv=conv, x=acts[i], y=acts[i + 1]):
            return lambda: y.copy_(F.gelu(conv(x)))

        with torch.inference_mode():
            us = graph_time_us([op() for _ in range(8)])
        lines.append(_line("conv2d+gelu (cuDNN)", f"encoder conv{i + 1}: {chunks} chunks, {cin}->{c} "
                           f"ch, out {ho}x{wo}", us, nbytes, flops=flops, bound="tensor"))
    # this library's kernels on the same inputs (csrc/conv.cu)
    packed = [kx.conv_pack_weight(conv.weight.detach().contiguous()) for conv in convs]
    x = [x0.view(chunks, 128, 100, 1)]
    for i, conv in enumerate(convs):
        x.append(kx.conv3x3s2_gelu(x[i], packed[i], conv.bias.detach(), c_out=c))
    for i, conv in enumerate(convs):
        cin = 1 if i == 0 else c
        ho, wo = shapes[i]
        flops = 2 * chunks * ho * wo * c * cin * 9
        nbytes = x[i].numel() * 2 + x[i + 1].numel() * 2 + conv.weight.numel() * 2

        def op(i=i, conv=conv):
            return lambda: kx.conv3x3s2_gelu(x[i], packed[i], conv.bias.detach(), c_out=c,
                                             out=x[i + 1])

        us = graph_time_us([op() for _ in range(8)])
        kind = "direct stencil" if i == 0 else "tcgen05 implicit GEMM"
        lines.append(_line(f"conv3x3s2_gelu ({kind})", f"encoder conv{i + 1}: {chunks} chunks, "
                           f"{cin}->{c} ch, out {ho}x{wo}, bias + GELU fused", us, nbytes,
                           flops=flops, bound="hbm" if i == 0 else "tensor"))
    flat = acts[3].permute(0, 3, 1, 2).reshape(chunks * 13, c * 16)
    y = torch.empty(chunks * 13, d, device=dev, dtype=torch.bfloat16)
    with torch.inference_mode():
        us = graph_time_us([lambda: torch.matmul(flat, out_w.T, out=y) for _ in range(8)])
    lines.append(_line("conv_out (cuBLAS)", f"{chunks} chunks x 13 tokens, 7680 -> 896", us,
                       flat.numel() * 2 + out_w.numel() * 2 + y.numel() * 2,
                       flops=2 * chunks * 13 * c * 16 * d, bound="tensor"))
    return lines


# --------------------------------------------------------------- store / pack


def store_rows(rows: int) -> dict:
    dev = torch.device("cuda")
    per_set = 4 * rows * 2048
    sets = _sets(per_set) if rows >= 1024 else 8
    nb = max(64, -(-rows * sets // 256) + 1)
    kc = torch.zeros(nb, 256, 8, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    runs = []
    for k in range(sets):
        qkv = torch.randn(rows, 4096, device=dev).bfloat16()
        key = qkv[:, 2048:3072].unflatten(1, (8, 128))
        val = qkv[:, 3072:].unflatten(1, (8, 128))
        slots = torch.arange(k * rows, (k + 1) * rows, dtype=torch.int32, device=dev)
        runs.append((key, val, slots))

    def op(r):
        key, val, slots = r
        return lambda: kx.store_kvcache(key, val, kc, vc, slots)

    us = graph_time_us([op(runs[i % sets]) for i in range(4 * sets)])
    return _line("store_kvcache", f"{rows} rows x 8 KV heads x 128 (K and V)", us, per_set,
                 bound="hbm" if rows >= 1024 else "latency")


def qk_norm_rope_rows(rows: int) -> dict:
    from voiceagent_b200.layers.norm import rope_table

    dev = torch.device("cuda")
    sets = 8 if rows < 1024 else 4
    nb = -(-rows * sets // 256) + 1
    kc = torch.zeros(nb, 256, 8, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    table = rope_table(128, 4096, 1e6, None).to(dev)
    qw = torch.ones(128, device=dev, dtype=torch.bfloat16)
    runs = []
    for k in range(sets):
        qkv = torch.randn(rows, 4096, device=dev).bfloat16()
        pos = torch.randint(0, 4096, (rows,), device=dev)
        slots = torch.arange(k * rows, (k + 1) * rows, dtype=torch.int32, device=dev)
        q = torch.empty(rows, 16, 128, device=dev, dtype=torch.bfloat16)
        runs.append((qkv, pos, slots, q))

    def op(r):
        qkv, pos, slots, q = r
        return lambda: kx.qk_norm_rope_store(qkv, pos, num_heads=16, num_kv_heads=8, head_dim=128,
                                             q_weight=qw, k_weight=qw, eps=1e-6,
                                             cos_sin_cache=table, q_out=q, k_cache=kc,
                                             v_cache=vc, slot_mapping=slots)

    us = graph_time_us([op(runs[i % sets]) for i in range(4 * sets)])
    nbytes = rows * (4096 * 2 + 2048 * 2 + 2048 * 2 + 8 + 4)  # qkv in; q out; k,v to cache
    return _line("qk_norm_rope_store", f"{rows} rows, 16/8 heads d128", us, nbytes,
                 bound="hbm" if rows >= 1024 else "latency")


def pack_decoder_batch() -> dict:
    """Mixed prefill batch metadata: 32 requests, ~4200 query tokens (config 3 prefill)."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(3)
    n = 32
    starts = np.zeros(n, np.int32)
    ends = rng.integers(60, 260, size=n).astype(np.int32)
    tlen = ((ends + 255) // 256).astype(np.int32)
    toff = np.concatenate([[0], np.cumsum(tlen)[:-1]]).astype(np.int32)
    tables = rng.permutation(4096)[:int(tlen.sum())].astype(np.int32)
    total = int(ends.sum())
    tokens = rng.integers(0, 150000, size=total).astype(np.int32)
    d = [torch.from_numpy(a).to(dev) for a in (starts, ends, toff, tlen, tables, tokens)]
    width = int(tlen.max())
    out = {"input_ids": torch.empty(total, dtype=torch.int64, device=dev),
           "positions": torch.empty(total, dtype=torch.int64, device=dev),
           "slot_mapping": torch.empty(total, dtype=torch.int32, device=dev),
           "cu_seqlens_q": torch.empty(n + 1, dtype=torch.int32, device=dev),
           "cu_seqlens_k": torch.empty(n + 1, dtype=torch.int32, device=dev),
           "max_seqlen": torch.empty(2, dtype=torch.int32, device=dev),
           "block_tables": torch.empty(n, width, dtype=torch.int32, device=dev),
           "last_token_index": torch.empty(n, dtype=torch.int64, device=dev)}
    us = graph_time_us([lambda: kx.pack_decoder(*d, total_tokens=total, width=width,
                                                block_size=256, out=out)] * 16)
    nbytes = total * (8 + 8 + 4) + n * (width * 4 + 16) + total * 4 + n * 16 + int(tlen.sum()) * 4
    return _line("pack_decoder", f"{n} requests, {total} query tokens", us, nbytes, bound="latency")


def linear_decode(m: int = 32) -> list[dict]:
    """Decode-step projections (0.6B shapes, ``m`` rows), 28 rotating layers of weights."""
    dev = torch.device("cuda")
    shapes = {"qkv_proj": (1024, 4096, False), "o_proj": (2048, 1024, False),
              "gate_up_proj+silu": (1024, 6144, True), "down_proj": (3072, 1024, False)}
    lines = []
    for name, (k, n, silu) in shapes.items():
        x = torch.randn(m, k, device=dev).bfloat16()
        ws = [(torch.randn(n, k, device=dev) * 0.02).bfloat16() for _ in range(28)]
        us = graph_time_us([(lambda w=w: kx.linear_small(x, w, silu=silu)) for w in ws])
        nbytes = n * k * 2 + m * k * 2 + m * (n // 2 if silu else n) * 2
        flops = 2 * m * n * k
        lines.append(_line("linear_small", f"{name} m={m} k={k} n={n}", us, nbytes, flops=flops,
                           bound="hbm (weight streaming)"))
        del ws
    torch.cuda.empty_cache()
    return lines


def lm_head(rows: int = 32, hidden: int = 1024, vocab: int = 151936) -> dict:
    """The decode step's lm_head projection alone: ``rows`` activation rows against the
    [vocab, hidden] bf16 weight (311 MB for the 0.6B model, 622 MB for the 1.7B: above L2,
    so each launch streams it from HBM), on the persistent streaming kernel."""
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(rows, hidden, device=dev, generator=gen).bfloat16()
    w = (torch.randn(vocab, hidden, device=dev, generator=gen) * 0.03).bfloat16()
    out = torch.empty(rows, vocab, dtype=torch.bfloat16, device=dev)
    us = graph_time_us([lambda: kx.linear_small(x, w, out=out)] * 16)
    nbytes = vocab * hidden * 2 + rows * hidden * 2 + rows * vocab * 2
    del w
    torch.cuda.empty_cache()
    return _line("linear_small (lm_head)", f"{rows} x {hidden} -> {vocab}", us, nbytes)


def argmax_rows(rows: int = 32) -> dict:
    dev = torch.device("cuda")
    per = rows * 151936 * 2
    sets = _sets(per)
    logits = [torch.randn(rows, 151936, device=dev).bfloat16() for _ in range(sets)]
    out = torch.empty(rows, dtype=torch.int64, device=dev)
    us = graph_time_us([(lambda l=l: kx.greedy_argmax(l, out=out)) for l in logits * 2])
    return _line("greedy_argmax", f"{rows} x 151936 bf16 logits", us, per + rows * 8)


def log_mel_config3() -> dict:
    from voiceagent_b200.audio.frontend import GpuMelFrontend
    from voiceagent_b200.workload import config3_clips

    dev = torch.device("cuda")
    fe = GpuMelFrontend(None)
    clips = config3_clips(128, seed=0)
    lens = np.asarray([c.size for c in clips], np.int64)
    frames = lens // 160
    wave = torch.from_numpy(np.concatenate(clips)).to(dev)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)])).to(dev)
    fs = torch.from_numpy(np.concatenate([[0], np.cumsum(frames)]).astype(np.int32)).to(dev)
    col = fs[:-1].clone()
    total = int(frames.sum())
    out = torch.empty(128, total, device=dev, dtype=torch.bfloat16)
    ws = torch.empty(kx.log_mel_workspace_size(len(clips), total), dtype=torch.uint8, device=dev)
    us = graph_time_us([lambda: kx.log_mel(wave, cu, fs, total_frames=total, tables=fe.tables,
                                           mel_filters=fe.filters, filter_range=fe.filter_range,
                                           out=out, out_col=col, workspace=ws)] * 4)
    nbytes = int(lens.sum()) * 4 + total * 128 * (2 + 4 + 4)  # waveform, out, scratch w+r
    flops = total * (201 * 400 * 4 + 2 * 201 * 128)
    return _line("log_mel (2 kernels)", f"config3 128 clips, {lens.sum() / 16000:.0f} s of audio",
                 us, nbytes, flops=flops, bound="fp32 DFT on CUDA cores",
                 audio_seconds_per_ms=round(float(lens.sum()) / 16000 / (us / 1000), 1))


class _DecodeRow:
    """The three things GraphRunner.run reads of a running request."""

    def __init__(self, length: int, block_table: list[int]):
        self.length, self.block_table, self.token_ids = length, block_table, [100]

    def __len__(self) -> int:
        return self.length


def decode_graph_step(fused: bool, iters: int = 64, l2_prefetch: bool = False,
                      profile_one: bool = False, preset: str = "0.6b", rows_n: int = 32) -> dict:
    """One whole decode step of Qwen3-ASR (random init) as the engine replays it: the
    bucket CUDA graph (28 layers of projections, norms, RoPE + KV store, paged attention,
    lm_head, argmax, descriptor advance) over `rows_n` rows of contexts U[80, 250], with
    the decoder's projections fused (five launches per layer) or not (eight). Defaults:
    the 0.6B model at 32 rows (benchmark configuration 3); preset "1.7b" with 64 rows is
    configuration 4's step."""
    import tempfile

    from voiceagent_b200.checkpoint import write_checkpoint
    from voiceagent_b200.engine.engine import AsrEngine

    path = write_checkpoint(Path(tempfile.mkdtemp()) / "ckpt", preset, weights=False)
    eng = AsrEngine(str(path), weights="random", seed=0, max_num_seqs=rows_n, max_model_len=1024,
                    num_kvcache_blocks=3 * rows_n, fused_decode=fused, l2_prefetch=l2_prefetch)
    gr = eng.model_runner.graph_runner
    rng = np.random.default_rng(3)
    lens = rng.integers(80, 251, size=rows_n)
    rows = [_DecodeRow(int(n), [3 * i, 3 * i + 1, 3 * i + 2]) for i, n in enumerate(lens)]
    gr.run(rows, 1)  # uploads the descriptor; each replay then advances it on the device
    graph = gr.graphs[(rows_n, True)]
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        graph.replay()
    e.record()
    e.synchronize()
    us = s.elapsed_time(e) * 1000.0 / iters
    if profile_one:  # one more replay between profiler start/stop (ncu --profile-from-start off)
        torch.cuda.profiler.start()
        graph.replay()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    t = eng.config.model_config.text
    hd = t.head_dim or t.hidden_size // t.num_attention_heads
    per_layer = (t.hidden_size * (t.num_attention_heads + 2 * t.num_key_value_heads) * hd
                 + t.num_attention_heads * hd * t.hidden_size + 3 * t.hidden_size * t.intermediate_size) * 2
    weights = t.num_hidden_layers * per_layer + t.vocab_size * t.hidden_size * 2
    ctx = int(lens.sum()) + rows_n * (3 + iters // 2)  # mean context over the timed replays
    kv = ctx * t.num_hidden_layers * t.num_key_value_heads * hd * 2 * 2
    launches = gr.kernels_per_replay[(rows_n, True)]
    del eng, gr, graph
    torch.cuda.empty_cache()
    what = ("fused projections" + (", next-layer L2 prefetch" if l2_prefetch else "")) if fused \
        else "unfused projections"
    return _line("decode_step_graph",
                 f"{preset.upper()} decode step, {rows_n} rows ctx~U[80,250], {what}",
                 us, weights + kv,
                 bound="hbm (weights + KV, latency-bound)", launches_per_step=launches,
                 timing=f"{iters} replays of the bucket-{rows_n} graph back to back")


BENCHES = {
    "decode": lambda: [decode_config1(), decode_config1(pdl=True)],
    "decode_step": lambda: [
        decode_config1(lo=80, hi=250, sets=16, max_seqlen_k=512,
                       label="config3 decode-step shape B=32 ctx~U[80,250], short-context kernel"),
        decode_config1(lo=80, hi=250, sets=16, max_seqlen_k=4096,
                       label="config3 decode-step shape B=32 ctx~U[80,250], stream-K kernel")],
    "lm_head": lambda: [lm_head(), lm_head(rows=64, hidden=2048)],
    "step": lambda: [decode_graph_step(True), decode_graph_step(True, l2_prefetch=True),
                     decode_graph_step(False)],
    "step_1p7b": lambda: [decode_graph_step(True, preset="1.7b", rows_n=64)],
    "decode_step_64": lambda: [
        decode_config1(lo=80, hi=250, sets=8, max_seqlen_k=512, batch=64,
                       label="config4 decode-step shape B=64 ctx~U[80,250], short-context kernel"),
        decode_config1(lo=80, hi=250, sets=8, max_seqlen_k=4096, batch=64,
                       label="config4 decode-step shape B=64 ctx~U[80,250], stream-K kernel")],
    "step_1p7b_profile": lambda: [decode_graph_step(True, iters=8, profile_one=True, preset="1.7b",
                                                    rows_n=64)],
    # one fused decode step bracketed for a profiler: its launch list is the step's kernels
    "step_profile": lambda: [decode_graph_step(True, iters=8, profile_one=True)],
    "prefill": lambda: [prefill_config2()],
    "window": lambda: [window_config2()],
    "encoder_conv": lambda: encoder_conv(),
    "store": lambda: [store_rows(32), store_rows(8192)],
    "rope": lambda: [qk_norm_rope_rows(32), qk_norm_rope_rows(4096)],
    "pack": lambda: [pack_decoder_batch()],
    "linear": lambda: linear_decode(32),
    "argmax": lambda: [argmax_rows(32)],
    "log_mel": lambda: [log_mel_config3()],
    "tts_decode": lambda: tts_pool_decode(),
    "tts_decode_variants": lambda: tts_pool_decode_variants(),
    # a 256 MB pool and four launches: the size for an ncu capture of one launch
    "tts_decode_profile": lambda: tts_pool_decode(iters=4, sets=1, pool_tokens=131072,
                                                  reference=False),
}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--only", nargs="*", choices=sorted(BENCHES), default=None)
    args = ap.parse_args()
    torch.cuda.set_device(0)
    for name, fn in BENCHES.items():
        if args.only and name not in args.only:
            continue
        for line in fn():
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
