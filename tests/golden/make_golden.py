"""Generate golden fixtures by running the reference's own Python on CPU.

Run in a container where the reference checkout exists (it is NOT available on
the GPU box; the fixtures it writes are committed next to this script):

    TORCHDYNAMO_DISABLE=1 TRITON_INTERPRET=1 python tests/golden/make_golden.py \
        --reference /path/to/VoiceAgent

``TORCHDYNAMO_DISABLE`` turns the reference's ``@torch.compile`` decorators into
plain eager calls; ``TRITON_INTERPRET`` runs its Triton kernels (the KV store and
the TTS paged decode) on the CPU interpreter. What each fixture pins:

* ``audio_pack.json``   -- ``audio/tokens.py`` + ``audio/batcher.py`` metadata
* ``decoder_pack.npz``  -- ``ModelRunner._prepare`` (model_runner.py:183-233)
* ``decode_bucket.npz`` -- ``GraphRunner.run`` staging (graph_runner.py:149-191)
* ``block_manager.json``-- ``BlockManager`` allocation traces with prefix caching
* ``store.npz``         -- ``store_kvcache`` Triton kernel (attention.py:31-67)
* ``paged_decode.npz``  -- TTS paged decode, its torch reference path
  (the Triton launcher refuses CPU tensors)
* ``tts_pool_decode.npz`` -- the same function in its own pool layout
  ``[pages, kv_heads, page_size, head_dim]``: the reference test's inputs, the fused
  current-token write, and talker-shaped cases with key-valid masks
* ``norm_rope.npz``     -- RMSNorm + RotaryEmbedding as used in qwen3.py:42-48
* ``elementwise.npz``   -- fused add-RMSNorm and SiluAndMul (layernorm.py, activation.py)
* ``sampler.npz``       -- greedy ``Sampler`` (sampler.py:16-27)
* ``model_tiny.npz``    -- upstream HF Qwen3-ASR thinker on a tiny seeded config
* ``frontend.npz``      -- ``AudioFrontend`` log-mel features (audio/frontend.py:71-94)
* ``ref_engine_hf.npz`` -- the upstream HF thinker in bf16 (CPU), teacher forced on the
  reference engine's tokens in ``ref_engine_tokens.npz`` (written on a B200 by
  ``make_ref_engine_tokens.py``; run that first): the reference's two implementations
  of the model compared position by position, with the same weights, audio and prompts
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))


def _f32(t):
    return t.detach().float().cpu().numpy()


# ------------------------------------------------------------------- requests


def _make_request(prompt_len, audio_offset, audio_length, block_size=256, seed_ids=None):
    import torch
    from qwen_asr_vllm.audio.frontend import AudioFeatures
    from qwen_asr_vllm.engine.request import AsrRequest, SamplingParams
    from qwen_asr_vllm.prompt import PromptLayout

    suffix = prompt_len - audio_offset - audio_length
    ids = (list(range(1000, 1000 + audio_offset)) + [151676] * audio_length
           + list(range(2000, 2000 + suffix)))
    if seed_ids is not None:
        ids = list(seed_ids)
    frames = max(1, audio_length * 100 // 13)
    return AsrRequest(
        features=AudioFeatures(mel=torch.zeros(128, frames), mel_frames=frames,
                               num_audio_tokens=audio_length, audio_seconds=audio_length / 13),
        layout=PromptLayout(token_ids=ids, audio_offset=audio_offset, audio_length=audio_length),
        sampling=SamplingParams(),
        block_size=block_size,
        stop_token_ids={151643, 151645},
    )


# -------------------------------------------------------------------- fixtures


def gen_audio_pack(out: Path):
    import torch
    from qwen_asr_vllm.audio.batcher import build_window_boundaries, pack_audio_batch
    from qwen_asr_vllm.audio.tokens import num_audio_tokens

    rng = np.random.default_rng(0)
    cases = [[350, 200, 105], [100], [7], [208 * 100 // 13 + 1], [2500], [99, 100, 101, 199, 200, 201]]
    cases += [list(map(int, rng.integers(1, 6000, size=int(rng.integers(1, 33))))) for _ in range(12)]
    packs = []
    for frames in cases:
        b = pack_audio_batch([torch.zeros(128, f) for f in frames], n_window_infer=800)
        packs.append({
            "mel_frames": frames,
            "chunk_lengths": b.chunk_lengths.tolist(),
            "chunk_valid_lens": b.chunk_valid_lens.tolist(),
            "cu_seqlens": b.cu_seqlens.tolist(),
            "audio_token_lens": list(b.audio_token_lens),
            "window_tokens": b.window_tokens,
            "max_seqlen": int(b.max_seqlen),
        })
    windows = [{"lens": lens, "window": w, "boundaries": build_window_boundaries(lens, w)}
               for lens, w in [([46, 26, 95], 104), ([250], 104), ([208], 104), ([1, 103, 104, 105], 104)]]
    data = {
        "num_audio_tokens": [num_audio_tokens(f) for f in range(1, 6000)],
        "packs": packs,
        "windows": windows,
    }
    (out / "audio_pack.json").write_text(json.dumps(data))


def _allocate_batch(manager, specs):
    """specs: list of (prompt_len, audio_offset, audio_len, n_decoded)."""
    reqs = []
    for prompt_len, off, alen, n_dec in specs:
        r = _make_request(prompt_len, off, alen)
        manager.allocate(r)
        for step in range(n_dec):
            r.num_computed_tokens = len(r)
            r.append_token(3000 + step)
            manager.may_append(r)
        reqs.append(r)
    return reqs


def gen_decoder_pack(out: Path):
    from types import SimpleNamespace

    from qwen_asr_vllm.engine.block_manager import BlockManager
    from qwen_asr_vllm.engine.model_runner import ModelRunner
    from qwen_asr_vllm.engine.scheduler import ModelBatch

    rng = np.random.default_rng(1)
    arrays = {}
    batches = [
        # (prefill specs, decode specs)
        ([(70, 9, 52, 0)], []),
        ([], [(70, 9, 52, 5)]),
        ([(300, 9, 270, 0), (40, 9, 13, 0)], [(256, 9, 200, 1), (255, 9, 200, 1), (600, 9, 560, 40)]),
        ([(700, 609, 46, 0)], [(62, 9, 46, 3)]),
    ]
    for _ in range(4):
        npre = int(rng.integers(0, 4))
        ndec = int(rng.integers(1 if npre == 0 else 0, 20))
        pre = [(int(p), 9, int(p) - 18, 0) for p in rng.integers(20, 900, size=npre)]
        dec = [(int(p), 9, int(p) - 18, int(d)) for p, d in zip(rng.integers(20, 900, size=ndec),
                                                               rng.integers(1, 300, size=ndec))]
        batches.append((pre, dec))

    stub = SimpleNamespace(block_size=256, device="cpu", _audio_span=ModelRunner._audio_span)
    for bi, (pre_specs, dec_specs) in enumerate(batches):
        manager = BlockManager(num_blocks=4096, block_size=256, enable_prefix_cache=False)
        # Shuffle physical block order so tables are not trivially contiguous.
        order = list(rng.permutation(4096))
        manager.free_block_ids = dict.fromkeys(int(i) for i in order)
        pre = _allocate_batch(manager, pre_specs)
        dec = _allocate_batch(manager, dec_specs)
        for r in dec:  # a decode row has computed everything but its last token
            r.num_computed_tokens = len(r) - 1
        batch = ModelBatch(prefill=pre, decode=dec)
        input_ids, positions, ctx, _ = ModelRunner._prepare(stub, batch)
        reqs = batch.requests
        p = f"b{bi}_"
        arrays[p + "starts"] = np.asarray([r.num_computed_tokens for r in reqs], np.int32)
        arrays[p + "ends"] = np.asarray([len(r) for r in reqs], np.int32)
        arrays[p + "table_lens"] = np.asarray([len(r.block_table) for r in reqs], np.int32)
        arrays[p + "tables_flat"] = np.asarray(sum((list(r.block_table) for r in reqs), []), np.int32)
        arrays[p + "token_lens"] = np.asarray([len(r.token_ids) for r in reqs], np.int32)
        arrays[p + "tokens_flat"] = np.asarray(sum((list(r.token_ids) for r in reqs), []), np.int64)
        arrays[p + "input_ids"] = input_ids.numpy()
        arrays[p + "positions"] = positions.numpy()
        arrays[p + "slot_mapping"] = ctx.slot_mapping.numpy()
        arrays[p + "cu_seqlens_q"] = ctx.cu_seqlens_q.numpy()
        arrays[p + "cu_seqlens_k"] = ctx.cu_seqlens_k.numpy()
        arrays[p + "max_seqlen"] = np.asarray([ctx.max_seqlen_q, ctx.max_seqlen_k], np.int32)
        arrays[p + "block_tables"] = ctx.block_tables.numpy()
    arrays["num_batches"] = np.asarray(len(batches))
    np.savez_compressed(out / "decoder_pack.npz", **arrays)


def gen_decode_bucket(out: Path):
    import torch
    from qwen_asr_vllm.engine.block_manager import BlockManager
    from qwen_asr_vllm.engine.graph_runner import GraphRunner

    class _Graph:
        def replay(self):
            pass

    rng = np.random.default_rng(2)
    arrays = {}
    cases = [(1, 1), (3, 4), (17, 24), (32, 32), (5, 8)]
    for ci, (b, bucket) in enumerate(cases):
        runner = GraphRunner.__new__(GraphRunner)
        runner.device = torch.device("cpu")
        runner.block_size = 256
        runner.config = type("C", (), {"max_model_len": 4096})()
        runner.max_blocks = 16
        runner.buckets = (1, 2, 4, 8, 16, 24, 32, 48, 64)
        runner.max_batch_size = 64
        runner._allocate_buffers()
        runner.graphs = {bucket: _Graph()}
        runner.outputs = {bucket: torch.zeros(bucket, 4)}
        manager = BlockManager(num_blocks=4096, block_size=256, enable_prefix_cache=False)
        manager.free_block_ids = dict.fromkeys(int(i) for i in rng.permutation(4096))
        specs = [(int(p), 9, int(p) - 18, int(d)) for p, d in zip(rng.integers(20, 1500, size=b),
                                                                 rng.integers(1, 500, size=b))]
        reqs = _allocate_batch(manager, specs)
        runner.run(reqs)
        p = f"c{ci}_"
        arrays[p + "bucket"] = np.asarray(bucket)
        arrays[p + "lens"] = np.asarray([len(r) for r in reqs], np.int32)
        arrays[p + "last_ids"] = np.asarray([r.last_token_id for r in reqs], np.int64)
        arrays[p + "table_lens"] = np.asarray([len(r.block_table) for r in reqs], np.int32)
        arrays[p + "tables_flat"] = np.asarray(sum((list(r.block_table) for r in reqs), []), np.int32)
        arrays[p + "input_ids"] = runner.input_ids[:bucket].numpy()
        arrays[p + "positions"] = runner.positions[:bucket].numpy()
        arrays[p + "slot_mapping"] = runner.slot_mapping[:bucket].numpy()
        arrays[p + "cu_seqlens_k"] = runner.cu_seqlens_k[: bucket + 1].numpy()
        arrays[p + "block_tables"] = runner.block_tables[:bucket].numpy()
    arrays["num_cases"] = np.asarray(len(cases))
    np.savez_compressed(out / "decode_bucket.npz", **arrays)


def gen_block_manager(out: Path):
    from qwen_asr_vllm.engine.block_manager import BlockManager

    traces = []
    for prefix_cache in (True, False):
        manager = BlockManager(num_blocks=24, block_size=256, enable_prefix_cache=prefix_cache)
        reqs = {}
        ops = [
            ("alloc", "a", (700, 609, 46)), ("alloc", "b", (700, 609, 46)),
            ("alloc", "c", (600, 0, 590)), ("append", "a", 260), ("dealloc", "b", None),
            ("alloc", "d", (700, 609, 46)), ("alloc", "e", (300, 9, 270)),
            ("append", "e", 300), ("dealloc", "a", None), ("dealloc", "c", None),
            ("alloc", "f", (1100, 900, 100)), ("alloc", "g", (1100, 900, 100)),
        ]
        log = []
        for op, name, arg in ops:
            if op == "alloc":
                r = _make_request(*arg)
                reqs[name] = r
                ok = manager.can_allocate(r)
                if ok:
                    manager.allocate(r)
                log.append({"op": op, "name": name, "arg": list(arg), "ok": ok,
                            "table": list(r.block_table), "cached": r.num_cached_tokens,
                            "computed": r.num_computed_tokens, "free": manager.num_free_blocks})
            elif op == "append":
                r = reqs[name]
                tables = []
                for step in range(arg):
                    r.append_token(5000 + step)
                    if manager.can_append(r):
                        manager.may_append(r)
                    tables.append(len(r.block_table))
                log.append({"op": op, "name": name, "arg": arg, "table": list(r.block_table),
                            "free": manager.num_free_blocks})
            else:
                manager.deallocate(reqs[name])
                log.append({"op": op, "name": name, "free": manager.num_free_blocks,
                            "free_order": list(manager.free_block_ids)})
        traces.append({"prefix_cache": prefix_cache, "log": log,
                       "hash_example": BlockManager.compute_hash(list(range(256)))})
    (out / "block_manager.json").write_text(json.dumps(traces))


def _bf16_bits(t):
    """bf16 tensor -> its raw uint16 bit patterns (exact and half the size of fp32)."""
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def gen_store(out: Path):
    import torch
    from qwen_asr_vllm.layers.attention import store_kvcache

    g = torch.Generator().manual_seed(3)
    t, hq, hkv, d, nblocks = 37, 4, 2, 64, 2
    qkv = torch.randn(t, (hq + 2 * hkv) * d, generator=g).bfloat16()
    k = qkv[:, hq * d : (hq + hkv) * d].view(t, hkv, d)
    v = qkv[:, (hq + hkv) * d :].view(t, hkv, d)
    kc = torch.randn(nblocks, 256, hkv, d, generator=g).bfloat16()
    vc = torch.randn(nblocks, 256, hkv, d, generator=g).bfloat16()
    slots = torch.randperm(nblocks * 256, generator=g)[:t].to(torch.int32)
    slots[[0, 5, 36]] = -1
    kc0, vc0 = kc.clone(), vc.clone()
    store_kvcache(k, v, kc, vc, slots)
    np.savez_compressed(out / "store.npz", qkv=_bf16_bits(qkv), k_cache_before=_bf16_bits(kc0),
                        v_cache_before=_bf16_bits(vc0), slots=slots.numpy(),
                        k_cache=_bf16_bits(kc), v_cache=_bf16_bits(vc),
                        dims=np.asarray([t, hq, hkv, d, nblocks]))


def gen_paged_decode(out: Path):
    """The reference's own paged decode (TTS module) in the TTS pool layout.

    Inputs are drawn in the engine's layout (N, 256, H_kv, D) and permuted to the
    TTS layout (N, H_kv, 256, D) for the call; the fixture stores the engine
    layout so consumers need no permutation.
    """
    import torch
    from qwen_asr_vllm.agent.qwen_tts_paged_attention import paged_attention_decode

    g = torch.Generator().manual_seed(4)
    b, hq, hkv, d, bs, nblocks = 5, 4, 2, 64, 256, 10
    lens = torch.tensor([1, 64, 255, 257, 520], dtype=torch.long)
    kc = (torch.randn(nblocks, bs, hkv, d, generator=g) / d**0.5).bfloat16()
    vc = (torch.randn(nblocks, bs, hkv, d, generator=g) / d**0.5).bfloat16()
    q = (torch.randn(b, hq, d, generator=g) / d**0.5).bfloat16()
    perm = torch.randperm(nblocks, generator=g)
    width = 3
    tables = torch.zeros(b, width, dtype=torch.long)
    cursor = 0
    for row, length in enumerate(lens.tolist()):
        need = (length + bs - 1) // bs
        tables[row, :need] = perm[cursor : cursor + need]
        cursor += need
    kp, vp = kc.permute(0, 2, 1, 3).contiguous(), vc.permute(0, 2, 1, 3).contiguous()
    ref = paged_attention_decode(q.float().unsqueeze(2), kp.float(), vp.float(), tables, lens,
                                 use_triton=False)
    np.savez_compressed(out / "paged_decode.npz", q=_bf16_bits(q), k_cache=_bf16_bits(kc),
                        v_cache=_bf16_bits(vc),
                        lens=lens.numpy().astype(np.int32), tables=tables.numpy().astype(np.int32),
                        out_reference=_f32(ref.squeeze(2)))


def gen_tts_pool_decode(out: Path):
    """``paged_attention_decode`` (agent/qwen_tts_paged_attention.py:383-516) through its
    torch path, on the layout the TTS talker's page pool uses.

    Case ``ref``: the reference test's own inputs (tests/test_qwen_tts_paged_attention_
    kernel.py:16-35; fp32, head_dim 4, page 2, left-padded mask), once without and once
    with the fused current-token write (its 144-177). Cases ``talker_*``: bf16 values
    (stored as bits, promoted to fp32 for the call), head_dim 128, GQA 2 and 4, pages of
    16 and 24 tokens, page tables padded with -1 as ``QwenPagedCache`` pads them
    (qwen_tts_outer_varlen.py:343-361), lengths on and around page boundaries, masks
    with left padding, and the current-token write.
    """
    import torch
    from qwen_asr_vllm.agent.qwen_tts_paged_attention import paged_attention_decode

    arrays = {}
    # -- the reference test's inputs, rebuilt exactly as its _inputs() does
    page_table = torch.tensor([[3, 5, 0], [1, 7, 2]], dtype=torch.long)
    seq_lens = torch.tensor([3, 5], dtype=torch.long)
    valid = torch.tensor([[True, True, True, False, False], [False, True, True, True, True]])
    k_pool = torch.zeros((8, 2, 2, 4), dtype=torch.float32)
    v_pool = torch.zeros_like(k_pool)
    torch.manual_seed(17)
    for page in (3, 5, 1, 7, 2):
        k_pool[page].normal_()
        v_pool[page].normal_()
    q = torch.ones((2, 4, 1, 4), dtype=torch.float32)
    g = torch.Generator().manual_seed(18)
    new_k = torch.randn((2, 2, 1, 4), generator=g)
    new_v = torch.randn((2, 2, 1, 4), generator=g)
    plain = paged_attention_decode(q, k_pool, v_pool, page_table, seq_lens, valid,
                                   use_triton=False)
    kw, vw = k_pool.clone(), v_pool.clone()
    fused = paged_attention_decode(q, kw, vw, page_table, seq_lens, valid, new_key=new_k,
                                   new_value=new_v, use_triton=False)
    arrays.update(ref_q=q.numpy(), ref_k_pool=k_pool.numpy(), ref_v_pool=v_pool.numpy(),
                  ref_page_table=page_table.numpy(), ref_seq_lens=seq_lens.numpy(),
                  ref_valid=valid.numpy(), ref_new_k=new_k.numpy(), ref_new_v=new_v.numpy(),
                  ref_out=plain.numpy(), ref_out_fused=fused.numpy(),
                  ref_k_pool_after=kw.numpy(), ref_v_pool_after=vw.numpy())

    # -- talker-shaped cases
    cases = {
        "talker_g2": dict(hq=16, hkv=8, ps=16, lens=[1, 15, 16, 17, 40, 70], seed=31),
        "talker_g4": dict(hq=8, hkv=2, ps=24, lens=[3, 24, 25, 200], seed=32),
    }
    for name, c in cases.items():
        g = torch.Generator().manual_seed(c["seed"])
        lens = torch.tensor(c["lens"], dtype=torch.long)
        b, hq, hkv, ps, d = len(c["lens"]), c["hq"], c["hkv"], c["ps"], 128
        need = [(n + ps - 1) // ps for n in c["lens"]]
        pages = sum(need) + 1
        kp = (torch.randn(pages, hkv, ps, d, generator=g) / d**0.5).bfloat16()
        vp = (torch.randn(pages, hkv, ps, d, generator=g) / d**0.5).bfloat16()
        q = (torch.randn(b, hq, 1, d, generator=g)).bfloat16()
        nk = (torch.randn(b, hkv, 1, d, generator=g) / d**0.5).bfloat16()
        nv = (torch.randn(b, hkv, 1, d, generator=g) / d**0.5).bfloat16()
        perm = torch.randperm(pages, generator=g)
        width = max(need) + 1
        table = torch.full((b, width), -1, dtype=torch.long)
        cursor = 0
        for row, n in enumerate(need):
            table[row, :n] = perm[cursor:cursor + n]
            cursor += n
        mask = torch.ones(b, max(c["lens"]), dtype=torch.bool)
        mask[1, :2] = False          # left padding
        mask[-1, :9] = False
        mask[-1, 20] = False
        kw, vw = kp.float(), vp.float()
        res = paged_attention_decode(q.float(), kw, vw, table, lens, mask, new_key=nk.float(),
                                     new_value=nv.float(), use_triton=False)
        arrays.update({f"{name}_q": _bf16_bits(q), f"{name}_k_pool": _bf16_bits(kp),
                       f"{name}_v_pool": _bf16_bits(vp), f"{name}_new_k": _bf16_bits(nk),
                       f"{name}_new_v": _bf16_bits(nv), f"{name}_page_table": table.numpy(),
                       f"{name}_seq_lens": lens.numpy(), f"{name}_valid": mask.numpy(),
                       f"{name}_out": _f32(res)})
    np.savez_compressed(out / "tts_pool_decode.npz", **arrays)


def gen_norm_rope(out: Path):
    import torch
    from qwen_asr_vllm.layers.layernorm import RMSNorm
    from qwen_asr_vllm.layers.rotary_embedding import RotaryEmbedding

    g = torch.Generator().manual_seed(5)
    t, hq, hkv, d = 12, 16, 8, 128
    qkv = (torch.randn(t, (hq + 2 * hkv) * d, generator=g) * 2).bfloat16()
    positions = torch.randint(0, 4096, (t,), generator=g)
    q_norm, k_norm = RMSNorm(d, 1e-6), RMSNorm(d, 1e-6)
    with torch.no_grad():
        q_norm.weight.copy_(torch.rand(d, generator=g) + 0.5)
        k_norm.weight.copy_(torch.rand(d, generator=g) + 0.5)
    q_norm, k_norm = q_norm.bfloat16(), k_norm.bfloat16()
    rope = RotaryEmbedding(d, 4096, 1_000_000.0)
    q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    qn = q_norm(q.reshape(-1, hq, d))
    kn = k_norm(k.reshape(-1, hkv, d))
    qr, kr = rope(positions, qn, kn)
    np.savez_compressed(out / "norm_rope.npz", qkv=_bf16_bits(qkv), positions=positions.numpy(),
                        q_weight=_bf16_bits(q_norm.weight), k_weight=_bf16_bits(k_norm.weight),
                        cos_sin_cache=_f32(rope.cos_sin_cache.squeeze(1)[positions]),
                        q_normed=_bf16_bits(qn), k_normed=_bf16_bits(kn), q_out=_bf16_bits(qr),
                        k_out=_bf16_bits(kr))


def gen_elementwise(out: Path):
    import torch
    from qwen_asr_vllm.layers.activation import SiluAndMul
    from qwen_asr_vllm.layers.layernorm import RMSNorm

    g = torch.Generator().manual_seed(6)
    x = torch.randn(19, 1024, generator=g).bfloat16()
    res = torch.randn(19, 1024, generator=g).bfloat16()
    norm = RMSNorm(1024, 1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(1024, generator=g) + 0.5)
    norm = norm.bfloat16()
    y_plain = norm(x.clone())
    y_add, r_add = norm(x.clone(), res.clone())
    gu = (torch.randn(19, 2 * 3072, generator=g) * 3).bfloat16()
    act = SiluAndMul()(gu)
    np.savez_compressed(out / "elementwise.npz", x=_bf16_bits(x), residual=_bf16_bits(res),
                        weight=_bf16_bits(norm.weight), rms=_bf16_bits(y_plain),
                        add_rms=_bf16_bits(y_add), add_residual=_bf16_bits(r_add),
                        gate_up=_bf16_bits(gu), silu_mul=_bf16_bits(act))


def gen_sampler(out: Path):
    import torch
    from qwen_asr_vllm.layers.sampler import Sampler

    g = torch.Generator().manual_seed(7)
    logits = torch.randn(5, 151936, generator=g).bfloat16()
    logits[1, 100] = 30.0
    logits[1, 90000] = 30.0  # tie: first index wins
    logits[2, :] = -5.0      # all equal
    logits[3, 151935] = 1e4  # last index
    logits[4, 0] = float("inf")
    logits[4, 7] = float("inf")
    ids = Sampler()(logits, torch.zeros(5))
    np.savez_compressed(out / "sampler.npz", logits=_bf16_bits(logits), ids=ids.numpy())


# -------------------------------------------------------------------- HF model


def tiny_thinker_config():
    """A small Qwen3-ASR configuration with the real structure (GQA, QK-norm, 3 convs)."""
    return {
        "audio": dict(num_mel_bins=128, d_model=64, encoder_layers=2, encoder_attention_heads=4,
                      encoder_ffn_dim=96, downsample_hidden_size=16, output_dim=96, n_window=50,
                      n_window_infer=800, conv_chunksize=500, max_source_positions=1500),
        "text": dict(vocab_size=512, hidden_size=96, intermediate_size=160, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6,
                     rope_theta=1_000_000.0, max_position_embeddings=4096, tie_word_embeddings=True),
        "audio_token_id": 500,
        "audio_start_token_id": 498,
        "audio_end_token_id": 499,
    }


def _import_hf_with_shims():
    """Import the upstream modeling file under transformers 5.x.

    Four runtime shims, no file edits (the file targets transformers 4.57):
    ``check_model_inputs`` callable with no arguments, a ``default`` RoPE init
    function, the same on the rotary class, and ``pad_token_id = None`` on configs
    (set in :func:`_build_hf_thinker`).
    """
    import functools

    import torch
    import transformers.utils.generic as generic
    from transformers import modeling_rope_utils

    original = generic.check_model_inputs
    if not getattr(original, "_golden_shim", False):
        def check_model_inputs(func=None, **kwargs):
            if func is None:
                return lambda f: original(f, **kwargs) if kwargs else original(f)
            return original(func, **kwargs) if kwargs else original(func)

        check_model_inputs._golden_shim = True
        generic.check_model_inputs = check_model_inputs

    def default_rope(config, device=None, *args, **kwargs):
        base = config.rope_theta
        dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).float().to(device) / dim))
        return inv, 1.0

    modeling_rope_utils.ROPE_INIT_FUNCTIONS.setdefault("default", default_rope)
    from reference import modeling_qwen3_asr as hf

    hf.Qwen3ASRThinkerTextRotaryEmbedding.compute_default_rope_parameters = staticmethod(
        functools.partial(default_rope))
    return hf


def _build_hf_thinker(hf, cfg: dict, weights, mrope_section=(8, 4, 4)):
    import torch
    from reference import configuration_qwen3_asr as hfc

    audio = hfc.Qwen3ASRAudioEncoderConfig(**cfg["audio"])
    text = hfc.Qwen3ASRTextConfig(**cfg["text"], rope_scaling={"mrope_section": list(mrope_section),
                                                               "rope_type": "default"})
    thinker_cfg = hfc.Qwen3ASRThinkerConfig(audio_config=audio.to_dict(), text_config=text.to_dict(),
                                            audio_token_id=cfg["audio_token_id"],
                                            audio_start_token_id=cfg["audio_start_token_id"])
    thinker_cfg.pad_token_id = None
    thinker_cfg.text_config.pad_token_id = None
    thinker_cfg._attn_implementation = "eager"
    thinker_cfg.audio_config._attn_implementation = "eager"
    thinker_cfg.text_config._attn_implementation = "eager"
    model = hf.Qwen3ASRThinkerForConditionalGeneration(thinker_cfg).float().eval()
    state = {k: v for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(state, strict=False)
    missing = [m for m in missing if m != "lm_head.weight"]
    if missing or unexpected:
        raise RuntimeError(f"weight mismatch: missing={missing[:5]} unexpected={unexpected[:5]}")
    with torch.no_grad():
        model.lm_head.weight.copy_(weights["lm_head.weight"])
    return model


def _hf_greedy(thinker, prompt, mel, frames, steps):
    """Manual greedy loop over ``forward`` with a DynamicCache (generate() needs
    ``cache_position`` that transformers 5.x leaves unset)."""
    import torch
    from transformers import DynamicCache

    ids = torch.tensor([prompt])
    cache = DynamicCache()
    mask = torch.ones_like(ids)
    out = thinker(input_ids=ids, input_features=mel.unsqueeze(0),
                  feature_attention_mask=torch.ones(1, frames, dtype=torch.long),
                  attention_mask=mask, past_key_values=cache, use_cache=True,
                  cache_position=torch.arange(ids.shape[1]))
    first_logits = out.logits[0, -1]
    tokens = [int(first_logits.argmax())]
    length = ids.shape[1]
    for _ in range(steps - 1):
        step_ids = torch.tensor([[tokens[-1]]])
        mask = torch.ones(1, length + 1, dtype=torch.long)
        out = thinker(input_ids=step_ids, attention_mask=mask, past_key_values=cache,
                      use_cache=True, cache_position=torch.tensor([length]),
                      position_ids=torch.tensor([[length]]))
        length += 1
        tokens.append(int(out.logits[0, -1].argmax()))
    return tokens, first_logits


def gen_model_tiny(out: Path):
    """Upstream HF thinker (reference/modeling_qwen3_asr.py) on a seeded tiny config."""
    import torch
    from oracle import model as omodel

    hf = _import_hf_with_shims()
    cfg = tiny_thinker_config()
    weights = omodel.init_weights(cfg, seed=11)
    thinker = _build_hf_thinker(hf, cfg, weights)

    g = torch.Generator().manual_seed(12)
    frames = 437
    mel = torch.randn(128, frames, generator=g) * 0.5
    n_audio = omodel.num_audio_tokens(frames)
    prompt = ([344, 13, 14, 345, 15, 344, 16, 17, 498]
              + [500] * n_audio + [499, 345, 15, 344, 18, 19, 20, 21, 22])
    with torch.no_grad():
        audio = thinker.get_audio_features(mel.unsqueeze(0),
                                           feature_attention_mask=torch.ones(1, frames, dtype=torch.long))
        tokens, logits0 = _hf_greedy(thinker, prompt, mel, frames, steps=12)
    np.savez_compressed(out / "model_tiny.npz", mel=mel.numpy(), prompt=np.asarray(prompt),
                        audio_features=_f32(audio), greedy=np.asarray(tokens),
                        first_logits=_f32(logits0), seed=np.asarray(11))


def gen_frontend(out: Path):
    """The reference's AudioFrontend (Whisper log-mel) on seeded clips of awkward lengths:
    a config-0 style mix of noise and sines, a clip that is not a multiple of the hop,
    a quiet one (the clip-max clamp bites) and the shortest that reflect padding allows."""
    import tempfile

    from qwen_asr_vllm.audio.frontend import AudioFrontend
    from voiceagent_b200.checkpoint import write_checkpoint
    from voiceagent_b200.workload import synthetic_waveform

    ckpt = write_checkpoint(Path(tempfile.mkdtemp()) / "ckpt", "tiny", weights=False)
    fe = AudioFrontend(str(ckpt))
    rng = np.random.default_rng(21)
    clips = [synthetic_waveform(1.0, rng), synthetic_waveform(0.77, rng)[:12321],
             (synthetic_waveform(0.5, rng) * 1e-4).astype(np.float32),
             rng.normal(0.0, 0.3, size=201).astype(np.float32)]
    mels = [fe(c, 16000).mel.float().numpy() for c in clips]
    lens = np.asarray([c.size for c in clips], np.int64)
    np.savez_compressed(out / "frontend.npz", wave=np.concatenate(clips), lens=lens,
                        mel=np.concatenate(mels, axis=1).astype(np.float32),
                        frames=np.asarray([m.shape[1] for m in mels], np.int64),
                        mel_filters=fe.extractor.mel_filters.astype(np.float32))


def gen_ref_engine_hf(out: Path):
    """The reference's upstream HF thinker (reference/modeling_qwen3_asr.py), 0.6B, the
    seeded bf16 checkpoint weights, bf16 on the CPU, teacher forced on the reference
    engine's greedy tokens (``ref_engine_tokens.npz``): per clip one forward over the
    prompt plus the engine's tokens, the argmax at every generated position. Audio comes
    from the reference's own frontend; prompts are the pinned template ids."""
    import tempfile

    import torch
    from qwen_asr_vllm.audio.frontend import AudioFrontend

    from voiceagent_b200.checkpoint import PRESETS, TOKEN_IDS, random_state_dict, write_checkpoint
    from voiceagent_b200.prompt import PromptBuilder

    sys.path.insert(0, str(HERE))
    from make_ref_engine_tokens import workload

    ref = np.load(out / "ref_engine_tokens.npz")
    tokens = ref["tokens"]
    meta = json.loads(str(ref["meta"]))
    hf = _import_hf_with_shims()
    cfg = {"audio": dict(PRESETS["0.6b"]["audio"]),
           "text": dict(PRESETS["0.6b"]["text"]), **TOKEN_IDS}
    weights = random_state_dict("0.6b", seed=0)  # bf16: the checkpoint's exact values
    weights["lm_head.weight"] = weights["model.embed_tokens.weight"]
    cfg_text = dict(cfg["text"])
    text_cfg = {"text": cfg_text}
    thinker = _build_hf_thinker(hf, {**cfg, **text_cfg}, {k: v.float() for k, v in weights.items()},
                                mrope_section=[24, 20, 20]).to(torch.bfloat16)
    ckpt = write_checkpoint(Path(tempfile.mkdtemp()) / "ckpt", "0.6b", weights=False)
    frontend = AudioFrontend(str(ckpt))
    builder = PromptBuilder()
    clips, n_tokens = workload()
    preds = np.full_like(tokens, -1)
    torch.set_num_threads(os.cpu_count() or 1)
    for i, (clip, n) in enumerate(zip(clips, n_tokens)):
        feats = frontend(clip, 16000)
        prompt = builder.build(feats.num_audio_tokens, language="English").token_ids
        assert len(prompt) == meta["prompt_tokens"][i], (len(prompt), meta["prompt_tokens"][i])
        ids = torch.tensor([prompt + [int(t) for t in tokens[i, :n - 1]]])
        mel = feats.mel.to(torch.bfloat16)
        with torch.no_grad():
            logits = thinker(input_ids=ids, input_features=mel.unsqueeze(0),
                             feature_attention_mask=torch.ones(1, mel.shape[1], dtype=torch.long),
                             attention_mask=torch.ones_like(ids), use_cache=False,
                             cache_position=torch.arange(ids.shape[1])).logits[0]
        preds[i, :n] = logits[len(prompt) - 1:].float().argmax(-1).numpy()
        print(f"clip {i}: {(preds[i, :n] == tokens[i, :n]).mean():.4f}", flush=True)
    valid = tokens >= 0
    agreement = float((preds == tokens)[valid].mean())
    np.savez_compressed(out / "ref_engine_hf.npz", hf_forced_tokens=preds,
                        agreement=np.asarray(agreement),
                        meta=np.array(json.dumps({
                            "generator": "tests/golden/make_golden.py --only ref_engine_hf",
                            "model": "reference/modeling_qwen3_asr.py thinker, bf16, CPU, eager "
                                     "attention, torch " + torch.__version__,
                            "teacher_forced_on": "ref_engine_tokens.npz tokens",
                            "agreement_with_reference_engine": agreement})))
    print("HF bf16 vs reference engine, teacher forced:", agreement)


GENERATORS = {
    "audio_pack": gen_audio_pack,
    "decoder_pack": gen_decoder_pack,
    "decode_bucket": gen_decode_bucket,
    "block_manager": gen_block_manager,
    "store": gen_store,
    "paged_decode": gen_paged_decode,
    "tts_pool_decode": gen_tts_pool_decode,
    "norm_rope": gen_norm_rope,
    "elementwise": gen_elementwise,
    "sampler": gen_sampler,
    "model_tiny": gen_model_tiny,
    "frontend": gen_frontend,
    "ref_engine_hf": gen_ref_engine_hf,
}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="VoiceAgent checkout")
    parser.add_argument("--only", nargs="*", default=None)
    args = parser.parse_args()
    if os.environ.get("TORCHDYNAMO_DISABLE") != "1":
        raise SystemExit("set TORCHDYNAMO_DISABLE=1 (eager reference semantics)")
    sys.path.insert(0, args.reference)
    for name, fn in GENERATORS.items():
        if args.only and name not in args.only:
            continue
        fn(HERE)
        print("wrote", name)


if __name__ == "__main__":
    main()
