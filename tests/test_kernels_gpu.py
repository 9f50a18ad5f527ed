"""CUDA kernels vs the reference (golden fixtures) and the CPU oracle.

Tolerances (north star): integer / byte work bit-exact; attention outputs within
bf16 tolerance -- max |err| <= 2e-2 and mean |err| <= 2e-3 against the float64
oracle; norm/rope/elementwise: >= 99.5 % of elements bit-identical to the
reference's eager output and all within one bf16 ulp.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kernels as K
from tests.conftest import bf16_bits_to_f32, load_json, load_npz

pytestmark = pytest.mark.gpu

ATOL_MAX = 2e-2
ATOL_MEAN = 2e-3


@pytest.fixture(scope="module")
def kx():
    from voiceagent_b200 import kernels

    return kernels


def dev(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def bf16(x):
    return torch.as_tensor(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).cuda()


def from_bits(bits):
    return bf16(bf16_bits_to_f32(bits))


def assert_attn_close(got: torch.Tensor, ref: np.ndarray, what: str):
    err = np.abs(got.float().cpu().numpy().astype(np.float64) - ref)
    assert np.isfinite(got.float().cpu().numpy()).all(), f"{what}: non-finite output"
    assert err.max() <= ATOL_MAX, f"{what}: max abs err {err.max():.3e}"
    assert err.mean() <= ATOL_MEAN, f"{what}: mean abs err {err.mean():.3e}"


def assert_bf16_match(got: torch.Tensor, ref: np.ndarray, what: str, exact_frac=0.995):
    g = got.float().cpu().numpy()
    same = np.mean(g == ref)
    assert same >= exact_frac, f"{what}: only {same:.4%} bit-identical"
    ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(g - ref) <= ulp + 1e-30), f"{what}: difference beyond one bf16 ulp"


# --------------------------------------------------------------------- packers


def _split(flat, lens):
    out, c = [], 0
    for n in lens:
        out.append(list(flat[c : c + n]))
        c += int(n)
    return out


def test_pack_decoder_matches_reference_prepare(kx):
    g = load_npz("decoder_pack.npz")
    for b in range(int(g["num_batches"])):
        p = f"b{b}_"
        starts, ends = g[p + "starts"], g[p + "ends"]
        tlens = g[p + "table_lens"]
        toks = _split(g[p + "tokens_flat"], g[p + "token_lens"])
        query = np.concatenate([np.asarray(t[s:e]) for t, s, e in zip(toks, starts, ends)])
        offs = np.concatenate([[0], np.cumsum(tlens)[:-1]]).astype(np.int32)
        batch, total = len(starts), int(query.size)
        width = int(tlens.max())
        out = {
            "input_ids": torch.empty(total, dtype=torch.int64, device="cuda"),
            "positions": torch.empty(total, dtype=torch.int64, device="cuda"),
            "slot_mapping": torch.empty(total, dtype=torch.int32, device="cuda"),
            "cu_seqlens_q": torch.empty(batch + 1, dtype=torch.int32, device="cuda"),
            "cu_seqlens_k": torch.empty(batch + 1, dtype=torch.int32, device="cuda"),
            "max_seqlen": torch.empty(2, dtype=torch.int32, device="cuda"),
            "block_tables": torch.empty(batch, width, dtype=torch.int32, device="cuda"),
            "last_token_index": torch.empty(batch, dtype=torch.int64, device="cuda"),
        }
        kx.pack_decoder(dev(starts, torch.int32), dev(ends, torch.int32), dev(offs, torch.int32),
                        dev(tlens, torch.int32), dev(g[p + "tables_flat"], torch.int32),
                        dev(query, torch.int32), total_tokens=total, width=width, block_size=256,
                        out=out)
        for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k",
                    "block_tables"):
            np.testing.assert_array_equal(out[key].cpu().numpy(), g[p + key], err_msg=f"{b} {key}")
        assert out["max_seqlen"].tolist() == g[p + "max_seqlen"].tolist()
        np.testing.assert_array_equal(out["last_token_index"].cpu().numpy(),
                                      g[p + "cu_seqlens_q"][1:].astype(np.int64) - 1)


def test_pack_decoder_large_batch_many_ctas(kx):
    rng = np.random.default_rng(5)
    batch = 700
    qlens = rng.integers(1, 40, size=batch)
    klens = qlens + rng.integers(0, 600, size=batch)
    tables = [list(rng.integers(0, 50000, size=(k + 255) // 256)) for k in klens]
    toks = [list(rng.integers(0, 151000, size=k)) for k in klens]
    ref = K.pack_decoder(klens - qlens, klens, tables, toks)
    query = np.concatenate([np.asarray(t[k - q:]) for t, q, k in zip(toks, qlens, klens)])
    tl = np.asarray([len(t) for t in tables], np.int32)
    total, width = int(query.size), int(tl.max())
    out = {k: torch.empty(n, dtype=d, device="cuda") for k, n, d in (
        ("input_ids", total, torch.int64), ("positions", total, torch.int64),
        ("slot_mapping", total, torch.int32), ("cu_seqlens_q", batch + 1, torch.int32),
        ("cu_seqlens_k", batch + 1, torch.int32), ("max_seqlen", 2, torch.int32),
        ("last_token_index", batch, torch.int64))}
    out["block_tables"] = torch.empty(batch, width, dtype=torch.int32, device="cuda")
    kx.pack_decoder(dev(klens - qlens, torch.int32), dev(klens, torch.int32),
                    dev(np.concatenate([[0], np.cumsum(tl)[:-1]]), torch.int32), dev(tl, torch.int32),
                    dev(np.concatenate(tables), torch.int32), dev(query, torch.int32),
                    total_tokens=total, width=width, block_size=256, out=out)
    for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k",
                "block_tables", "last_token_indices"):
        got_key = "last_token_index" if key == "last_token_indices" else key
        np.testing.assert_array_equal(out[got_key].cpu().numpy(), ref[key], err_msg=key)


def test_pack_decode_bucket_matches_reference_staging(kx):
    g = load_npz("decode_bucket.npz")
    for c in range(int(g["num_cases"])):
        p = f"c{c}_"
        bucket = int(g[p + "bucket"])
        lens, tl = g[p + "lens"], g[p + "table_lens"]
        batch = len(lens)
        offs = np.concatenate([[0], np.cumsum(tl)[:-1]]).astype(np.int32)
        bufs = dict(input_ids=torch.full((64,), 7, dtype=torch.int64, device="cuda"),
                    positions=torch.full((64,), 7, dtype=torch.int64, device="cuda"),
                    slot_mapping=torch.zeros(64, dtype=torch.int32, device="cuda"),
                    cu_seqlens_k=torch.zeros(65, dtype=torch.int32, device="cuda"),
                    block_tables=torch.full((64, 16), 9, dtype=torch.int32, device="cuda"))
        kx.pack_decode_bucket(dev(lens, torch.int32), dev(g[p + "last_ids"], torch.int32),
                              dev(offs, torch.int32), dev(tl, torch.int32),
                              dev(g[p + "tables_flat"], torch.int32), batch=batch, bucket=bucket,
                              max_blocks=16, block_size=256, **bufs)
        np.testing.assert_array_equal(bufs["input_ids"][:batch].cpu(), g[p + "input_ids"][:batch])
        np.testing.assert_array_equal(bufs["positions"][:batch].cpu(), g[p + "positions"][:batch])
        np.testing.assert_array_equal(bufs["slot_mapping"][:bucket].cpu(), g[p + "slot_mapping"])
        np.testing.assert_array_equal(bufs["cu_seqlens_k"][: bucket + 1].cpu(), g[p + "cu_seqlens_k"])
        np.testing.assert_array_equal(bufs["block_tables"][:bucket].cpu(), g[p + "block_tables"])


@pytest.mark.parametrize("index", range(18))
def test_pack_audio_matches_reference(kx, index):
    case = load_json("audio_pack.json")["packs"][index]
    frames = np.asarray(case["mel_frames"], np.int32)
    nc, nw = len(case["chunk_lengths"]), len(case["cu_seqlens"]) - 1
    out = dict(chunk_lengths=torch.empty(nc, dtype=torch.int64, device="cuda"),
               chunk_valid_lens=torch.empty(nc, dtype=torch.int64, device="cuda"),
               chunk_start=torch.empty(nc, dtype=torch.int32, device="cuda"),
               audio_token_lens=torch.empty(len(frames), dtype=torch.int32, device="cuda"),
               cu_seqlens=torch.empty(nw + 1, dtype=torch.int32, device="cuda"),
               counts=torch.empty(3, dtype=torch.int32, device="cuda"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kx.pack_audio(dev(frames, torch.int32), chunk_frames=100, window_tokens=case["window_tokens"],
                  max_chunks=nc, max_windows=nw, out=out, error_flag=err)
    assert err.item() == 0
    assert out["chunk_lengths"].tolist() == case["chunk_lengths"]
    assert out["chunk_valid_lens"].tolist() == case["chunk_valid_lens"]
    assert out["cu_seqlens"].tolist() == case["cu_seqlens"]
    assert out["audio_token_lens"].tolist() == case["audio_token_lens"]
    assert out["counts"].tolist() == [nc, nw, case["max_seqlen"]]
    starts = np.concatenate([[0], np.cumsum(case["chunk_lengths"])[:-1]])
    np.testing.assert_array_equal(out["chunk_start"].cpu().numpy(), starts)


def test_pack_audio_flags_capacity_overflow(kx):
    out = dict(chunk_lengths=torch.empty(1, dtype=torch.int64, device="cuda"),
               chunk_valid_lens=torch.empty(1, dtype=torch.int64, device="cuda"),
               chunk_start=torch.empty(1, dtype=torch.int32, device="cuda"),
               audio_token_lens=torch.empty(1, dtype=torch.int32, device="cuda"),
               cu_seqlens=torch.empty(2, dtype=torch.int32, device="cuda"),
               counts=torch.empty(3, dtype=torch.int32, device="cuda"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kx.pack_audio(dev(np.array([350], np.int32)), chunk_frames=100, window_tokens=104,
                  max_chunks=1, max_windows=1, out=out, error_flag=err)
    assert err.item() == 8 and out["counts"].tolist()[:2] == [4, 1]


def test_audio_chunk_pad_matches_oracle(kx):
    rng = np.random.default_rng(9)
    frames = [350, 7, 100, 201]
    meta = K.pack_audio_metadata(frames)
    mel = K.bf16_round(rng.standard_normal((128, sum(frames))).astype(np.float32))
    starts = np.concatenate([[0], np.cumsum(meta["chunk_lengths"])[:-1]]).astype(np.int32)
    out = torch.full((len(starts), 128, 100), 5.0, dtype=torch.bfloat16, device="cuda")
    kx.audio_chunk_pad(bf16(mel), dev(starts), dev(meta["chunk_lengths"]), len(starts), 100, out)
    np.testing.assert_array_equal(out.float().cpu().numpy(),
                                  K.chunk_and_pad(mel, meta["chunk_lengths"]))


@pytest.mark.parametrize("frames,d", [([350, 7, 100, 201], 896), ([1, 99, 100, 101, 3000], 64)])
def test_audio_gather_pos_matches_reference_mask_select(kx, frames, d):
    """Positional add + valid-token gather of the conv front against the reference's
    eager form (models/audio_encoder.py:169-173: ``embed + pos.to(bf16)``, rounded once,
    then ``embed[positions < chunk_valid_lens]``), bit for bit; padding rows are zero."""
    rng = np.random.default_rng(len(frames))
    meta = K.pack_audio_metadata(frames)
    valid = np.asarray(meta["chunk_valid_lens"])
    chunks, per = len(valid), 13
    embed = K.bf16_round(rng.standard_normal((chunks, per, d)).astype(np.float32))
    pos = K.bf16_round(rng.standard_normal((per, d)).astype(np.float32))
    mask = np.arange(per)[None, :] < valid[:, None]
    want = K.bf16_round((embed + pos[None]).astype(np.float32))[mask]
    index = np.flatnonzero(mask.ravel()).astype(np.int64)
    rows = len(index) + 11
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = kx.audio_gather_pos(bf16(embed), bf16(pos), dev(index), rows, error_flag=err)
    assert err.item() == 0
    np.testing.assert_array_equal(got[:len(index)].float().cpu().numpy(), want)
    assert not got[len(index):].float().abs().sum().item()
    # an index past the conv output is flagged and its row zeroed, the others kept
    bad = index.copy()
    bad[1] = chunks * per
    got = kx.audio_gather_pos(bf16(embed), bf16(pos), dev(bad), len(bad), error_flag=err)
    assert err.item() == 8 and not got[1].float().abs().sum().item()
    np.testing.assert_array_equal(got[2:].float().cpu().numpy(), want[2:])


# -------------------------------------------------------------------- KV store


def test_store_matches_reference_triton_kernel(kx):
    g = load_npz("store.npz")
    t, hq, hkv, d, nblocks = g["dims"].tolist()
    qkv = from_bits(g["qkv"])
    k = qkv[:, hq * d : (hq + hkv) * d].view(t, hkv, d)
    v = qkv[:, (hq + hkv) * d :].view(t, hkv, d)
    kc, vc = from_bits(g["k_cache_before"]), from_bits(g["v_cache_before"])
    kx.store_kvcache(k, v, kc, vc, dev(g["slots"], torch.int32))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kc.float().cpu().numpy(), bf16_bits_to_f32(g["k_cache"]))
    np.testing.assert_array_equal(vc.float().cpu().numpy(), bf16_bits_to_f32(g["v_cache"]))


def test_store_flags_out_of_range_slot(kx):
    kc = torch.zeros(2, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    k = torch.ones(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kx.store_kvcache(k, k, kc, vc, dev(np.array([3, 512], np.int32)), error_flag=err)
    assert err.item() == 1
    assert kc.view(512, 1024)[3].eq(1).all() and kc.sum().item() == 1024


# ------------------------------------------------------- norms, rope, elementwise


def test_qk_norm_rope_store_matches_reference(kx):
    g = load_npz("norm_rope.npz")
    qkv = from_bits(g["qkv"])
    t = qkv.shape[0]
    positions = dev(g["positions"], torch.int64)
    table = torch.zeros(4096, 128, dtype=torch.float32, device="cuda")
    table[positions] = dev(g["cos_sin_cache"], torch.float32)
    kc = torch.zeros(4, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.arange(t, dtype=torch.int32, device="cuda") * 37 % 1024
    slots[3] = -1
    q = torch.empty(t, 16, 128, dtype=torch.bfloat16, device="cuda")
    k_out = torch.empty(t, 8, 128, dtype=torch.bfloat16, device="cuda")
    kx.qk_norm_rope_store(qkv, positions, num_heads=16, num_kv_heads=8, head_dim=128,
                          q_weight=from_bits(g["q_weight"]), k_weight=from_bits(g["k_weight"]),
                          eps=1e-6, cos_sin_cache=table, q_out=q, k_cache=kc, v_cache=vc,
                          slot_mapping=slots, k_out=k_out)
    assert_bf16_match(q, bf16_bits_to_f32(g["q_out"]), "q")
    assert_bf16_match(k_out, bf16_bits_to_f32(g["k_out"]), "k")
    kflat, vflat = kc.view(-1, 8, 128), vc.view(-1, 8, 128)
    for i in range(t):
        s = int(slots[i])
        if s < 0:
            continue
        assert torch.equal(kflat[s], k_out[i])
        assert torch.equal(vflat[s], qkv[i, 3072:].view(8, 128))
    assert kflat.float().abs().sum().item() > 0


def test_rmsnorm_and_add_rmsnorm_match_reference(kx):
    g = load_npz("elementwise.npz")
    x, r, w = from_bits(g["x"]), from_bits(g["residual"]), from_bits(g["weight"])
    assert_bf16_match(kx.rmsnorm(x, w, 1e-6), bf16_bits_to_f32(g["rms"]), "rms")
    res = r.clone()
    y = kx.rmsnorm(x, w, 1e-6, residual=res)
    np.testing.assert_array_equal(res.float().cpu().numpy(), bf16_bits_to_f32(g["add_residual"]))
    assert_bf16_match(y, bf16_bits_to_f32(g["add_rms"]), "add_rms")


def test_silu_mul_matches_reference(kx):
    g = load_npz("elementwise.npz")
    out = kx.silu_mul(from_bits(g["gate_up"]))
    assert_bf16_match(out, bf16_bits_to_f32(g["silu_mul"]), "silu_mul", exact_frac=0.99)


# --------------------------------------------------------------------- sampler


def test_greedy_argmax_matches_reference_sampler(kx):
    g = load_npz("sampler.npz")
    ids = kx.greedy_argmax(from_bits(g["logits"]))
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])


def test_greedy_argmax_random_rows_and_ties(kx):
    rng = np.random.default_rng(2)
    logits = K.bf16_round(rng.standard_normal((33, 151936)).astype(np.float32) * 3)
    logits[5, [10, 150000]] = 50.0
    logits[6, :] = 1.0
    logits[7, 151935] = 60.0
    logits[8, [3, 99]] = np.nan
    ids = kx.greedy_argmax(bf16(logits)).cpu().numpy()
    ref = K.greedy_argmax(logits)
    ref[8] = 3  # torch/numpy: first NaN wins
    np.testing.assert_array_equal(ids, ref)
    odd = bf16(logits[:4, :1001])  # vocab not a multiple of 8, unaligned rows
    np.testing.assert_array_equal(kx.greedy_argmax(odd).cpu().numpy(),
                                  K.greedy_argmax(logits[:4, :1001]))


# ------------------------------------------------------------------ attention


def _decode_case(rng, lens, nblocks=4096, hq=16, hkv=8, d=128):
    b = len(lens)
    kc = K.bf16_round(rng.standard_normal((nblocks, 256, hkv, d)).astype(np.float32) / np.sqrt(d))
    vc = K.bf16_round(rng.standard_normal((nblocks, 256, hkv, d)).astype(np.float32) / np.sqrt(d))
    q = K.bf16_round(rng.standard_normal((b, hq, d)).astype(np.float32) / np.sqrt(d))
    perm = rng.permutation(nblocks)
    width = max((int(l) + 255) // 256 for l in lens)
    tables = np.zeros((b, width), np.int32)
    c = 0
    for i, l in enumerate(lens):
        n = (int(l) + 255) // 256
        tables[i, :n] = perm[c : c + n]
        c += n
    cu_k = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return q, kc, vc, tables, cu_k


def _run_decode(kx, q, kc, vc, tables, cu_k, max_len, err=None):
    qd, kcd, vcd = bf16(q), bf16(kc), bf16(vc)
    out = torch.zeros_like(qd)
    ws = torch.zeros(kx.paged_decode_workspace_size(q.shape[0], max_len, q.shape[1]) // 4 + 64,
                     dtype=torch.float32, device="cuda")
    kx.paged_decode(qd, kcd, vcd, dev(cu_k, torch.int32), dev(tables, torch.int32),
                    max_seqlen_k=max_len, scale=q.shape[-1] ** -0.5, out=out, workspace=ws,
                    error_flag=err)
    return out


def test_paged_decode_matches_reference_torch_path(kx):
    """Same inputs as the reference's own paged-decode oracle (TTS module)."""
    g = load_npz("paged_decode.npz")
    q = bf16_bits_to_f32(g["q"])
    kc, vc = bf16_bits_to_f32(g["k_cache"]), bf16_bits_to_f32(g["v_cache"])
    lens = g["lens"]
    cu_k = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    # the fixture has 4 query / 2 KV heads of dim 64; lift it into the engine's
    # head_dim 128 by zero-padding dims (scores unchanged when the scale is kept)
    pad = lambda x: np.concatenate([x, np.zeros_like(x)], axis=-1)
    qd, kcd, vcd = bf16(pad(q)), bf16(pad(kc)), bf16(pad(vc))
    out = torch.zeros_like(qd)
    ws = torch.zeros(1 << 22, dtype=torch.float32, device="cuda")
    kx.paged_decode(qd, kcd, vcd, dev(cu_k, torch.int32), dev(g["tables"], torch.int32),
                    max_seqlen_k=int(lens.max()), scale=64 ** -0.5, out=out, workspace=ws)
    assert_attn_close(out[..., :64], g["out_reference"].astype(np.float64), "decode vs reference")


@pytest.mark.parametrize("lens", [
    [1], [63], [64], [65], [255], [256], [257], [1023, 1024, 1025], [4096],
    [1, 2, 3, 4, 5, 300, 700, 128],
])
@pytest.mark.parametrize("max_len", ["tight", 4096])
def test_paged_decode_edges(kx, lens, max_len):
    """Both decode kernels: max_seqlen_k <= 512 selects one CTA per (sequence, KV head),
    larger bounds the stream-K split."""
    rng = np.random.default_rng(sum(lens))
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=64)
    out = _run_decode(kx, q, kc, vc, tables, cu_k, max(lens) if max_len == "tight" else max_len)
    ref = K.paged_attention(q, kc, vc, np.arange(len(lens) + 1), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, f"decode {lens} max_seqlen_k={max_len}")


@pytest.mark.parametrize("max_len", [512, 4096])
def test_paged_decode_step_shape_both_kernels(kx, max_len):
    """Config-3 decode-step shape (32 sequences of 80-250 tokens, random tables) through
    the short-context kernel (512) and the stream-K kernel (4096)."""
    rng = np.random.default_rng(77)
    lens = rng.integers(80, 251, size=32)
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=128)
    out = _run_decode(kx, q, kc, vc, tables, cu_k, max_len)
    ref = K.paged_attention(q, kc, vc, np.arange(33), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, f"decode step shape max_seqlen_k={max_len}")


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 4), (16, 8)])
@pytest.mark.parametrize("max_len", [512, 4096])
def test_paged_decode_query_groups(kx, hq, hkv, max_len):
    """Query heads per KV head G = 1, 4 and 2 through both kernels (peaked scores, lengths
    across stage and block boundaries)."""
    rng = np.random.default_rng(hq * 10 + hkv)
    lens = [1, 17, 64, 65, 200, 256, 300, 511]
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=64, hq=hq, hkv=hkv)
    q, kc = K.bf16_round(q * 2 * np.sqrt(128)), K.bf16_round(kc * 2 * np.sqrt(128))
    vc = vc * 8
    out = _run_decode(kx, q, kc, vc, tables, cu_k, max_len)
    ref = K.paged_attention(q, kc, vc, np.arange(len(lens) + 1), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, f"decode G={hq // hkv} max_seqlen_k={max_len}")


@pytest.mark.parametrize("max_len", [512, 4096])
def test_paged_decode_peaked_scores(kx, max_len):
    """Scores with a spread of ~9 (q, k ~ 3 N(0, 1) after the 1/sqrt(d) scale): the
    running-max rescale across stages and the split merge carry the result, not a
    near-uniform average. Lengths cross stage, 64-token and block boundaries."""
    rng = np.random.default_rng(9)
    lens = [70, 118, 1, 1, 257, 500, 33, 190]
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=64)
    q, kc = K.bf16_round(q * 3 * np.sqrt(128)), K.bf16_round(kc * 3 * np.sqrt(128))
    vc = vc * 8  # values ~ N(0, 0.5); a power of two keeps them exact in bf16
    out = _run_decode(kx, q, kc, vc, tables, cu_k, max_len)
    ref = K.paged_attention(q, kc, vc, np.arange(len(lens) + 1), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, f"decode peaked scores max_seqlen_k={max_len}")


@pytest.mark.parametrize("batch", [64, 160])
@pytest.mark.parametrize("pdl", [False, True])
def test_paged_decode_short_several_units_per_cta(kx, batch, pdl):
    """The short-context kernel when a CTA takes several (sequence, KV head) units
    (B x 8 units over at most 2 CTAs per SM: the decode graph's 64-row bucket and more)
    and contexts of up to eight 64-token stages, so each of its two consumer groups waits
    on ring slots the other group's stages occupied: eager, and as a PDL chain of graph
    launches back to back. Results against the oracle; the device error word stays zero
    (no bounded wait may time out)."""
    rng = np.random.default_rng(batch + pdl)
    lens = rng.integers(1, 512, size=batch)
    lens[:4] = [511, 449, 193, 1]
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=int(sum((lens + 255) // 256)))
    qd, kcd, vcd = bf16(q), bf16(kc), bf16(vc)
    cu, tb = dev(cu_k, torch.int32), dev(tables, torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.float32, device="cuda")
    out = torch.zeros_like(qd)
    kx.set_pdl(pdl)
    try:
        def run():
            kx.paged_decode(qd, kcd, vcd, cu, tb, max_seqlen_k=512, scale=128 ** -0.5, out=out,
                            workspace=ws, error_flag=err)

        run()
        torch.cuda.synchronize()
        assert err.item() == 0
        ref = K.paged_attention(q, kc, vc, np.arange(batch + 1), cu_k, tables, 128 ** -0.5)
        assert_attn_close(out, ref, f"short kernel, {batch} sequences, pdl={pdl}")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(8):
                run()
        out.zero_()
        for _ in range(4):
            graph.replay()
        torch.cuda.synchronize()
        del graph
    finally:
        kx.set_pdl(False)
    assert err.item() == 0
    assert_attn_close(out, ref, f"short kernel graph chain, {batch} sequences, pdl={pdl}")


@pytest.mark.parametrize("max_len", [512, 4096])
def test_paged_decode_newest_row_written_just_before_with_pdl(kx, max_len):
    """Both decode kernels request stages before their PDL wait, except those holding a
    sequence's newest token: with PDL on, a store of each sequence's newest K/V row
    immediately before the decode (in a graph) must be seen, as without PDL."""
    rng = np.random.default_rng(21)
    lens = [70, 128, 129, 200, 1, 64, 65, 250]
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=32)
    qd, kcd, vcd = bf16(q), bf16(kc), bf16(vc)
    cu, tb = dev(cu_k, torch.int32), dev(tables, torch.int32)
    newest = [int(tables[i, (n - 1) // 256]) * 256 + (n - 1) % 256 for i, n in enumerate(lens)]
    slots = dev(np.asarray(newest, np.int32), torch.int32)
    g = torch.Generator(device="cuda").manual_seed(5)
    new_k = (torch.randn(len(lens), 8, 128, device="cuda", generator=g) * 0.3).bfloat16()
    new_v = torch.randn(len(lens), 8, 128, device="cuda", generator=g).bfloat16()
    ws = torch.zeros(1 << 20, dtype=torch.float32, device="cuda")
    outs = []
    for pdl in (False, True):
        kx.set_pdl(pdl)
        try:
            k_run, v_run = kcd.clone(), vcd.clone()
            out = torch.zeros_like(qd)

            def step():
                kx.store_kvcache(new_k, new_v, k_run, v_run, slots)
                kx.paged_decode(qd, k_run, v_run, cu, tb, max_seqlen_k=max_len,
                                scale=128 ** -0.5, out=out, workspace=ws)

            step()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            for _ in range(3):  # the newest rows are rewritten each replay
                k_run.copy_(kcd)
                v_run.copy_(vcd)
                graph.replay()
            torch.cuda.synchronize()
            outs.append(out.clone())
            del graph
        finally:
            kx.set_pdl(False)
    assert torch.equal(outs[0], outs[1])
    kc2, vc2 = kc.copy(), vc.copy()
    for i, s in enumerate(newest):
        kc2.reshape(-1, 8, 128)[s] = new_k[i].float().cpu().numpy()
        vc2.reshape(-1, 8, 128)[s] = new_v[i].float().cpu().numpy()
    ref = K.paged_attention(q, kc2, vc2, np.arange(len(lens) + 1), cu_k, tables, 128 ** -0.5)
    assert_attn_close(outs[1], ref, "decode after a PDL store of the newest rows")


def test_paged_decode_config1(kx):
    """Benchmark configuration 1: B=32, ctx ~ U[64, 1024], 4096-block pool, random tables."""
    rng = np.random.default_rng(0)
    lens = rng.integers(64, 1025, size=32)
    q, kc, vc, tables, cu_k = _decode_case(rng, lens)
    out = _run_decode(kx, q, kc, vc, tables, cu_k, 4096)
    ref = K.paged_attention(q, kc, vc, np.arange(33), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, "decode config1")


def test_paged_decode_padding_rows_and_bad_block(kx):
    rng = np.random.default_rng(4)
    lens = [300, 1, 1]  # a real row and two graph padding rows (key length 1, block 0)
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=8)
    tables[1:] = 0
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = _run_decode(kx, q, kc, vc, tables, cu_k, 4096, err)
    ref = K.paged_attention(q, kc, vc, np.arange(4), cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, "decode padded")
    assert err.item() == 0
    tables[0, 1] = 99  # out of the 8-block pool: flagged, memory-safe
    _run_decode(kx, q, kc, vc, tables, cu_k, 4096, err)
    assert err.item() & 2


def _prefill_case(rng, q_lens, k_lens, nblocks=256):
    hq, hkv, d = 16, 8, 128
    kc = K.bf16_round(rng.standard_normal((nblocks, 256, hkv, d)).astype(np.float32))
    vc = K.bf16_round(rng.standard_normal((nblocks, 256, hkv, d)).astype(np.float32))
    tq = int(sum(q_lens))
    q = K.bf16_round(rng.standard_normal((tq, hq, d)).astype(np.float32))
    perm = rng.permutation(nblocks)
    width = max((k + 255) // 256 for k in k_lens)
    tables = np.full((len(q_lens), width), -1, np.int32)
    c = 0
    for i, k in enumerate(k_lens):
        n = (k + 255) // 256
        tables[i, :n] = perm[c : c + n]
        c += n
    cu_q = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(k_lens)]).astype(np.int32)
    return q, kc, vc, tables, cu_q, cu_k


def _run_prefill(kx, q, kc, vc, tables, cu_q, cu_k, err=None):
    qd = bf16(q)
    out = torch.zeros_like(qd)
    kx.paged_prefill(qd, bf16(kc), bf16(vc), dev(cu_q, torch.int32), dev(cu_k, torch.int32),
                     dev(tables, torch.int32), max_seqlen_q=int(np.diff(cu_q).max()),
                     scale=128 ** -0.5, out=out, error_flag=err)
    return out


@pytest.mark.parametrize("q_lens,k_lens", [
    ([76], [76]),
    ([1], [1]),
    ([64, 65, 63, 128, 129], [64, 65, 63, 128, 129]),
    ([76, 1, 300, 1, 40], [76, 257, 300, 1000, 552]),   # mixed prefill/decode, cached prefixes
    ([700], [700]),
])
def test_paged_prefill_matches_oracle(kx, q_lens, k_lens):
    rng = np.random.default_rng(len(q_lens) * 7 + sum(k_lens))
    q, kc, vc, tables, cu_q, cu_k = _prefill_case(rng, q_lens, k_lens)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = _run_prefill(kx, q, kc, vc, tables, cu_q, cu_k, err)
    ref = K.paged_attention(q, kc, vc, cu_q, cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, f"prefill {q_lens}/{k_lens}")
    assert err.item() == 0


def test_paged_prefill_config2_lengths(kx):
    """Benchmark configuration 2, decoder part: 32 prompts of 13*s + 24 tokens, s ~ U(2, 30)."""
    rng = np.random.default_rng(2)
    secs = rng.uniform(2, 30, size=32)
    lens = [int(K.num_audio_tokens(int(100 * s))) + 24 for s in secs]
    q, kc, vc, tables, cu_q, cu_k = _prefill_case(rng, lens, lens, nblocks=128)
    out = _run_prefill(kx, q, kc, vc, tables, cu_q, cu_k)
    ref = K.paged_attention(q, kc, vc, cu_q, cu_k, tables, 128 ** -0.5)
    assert_attn_close(out, ref, "prefill config2")


def _poison_unused(kc, vc, tables, k_lens, block=256):
    """NaN in every cache slot that no sequence holds: never-written pages and the tails of
    the sequences' last pages (what a freshly allocated cache may contain). flash-attn's
    paged kernels never let those slots reach an output; neither may ours."""
    used = np.zeros(kc.shape[:2], bool)
    for i, n in enumerate(k_lens):
        for b in range((int(n) + block - 1) // block):
            used[tables[i, b], : min(block, int(n) - b * block)] = True
    kc, vc = kc.copy(), vc.copy()
    kc[~used] = np.nan
    vc[~used] = np.nan
    return kc, vc


@pytest.mark.parametrize("q_lens,k_lens", [
    ([76, 1, 300, 1, 40], [76, 257, 300, 1000, 552]),
    ([63, 130, 1], [63, 130, 1]),
])
def test_paged_prefill_ignores_unwritten_cache_slots(kx, q_lens, k_lens):
    rng = np.random.default_rng(sum(k_lens) + 5)
    q, kc, vc, tables, cu_q, cu_k = _prefill_case(rng, q_lens, k_lens)
    ref = K.paged_attention(q, kc, vc, cu_q, cu_k, tables, 128 ** -0.5)
    kc, vc = _poison_unused(kc, vc, tables, k_lens)
    out = _run_prefill(kx, q, kc, vc, tables, cu_q, cu_k)
    assert torch.isfinite(out).all()
    assert_attn_close(out, ref, f"prefill over a NaN-filled cache {q_lens}/{k_lens}")


@pytest.mark.parametrize("max_len", [512, 4096])
def test_paged_decode_ignores_unwritten_cache_slots(kx, max_len):
    rng = np.random.default_rng(31)
    lens = [1, 17, 64, 65, 200, 256, 300, 511]
    q, kc, vc, tables, cu_k = _decode_case(rng, lens, nblocks=64)
    ref = K.paged_attention(q, kc, vc, np.arange(len(lens) + 1), cu_k, tables, 128 ** -0.5)
    kc, vc = _poison_unused(kc, vc, tables, lens)
    out = _run_decode(kx, q, kc, vc, tables, cu_k, max_len)
    assert torch.isfinite(out).all()
    assert_attn_close(out, ref, f"decode over a NaN-filled cache max_seqlen_k={max_len}")


def _window_case(rng, token_lens, heads=14, d=64):
    cu = np.asarray(K.build_window_boundaries(token_lens, 104), np.int32)
    t = int(cu[-1])
    qkv = K.bf16_round(rng.standard_normal((t, 3, heads, d)).astype(np.float32))
    return qkv, cu


@pytest.mark.parametrize("token_lens", [[46, 26, 95], [250], [208], [1], [104, 1, 103, 400]])
def test_varlen_window_attention_matches_oracle(kx, token_lens):
    rng = np.random.default_rng(sum(token_lens))
    qkv, cu = _window_case(rng, token_lens)
    d = bf16(qkv.reshape(qkv.shape[0], -1))
    q = d[:, : 14 * 64].view(-1, 14, 64)
    k = d[:, 14 * 64 : 28 * 64].view(-1, 14, 64)
    v = d[:, 28 * 64 :].view(-1, 14, 64)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = kx.varlen_attention(q, k, v, dev(cu, torch.int32), int(np.diff(cu).max()), 64 ** -0.5,
                              error_flag=err)
    ref = K.varlen_attention(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, 64 ** -0.5)
    assert_attn_close(out, ref, f"window {token_lens}")
    assert err.item() == 0


def test_varlen_window_segments_stay_independent(kx):
    """A segment's 128-row tile reaches into the next segments: NaN in one segment's K
    and V must not leak into the segment before it (the reference's varlen kernel keeps
    segments apart)."""
    rng = np.random.default_rng(12)
    token_lens = [46, 26, 95, 30]
    qkv, cu = _window_case(rng, token_lens)
    ref = K.varlen_attention(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, 64 ** -0.5)
    poisoned = qkv.copy()
    bad = slice(int(cu[1]), int(cu[2]))  # segment 1
    poisoned[bad, 1:] = np.nan
    d = bf16(poisoned.reshape(poisoned.shape[0], -1))
    q = d[:, : 14 * 64].view(-1, 14, 64)
    k = d[:, 14 * 64 : 28 * 64].view(-1, 14, 64)
    v = d[:, 28 * 64 :].view(-1, 14, 64)
    out = kx.varlen_attention(q, k, v, dev(cu, torch.int32), int(np.diff(cu).max()), 64 ** -0.5)
    keep = np.ones(qkv.shape[0], bool)
    keep[bad] = False
    got = out[torch.from_numpy(keep).cuda()]
    assert torch.isfinite(got).all()
    assert_attn_close(got, ref[keep], "window segments next to a NaN segment")


# ------------------------------------------------------------------ mel frontend


def _bf16_ulp_close(got, want, atol=1e-3):
    """(fraction of bit-identical bf16 values, all within one bf16 ulp or ``atol``, worst).

    The absolute floor covers values near zero: (x + 4) / 4 cancels there, a bf16 ulp
    shrinks with the value, and fp32 STFT rounding (~1e-6) can exceed it."""
    w = torch.as_tensor(np.ascontiguousarray(want, dtype=np.float32)).to(torch.bfloat16).float()
    g = got.float().cpu()
    exact = (g == w).float().mean().item()
    ulp = torch.exp2(torch.floor(torch.log2(w.abs().clamp_min(1e-30))) - 7)
    err = (g - w).abs()
    ok = err <= torch.maximum(ulp, torch.full_like(ulp, atol))
    i = int(torch.argmax(err / torch.maximum(ulp, torch.full_like(ulp, atol))))
    worst = (float(g.flatten()[i]), float(w.flatten()[i]), float(err.flatten()[i]))
    return exact, bool(ok.all()), worst


def _render(frontend, clips, columns=None, width=None):
    feats = [frontend(c) for c in clips]
    frames = [f.mel_frames for f in feats]
    if columns is None:
        columns = list(np.concatenate([[0], np.cumsum(frames)])[:-1])
        width = int(sum(frames))
    out = torch.full((128, width), float("nan"), dtype=torch.bfloat16, device="cuda")
    frontend.render(feats, out, [int(c) for c in columns])
    torch.cuda.synchronize()
    return out, frames


@pytest.fixture(scope="module")
def gpu_frontend():
    from voiceagent_b200.audio.frontend import GpuMelFrontend

    return GpuMelFrontend(None)


def test_log_mel_matches_reference_frontend(gpu_frontend):
    z = load_npz("frontend.npz")
    off = np.concatenate([[0], np.cumsum(z["lens"])])
    clips = [z["wave"][off[i]:off[i + 1]] for i in range(len(z["lens"]))]
    out, frames = _render(gpu_frontend, clips)
    assert frames == list(z["frames"])
    exact, within, worst = _bf16_ulp_close(out, z["mel"])
    assert exact >= 0.995 and within, (exact, worst)


def test_log_mel_matches_oracle_on_mixed_lengths(gpu_frontend):
    from voiceagent_b200.workload import config0_clip, synthetic_waveform

    rng = np.random.default_rng(5)
    clips = [config0_clip(0), synthetic_waveform(2.3456, rng), rng.normal(0, 0.2, 201).astype(np.float32),
             (synthetic_waveform(0.9, rng) * 1e-5).astype(np.float32), synthetic_waveform(12.0, rng)]
    filters = np.asarray(gpu_frontend.extractor.mel_filters)
    # scattered, out-of-order output columns with untouched gaps between them
    frames = [c.size // 160 for c in clips]
    columns, at = [], 7
    for f in reversed(frames):
        columns.insert(0, at)
        at += f + 5
    out, _ = _render(gpu_frontend, clips, columns=columns, width=at)
    covered = torch.zeros(at, dtype=torch.bool)
    for c, f, clip in zip(columns, frames, clips):
        exact, within, worst = _bf16_ulp_close(out[:, c:c + f], K.log_mel(clip, filters))
        assert exact >= 0.995 and within, (exact, worst, clip.size)
        covered[c:c + f] = True
    assert torch.isnan(out[:, ~covered.cuda()].float()).all()  # nothing written outside


@pytest.mark.parametrize("staged", [(0, 1, 2, 3, 4), (1, 3), (0, 4), (2,)])
def test_log_mel_of_clips_staged_ahead_is_identical(gpu_frontend, staged):
    """Clips copied into pinned memory ahead of their batch (GpuMelFrontend.stage, as the
    engine does while a decoder call runs) render exactly as clips staged with the batch,
    for every pattern of staged / not staged runs; the staged buffers are released."""
    from voiceagent_b200.workload import synthetic_waveform

    rng = np.random.default_rng(9)
    clips = [synthetic_waveform(s, rng) for s in (1.7, 3.05, 0.4, 7.3, 2.0)]
    want, frames = _render(gpu_frontend, clips)
    feats = [gpu_frontend(c) for c in clips]
    for i in staged:
        assert gpu_frontend.stage(feats[i]) and not gpu_frontend.stage(feats[i])
    columns = list(np.concatenate([[0], np.cumsum(frames)])[:-1])
    got = torch.full_like(want, float("nan"))
    gpu_frontend.render(feats, got, [int(c) for c in columns])
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert all(f.staged is None for f in feats)


def test_log_mel_rejects_short_clips(gpu_frontend):
    with pytest.raises(ValueError):
        gpu_frontend(np.zeros(200, np.float32))


# ------------------------------------------------------------------ decode linears


def _close_to(got, ref, rel=1e-2):
    """bf16 GEMM output vs an fp32 reference of the same math."""
    scale = ref.abs().max().item()
    err = (got.float() - ref).abs()
    ulp_ok = (got.float() == ref.bfloat16().float()).float().mean().item()
    return err.max().item() <= rel * scale and err.mean().item() <= 2e-3 * scale, ulp_ok


@pytest.mark.parametrize("m,k,n", [(1, 1024, 4096), (7, 1024, 1024), (32, 2048, 1024),
                                   (32, 3072, 1024), (33, 1024, 4096), (64, 2048, 2048),
                                   (16, 6144, 2048)])
def test_linear_small_matches_fp32_matmul(kx, m, k, n):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + k + n)
    base = torch.randn(m, k + 64, device="cuda", generator=g).bfloat16()
    x = base[:, :k]  # row stride k + 64: a strided view
    w = (torch.randn(n, k, device="cuda", generator=g) * k ** -0.5).bfloat16()
    y = kx.linear_small(x, w)
    ref = x.float() @ w.float().T
    ok, exact = _close_to(y, ref)
    assert ok and exact >= 0.98, exact


@pytest.mark.parametrize("m,k,inner", [(1, 1024, 3072), (32, 1024, 3072), (64, 2048, 6144)])
def test_linear_small_fused_silu_mul(kx, m, k, inner):
    import torch.nn.functional as F

    g = torch.Generator(device="cuda").manual_seed(m + inner)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * inner, k, device="cuda", generator=g) * k ** -0.5).bfloat16()
    y = kx.linear_small(x, w, silu=True)
    proj = (x.float() @ w.float().T).bfloat16().float()  # the unfused path's bf16 projection
    gate, up = proj[:, :inner], proj[:, inner:]
    ref = (F.silu(gate).bfloat16().float() * up)
    ok, exact = _close_to(y, ref, rel=2e-2)
    assert y.shape == (m, inner) and ok and exact >= 0.97, exact


def test_linear_small_lm_head_width(kx):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(32, 1024, device="cuda", generator=g).bfloat16()
    w = (torch.randn(151936, 1024, device="cuda", generator=g) * 0.03).bfloat16()
    y = kx.linear_small(x, w)
    ok, exact = _close_to(y, x.float() @ w.float().T)
    assert ok and exact >= 0.98, exact


@pytest.mark.parametrize("m,k,tiles", [(32, 1024, 1187), (1, 1024, 297), (17, 2048, 700),
                                       (64, 2048, 1187), (40, 1024, 333)])
def test_linear_small_persistent_stream_equals_one_cta_per_tile(kx, m, k, tiles):
    """Projections with more 128-row tiles than two waves of CTAs (the lm_head) run on the
    persistent streaming kernel; its output is bit-identical to the one-CTA-per-tile
    kernel's, which even slices of 120-256 tiles still take (no K split at that many
    tiles, so the same summation order), and close to fp32."""
    g = torch.Generator(device="cuda").manual_seed(m + k + tiles)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(tiles * 128, k, device="cuda", generator=g) * 0.03).bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = kx.linear_small(x, w, error_flag=err)
    cuts = np.linspace(0, tiles, -(-tiles // 256) + 1).round().astype(int) * 128
    assert all(120 * 128 <= b - a <= 256 * 128 for a, b in zip(cuts[:-1], cuts[1:]))
    parts = [kx.linear_small(x, w[a:b], error_flag=err) for a, b in zip(cuts[:-1], cuts[1:])]
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.equal(y, torch.cat(parts, dim=1))
    ok, exact = _close_to(y, x.float() @ w.float().T)
    assert ok and exact >= 0.98, exact


def _within_one_ulp(got, ref, exact_frac=0.99):
    """bf16 tensors that differ only by fp32 summation order upstream."""
    g, r = got.float(), ref.float()
    same = (g == r).float().mean().item()
    ulp = r.abs().clamp_min(1e-30) * 2.0 ** -7
    return same >= exact_frac and bool(((g - r).abs() <= ulp).all()), same


@pytest.mark.parametrize("m", [1, 17, 32, 64])
def test_linear_small_add_matches_unfused(kx, m):
    """o_proj / down_proj + residual add: residual and h bit-exact against linear_small
    followed by the add of rmsnorm; tile sums of h^2 against float64."""
    g = torch.Generator(device="cuda").manual_seed(m)
    # 0.6B o_proj / down_proj, then the 1.7B ones (K = 6144 streams past the ring)
    for k, n in ((2048, 1024), (3072, 1024), (2048, 2048), (6144, 2048)):
        x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(n, k, device="cuda", generator=g) * k ** -0.5).bfloat16()
        res = torch.randn(m, n, device="cuda", generator=g).bfloat16()
        state = kx.NormState(m, n, "cuda")
        res_fused = res.clone()
        kx.linear_small_add(x, w, res_fused, state)
        y = kx.linear_small(x, w)
        h_ref = y.float() + res.float()
        assert torch.equal(state.h, h_ref)
        assert torch.equal(res_fused, h_ref.bfloat16())
        ss_ref = (h_ref.double() ** 2).reshape(m, n // 128, 128).sum(-1)
        torch.testing.assert_close(state.ss.double(), ss_ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("m", [1, 32, 64])
@pytest.mark.parametrize("silu", [False, True])
@pytest.mark.parametrize("hidden,inner", [(1024, 3072), (2048, 6144)])  # 0.6B, 1.7B
def test_linear_small_norm_matches_unfused(kx, m, silu, hidden, inner):
    """RMSNorm prologue: the same as rmsnorm(y, residual) then linear_small, up to the
    order of the fp32 sum of squares (outputs within one bf16 ulp, nearly all equal)."""
    g = torch.Generator(device="cuda").manual_seed(100 + m + hidden)
    n = 2 * inner if silu else 4096
    y = torch.randn(m, hidden, device="cuda", generator=g).bfloat16()
    res = torch.randn(m, hidden, device="cuda", generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).bfloat16()
    w = (torch.randn(n, hidden, device="cuda", generator=g) * hidden ** -0.5).bfloat16()
    state = kx.rms_stats(y, kx.NormState(m, hidden, "cuda"), residual=res.clone())
    fused = kx.linear_small_norm(state, nw, 1e-6, w, silu=silu)
    # an L2 prefetch hint of two ranges changes nothing
    hinted = kx.linear_small_norm(state, nw, 1e-6, w, silu=silu,
                                  prefetch=kx.l2_prefetch(ranges=(w, nw)))
    assert torch.equal(fused, hinted)
    normed = kx.rmsnorm(y, nw, 1e-6, residual=res.clone())
    # the normalised activation itself, as the prologue builds it: bf16(bf16(h * rs) * w)
    # with rs from another fp32 summation order, so the inner rounding can move one ulp
    # and the outer one can turn that into two
    applied = kx.norm_apply(state, nw, 1e-6)
    ok, same = _within_one_ulp(applied, normed, 0.995)
    if not ok:
        a, r = applied.float(), normed.float()
        assert same >= 0.995 and bool(((a - r).abs() <= r.abs().clamp_min(1e-30) * 2.0 ** -6).all()), same
    unfused = kx.linear_small(normed, w, silu=silu)
    ok, same = _within_one_ulp(fused, unfused, 0.97)
    if not ok:  # an input that moved by one ulp moves the sum by more: bound it instead
        err = (fused.float() - unfused.float()).abs().max().item()
        assert err <= 2e-2 * unfused.float().abs().max().item() and same >= 0.97, (err, same)


@pytest.mark.parametrize("m", [1, 33, 64])
@pytest.mark.parametrize("hidden", [1024, 2048])  # 0.6B, 1.7B
def test_linear_small_qk_rope_matches_unfused(kx, m, hidden):
    """qkv_proj on a normalised x + q/k norm + RoPE + KV store in one kernel: q, K and V
    bit-exact against linear_small followed by qk_norm_rope_store (same K split, same
    per-head arithmetic); slot -1 rows leave the cache untouched."""
    from voiceagent_b200.layers.norm import rope_table

    g = torch.Generator(device="cuda").manual_seed(11 + m + hidden)
    hq, hkv, d = 16, 8, 128
    base = torch.randn(m, hidden + 64, device="cuda", generator=g).bfloat16()
    x = base[:, :hidden]  # a strided view
    w = (torch.randn((hq + 2 * hkv) * d, hidden, device="cuda", generator=g) * 0.03).bfloat16()
    qw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    positions = torch.randint(0, 4096, (m,), device="cuda", generator=g)
    nslots = 4 * 256
    slots = torch.randperm(nslots, device="cuda", generator=g)[:m].int()
    slots[::5] = -1
    table = rope_table(d, 4096, 1e6, "cuda")
    outs = []
    for fused in (True, False):
        kc = torch.full((4, 256, hkv, d), 7.0, device="cuda").bfloat16()
        vc = kc.clone()
        q = torch.empty(m, hq, d, device="cuda", dtype=torch.bfloat16)
        heads = dict(num_heads=hq, num_kv_heads=hkv, head_dim=d, q_weight=qw, k_weight=kw,
                     cos_sin_cache=table, q_out=q, k_cache=kc, v_cache=vc, slot_mapping=slots)
        if fused:
            kx.linear_small_qk_rope(x, w, positions, qk_eps=1e-6, **heads)
        else:
            kx.qk_norm_rope_store(kx.linear_small(x, w), positions, eps=1e-6, **heads)
        outs.append((q, kc, vc))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    untouched = torch.ones(nslots, dtype=torch.bool, device="cuda")
    untouched[slots[slots >= 0].long()] = False
    assert bool((outs[0][1].view(nslots, -1)[untouched] == 7.0).all())


@pytest.mark.parametrize("m", [1, 32, 64])
@pytest.mark.parametrize("hidden", [1024, 2048])  # 0.6B, 1.7B
def test_linear_small_norm_qk_rope_matches_unfused(kx, m, hidden):
    """qkv_proj (RMSNorm prologue) + q/k norm + RoPE + KV store in one kernel: q, K and V
    bit-exact against linear_small_norm followed by qk_norm_rope_store (same K split,
    same per-head arithmetic); slot -1 rows leave the cache untouched."""
    g = torch.Generator(device="cuda").manual_seed(7 + m + hidden)
    hq, hkv, d = 16, 8, 128
    y = torch.randn(m, hidden, device="cuda", generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).bfloat16()
    w = (torch.randn((hq + 2 * hkv) * d, hidden, device="cuda", generator=g) * 0.03).bfloat16()
    qw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    positions = torch.randint(0, 4096, (m,), device="cuda", generator=g)
    nslots = 4 * 256
    slots = torch.randperm(nslots, device="cuda", generator=g)[:m].int()
    slots[::5] = -1
    from voiceagent_b200.layers.norm import rope_table

    table = rope_table(d, 4096, 1e6, "cuda")
    state = kx.rms_stats(y, kx.NormState(m, hidden, "cuda"))
    # an L2 prefetch hint (K/V over ragged sequences, one with an out-of-pool block that is
    # skipped, and two ranges) changes nothing
    pf_lens = torch.tensor([0, 300, 1, 700, 255], dtype=torch.int32, device="cuda")
    pf_cu = torch.cat([torch.zeros(1, dtype=torch.int32, device="cuda"), pf_lens.cumsum(0).int()])
    pf_tables = torch.tensor([[0, 0, 0], [1, 2, 0], [3, 0, 0], [0, 1, 99], [2, 0, 0]],
                             dtype=torch.int32, device="cuda")
    pf_k = torch.zeros(4, 256, hkv, d, device="cuda", dtype=torch.bfloat16)
    outs = []
    for fused in (True, "prefetch", False):
        kc = torch.full((4, 256, hkv, d), 7.0, device="cuda").bfloat16()
        vc = kc.clone()
        q = torch.empty(m, hq, d, device="cuda", dtype=torch.bfloat16)
        if fused:
            kx.linear_small_norm_qk_rope(state, nw, 1e-6, w, positions, num_heads=hq,
                                         num_kv_heads=hkv, head_dim=d, q_weight=qw, k_weight=kw,
                                         qk_eps=1e-6, cos_sin_cache=table, q_out=q, k_cache=kc,
                                         v_cache=vc, slot_mapping=slots,
                                         prefetch=kx.l2_prefetch(
                                             kv=(pf_cu, pf_tables, pf_k, pf_k), ranges=(w, table))
                                         if fused == "prefetch" else None)
        else:
            qkv = kx.linear_small_norm(state, nw, 1e-6, w)
            kx.qk_norm_rope_store(qkv, positions, num_heads=hq, num_kv_heads=hkv, head_dim=d,
                                  q_weight=qw, k_weight=kw, eps=1e-6, cos_sin_cache=table,
                                  q_out=q, k_cache=kc, v_cache=vc, slot_mapping=slots)
        outs.append((q, kc, vc))
    for a, b, c in zip(*outs):
        assert torch.equal(a, c) and torch.equal(b, c)
    untouched = torch.ones(nslots, dtype=torch.bool, device="cuda")
    untouched[slots[slots >= 0].long()] = False
    assert bool((outs[0][1].view(nslots, -1)[untouched] == 7.0).all())


def test_fused_step_rejects_bad_slot(kx):
    """An out-of-range slot raises the error flag and stores nothing (memory safe)."""
    hidden, hq, hkv, d, m = 1024, 16, 8, 128, 4
    y = torch.randn(m, hidden, device="cuda").bfloat16()
    ones = torch.ones(hidden, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn((hq + 2 * hkv) * d, hidden, device="cuda") * 0.03).bfloat16()
    from voiceagent_b200.layers.norm import rope_table

    kc = torch.zeros(2, 256, hkv, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    state = kx.rms_stats(y, kx.NormState(m, hidden, "cuda"))
    kx.linear_small_norm_qk_rope(
        state, ones, 1e-6, w, torch.zeros(m, dtype=torch.int64, device="cuda"), num_heads=hq,
        num_kv_heads=hkv, head_dim=d, q_weight=ones[:d], k_weight=ones[:d], qk_eps=1e-6,
        cos_sin_cache=rope_table(d, 16, 1e6, "cuda"),
        q_out=torch.empty(m, hq, d, device="cuda", dtype=torch.bfloat16), k_cache=kc, v_cache=vc,
        slot_mapping=torch.tensor([0, 1, 512, -1], dtype=torch.int32, device="cuda"),
        error_flag=err)
    torch.cuda.synchronize()
    assert err.item() != 0
    assert bool((kc.view(512, -1)[2:] == 0).all()) and bool((vc.view(512, -1)[2:] == 0).all())


def test_linear_small_chain_with_pdl_in_a_graph(kx):
    """Dependent linear_small / rmsnorm launches with PDL, captured in a graph, give the
    same bytes as without PDL (the waits order every read after its producer)."""
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(32, 1024, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(1024, 1024, device="cuda", generator=g) * 0.03).bfloat16() for _ in range(6)]
    nw = torch.ones(1024, device="cuda", dtype=torch.bfloat16)

    def chain():
        h = x
        for w in ws:
            h = kx.rmsnorm(kx.linear_small(h, w), nw, 1e-6)
        return h

    outs = []
    for pdl in (False, True):
        kx.set_pdl(pdl)
        try:
            chain()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                y = chain()
            graph.replay()
            torch.cuda.synchronize()
            outs.append(y.clone())
        finally:
            kx.set_pdl(False)
    assert torch.equal(outs[0], outs[1])


def test_paged_decode_reuses_its_workspace_across_calls(kx):
    """Config-1-sized calls three times in a row on one workspace with different data: the
    merge counters the kernel leaves behind must not leak into the next call."""
    rng = np.random.default_rng(41)
    b, h, hkv, d, nb = 32, 16, 8, 128, 320
    ws = torch.zeros(kx.paged_decode_workspace_size(b, 4096, h) // 4 + 64, dtype=torch.float32,
                     device="cuda")
    for call in range(3):
        lens = rng.integers(64, 1025, size=b)
        kc = K.bf16_round(rng.standard_normal((nb, 256, hkv, d)).astype(np.float32) / 11.3)
        vc = K.bf16_round(rng.standard_normal((nb, 256, hkv, d)).astype(np.float32) / 11.3)
        q = K.bf16_round(rng.standard_normal((b, h, d)).astype(np.float32) / 11.3)
        perm = rng.permutation(nb)
        tables = np.zeros((b, 5), np.int32)
        c = 0
        for i, n in enumerate(lens):
            m = (int(n) + 255) // 256
            tables[i, :m] = perm[c:c + m]
            c += m
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        out = torch.full((b, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        kx.paged_decode(bf16(q), bf16(kc), bf16(vc), dev(cu, torch.int32), dev(tables, torch.int32),
                        max_seqlen_k=4096, scale=d ** -0.5, out=out, workspace=ws, error_flag=err)
        ref = K.paged_attention(q, kc, vc, np.arange(b + 1), cu, tables, d ** -0.5)
        e = np.abs(out.float().cpu().numpy() - ref)
        assert err.item() == 0
        assert e.max() <= ATOL_MAX and e.mean() <= ATOL_MEAN, (call, e.max())
    assert int(ws[:4096 // 4].view(torch.int32).abs().sum().item()) == 0  # header left at zero
