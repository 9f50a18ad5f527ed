"""The CPU oracle reproduces the reference's own outputs (fixtures in tests/golden).

These pin ``oracle/`` before it is trusted as the checker for the CUDA kernels.
Integer fixtures must match exactly; floating-point fixtures within the stated
tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kernels as K
from oracle import model as M
from tests.conftest import bf16_bits_to_f32, load_json, load_npz


# --------------------------------------------------------------- audio packing


def test_num_audio_tokens_all_frame_counts():
    golden = load_json("audio_pack.json")["num_audio_tokens"]
    assert [K.num_audio_tokens(f) for f in range(1, 6000)] == golden


def test_window_boundaries_known_answers():
    for case in load_json("audio_pack.json")["windows"]:
        assert K.build_window_boundaries(case["lens"], case["window"]) == case["boundaries"]
    # test_units.py:74-88 of the reference
    assert K.attention_window_tokens(800) == 104
    assert K.build_window_boundaries([46, 26, 95], 104) == [0, 46, 72, 167]
    assert K.build_window_boundaries([250], 104) == [0, 104, 208, 250]
    assert K.build_window_boundaries([208], 104) == [0, 104, 208]


@pytest.mark.parametrize("index", range(18))
def test_pack_audio_metadata(index):
    case = load_json("audio_pack.json")["packs"][index]
    got = K.pack_audio_metadata(case["mel_frames"], 800)
    assert got["chunk_lengths"].tolist() == case["chunk_lengths"]
    assert got["chunk_valid_lens"].tolist() == case["chunk_valid_lens"]
    assert got["cu_seqlens"].tolist() == case["cu_seqlens"]
    assert got["audio_token_lens"].tolist() == case["audio_token_lens"]
    assert got["max_seqlen"] == case["max_seqlen"]
    assert got["window_tokens"] == case["window_tokens"]


def test_pack_audio_reference_unit_case():
    # test_units.py:89-98: (350, 200, 105) frames
    got = K.pack_audio_metadata([350, 200, 105])
    assert got["audio_token_lens"].tolist() == [46, 26, 14]
    assert got["chunk_lengths"].tolist() == [100, 100, 100, 50, 100, 100, 100, 5]


def test_chunk_lengths_reject_empty():
    with pytest.raises(ValueError):
        K.chunk_lengths_for(0)


# ------------------------------------------------------------- decoder packing


def _split(flat, lens):
    out, c = [], 0
    for n in lens:
        out.append(list(flat[c : c + n]))
        c += int(n)
    return out


def test_pack_decoder_matches_prepare():
    g = load_npz("decoder_pack.npz")
    for b in range(int(g["num_batches"])):
        p = f"b{b}_"
        tables = _split(g[p + "tables_flat"], g[p + "table_lens"])
        toks = _split(g[p + "tokens_flat"], g[p + "token_lens"])
        got = K.pack_decoder(g[p + "starts"], g[p + "ends"], tables, toks)
        for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k",
                    "block_tables"):
            np.testing.assert_array_equal(got[key], g[p + key], err_msg=f"batch {b} {key}")
        assert [got["max_seqlen_q"], got["max_seqlen_k"]] == g[p + "max_seqlen"].tolist()


def test_pack_decode_bucket_matches_graph_staging():
    g = load_npz("decode_bucket.npz")
    for c in range(int(g["num_cases"])):
        p = f"c{c}_"
        bucket = int(g[p + "bucket"])
        lens = g[p + "lens"]
        tables = _split(g[p + "tables_flat"], g[p + "table_lens"])
        got = K.pack_decode_bucket(lens, g[p + "last_ids"], tables, bucket, 16)
        b = len(lens)
        np.testing.assert_array_equal(got["input_ids"][:b], g[p + "input_ids"][:b])
        np.testing.assert_array_equal(got["positions"][:b], g[p + "positions"][:b])
        for key in ("slot_mapping", "cu_seqlens_k", "block_tables"):
            np.testing.assert_array_equal(got[key], g[p + key], err_msg=f"case {c} {key}")


# -------------------------------------------------------------------- KV store


def test_store_matches_triton_kernel():
    g = load_npz("store.npz")
    t, hq, hkv, d, nblocks = g["dims"].tolist()
    qkv = bf16_bits_to_f32(g["qkv"])
    k = qkv[:, hq * d : (hq + hkv) * d].reshape(t, hkv, d)
    v = qkv[:, (hq + hkv) * d :].reshape(t, hkv, d)
    kc = bf16_bits_to_f32(g["k_cache_before"]).copy()
    vc = bf16_bits_to_f32(g["v_cache_before"]).copy()
    K.store_kvcache(k, v, kc, vc, g["slots"])
    np.testing.assert_array_equal(kc, bf16_bits_to_f32(g["k_cache"]))
    np.testing.assert_array_equal(vc, bf16_bits_to_f32(g["v_cache"]))


# ------------------------------------------------------------------- attention


def test_paged_decode_matches_reference_torch_path():
    g = load_npz("paged_decode.npz")
    q = bf16_bits_to_f32(g["q"])
    kc, vc = bf16_bits_to_f32(g["k_cache"]), bf16_bits_to_f32(g["v_cache"])
    lens = g["lens"]
    b = len(lens)
    cu_q = np.arange(b + 1, dtype=np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    got = K.paged_attention(q, kc, vc, cu_q, cu_k, g["tables"], q.shape[-1] ** -0.5)
    np.testing.assert_allclose(got, g["out_reference"], atol=2e-5, rtol=1e-4)


def test_pool_decode_matches_reference_test_inputs():
    """The reference test's own case (fp32, head_dim 4, page 2, left-padded mask), with
    and without the fused current-token write."""
    g = load_npz("tts_pool_decode.npz")
    args = (g["ref_q"], g["ref_k_pool"].copy(), g["ref_v_pool"].copy(), g["ref_page_table"],
            g["ref_seq_lens"], 0.5)
    got = K.pool_paged_attention(*args, key_valid_mask=g["ref_valid"])
    np.testing.assert_allclose(got, g["ref_out"], atol=1e-6, rtol=1e-5)
    kp, vp = g["ref_k_pool"].copy(), g["ref_v_pool"].copy()
    got = K.pool_paged_attention(g["ref_q"], kp, vp, g["ref_page_table"], g["ref_seq_lens"], 0.5,
                                 key_valid_mask=g["ref_valid"], new_key=g["ref_new_k"],
                                 new_value=g["ref_new_v"])
    np.testing.assert_allclose(got, g["ref_out_fused"], atol=1e-6, rtol=1e-5)
    np.testing.assert_array_equal(kp, g["ref_k_pool_after"])
    np.testing.assert_array_equal(vp, g["ref_v_pool_after"])


@pytest.mark.parametrize("case", ["talker_g2", "talker_g4"])
def test_pool_decode_matches_reference_talker_cases(case):
    g = load_npz("tts_pool_decode.npz")
    f = {k[len(case) + 1:]: v for k, v in g.items() if k.startswith(case + "_")}
    bf = {k: bf16_bits_to_f32(f[k]) for k in ("q", "k_pool", "v_pool", "new_k", "new_v")}
    got = K.pool_paged_attention(bf["q"], bf["k_pool"].copy(), bf["v_pool"].copy(),
                                 f["page_table"], f["seq_lens"], 128 ** -0.5,
                                 key_valid_mask=f["valid"], new_key=bf["new_k"],
                                 new_value=bf["new_v"])
    np.testing.assert_allclose(got, f["out"], atol=2e-5, rtol=1e-4)


def test_pool_decode_edge_semantics():
    """Fully masked rows give zeros (the reference kernel's guard); kernel_seq_len bounds
    the attended positions as the reference kernel's loop does; mask columns beyond the
    mask's width are valid."""
    rng = np.random.default_rng(3)
    kp = rng.standard_normal((4, 1, 2, 8)).astype(np.float32)
    vp = rng.standard_normal((4, 1, 2, 8)).astype(np.float32)
    q = rng.standard_normal((1, 2, 1, 8)).astype(np.float32)
    table = np.array([[2, 0, 3]])
    mask = np.zeros((1, 6), dtype=bool)
    assert not K.pool_paged_attention(q, kp, vp, table, [5], 0.3, key_valid_mask=mask).any()
    short = K.pool_paged_attention(q, kp, vp, table, [5], 0.3, kernel_seq_len=3)
    np.testing.assert_allclose(short, K.pool_paged_attention(q, kp, vp, table, [3], 0.3))
    narrow = np.array([[False, True]])
    full = np.array([[False, True, True, True, True]])
    np.testing.assert_allclose(K.pool_paged_attention(q, kp, vp, table, [5], 0.3,
                                                      key_valid_mask=narrow),
                               K.pool_paged_attention(q, kp, vp, table, [5], 0.3,
                                                      key_valid_mask=full))


def test_paged_prefill_is_bottom_right_causal():
    """A request prefilled in one pass equals the same request decoded one token at a
    time -- the property FlashAttention's bottom-right alignment provides."""
    rng = np.random.default_rng(0)
    hq, hkv, d, n = 4, 2, 16, 300
    kc = rng.standard_normal((4, 256, hkv, d)).astype(np.float32)
    vc = rng.standard_normal((4, 256, hkv, d)).astype(np.float32)
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    table = np.array([[2, 0, 3, 1]], dtype=np.int32)
    full = K.paged_attention(q, kc, vc, np.array([0, n]), np.array([0, n]), table, 0.25)
    for i in (0, 1, 255, 256, 299):
        one = K.paged_attention(q[i : i + 1], kc, vc, np.array([0, 1]), np.array([0, i + 1]),
                                table, 0.25)
        np.testing.assert_allclose(one[0], full[i], atol=1e-12)
    # a partial prefill (query tail of 40 over 300 keys) matches the tail of the full one
    tail = K.paged_attention(q[260:], kc, vc, np.array([0, 40]), np.array([0, n]), table, 0.25)
    np.testing.assert_allclose(tail, full[260:], atol=1e-12)


def test_varlen_attention_is_block_diagonal():
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((30, 3, 8)) for _ in range(3))
    cu = np.array([0, 10, 11, 30])
    got = K.varlen_attention(q, k, v, cu, 0.5)
    for a, b in zip(cu[:-1], cu[1:]):
        np.testing.assert_allclose(got[a:b], K.varlen_attention(q[a:b], k[a:b], v[a:b],
                                                                np.array([0, b - a]), 0.5))


# ------------------------------------------------------- norms, rope, elementwise


def test_qk_norm_rope_matches_reference_layers():
    g = load_npz("norm_rope.npz")
    qkv = bf16_bits_to_f32(g["qkv"])
    t = qkv.shape[0]
    qw, kw = bf16_bits_to_f32(g["q_weight"]), bf16_bits_to_f32(g["k_weight"])
    qn = K.rms_norm(qkv[:, :2048].reshape(t, 16, 128), qw)
    kn = K.rms_norm(qkv[:, 2048:3072].reshape(t, 8, 128), kw)
    np.testing.assert_array_equal(qn, bf16_bits_to_f32(g["q_normed"]))
    np.testing.assert_array_equal(kn, bf16_bits_to_f32(g["k_normed"]))
    # The table itself: torch's fp32 cos/sin are within 3e-4 of the exact values.
    own = K.rope_cache(128, 4096, 1_000_000.0)
    np.testing.assert_allclose(own[g["positions"]], g["cos_sin_cache"], atol=3e-4)
    # The rotation, given the reference's table, is bit-exact.
    cache = np.zeros((4096, 128), dtype=np.float32)
    cache[g["positions"]] = g["cos_sin_cache"]
    q, k, v = K.qk_norm_rope(qkv, g["positions"], qw, kw, cache, 16, 8, 128)
    np.testing.assert_array_equal(q, bf16_bits_to_f32(g["q_out"]))
    np.testing.assert_array_equal(k, bf16_bits_to_f32(g["k_out"]))
    np.testing.assert_array_equal(v, qkv[:, 3072:].reshape(-1, 8, 128))


def test_rms_and_add_rms_match_reference():
    g = load_npz("elementwise.npz")
    x, r, w = (bf16_bits_to_f32(g[k]) for k in ("x", "residual", "weight"))
    np.testing.assert_array_equal(K.rms_norm(x, w), bf16_bits_to_f32(g["rms"]))
    y, res = K.add_rms_norm(x, r, w)
    np.testing.assert_array_equal(res, bf16_bits_to_f32(g["add_residual"]))
    np.testing.assert_array_equal(y, bf16_bits_to_f32(g["add_rms"]))


def test_silu_mul_matches_reference():
    g = load_npz("elementwise.npz")
    got = K.silu_mul(bf16_bits_to_f32(g["gate_up"]))
    ref = bf16_bits_to_f32(g["silu_mul"])
    assert np.mean(got != ref) < 0.01
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-6)


def test_greedy_argmax_matches_sampler():
    g = load_npz("sampler.npz")
    np.testing.assert_array_equal(K.greedy_argmax(bf16_bits_to_f32(g["logits"])), g["ids"])


def test_bf16_round_matches_torch():
    x = np.random.default_rng(3).standard_normal(10000).astype(np.float32) * 100
    ref = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(K.bf16_round(x), ref)


# ------------------------------------------------------------------ model oracle


def test_model_oracle_matches_hf_thinker():
    import sys
    sys.path.insert(0, str(__import__("pathlib").Path(__file__).parent / "golden"))
    from make_golden import tiny_thinker_config

    g = load_npz("model_tiny.npz")
    cfg = tiny_thinker_config()
    thinker = M.OracleThinker(cfg, M.init_weights(cfg, seed=int(g["seed"])))
    mel = torch.from_numpy(g["mel"])
    audio = thinker.encode_audio(mel)
    np.testing.assert_allclose(audio.numpy(), g["audio_features"], atol=2e-5, rtol=1e-4)
    tokens, _ = thinker.greedy(g["prompt"].tolist(), audio, steps=len(g["greedy"]))
    assert tokens == g["greedy"].tolist()


def test_log_mel_oracle_matches_reference_frontend():
    """oracle.log_mel (float64) vs the reference AudioFrontend (fp32 torch STFT)."""
    z = load_npz("frontend.npz")
    off = np.concatenate([[0], np.cumsum(z["lens"])])
    col = np.concatenate([[0], np.cumsum(z["frames"])])
    for i in range(len(z["lens"])):
        want = z["mel"][:, col[i]:col[i + 1]]
        got = K.log_mel(z["wave"][off[i]:off[i + 1]], z["mel_filters"])
        assert got.shape == want.shape == (128, z["lens"][i] // 160)
        assert np.abs(got - want).max() <= 5e-5


def test_log_mel_oracle_rejects_clips_too_short_to_reflect():
    with pytest.raises(ValueError):
        K.log_mel(np.zeros(200, np.float32), np.zeros((201, 128)))
