"""TTS talker paged decode over a page pool (agent/qwen_tts_paged_attention.py).

CPU tests: the drop-in module's validation (the reference's messages and exception
class) and the C-ABI's host checks. GPU tests: the kernel against the reference's own
outputs (tests/golden/tts_pool_decode.npz, written by its torch path) and against the
oracle (``oracle.kernels.pool_paged_attention``) on seeded sweeps of dtype, group size,
head_dim, page size, masks, lengths and strides; the fused current-token write is
bit-exact. Tolerances: fp32 inputs 2e-3 abs/rel (the reference's own GPU test); bf16 /
fp16 outputs max |err| <= 2e-2 and mean <= 2e-3 (the attention bar of this path).
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kernels as K
from tests.conftest import bf16_bits_to_f32, load_npz

REPO = Path(__file__).resolve().parents[1]


def _ref_inputs():
    """The reference test's _inputs() (tests/test_qwen_tts_paged_attention_kernel.py:16-35),
    from the golden fixture."""
    g = load_npz("tts_pool_decode.npz")
    return (torch.from_numpy(g["ref_q"]), torch.from_numpy(g["ref_k_pool"]),
            torch.from_numpy(g["ref_v_pool"]), torch.from_numpy(g["ref_page_table"]),
            torch.from_numpy(g["ref_seq_lens"]), torch.from_numpy(g["ref_valid"])), g


# --------------------------------------------------------------------------- CPU


def test_rejects_invalid_page_table():
    from voiceagent_b200.agent.qwen_tts_paged_attention import (
        PagedAttentionKernelError, paged_attention_decode)

    (q, kp, vp, table, lens, valid), _ = _ref_inputs()
    table = table.clone()
    table[0, 0] = 99
    with pytest.raises(PagedAttentionKernelError, match="page table"):
        paged_attention_decode(q, kp, vp, table, lens, valid)


@pytest.mark.parametrize("mutate,match", [
    (lambda a: a.update(q=a["q"][:, :, 0]), "query must have shape"),
    (lambda a: a.update(vp=a["vp"][:4]), "KV pool must have shape"),
    (lambda a: a.update(lens=a["lens"].int()), "seq_lens must be a torch.long"),
    (lambda a: a.update(table=a["table"].int()), "page_table must be a torch.long"),
    (lambda a: a.update(lens=torch.tensor([3, 0])), "sequence lengths must be positive"),
    (lambda a: a.update(lens=torch.tensor([3, 7])), "exceeds page table capacity"),
    (lambda a: a.update(valid=a["valid"][:, :4]), "shorter than sequence length"),
    (lambda a: a.update(valid=a["valid"].int()), "key_valid_mask must be"),
    (lambda a: a.update(q=torch.ones(2, 3, 1, 4)), "divisible by KV heads"),
    (lambda a: a.update(q=a["q"].double()), "share a dtype"),
])
def test_validation_matches_reference_messages(mutate, match):
    from voiceagent_b200.agent.qwen_tts_paged_attention import (
        PagedAttentionKernelError, paged_attention_decode)

    (q, kp, vp, table, lens, valid), _ = _ref_inputs()
    a = dict(q=q, kp=kp, vp=vp, table=table, lens=lens, valid=valid)
    mutate(a)
    with pytest.raises(PagedAttentionKernelError, match=match):
        paged_attention_decode(a["q"], a["kp"], a["vp"], a["table"], a["lens"], a["valid"])


def test_new_kv_contract_and_no_cpu_path():
    from voiceagent_b200.agent.qwen_tts_paged_attention import (
        PagedAttentionKernelError, paged_attention_decode)

    (q, kp, vp, table, lens, valid), _ = _ref_inputs()
    with pytest.raises(PagedAttentionKernelError, match="provided together"):
        paged_attention_decode(q, kp, vp, table, lens, valid, new_key=torch.zeros(2, 2, 1, 4))
    with pytest.raises(PagedAttentionKernelError, match="new KV must have shape"):
        paged_attention_decode(q, kp, vp, table, lens, valid, new_key=torch.zeros(2, 1, 1, 4),
                               new_value=torch.zeros(2, 1, 1, 4))
    # the product path never falls back to a CPU computation
    with pytest.raises(PagedAttentionKernelError, match="CUDA kernel"):
        paged_attention_decode(q, kp, vp, table, lens, valid)
    with pytest.raises(PagedAttentionKernelError, match="CUDA kernel"):
        paged_attention_decode(q, kp, vp, table, lens, valid, use_triton=False)


def test_oracle_is_independent_of_page_placement():
    """Moving a row's pages to other physical slots (table updated to match) leaves the
    attention unchanged: only the logical order of positions matters."""
    rng = np.random.default_rng(11)
    c = _random_case(rng, batch=3, hq=8, hkv=4, d=16, ps=4, lens=[3, 9, 14], dtype=torch.float32,
                     mask=True)
    want = K.pool_paged_attention(c["q"], c["kp"].copy(), c["vp"].copy(), c["table"], c["lens"],
                                  0.25, key_valid_mask=c["valid"])
    perm = rng.permutation(c["kp"].shape[0])
    inv = np.argsort(perm)
    kp2, vp2 = c["kp"][perm], c["vp"][perm]  # physical page p moves to slot inv[p]
    table2 = np.where(c["table"] >= 0, inv[np.maximum(c["table"], 0)], -1)
    got = K.pool_paged_attention(c["q"], kp2, vp2, table2, c["lens"], 0.25,
                                 key_valid_mask=c["valid"])
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_oracle_fused_write_equals_prewritten_pool():
    """Attending with new_key/new_value equals attending over a pool that already holds
    the current token's row (the reference's fused-write contract)."""
    rng = np.random.default_rng(12)
    c = _random_case(rng, batch=2, hq=4, hkv=2, d=8, ps=4, lens=[6, 13], dtype=torch.float32)
    kw, vw = c["kp"].copy(), c["vp"].copy()
    fused = K.pool_paged_attention(c["q"], kw, vw, c["table"], c["lens"], 0.3, new_key=c["nk"],
                                   new_value=c["nv"])
    kp, vp = c["kp"].copy(), c["vp"].copy()
    K.write_current_kv(kp, vp, c["table"], c["lens"], c["nk"], c["nv"])
    np.testing.assert_array_equal(kp, kw)
    np.testing.assert_array_equal(vp, vw)
    np.testing.assert_allclose(fused, K.pool_paged_attention(c["q"], kp, vp, c["table"],
                                                             c["lens"], 0.3), rtol=0, atol=0)


def _capi_call(lib, **over):
    dummy = ctypes.c_void_p(256)
    args = dict(dtype=0, batch=2, num_heads=16, num_kv_heads=8, head_dim=128, query=dummy,
                q_sb=2048, q_sh=128, kp=dummy, vp=dummy, num_pages=8, page_size=16,
                sp=16384, sh=2048, ss=128, table=dummy, table_stride=4, table_width=4,
                lens=dummy, mask=None, vstride=0, vlen=0, nk=None, nv=None, nsb=0, nsh=0,
                out=dummy, osb=2048, osh=128, max_seq_len=64, tpc=0, scale=1.0, ws=dummy,
                ws_bytes=1 << 30, err=None, stream=None)
    args.update(over)
    return lib.b200asr_pool_paged_decode(*args.values())


def test_capi_host_checks_without_gpu():
    from voiceagent_b200._lib import lib

    def err():
        return lib.b200asr_last_error().decode()

    assert _capi_call(lib, batch=0) == 0  # empty batch: nothing to launch
    assert _capi_call(lib, dtype=7) == 1 and "dtype" in err()
    assert _capi_call(lib, num_heads=24) == 3 and "group size" in err()
    assert _capi_call(lib, num_heads=15) == 1 and "divisible" in err()
    assert _capi_call(lib, dtype=1, head_dim=4) == 3 and "16 bytes" in err()
    assert _capi_call(lib, nk=ctypes.c_void_p(256)) == 1 and "together" in err()
    assert _capi_call(lib, q_sh=100) == 1 and "strides" in err()
    assert _capi_call(lib, query=ctypes.c_void_p(264)) == 1 and "aligned" in err()
    assert _capi_call(lib, tpc=32) == 1 and "tokens_per_cta" in err()
    need = lib.b200asr_pool_paged_decode_workspace_size(2, 16, 128, 64)
    assert _capi_call(lib, ws_bytes=need - 1) == 4 and "workspace" in err()


# --------------------------------------------------------------------------- GPU


def _dev(t):
    return t.cuda() if torch.is_tensor(t) else torch.from_numpy(np.ascontiguousarray(t)).cuda()


@pytest.mark.gpu
def test_reference_test_inputs_on_gpu():
    """test_paged_decode_triton_matches_reference_on_cuda and ..._fused_write_... of the
    reference, against the outputs its torch path produced."""
    from voiceagent_b200.agent.qwen_tts_paged_attention import paged_attention_decode

    (q, kp, vp, table, lens, valid), g = _ref_inputs()
    q, kp, vp, table, lens, valid = map(_dev, (q, kp, vp, table, lens, valid))
    out = paged_attention_decode(q, kp, vp, table, lens, valid)
    assert torch.allclose(out.cpu(), torch.from_numpy(g["ref_out"]), atol=2e-3, rtol=2e-3)

    kw, vw = kp.clone(), vp.clone()
    out = paged_attention_decode(q, kw, vw, table, lens, valid, new_key=_dev(g["ref_new_k"]),
                                 new_value=_dev(g["ref_new_v"]))
    torch.cuda.synchronize()
    assert torch.equal(kw.cpu(), torch.from_numpy(g["ref_k_pool_after"]))
    assert torch.equal(vw.cpu(), torch.from_numpy(g["ref_v_pool_after"]))
    assert torch.allclose(out.cpu(), torch.from_numpy(g["ref_out_fused"]), atol=2e-3, rtol=2e-3)


def _bf16_tensor(bits):
    return torch.from_numpy(bf16_bits_to_f32(bits)).bfloat16()


def _assert_close(got, want, what):
    err = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, f"{what}: max {err.max():.3e} mean {err.mean():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["talker_g2", "talker_g4"])
def test_talker_golden_cases(case):
    from voiceagent_b200.agent.qwen_tts_paged_attention import paged_attention_decode

    g = load_npz("tts_pool_decode.npz")
    f = {k[len(case) + 1:]: v for k, v in g.items() if k.startswith(case + "_")}
    t = {k: _dev(_bf16_tensor(f[k])) for k in ("q", "k_pool", "v_pool", "new_k", "new_v")}
    kp0 = t["k_pool"].clone()
    out = paged_attention_decode(t["q"], t["k_pool"], t["v_pool"], _dev(f["page_table"]),
                                 _dev(f["seq_lens"]), _dev(f["valid"]), new_key=t["new_k"],
                                 new_value=t["new_v"])
    _assert_close(out.float().cpu().numpy(), f["out"], case)
    # the write: exactly the new rows, nothing else
    kw = kp0.float().cpu().numpy()
    vw = _bf16_tensor(f["v_pool"]).float().numpy()
    K.write_current_kv(kw, vw, f["page_table"], f["seq_lens"],
                       bf16_bits_to_f32(f["new_k"]), bf16_bits_to_f32(f["new_v"]))
    np.testing.assert_array_equal(t["k_pool"].float().cpu().numpy(), kw)
    np.testing.assert_array_equal(t["v_pool"].float().cpu().numpy(), vw)


def _random_case(rng, *, batch, hq, hkv, d, ps, lens, dtype, mask=False, spare_pages=3):
    need = [(n + ps - 1) // ps for n in lens]
    pages = sum(need) + spare_pages
    kp = rng.standard_normal((pages, hkv, ps, d)).astype(np.float32) / np.sqrt(d)
    vp = rng.standard_normal((pages, hkv, ps, d)).astype(np.float32)
    q = rng.standard_normal((batch, hq, 1, d)).astype(np.float32)
    nk = rng.standard_normal((batch, hkv, 1, d)).astype(np.float32) / np.sqrt(d)
    nv = rng.standard_normal((batch, hkv, 1, d)).astype(np.float32)
    # values exactly representable in the kernel's element type (float32 arrays)
    kp, vp, q, nk, nv = (x.astype(np.float32) for x in (kp, vp, q, nk, nv))
    if dtype != torch.float32:
        rnd = (lambda x: K.bf16_round(x)) if dtype == torch.bfloat16 else (
            lambda x: x.astype(np.float16).astype(np.float32))
        kp, vp, q, nk, nv = map(rnd, (kp, vp, q, nk, nv))
    perm = rng.permutation(pages)
    width = max(need) + 1
    table = np.full((batch, width), -1, np.int64)
    cur = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[cur:cur + n]
        cur += n
    valid = None
    if mask:
        valid = rng.random((batch, max(lens))) > 0.2
        valid[:, :3] = False  # left padding
    return dict(q=q, kp=kp, vp=vp, nk=nk, nv=nv, table=table,
                lens=np.asarray(lens, np.int64), valid=valid)


SWEEP = [
    # dtype, hq, hkv, d, page, lens, mask, tokens_per_cta
    (torch.bfloat16, 16, 8, 128, 16, [1, 16, 17, 300, 1000, 3001], True, 0),
    (torch.bfloat16, 16, 8, 128, 16, [5, 700, 2049], False, 64),
    (torch.bfloat16, 16, 16, 64, 256, [1, 255, 256, 257, 1500], True, 0),
    (torch.bfloat16, 16, 4, 128, 24, [3, 48, 49, 999], True, 0),
    (torch.bfloat16, 32, 4, 128, 16, [2, 100, 1777], False, 0),
    (torch.bfloat16, 8, 4, 256, 16, [9, 333, 1024], True, 0),
    (torch.float16, 16, 8, 128, 16, [1, 31, 32, 33, 900], True, 0),
    (torch.float16, 8, 1, 128, 32, [70, 1200], False, 0),
    (torch.float32, 16, 8, 128, 16, [4, 400, 1300], True, 0),
    (torch.float32, 4, 2, 256, 8, [1, 64, 513], False, 0),
    (torch.float32, 4, 2, 4, 2, [1, 2, 3, 150], True, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hq,hkv,d,ps,lens,mask,tpc", SWEEP)
def test_sweep_against_oracle(dtype, hq, hkv, d, ps, lens, mask, tpc):
    from voiceagent_b200 import kernels as kx

    rng = np.random.default_rng(hash((hq, hkv, d, ps, len(lens))) % 2**32)
    c = _random_case(rng, batch=len(lens), hq=hq, hkv=hkv, d=d, ps=ps, lens=lens, dtype=dtype,
                     mask=mask)
    t = {k: torch.from_numpy(c[k]).to(dtype).cuda() for k in ("q", "kp", "vp", "nk", "nv")}
    # a strided query/out, as the talker's transpose(1, 2) hands them over
    qs = t["q"].transpose(1, 2).contiguous().transpose(1, 2)
    out = torch.empty_like(qs)
    max_len = max(lens)
    kx.pool_paged_decode(qs, t["kp"], t["vp"], _dev(c["table"]), _dev(c["lens"]),
                         max_seq_len=max_len, scale=d ** -0.5, out=out,
                         key_valid_mask=None if c["valid"] is None else _dev(c["valid"]),
                         new_key=t["nk"], new_value=t["nv"], tokens_per_cta=tpc)
    kw, vw = c["kp"].copy(), c["vp"].copy()
    want = K.pool_paged_attention(c["q"], kw, vw, c["table"], c["lens"], d ** -0.5,
                                  key_valid_mask=c["valid"], new_key=c["nk"], new_value=c["nv"])
    got = out.float().cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, atol=2e-3, rtol=2e-3)
    else:
        _assert_close(got, want, f"{dtype} hq{hq} hkv{hkv} d{d} ps{ps}")
    np.testing.assert_array_equal(t["kp"].float().cpu().numpy(), kw)
    np.testing.assert_array_equal(t["vp"].float().cpu().numpy(), vw)


@pytest.mark.gpu
def test_strided_lengths_and_table_views():
    """Lengths and page tables handed over as strided views (as sliced metadata would be)."""
    from voiceagent_b200 import kernels as kx

    rng = np.random.default_rng(7)
    c = _random_case(rng, batch=3, hq=16, hkv=8, d=128, ps=16, lens=[5, 300, 77],
                     dtype=torch.bfloat16)
    t = {k: torch.from_numpy(c[k]).bfloat16().cuda() for k in ("q", "kp", "vp")}
    lens2 = torch.from_numpy(np.stack([c["lens"], c["lens"] * 0 + 9], 1)).cuda()[:, 0]
    wide = np.full((3, c["table"].shape[1] * 2), -1, np.int64)
    wide[:, ::2] = c["table"]
    table2 = torch.from_numpy(wide).cuda()[:, ::2]
    assert lens2.stride(0) != 1 and table2.stride(-1) != 1
    out = kx.pool_paged_decode(t["q"], t["kp"], t["vp"], table2, lens2, max_seq_len=300,
                               scale=0.1)
    want = K.pool_paged_attention(c["q"], c["kp"], c["vp"], c["table"], c["lens"], 0.1)
    _assert_close(out.float().cpu().numpy(), want, "strided views")


@pytest.mark.gpu
def test_truncation_flags_and_bad_pages():
    """kernel_seq_len below a length attends the first kernel_seq_len positions (the
    reference kernel's loop bound) and raises LENGTH; a page outside the pool is skipped
    with BLOCK raised."""
    from voiceagent_b200 import kernels as kx

    rng = np.random.default_rng(5)
    c = _random_case(rng, batch=3, hq=16, hkv=8, d=128, ps=16, lens=[40, 200, 90],
                     dtype=torch.bfloat16)
    t = {k: torch.from_numpy(c[k]).bfloat16().cuda() for k in ("q", "kp", "vp")}
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = kx.pool_paged_decode(t["q"], t["kp"], t["vp"], _dev(c["table"]), _dev(c["lens"]),
                               max_seq_len=128, scale=0.1, error_flag=flag)
    want = K.pool_paged_attention(c["q"], c["kp"], c["vp"], c["table"], c["lens"], 0.1,
                                  kernel_seq_len=128)
    _assert_close(out.float().cpu().numpy(), want, "truncated")
    assert int(flag.item()) & 8  # B200ASR_DEVERR_LENGTH

    table = c["table"].copy()
    table[2, 1] = 10_000  # outside the pool
    flag.zero_()
    out = kx.pool_paged_decode(t["q"], t["kp"], t["vp"], _dev(table), _dev(c["lens"]),
                               max_seq_len=200, scale=0.1, error_flag=flag)
    assert int(flag.item()) == 2  # B200ASR_DEVERR_BLOCK only
    valid = np.ones((3, 200), bool)
    valid[2, 16:32] = False  # the skipped page
    want = K.pool_paged_attention(c["q"], c["kp"], c["vp"], c["table"], c["lens"], 0.1,
                                  key_valid_mask=valid)
    _assert_close(out.float().cpu().numpy(), want, "bad page skipped")


@pytest.mark.gpu
def test_fully_masked_row_is_zero_and_graph_replay_is_stable():
    from voiceagent_b200 import kernels as kx

    rng = np.random.default_rng(6)
    c = _random_case(rng, batch=4, hq=16, hkv=8, d=128, ps=16, lens=[3, 500, 1900, 64],
                     dtype=torch.bfloat16)
    t = {k: torch.from_numpy(c[k]).bfloat16().cuda() for k in ("q", "kp", "vp")}
    valid = np.ones((4, 1900), bool)
    valid[0, :3] = False
    table, lens, vm = _dev(c["table"]), _dev(c["lens"]), _dev(valid)
    out = torch.empty_like(t["q"])
    ws = kx.pool_decode_workspace(4, 16, 128, 1900, "cuda")

    def run():
        kx.pool_paged_decode(t["q"], t["kp"], t["vp"], table, lens, max_seq_len=1900, scale=0.1,
                             out=out, key_valid_mask=vm, workspace=ws, tokens_per_cta=64)

    run()
    first = out.clone()
    assert not first[0].float().abs().any()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)  # merge counters are reset by every launch
    want = K.pool_paged_attention(c["q"], c["kp"], c["vp"], c["table"], c["lens"], 0.1,
                                  key_valid_mask=valid)
    _assert_close(first.float().cpu().numpy(), want, "masked + long rows")


def _reference_triton():
    """The reference's own Triton kernel from its installed copy, when present."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "qwen_asr_vllm").is_dir():
        return None
    sys.path.insert(0, str(ref))
    try:
        from qwen_asr_vllm.agent import qwen_tts_paged_attention as m
    except Exception:  # noqa: BLE001 - optional cross-check
        return None
    finally:
        sys.path.remove(str(ref))
    return m if m.HAS_TRITON else None


@pytest.mark.gpu
def test_matches_reference_triton_kernel_live():
    """Both kernels on the same talker-shaped inputs, the fused write included."""
    m = _reference_triton()
    if m is None:
        pytest.skip("reference install (baseline/_ref) with Triton not available")
    from voiceagent_b200.agent.qwen_tts_paged_attention import paged_attention_decode

    rng = np.random.default_rng(8)
    c = _random_case(rng, batch=6, hq=16, hkv=8, d=128, ps=16, lens=[1, 17, 64, 333, 800, 1200],
                     dtype=torch.bfloat16, mask=True)
    t = {k: torch.from_numpy(c[k]).bfloat16().cuda() for k in ("q", "kp", "vp", "nk", "nv")}
    table = _dev(c["table"])
    lens = _dev(c["lens"])
    valid = _dev(c["valid"])
    k1, v1, k2, v2 = t["kp"].clone(), t["vp"].clone(), t["kp"].clone(), t["vp"].clone()
    mine = paged_attention_decode(t["q"], k1, v1, table, lens, valid, new_key=t["nk"],
                                  new_value=t["nv"])
    theirs = m.paged_attention_decode(t["q"], k2, v2, table, lens, valid,
                                      new_key=t["nk"], new_value=t["nv"])
    torch.cuda.synchronize()
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    _assert_close(mine.float().cpu().numpy(), theirs.float().cpu().numpy(), "vs reference Triton")


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv", [(16, 8), (8, 8), (16, 4), (4, 2)])
def test_stream_k_path_matches_chunked_kernel(hq, hkv):
    """The talker's case (bf16, head_dim 128, 16-position pages, heads contiguous) runs on
    the stream-K decode kernel; tokens_per_cta != 0 keeps the chunked CUDA-core kernel.
    Both against the oracle and each other on the awkward rows: one fully masked, one whose
    current token lies past max_seq_len (stored, not attended), one page outside the pool,
    long rows split over several CTAs -- with the same pool writes and error bits."""
    from voiceagent_b200 import kernels as kx

    rng = np.random.default_rng(hq * 31 + hkv)
    lens = [3, 500, 1900, 64, 16, 1301]
    c = _random_case(rng, batch=len(lens), hq=hq, hkv=hkv, d=128, ps=16, lens=lens,
                     dtype=torch.bfloat16)
    max_len = 1500  # row 2 (1900) is cut off: its current token is stored, not attended
    valid = rng.random((len(lens), 1400)) > 0.1
    valid[0, :] = False  # row 0: nothing attended -> zeros
    table = c["table"].copy()
    table[5, 3] = 10**6  # a page outside the pool: skipped, BLOCK raised
    outs, pools, flags = [], [], []
    for tpc in (0, 64):
        t = {k: torch.from_numpy(c[k]).bfloat16().cuda() for k in ("q", "kp", "vp", "nk", "nv")}
        qs = t["q"].transpose(1, 2).contiguous().transpose(1, 2)
        out = torch.empty_like(qs)
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        kx.pool_paged_decode(qs, t["kp"], t["vp"], _dev(table), _dev(c["lens"]),
                             max_seq_len=max_len, scale=128 ** -0.5, out=out,
                             key_valid_mask=_dev(valid), new_key=t["nk"], new_value=t["nv"],
                             tokens_per_cta=tpc, error_flag=flag)
        outs.append(out.float().cpu().numpy())
        pools.append((t["kp"].float().cpu().numpy(), t["vp"].float().cpu().numpy()))
        flags.append(int(flag.item()))
    kw, vw = c["kp"].copy(), c["vp"].copy()
    attend = np.ones((len(lens), max(lens)), bool)
    attend[:, :1400] = valid
    p_bad = 3 * 16
    attend[5, p_bad:p_bad + 16] = False
    want = K.pool_paged_attention(c["q"], kw, vw, table, c["lens"], 128 ** -0.5,
                                  key_valid_mask=attend, new_key=c["nk"], new_value=c["nv"],
                                  kernel_seq_len=max_len)
    for got, what in zip(outs, ("stream-K", "chunked")):
        assert not np.abs(got[0]).any(), what
        _assert_close(got, want, what)
    np.testing.assert_array_equal(pools[0][0], pools[1][0])
    np.testing.assert_array_equal(pools[0][1], pools[1][1])
    assert flags[0] == flags[1] == (2 | 8)  # BLOCK (the bad page) | LENGTH (row 2)
