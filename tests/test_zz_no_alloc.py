"""The allocation-free decode entry point against the workspace one.

``b200asr_paged_decode_noalloc`` serves callers that cannot give the library device
scratch: hosts reaching it through a foreign-function interface with no CUDA
allocator of their own, servers whose memory pool is entirely reserved for the KV
cache at start-up, and code that runs while a CUDA graph is being captured (where
cudaMalloc is illegal). Its split-K partials live in a static device array inside
the library instead. These tests call it through the C ABI, twice in a row with
different inputs (the array keeps the previous call's contents, which must not
leak into the next result), and compare with ``b200asr_paged_decode`` under the
attention tolerance used throughout the suite. They pass alone in a fresh process
and after the rest of the suite: nothing depends on earlier tests' state.

Every call clears the array's merge counters on the caller's stream before its kernel,
so the very first call in a process may come from a non-blocking side stream (checked
in a child process, against the float64 oracle as well as the workspace entry point),
and the largest batch the array accepts is checked against the workspace entry point.
"""

from __future__ import annotations

import json
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def _case(seed: int, batch: int, nblocks: int = 96):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 1100, size=batch)
    lens[0] = 1024  # a sequence long enough to need several partials
    gen = torch.Generator(device="cuda").manual_seed(seed)
    kc = (torch.randn(nblocks, 256, 8, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    vc = (torch.randn(nblocks, 256, 8, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    q = (torch.randn(batch, 16, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    perm = rng.permutation(nblocks)
    tables = np.zeros((batch, 5), np.int32)
    c = 0
    for i, n in enumerate(lens):
        k = (int(n) + 255) // 256
        tables[i, :k] = perm[c:c + k]
        c += k
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return q, kc, vc, torch.from_numpy(cu).cuda(), torch.from_numpy(tables).cuda()


def _noalloc(lib, q, kc, vc, cu, bt, max_len, out, err=None, num_heads=16):
    return lib.b200asr_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], 256, num_heads, 8, 128,
        cu.data_ptr(), bt.data_ptr(), bt.stride(0), q.shape[0], max_len, 128 ** -0.5,
        out.data_ptr(), out.stride(0), None if err is None else err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_twice():
    from voiceagent_b200 import kernels as kx
    from voiceagent_b200._lib import lib

    for seed, batch in ((1, 32), (2, 7)):
        q, kc, vc, cu, bt = _case(seed, batch)
        ref = torch.empty_like(q)
        ws = torch.zeros(kx.paged_decode_workspace_size(batch, 1280, 16) // 4 + 64,
                         dtype=torch.float32, device="cuda")
        kx.paged_decode(q, kc, vc, cu, bt, max_seqlen_k=1280, scale=128 ** -0.5, out=ref,
                        workspace=ws)
        got = torch.full_like(q, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert _noalloc(lib, q, kc, vc, cu, bt, 1280, got, err) == 0, \
            lib.b200asr_last_error().decode()
        torch.cuda.synchronize()
        assert err.item() == 0
        diff = (got.float() - ref.float()).abs()
        assert torch.isfinite(got.float()).all()
        assert diff.max().item() <= ATOL_MAX and diff.mean().item() <= ATOL_MEAN


def test_noalloc_rejects_requests_beyond_its_scratch():
    from voiceagent_b200._lib import lib

    q, kc, vc, cu, bt = _case(3, 4)
    out = torch.zeros_like(q)
    rc = _noalloc(lib, q, kc, vc, cu, bt, 1024, out, num_heads=128)  # partials beyond 12 MiB
    assert rc == 4
    assert "scratch" in lib.b200asr_last_error().decode()
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0  # nothing launched


def test_noalloc_largest_accepted_batch():
    """1024 sequences x 16 heads: the largest request the static array takes."""
    from voiceagent_b200 import kernels as kx
    from voiceagent_b200._lib import lib

    batch, nblocks = 1024, 64
    need = kx.paged_decode_workspace_size(batch, 1280, 16)
    assert need <= 12 << 20  # B200ASR_NOALLOC_SCRATCH_BYTES
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 700, size=batch)
    lens[::97] = 1024  # some sequences long enough to be split over several CTAs
    gen = torch.Generator(device="cuda").manual_seed(11)
    kc = (torch.randn(nblocks, 256, 8, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    vc = (torch.randn(nblocks, 256, 8, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    q = (torch.randn(batch, 16, 128, device="cuda", generator=gen) / 128 ** 0.5).bfloat16()
    tables = torch.from_numpy(rng.integers(0, nblocks, size=(batch, 5)).astype(np.int32)).cuda()
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    ref = torch.empty_like(q)
    ws = torch.zeros(need // 4 + 64, dtype=torch.float32, device="cuda")
    kx.paged_decode(q, kc, vc, cu, tables, max_seqlen_k=1280, scale=128 ** -0.5, out=ref,
                    workspace=ws)
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert _noalloc(lib, q, kc, vc, cu, tables, 1280, got, err) == 0, \
            lib.b200asr_last_error().decode()
        torch.cuda.synchronize()
        assert err.item() == 0
        diff = (got.float() - ref.float()).abs()
        assert torch.isfinite(got.float()).all()
        assert diff.max().item() <= ATOL_MAX and diff.mean().item() <= ATOL_MEAN


_FIRST_CALL_ON_SIDE_STREAM = textwrap.dedent("""
    import json, sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    from oracle import kernels as K
    from voiceagent_b200 import kernels as kx
    from voiceagent_b200._lib import lib

    rng = np.random.default_rng(5)
    batch, nblocks = 8, 24
    report = []
    side = torch.cuda.Stream()  # non-blocking with respect to the legacy default stream
    for call in range(2):
        lens = rng.integers(1, 1100, size=batch)
        lens[call] = 1024
        kc = K.bf16_round(rng.standard_normal((nblocks, 256, 8, 128)).astype(np.float32) / 11.3)
        vc = K.bf16_round(rng.standard_normal((nblocks, 256, 8, 128)).astype(np.float32) / 11.3)
        q = K.bf16_round(rng.standard_normal((batch, 16, 128)).astype(np.float32) / 11.3)
        tables = rng.integers(0, nblocks, size=(batch, 5)).astype(np.int32)
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        dev = lambda x, dt: torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dt)
        with torch.cuda.stream(side):
            gq, gk, gv = dev(q, torch.bfloat16), dev(kc, torch.bfloat16), dev(vc, torch.bfloat16)
            gcu, gbt = dev(cu, torch.int32), dev(tables, torch.int32)
            got = torch.full_like(gq, float("nan"))
            err = torch.zeros(1, dtype=torch.int32, device="cuda")
            rc = lib.b200asr_paged_decode_noalloc(
                gq.data_ptr(), gq.stride(0), gk.data_ptr(), gv.data_ptr(), nblocks, 256, 16, 8,
                128, gcu.data_ptr(), gbt.data_ptr(), gbt.stride(0), batch, 1280, 128 ** -0.5,
                got.data_ptr(), got.stride(0), err.data_ptr(), side.cuda_stream)
            ref = torch.empty_like(gq)
            ws = torch.zeros(kx.paged_decode_workspace_size(batch, 1280, 16) // 4 + 64,
                             dtype=torch.float32, device="cuda")
            kx.paged_decode(gq, gk, gv, gcu, gbt, max_seqlen_k=1280, scale=128 ** -0.5,
                            out=ref, workspace=ws)
        side.synchronize()
        oracle = K.paged_attention(q, kc, vc, np.arange(batch + 1), cu, tables, 128 ** -0.5)
        g = got.float().cpu().numpy()
        report.append({"rc": rc, "err": int(err.item()), "finite": bool(np.isfinite(g).all()),
                       "vs_oracle_max": float(np.abs(g - oracle).max()),
                       "vs_oracle_mean": float(np.abs(g - oracle).mean()),
                       "vs_workspace_max": float((got.float() - ref.float()).abs().max())})
    print(json.dumps(report))
""")


def test_noalloc_first_call_from_a_non_blocking_stream():
    """A fresh process whose first no-alloc call runs on a non-blocking side stream:
    the counter clear is ordered with the kernel on that stream, so both calls match
    the oracle and the workspace entry point."""
    repo = Path(__file__).resolve().parents[1]
    proc = subprocess.run([sys.executable, "-c", _FIRST_CALL_ON_SIDE_STREAM, str(repo)],
                          capture_output=True, text=True, timeout=600, cwd=repo)
    assert proc.returncode == 0, proc.stderr[-2000:]
    report = json.loads(proc.stdout.strip().splitlines()[-1])
    assert len(report) == 2
    for r in report:
        assert r["rc"] == 0 and r["err"] == 0 and r["finite"], r
        assert r["vs_oracle_max"] <= ATOL_MAX and r["vs_oracle_mean"] <= ATOL_MEAN, r
        assert r["vs_workspace_max"] <= ATOL_MAX, r
