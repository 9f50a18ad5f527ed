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
"""

from __future__ import annotations

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
