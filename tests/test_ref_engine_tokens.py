"""Greedy tokens of this engine against the reference engine's own, on identical inputs.

The fixture ``tests/golden/ref_engine_tokens.npz`` holds what ``qwen_asr_vllm.AsrEngine``
(the reference, installed unmodified; flash-attn varlen attention, its Triton KV store
and CUDA-graph decode) produced on a B200 for the seeded random-init 0.6B checkpoint:
the config-0 clip with 48 greedy tokens and the first 24 config-3 clips with 64,
language "en", EOS ignored, plus the two largest logits at every position
(``tests/golden/make_ref_engine_tokens.py`` made it; it mirrors the reference's gates in
tests/test_end_to_end_parity.py:86 and tests/test_cuda_graph.py:98-104, driven through
engine/engine.py:539-627 transcribe).

The random-init model's logits sit around 2.7, where one bf16 step is 1/64, and are
full of near-ties (exact bf16 ties at 0.5 % of positions, gaps of at most one step at
~3 %), so any two correct bf16 implementations pick different tokens at some of them.
Two measurements of the reference against itself bound what that costs:

* its eager decode against its graph decode (``ref_engine_tokens.npz``): the same
  kernels run twice -- repeatability of one implementation (99.87 % teacher forced);
* its own upstream model (reference/modeling_qwen3_asr.py, bf16) teacher forced on the
  engine's tokens (``ref_engine_hf.npz``, made by ``tests/golden/make_golden.py --only
  ref_engine_hf``): the reference's two implementations of the model compared
  (98.30 %), every difference at a top-2 gap of at most three bf16 steps.

This engine is a third implementation, so it is held to the second: strict token
equality, never looser than that cross-implementation agreement and never above the
north star's 99 %:

* teacher forced: this engine, fed the reference's tokens through ``AsrEngine.transcribe``
  (one CUDA-graph decode step per call), samples the reference's token at >= that many
  positions, and every position where it does not lies at a reference top-2 gap of at
  most three bf16 steps (the largest among the reference's own disagreements);
* free running: each clip's tokens equal the reference's up to its first difference, and
  that first difference lies at such a near-tie (after a near-tie flips, the two
  continuations are different texts and positional equality stops meaning anything).

Rates are reported as warnings so they show in the test summary.
"""

from __future__ import annotations

import json
import warnings

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"

GATE = 0.99


NEAR_TIE_STEPS = 3  # the widest top-2 gap among the reference's own disagreements


@pytest.fixture(scope="module")
def fixture():
    with np.load(GOLDEN / "ref_engine_tokens.npz") as npz:
        data = {k: npz[k] for k in npz.files}
    data["meta"] = json.loads(str(data["meta"]))
    with np.load(GOLDEN / "ref_engine_hf.npz") as npz:
        data["hf_forced_tokens"] = npz["hf_forced_tokens"]
        data["hf_agreement"] = float(npz["agreement"])
    return data


def _bf16_step(x: float) -> float:
    """One bf16 step (8 significand bits) at magnitude |x|."""
    return float(2.0 ** (np.floor(np.log2(abs(x))) - 7))


def test_fixture_is_self_consistent(fixture):
    tokens, top2 = fixture["tokens"], fixture["top2"]
    valid = tokens >= 0
    assert valid.sum() == 48 + (tokens.shape[0] - 1) * 64
    # the recorded token is the largest logit (or tied with the second)
    assert (top2[..., 0] >= top2[..., 1])[valid].all()
    # the reference's two implementations differ only at near-ties
    hf = fixture["hf_forced_tokens"]
    assert float(((hf == tokens)[valid]).mean()) == pytest.approx(fixture["hf_agreement"])
    for i, j in zip(*np.nonzero((hf != tokens) & valid)):
        gap = top2[i, j, 0] - top2[i, j, 1]
        assert gap <= NEAR_TIE_STEPS * _bf16_step(top2[i, j, 0]), (i, j, gap)


def _engine(tmp_path, **settings):
    import sys

    sys.path.insert(0, str(GOLDEN))
    from make_ref_engine_tokens import ENGINE_SETTINGS

    from voiceagent_b200.checkpoint import write_checkpoint
    from voiceagent_b200.engine.engine import AsrEngine

    ckpt = write_checkpoint(tmp_path / "ckpt", "0.6b", seed=0, weights=False)
    return AsrEngine(str(ckpt), weights="random", seed=0, device="cuda:0",
                     **{**ENGINE_SETTINGS, **settings})


def _transcribe(engine):
    from make_ref_engine_tokens import TOKENS_CONFIG0, TOKENS_CONFIG3, workload

    from voiceagent_b200.engine.request import SamplingParams

    clips, n_tokens = workload()
    outs = engine.transcribe(clips[:1], language="en",
                             sampling=SamplingParams(max_new_tokens=TOKENS_CONFIG0, ignore_eos=True))
    outs += engine.transcribe(clips[1:], language="en",
                              sampling=SamplingParams(max_new_tokens=TOKENS_CONFIG3,
                                                      ignore_eos=True))
    return outs, n_tokens


def _force(engine, forced: np.ndarray) -> dict[int, list[int]]:
    """Teacher forcing: every call of the model runner returns the reference's token for
    each request (by admission order) while what the engine sampled is recorded."""
    admit, run = engine.add_request, engine.model_runner.run
    clip_of: dict[int, int] = {}
    sampled: dict[int, list[int]] = {}

    def add_request(*args, **kwargs):
        request = admit(*args, **kwargs)
        clip_of[request.request_id] = len(clip_of)
        return request

    def forced_run(batch):
        fed = []
        for request, token in zip(batch.requests, run(batch)):
            mine = sampled.setdefault(clip_of[request.request_id], [])
            mine.append(int(token))
            fed.append(int(forced[clip_of[request.request_id], len(mine) - 1]))
        return fed

    engine.add_request, engine.model_runner.run = add_request, forced_run
    return sampled


@pytest.mark.gpu
def test_teacher_forced_tokens_match_reference_engine(fixture, tmp_path):
    ref = fixture["tokens"]
    engine = _engine(tmp_path, decode_steps=1)  # one token per call: each step is forced
    sampled = _force(engine, ref)
    outs, n_tokens = _transcribe(engine)
    assert [o.num_prompt_tokens for o in outs] == fixture["meta"]["prompt_tokens"]
    same = total = 0
    steps = []
    top2 = fixture["top2"]
    for i, n in enumerate(n_tokens):
        got = np.asarray(sampled[i], np.int64)
        assert got.shape == (n,), got.shape
        eq = got == ref[i, :n]
        same, total = same + int(eq.sum()), total + n
        steps += [float((top2[i, j, 0] - top2[i, j, 1]) / _bf16_step(top2[i, j, 0]))
                  for j in np.flatnonzero(~eq)]
    strict = same / total
    floor = fixture["hf_agreement"]
    gate = min(GATE, floor)
    repeat = fixture["meta"]["self_agreement_graph_vs_eager_teacher_forced"]
    warnings.warn(f"teacher-forced greedy tokens vs the reference engine: strict {strict:.4f} over "
                  f"{total} positions (gate {gate:.4f} = min(0.99, the reference's upstream model "
                  f"vs its engine {floor:.4f}); the reference's eager vs graph decode {repeat:.4f}); "
                  f"reference top-2 gaps where they differ, in bf16 steps: {steps}")
    assert strict >= gate, (strict, steps)
    assert all(x <= NEAR_TIE_STEPS for x in steps), steps


@pytest.mark.gpu
def test_free_running_tokens_follow_reference_engine(fixture, tmp_path):
    ref, top2 = fixture["tokens"], fixture["top2"]
    outs, n_tokens = _transcribe(_engine(tmp_path))
    assert [o.num_prompt_tokens for o in outs] == fixture["meta"]["prompt_tokens"]
    same = total = 0
    first = []
    for i, (out, n) in enumerate(zip(outs, n_tokens)):
        got = np.asarray(out.output_token_ids, np.int64)
        assert got.shape == (n,), got.shape
        eq = got == ref[i, :n]
        same, total = same + int(eq.sum()), total + n
        if not eq.all():
            j = int(np.argmin(eq))
            first.append((i, j, float(top2[i, j, 0] - top2[i, j, 1]), float(top2[i, j, 0])))
    strict = same / total
    floor = fixture["meta"]["self_agreement_graph_vs_eager"]
    warnings.warn(f"free-running greedy tokens vs the reference engine: {strict:.4f} of {total} "
                  f"positions equal (the reference's eager vs graph decode: {floor:.4f}); first "
                  f"differences (clip, position, reference top-2 gap, top logit): {first}")
    for clip, pos, gap, top in first:
        assert gap <= NEAR_TIE_STEPS * _bf16_step(top), (clip, pos, gap)
