"""Generate ``tests/golden/ref_engine_tokens.npz``: greedy tokens of the reference engine.

Run on a GPU box where the reference is installed under ``baseline/_ref`` (see
``baseline/ref_engine.py``)::

    python tests/golden/make_ref_engine_tokens.py [--out tests/golden/ref_engine_tokens.npz]

It builds the seeded random-init Qwen3-ASR-0.6B checkpoint (``voiceagent_b200.checkpoint``,
seed 0, bf16) and transcribes, through ``qwen_asr_vllm.AsrEngine.transcribe``
(engine/engine.py:539-627; flash-attn varlen attention, the Triton KV store, CUDA-graph
decode), the config-0 clip (4.0 s, 48 greedy tokens) and the first 24 clips of the
config-3 workload (64 greedy tokens each), language "en", EOS ignored. It records each
request's sampled tokens and, at every position, the two largest logits its greedy
sampler compared (layers/sampler.py:16-20), read through a wrapper around
``ModelRunner._sample`` that returns the engine's own sample.

The same transcription is then repeated twice with ``enforce_eager=True`` (the
reference's eager decode against its own graph decode, the comparison its
tests/test_cuda_graph.py makes): once free running, and once teacher forced -- fed the
graph run's tokens through the same sampling hook while recording what it would have
sampled. The two agreement rates measure how often the reference disagrees with itself
on this random-init model (whose logits are full of near-ties); they are stored beside
the tokens as the floor below which no parity gate may be set.
"""

from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

N_CONFIG3_CLIPS = 24
TOKENS_CONFIG0, TOKENS_CONFIG3 = 48, 64
ENGINE_SETTINGS = dict(max_num_seqs=32, max_model_len=4096, max_num_batched_tokens=8192,
                       max_audio_batch_size=32, num_kvcache_blocks=256)


def workload():
    """(clips, tokens per clip): the config-0 clip, then the first config-3 clips."""
    from voiceagent_b200.workload import config0_clip, config3_clips

    clips = [config0_clip(0)] + config3_clips(512, seed=0)[:N_CONFIG3_CLIPS]
    return clips, [TOKENS_CONFIG0] + [TOKENS_CONFIG3] * N_CONFIG3_CLIPS


def run_reference(checkpoint: str, eager: bool, forced: np.ndarray | None = None):
    """(tokens, top-2 logits, prompt lengths) of one reference run; teacher forced to
    ``forced`` (clip x position) when given, the tokens being then what it sampled."""
    import torch

    from baseline import ref_engine

    clips, n_tokens = workload()
    engine = ref_engine.build_engine(checkpoint, device="cuda:0", enforce_eager=eager,
                                     **ENGINE_SETTINGS)
    steps = ref_engine.record_greedy_steps(engine)
    if forced is not None:
        ref_engine.force_tokens(engine, {i: list(row[row >= 0]) for i, row in enumerate(forced)})
    outs = engine.transcribe(clips[:1], language="en",
                             sampling=ref_engine.sampling_params(TOKENS_CONFIG0))
    outs += engine.transcribe(clips[1:], language="en",
                              sampling=ref_engine.sampling_params(TOKENS_CONFIG3))
    width = max(n_tokens)
    tokens = np.full((len(clips), width), -1, np.int64)
    top = np.zeros((len(clips), width, 2), np.float32)
    for i, (out, n) in enumerate(zip(outs, n_tokens)):
        rec = steps[out.request_id]
        assert len(rec) == n, (len(rec), n)
        tokens[i, :n] = [t for t, _, _ in rec]
        top[i, :n] = [(a, b) for _, a, b in rec]
    del engine
    torch.cuda.empty_cache()
    return tokens, top, [int(o.num_prompt_tokens) for o in outs]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--out", default=str(REPO / "tests" / "golden" / "ref_engine_tokens.npz"))
    args = parser.parse_args()

    import flash_attn
    import torch

    from voiceagent_b200.checkpoint import write_checkpoint

    ckpt = write_checkpoint(Path(tempfile.mkdtemp(prefix="ref_tokens_")) / "ckpt", "0.6b",
                            seed=0, weights=True)
    graph_tokens, graph_top, prompts = run_reference(str(ckpt), eager=False)
    eager_tokens, _, _ = run_reference(str(ckpt), eager=True)
    forced_tokens, _, _ = run_reference(str(ckpt), eager=True, forced=graph_tokens)
    valid = graph_tokens >= 0
    self_agreement = float((graph_tokens == eager_tokens)[valid].mean())
    self_agreement_forced = float((graph_tokens == forced_tokens)[valid].mean())
    meta = {
        "generator": "tests/golden/make_ref_engine_tokens.py",
        "reference": "qwen_asr_vllm.AsrEngine (baseline/_ref), CUDA-graph decode; eager rerun",
        "checkpoint": "voiceagent_b200.checkpoint.write_checkpoint('0.6b', seed=0), bf16",
        "clips": f"config0_clip(0) with 48 tokens, then config3_clips(512, seed=0)[:{N_CONFIG3_CLIPS}] with 64",
        "language": "en", "ignore_eos": True, "engine_settings": ENGINE_SETTINGS,
        "prompt_tokens": prompts, "self_agreement_graph_vs_eager": self_agreement,
        "self_agreement_graph_vs_eager_teacher_forced": self_agreement_forced,
        "gpu": torch.cuda.get_device_name(0), "torch": torch.__version__,
        "flash_attn": flash_attn.__version__,
    }
    np.savez_compressed(args.out, tokens=graph_tokens, top2=graph_top, eager_tokens=eager_tokens,
                        eager_forced_tokens=forced_tokens, meta=np.array(json.dumps(meta)))
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
