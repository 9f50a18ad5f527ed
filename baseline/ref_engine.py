"""Runs the reference's own GPU engine, installed unmodified under ``baseline/_ref``.

The reference (``qwen_asr_vllm``, DingdongD/VoiceAgent) is installed with
``pip install --no-index --no-build-isolation --no-deps --target baseline/_ref <copy of
the reference>``. This module is the launcher that ``bench.py`` (the like-for-like
engine comparison) and ``tests/golden/make_ref_engine_tokens.py`` (the reference-engine
token fixture) share. It is not part of the product: nothing in ``voiceagent_b200``
imports it.

The only stand-in is the tokenizer: the checkpoint tokenizer's files do not exist
offline, and the engine only asks its tokenizer to encode the chat template (once per
context/language pair), for the EOS id, and to decode output text.
:class:`TemplateTokenizer` returns the template ids the reference's tests/test_prompt.py
pins (the same ids ``voiceagent_b200.prompt`` builds), so both engines see prompts of
identical length and content; text output is empty. Frontend, scheduler, model,
flash-attn, the Triton store and the CUDA graphs are the reference's own code.
"""

from __future__ import annotations

import sys
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"


def available() -> tuple[bool, str]:
    """Whether the reference package is installed here, and why not."""
    if not (REF / "qwen_asr_vllm").is_dir():
        return False, "baseline/_ref is not installed (pip install --target baseline/_ref)"
    try:
        import flash_attn  # noqa: F401  (the reference engine's attention)
    except Exception as exc:  # pragma: no cover - depends on the box
        return False, f"flash_attn does not import: {type(exc).__name__}: {exc}"
    return True, ""


class TemplateTokenizer:
    """The tokenizer stand-in described in the module docstring."""

    eos_token_id = 151645

    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        return cls()

    def encode(self, text: str) -> list[int]:
        from voiceagent_b200.prompt import PromptBuilder

        head, sep, tail = text.partition("<|im_start|>assistant\n")
        if not sep or "<|im_start|>system\n<|im_end|>" not in head:
            raise ValueError("template tokenizer: only the empty-context ASR template is known")
        language = tail[len("language "):].replace("<asr_text>", "") if tail else None
        return PromptBuilder().template(None, language or None)[0]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return ""


def import_reference():
    """Import the installed reference with the tokenizer stand-in in place."""
    ok, why = available()
    if not ok:
        raise RuntimeError(why)
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import qwen_asr_vllm.prompt as ref_prompt

    ref_prompt.AutoTokenizer = TemplateTokenizer
    import qwen_asr_vllm

    return qwen_asr_vllm


def build_engine(checkpoint: str, **settings):
    """``qwen_asr_vllm.AsrEngine(model=checkpoint, **settings)``."""
    ref = import_reference()
    return ref.AsrEngine(model=str(checkpoint), **settings)


def sampling_params(max_new_tokens: int, ignore_eos: bool = True):
    import_reference()
    from qwen_asr_vllm.engine.request import SamplingParams

    return SamplingParams(max_new_tokens=max_new_tokens, ignore_eos=ignore_eos)


def record_greedy_steps(engine) -> dict[int, list[tuple[int, float, float]]]:
    """Wrap the engine's ``ModelRunner._sample`` (engine/model_runner.py:337-343) to
    record, per request id and in order, (sampled token, largest logit, second largest
    logit) as fp32 -- the values its greedy sampler (layers/sampler.py:16-20) compares.
    The wrapped call still returns the engine's own sample."""
    runner = engine.model_runner
    inner = runner._sample
    steps: dict[int, list[tuple[int, float, float]]] = {}

    def sample(logits, requests):
        out = inner(logits, requests)
        top = logits.float().topk(2, dim=-1)
        vals, idx = top.values.tolist(), top.indices.tolist()
        for row, (request, token) in enumerate(zip(requests, out)):
            steps.setdefault(request.request_id, []).append(
                (int(token), float(vals[row][0]), float(vals[row][1])))
            assert idx[row][0] == token or vals[row][0] == vals[row][1], "greedy sample"
        return out

    runner._sample = sample
    return steps


def force_tokens(engine, forced: dict[int, list[int]]) -> dict[int, list[int]]:
    """Teacher forcing through the engine's own sampling hook: wrap
    ``ModelRunner._sample`` (engine/model_runner.py:337-343) so that the engine keeps
    generating from ``forced[clip]`` instead of its own samples, while recording what it
    sampled at each position. ``forced`` is keyed by the clip's admission order (0, 1,
    ... across this engine's ``add_request`` calls). Returns {clip: [sampled tokens]}."""
    admit = engine.add_request
    clip_of: dict[int, int] = {}
    sampled: dict[int, list[int]] = {}

    def add_request(*args, **kwargs):
        request = admit(*args, **kwargs)
        clip_of[request.request_id] = len(clip_of)
        return request

    runner = engine.model_runner
    inner = runner._sample

    def sample(logits, requests):
        out = inner(logits, requests)
        fed = []
        for request, token in zip(requests, out):
            clip = clip_of[request.request_id]
            mine = sampled.setdefault(clip, [])
            mine.append(int(token))
            fed.append(int(forced[clip][len(mine) - 1]))
        return fed

    engine.add_request = add_request
    runner._sample = sample
    return sampled
