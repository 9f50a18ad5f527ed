"""One transcription request and the stages it moves through.

Stage graph (same stages and meaning as qwen-asr-vllm's engine/request.py:15-24,
89-199, whose scheduler decisions this engine reproduces):

    WAITING_ENCODE --encoded--> WAITING_PREFILL --first token--> RUNNING_DECODE
          |                        ^      |                            |
          |                        +------|------- preempted ----------+
          +------------------------+------+--> FINISHED <--------------+

Token bookkeeping: ``token_ids`` is the prompt followed by every sampled token.
``num_computed_tokens`` counts the leading positions whose K/V already sit in the
cache (prefix-cache hits included), so the next forward pass always feeds the tail
``token_ids[num_computed_tokens:]`` -- the whole prompt (or the part after a cached
prefix) for a prefill, one token for a decode.
"""

from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass

import torch

from voiceagent_b200.audio.frontend import AudioFeatures
from voiceagent_b200.prompt import PromptLayout

# Default output cap when a caller gives none: generous for the short utterances the
# engine mostly sees, and scaled with the recording for long-form audio.
DEFAULT_MAX_NEW_TOKENS = 440
TOKENS_PER_AUDIO_SECOND = 8
TOKEN_CAP_MARGIN = 64


class RequestStage(enum.Enum):
    WAITING_ENCODE = enum.auto()
    WAITING_PREFILL = enum.auto()
    RUNNING_DECODE = enum.auto()
    FINISHED = enum.auto()


# Transitions the engine performs; anything else is a bug in the caller.
_ALLOWED = {
    RequestStage.WAITING_ENCODE: {RequestStage.WAITING_PREFILL, RequestStage.FINISHED},
    RequestStage.WAITING_PREFILL: {RequestStage.RUNNING_DECODE, RequestStage.FINISHED},
    RequestStage.RUNNING_DECODE: {RequestStage.WAITING_PREFILL, RequestStage.FINISHED},
    RequestStage.FINISHED: set(),
}


@dataclass
class SamplingParams:
    """Per-request decoding controls: temperature 0 is greedy; ``ignore_eos`` keeps
    generating past stop tokens until ``max_new_tokens``."""

    temperature: float = 0.0
    max_new_tokens: int = DEFAULT_MAX_NEW_TOKENS
    ignore_eos: bool = False

    @classmethod
    def for_audio(cls, audio_seconds: float, max_new_tokens: int = 0, **kwargs) -> "SamplingParams":
        """An explicit positive cap wins; otherwise the default cap, raised for long
        audio to ``TOKENS_PER_AUDIO_SECOND`` per second plus a fixed margin."""
        if max_new_tokens <= 0:
            scaled = int(audio_seconds * TOKENS_PER_AUDIO_SECOND) + TOKEN_CAP_MARGIN
            max_new_tokens = max(DEFAULT_MAX_NEW_TOKENS, scaled)
        return cls(max_new_tokens=max_new_tokens, **kwargs)


class RequestTimings:
    """Wall-clock milestones of a request (``time.perf_counter`` seconds, None until
    reached) and the stage durations between them."""

    MILESTONES = ("arrival", "encode_start", "encode_end", "prefill_end", "finish")

    def __init__(self) -> None:
        self.arrival: float | None = time.perf_counter()
        self.encode_start: float | None = None
        self.encode_end: float | None = None
        self.prefill_end: float | None = None
        self.finish: float | None = None

    def _between(self, first: str, last: str) -> float:
        a, b = getattr(self, first), getattr(self, last)
        return b - a if a is not None and b is not None else 0.0

    queue_seconds = property(lambda self: self._between("arrival", "encode_start"))
    encode_seconds = property(lambda self: self._between("encode_start", "encode_end"))
    prefill_seconds = property(lambda self: self._between("encode_end", "prefill_end"))
    decode_seconds = property(lambda self: self._between("prefill_end", "finish"))
    total_seconds = property(lambda self: self._between("arrival", "finish"))

    def __repr__(self) -> str:
        return "RequestTimings(" + ", ".join(f"{m}={getattr(self, m)}" for m in self.MILESTONES) + ")"


_request_ids = itertools.count()


class AsrRequest:
    """Everything the scheduler, block manager and model runner track for one clip."""

    def __init__(self, features: AudioFeatures, layout: PromptLayout, sampling: SamplingParams,
                 block_size: int, stop_token_ids: set[int], language: str | None = None):
        self.request_id = next(_request_ids)
        self.features, self.layout, self.sampling = features, layout, sampling
        self.block_size = block_size
        self.stop_token_ids = stop_token_ids
        self.language = language
        self.token_ids: list[int] = list(layout.token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        # KV-cache state, owned by the block manager and the scheduler
        self.block_table: list[int] = []
        self.num_computed_tokens = 0
        self.num_cached_tokens = 0
        # encoder output, kept until the request finishes so a preempted request
        # re-prefills without re-encoding
        self.audio_embeds: torch.Tensor | None = None
        self.stage = RequestStage.WAITING_ENCODE
        self.finish_reason: str | None = None
        self.cancel_requested = False  # set while the request is inside a running step
        self.timings = RequestTimings()

    # ---------------------------------------------------------------- tokens

    def __len__(self) -> int:
        return len(self.token_ids)

    @property
    def output_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_output_tokens(self) -> int:
        return len(self) - self.num_prompt_tokens

    @property
    def last_token_id(self) -> int:
        return self.token_ids[-1]

    @property
    def num_tokens_to_compute(self) -> int:
        """Query length of the next forward pass."""
        return len(self) - self.num_computed_tokens

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)

    # ---------------------------------------------------------------- blocks

    @property
    def num_blocks(self) -> int:
        """Cache blocks the current tokens occupy."""
        return (len(self) + self.block_size - 1) // self.block_size

    def block(self, index: int) -> list[int]:
        """Token ids held by cache block ``index``."""
        lo = index * self.block_size
        return self.token_ids[lo:lo + self.block_size]

    @property
    def num_cacheable_blocks(self) -> int:
        """Leading blocks safe to share through the prefix cache: those that end before
        the audio span. Every audio position carries the same placeholder id, so a
        block containing audio (and every block after it) depends on the recording,
        not on its token ids."""
        return self.layout.audio_offset // self.block_size

    # ---------------------------------------------------------------- stages

    def move_to(self, stage: RequestStage) -> None:
        if stage not in _ALLOWED[self.stage]:
            raise RuntimeError(f"request {self.request_id}: {self.stage.name} -> {stage.name} "
                               "is not a valid stage change")
        self.stage = stage

    def mark_encoding(self) -> None:
        """Encoder output attached: ready for prefill."""
        self.move_to(RequestStage.WAITING_PREFILL)
        self.timings.encode_end = time.perf_counter()

    def mark_prefilled(self) -> None:
        """First token sampled: decoding from now on."""
        self.move_to(RequestStage.RUNNING_DECODE)
        self.timings.prefill_end = time.perf_counter()

    def finish(self, reason: str) -> None:
        self.stage = RequestStage.FINISHED  # any stage may end (cancel, abort, stop)
        self.finish_reason = reason
        self.timings.finish = time.perf_counter()

    def check_finished(self) -> bool:
        """Ends the request on a stop token (unless ignored) or at the output cap;
        returns whether it ended."""
        if self.last_token_id in self.stop_token_ids and not self.sampling.ignore_eos:
            reason = "stop"
        elif self.num_output_tokens >= self.sampling.max_new_tokens:
            reason = "length"
        else:
            return False
        self.finish(reason)
        return True

    @property
    def is_finished(self) -> bool:
        return self.stage is RequestStage.FINISHED
