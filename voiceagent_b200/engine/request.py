"""Request state machine (engine/request.py of the reference).

    WAITING_ENCODE -> WAITING_PREFILL -> RUNNING_DECODE -> FINISHED

``num_computed_tokens`` counts prompt/output positions that already have KV state
(prefix-cache hits included), so the query length of the next forward pass is
``len(request) - num_computed_tokens`` for prefill and decode alike.
"""

from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field

import torch

from voiceagent_b200.audio.frontend import AudioFeatures
from voiceagent_b200.prompt import PromptLayout


class RequestStage(enum.Enum):
    WAITING_ENCODE = enum.auto()
    WAITING_PREFILL = enum.auto()
    RUNNING_DECODE = enum.auto()
    FINISHED = enum.auto()


@dataclass
class SamplingParams:
    temperature: float = 0.0
    max_new_tokens: int = 440
    ignore_eos: bool = False

    @classmethod
    def for_audio(cls, audio_seconds: float, max_new_tokens: int = 0, **kwargs) -> "SamplingParams":
        """A cap scaled to the audio: 8 tokens per second + 64, at least 440."""
        if max_new_tokens > 0:
            return cls(max_new_tokens=max_new_tokens, **kwargs)
        return cls(max_new_tokens=max(440, int(audio_seconds * 8) + 64), **kwargs)


@dataclass
class RequestTimings:
    arrival: float = field(default_factory=time.perf_counter)
    encode_start: float | None = None
    encode_end: float | None = None
    prefill_end: float | None = None
    finish: float | None = None

    @staticmethod
    def _span(a, b) -> float:
        return 0.0 if a is None or b is None else b - a

    @property
    def queue_seconds(self) -> float:
        return self._span(self.arrival, self.encode_start)

    @property
    def encode_seconds(self) -> float:
        return self._span(self.encode_start, self.encode_end)

    @property
    def prefill_seconds(self) -> float:
        return self._span(self.encode_end, self.prefill_end)

    @property
    def decode_seconds(self) -> float:
        return self._span(self.prefill_end, self.finish)

    @property
    def total_seconds(self) -> float:
        return self._span(self.arrival, self.finish)


class AsrRequest:
    _ids = itertools.count()

    def __init__(self, features: AudioFeatures, layout: PromptLayout, sampling: SamplingParams,
                 block_size: int, stop_token_ids: set[int], language: str | None = None):
        self.request_id = next(AsrRequest._ids)
        self.features = features
        self.layout = layout
        self.sampling = sampling
        self.block_size = block_size
        self.stop_token_ids = stop_token_ids
        self.language = language
        self.stage = RequestStage.WAITING_ENCODE
        self.timings = RequestTimings()
        self.audio_embeds: torch.Tensor | None = None
        self.token_ids: list[int] = list(layout.token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_computed_tokens = 0
        self.num_cached_tokens = 0
        self.block_table: list[int] = []
        self.finish_reason: str | None = None
        self.cancel_requested = False

    def __len__(self) -> int:
        return len(self.token_ids)

    @property
    def num_output_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def output_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def last_token_id(self) -> int:
        return self.token_ids[-1]

    @property
    def num_blocks(self) -> int:
        return -(-len(self.token_ids) // self.block_size)

    def block(self, index: int) -> list[int]:
        return self.token_ids[index * self.block_size:(index + 1) * self.block_size]

    @property
    def num_cacheable_blocks(self) -> int:
        """Blocks entirely before the audio span (audio placeholders all share one id,
        so a block holding audio -- and any block after it -- is unsafe to reuse)."""
        return self.layout.audio_offset // self.block_size

    @property
    def num_tokens_to_compute(self) -> int:
        return len(self.token_ids) - self.num_computed_tokens

    def mark_encoding(self) -> None:
        self.stage = RequestStage.WAITING_PREFILL
        self.timings.encode_end = time.perf_counter()

    def mark_prefilled(self) -> None:
        self.stage = RequestStage.RUNNING_DECODE
        self.timings.prefill_end = time.perf_counter()

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)

    def check_finished(self) -> bool:
        if not self.sampling.ignore_eos and self.last_token_id in self.stop_token_ids:
            self.finish("stop")
            return True
        if self.num_output_tokens >= self.sampling.max_new_tokens:
            self.finish("length")
            return True
        return False

    def finish(self, reason: str) -> None:
        self.stage = RequestStage.FINISHED
        self.finish_reason = reason
        self.timings.finish = time.perf_counter()

    @property
    def is_finished(self) -> bool:
        return self.stage is RequestStage.FINISHED
