"""Three-stage scheduling with mixed prefill/decode batches.

Semantics of the reference scheduler (engine/scheduler.py:62-309): an audio-encode
stage packs several requests into one encoder call (backlog capped at
``max_num_seqs``); each decoder step takes every running decode first (preempting
the newest when blocks run out, aborting a lone request that cannot grow), then
admits prefills under the token and sequence budgets; OOM rollbacks restore batches
exactly and halve the caps, ``relax_limits`` doubles them back.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.block_manager import BlockManager
from voiceagent_b200.engine.request import AsrRequest, RequestStage


@dataclass
class ModelBatch:
    prefill: list[AsrRequest] = field(default_factory=list)
    decode: list[AsrRequest] = field(default_factory=list)

    @property
    def requests(self) -> list[AsrRequest]:
        return self.prefill + self.decode

    @property
    def num_tokens(self) -> int:
        return sum(r.num_tokens_to_compute for r in self.requests)

    def __bool__(self) -> bool:
        return bool(self.prefill or self.decode)


@dataclass
class SchedulerStats:
    num_encode_batches: int = 0
    num_model_steps: int = 0
    num_mixed_steps: int = 0
    num_preemptions: int = 0
    num_encoded_requests: int = 0
    num_prefilled_tokens: int = 0
    num_decoded_tokens: int = 0
    num_model_ooms: int = 0
    num_audio_ooms: int = 0


class Scheduler:
    def __init__(self, config: EngineConfig, block_manager: BlockManager):
        self.config = config
        self.block_manager = block_manager
        self.waiting_encode: deque[AsrRequest] = deque()
        self.waiting_prefill: deque[AsrRequest] = deque()
        self.running: deque[AsrRequest] = deque()
        self.aborted: list[AsrRequest] = []
        self.tracked: dict[int, AsrRequest] = {}
        self.stats = SchedulerStats()
        self.model_batch_limit = config.max_num_seqs
        self.audio_frame_limit = config.max_audio_batch_frames

    # -------------------------------------------------------------- queues

    def add(self, request: AsrRequest) -> None:
        self.waiting_encode.append(request)
        self.tracked[request.request_id] = request

    def admit_prefill(self, requests: list[AsrRequest]) -> None:
        self.waiting_prefill.extend(requests)

    def drain_aborted(self) -> list[AsrRequest]:
        out, self.aborted = self.aborted, []
        return out

    def cancel(self, request_id: int) -> bool:
        request = self.tracked.get(request_id)
        if request is None:
            return False
        for queue in (self.waiting_encode, self.waiting_prefill, self.running):
            if request in queue:
                queue.remove(request)
                self._give_up(request, "cancelled")
                return True
        request.cancel_requested = True  # inside the batch being executed
        return True

    @property
    def has_work(self) -> bool:
        return bool(self.waiting_encode or self.waiting_prefill or self.running)

    @property
    def num_in_flight(self) -> int:
        return len(self.waiting_encode) + len(self.waiting_prefill) + len(self.running)

    # ---------------------------------------------------------- scheduling

    def schedule_audio(self) -> list[AsrRequest]:
        capacity = self.config.max_num_seqs - len(self.waiting_prefill)
        if capacity <= 0 or not self.waiting_encode:
            return []
        limit = min(capacity, self.config.max_audio_batch_size)
        picked: list[AsrRequest] = []
        frames = 0
        while self.waiting_encode and len(picked) < limit:
            request = self.waiting_encode[0]
            n = request.features.mel_frames
            if picked and frames + n > self.audio_frame_limit:
                break
            self.waiting_encode.popleft()
            request.timings.encode_start = time.perf_counter()
            picked.append(request)
            frames += n
        if picked:
            self.stats.num_encode_batches += 1
            self.stats.num_encoded_requests += len(picked)
        return picked

    def _preempt(self, request: AsrRequest) -> None:
        self.block_manager.deallocate(request)
        request.num_computed_tokens = 0
        request.stage = RequestStage.WAITING_PREFILL
        self.waiting_prefill.appendleft(request)
        self.stats.num_preemptions += 1

    def schedule_model(self) -> ModelBatch:
        batch = ModelBatch()
        while self.running:
            request = self.running[0]
            if self.block_manager.can_append(request):
                batch.decode.append(self.running.popleft())
                continue
            if len(self.running) > 1:
                self._preempt(self.running.pop())
                continue
            self.running.popleft()
            request.finish("aborted:out_of_kv_blocks")
            self.block_manager.deallocate(request)
            request.audio_embeds = None
            self.aborted.append(request)
            break

        tokens_left = self.config.max_num_batched_tokens - len(batch.decode)
        seqs_left = self.model_batch_limit - len(batch.decode)
        while self.waiting_prefill and seqs_left > 0:
            request = self.waiting_prefill[0]
            if len(request) > tokens_left:
                break
            if not self.block_manager.can_ever_allocate(request):
                self.waiting_prefill.popleft()
                request.finish("aborted:kv_cache_too_small")
                request.audio_embeds = None
                self.aborted.append(request)
                continue
            if not self.block_manager.can_allocate(request):
                break
            self.waiting_prefill.popleft()
            self.block_manager.allocate(request)
            batch.prefill.append(request)
            tokens_left -= request.num_tokens_to_compute
            seqs_left -= 1

        if batch:
            self.stats.num_model_steps += 1
            if batch.prefill and batch.decode:
                self.stats.num_mixed_steps += 1
            self.stats.num_prefilled_tokens += sum(r.num_tokens_to_compute for r in batch.prefill)
            self.stats.num_decoded_tokens += len(batch.decode)
        return batch

    # ------------------------------------------------------------ recovery

    def _give_up(self, request: AsrRequest, reason: str) -> None:
        self.block_manager.deallocate(request)
        request.num_computed_tokens = 0
        request.audio_embeds = None
        request.finish(reason)
        self.tracked.pop(request.request_id, None)
        self.aborted.append(request)

    def on_model_oom(self, batch: ModelBatch) -> None:
        """Put a failed decoder batch back exactly (nothing was mutated) and halve the cap."""
        self.stats.num_model_ooms += 1
        attempted = len(batch.requests)
        for request in reversed(batch.prefill):
            self.block_manager.deallocate(request)
            request.num_computed_tokens = 0
            self.waiting_prefill.appendleft(request)
        for request in reversed(batch.decode):
            self.running.appendleft(request)
        if attempted <= 1:
            self.model_batch_limit = 1
            if self.running:
                self._give_up(self.running.pop(), "aborted:out_of_memory")
            elif self.waiting_prefill:
                self._give_up(self.waiting_prefill.popleft(), "aborted:out_of_memory")
            return
        self.model_batch_limit = max(1, attempted // 2)

    def on_audio_oom(self, requests: list[AsrRequest]) -> None:
        self.stats.num_audio_ooms += 1
        frames = sum(r.features.mel_frames for r in requests)
        for request in reversed(requests):
            request.timings.encode_start = None
            request.audio_embeds = None
            self.waiting_encode.appendleft(request)
        if len(requests) <= 1:
            self._give_up(self.waiting_encode.popleft(), "aborted:out_of_memory")
            return
        self.audio_frame_limit = max(1, frames // 2)

    def relax_limits(self) -> None:
        if self.model_batch_limit < self.config.max_num_seqs:
            self.model_batch_limit = min(self.config.max_num_seqs, self.model_batch_limit * 2)
        if self.audio_frame_limit < self.config.max_audio_batch_frames:
            self.audio_frame_limit = min(self.config.max_audio_batch_frames,
                                         self.audio_frame_limit * 2)

    def decode_steps_for(self, batch: ModelBatch, limit: int, max_model_len: int) -> int:
        """How many decode steps a decode-only batch can run in one call (>= 1): bounded
        by ``limit``, every request's remaining token budget and the model length, and
        by free blocks for the positions those steps write (taken when > 1 is returned).

        Running several steps before the host sees their tokens changes no output: a
        request that stops early (EOS) has its later tokens discarded. It can delay the
        admission of a waiting request by up to ``steps - 1`` steps."""
        if limit <= 1 or batch.prefill or not batch.decode:
            return 1
        steps = limit
        for r in batch.decode:
            if r.cancel_requested:
                return 1
            steps = min(steps, r.sampling.max_new_tokens - r.num_output_tokens,
                        max_model_len - len(r) + 1)
        if steps <= 1:
            return 1
        need = sum(self.block_manager.blocks_ahead(r, steps) for r in batch.decode)
        if need > self.block_manager.num_free_blocks:
            return 1
        for r in batch.decode:
            self.block_manager.append_ahead(r, steps)
        return steps

    def postprocess_steps(self, batch: ModelBatch, tokens: list[list[int]]) -> list[AsrRequest]:
        """``postprocess`` for several decode steps of a decode-only batch: tokens[k][i] is
        request i's token of step k; a request stops at its first finishing token."""
        requests = batch.decode
        if batch.prefill or any(len(step) != len(requests) for step in tokens):
            raise ValueError("multi-step results do not match the decode batch")
        finished: list[AsrRequest] = []
        for i, request in enumerate(requests):
            done = False
            for step in tokens:
                request.num_computed_tokens = len(request)
                request.append_token(step[i])
                if request.cancel_requested:
                    request.finish("cancelled")
                    done = True
                elif request.check_finished():
                    done = True
                if done:
                    break
            if not done:
                self.block_manager.may_append(request)
                self.running.append(request)
                continue
            self.block_manager.deallocate(request)
            request.audio_embeds = None
            self.tracked.pop(request.request_id, None)
            finished.append(request)
        extra = len(tokens) - 1
        self.stats.num_model_steps += extra
        self.stats.num_decoded_tokens += extra * len(requests)
        return finished

    def postprocess(self, batch: ModelBatch, token_ids: list[int]) -> list[AsrRequest]:
        requests = batch.requests
        if len(requests) != len(token_ids):
            raise ValueError(f"sampler returned {len(token_ids)} tokens for {len(requests)} requests")
        finished: list[AsrRequest] = []
        for request, token_id in zip(requests, token_ids):
            request.num_computed_tokens = len(request)
            request.append_token(token_id)
            if request.stage is RequestStage.WAITING_PREFILL:
                request.mark_prefilled()
            if request.cancel_requested:
                request.finish("cancelled")
            elif not request.check_finished():
                self.block_manager.may_append(request)
                self.running.append(request)
                continue
            self.block_manager.deallocate(request)
            request.audio_embeds = None
            self.tracked.pop(request.request_id, None)
            finished.append(request)
        return finished
