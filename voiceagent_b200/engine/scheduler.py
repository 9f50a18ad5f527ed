"""Scheduling of the engine's three stages: audio encode, prefill, decode.

The decisions are the ones qwen-asr-vllm's scheduler makes (engine/scheduler.py:62-309),
because the slot mappings and block tables this engine must reproduce follow from them:

* Encode: requests leave the encode queue in arrival order, several per encoder call,
  while the prefill backlog has room (at most ``max_num_seqs`` encoded-but-unprefilled
  requests, since their embeddings occupy device memory), the call stays within
  ``max_audio_batch_size`` requests and the frame cap (the first request always fits).
* Decode first: every running request joins the step in order if its next token has
  a cache slot. When one does not, the most recently started running request is
  preempted -- its blocks freed, its embeddings kept, back to the front of the prefill
  queue -- and the check repeats; a request that is the only one running and still
  cannot grow ends as ``aborted:out_of_kv_blocks``.
* Then prefill, in queue order, while the step has sequence slots (the adaptive cap)
  and token budget (``max_num_batched_tokens``, decodes count one each): a request
  longer than the remaining budget, or whose blocks are not free now, waits at the
  head; one needing more blocks than the whole cache ends as
  ``aborted:kv_cache_too_small``.
* Out of memory: the failed step is undone exactly (its requests back at the front of
  their queues, prefill blocks freed) and its cap halves (``max(1, attempted // 2)``
  sequences, or half the failed call's frames for the encoder); a failed step of one
  request gives that request up. Each successful step doubles the caps back toward
  their configured values.
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
    """The requests of one decoder forward pass: prefills first, then decodes."""

    prefill: list[AsrRequest] = field(default_factory=list)
    decode: list[AsrRequest] = field(default_factory=list)

    @property
    def requests(self) -> list[AsrRequest]:
        return [*self.prefill, *self.decode]

    @property
    def num_tokens(self) -> int:
        return sum(r.num_tokens_to_compute for r in self.requests)

    def __bool__(self) -> bool:
        return len(self.prefill) + len(self.decode) > 0


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


class AdaptiveCap:
    """A limit that drops after an out-of-memory failure and climbs back by doubling
    after each success, never above its configured ceiling."""

    def __init__(self, ceiling: int):
        self.ceiling = ceiling
        self.value = ceiling

    def cut_to(self, value: int) -> None:
        self.value = max(1, value)

    def relax(self) -> None:
        if self.value < self.ceiling:
            self.value = min(self.ceiling, 2 * self.value)


class Scheduler:
    def __init__(self, config: EngineConfig, block_manager: BlockManager):
        self.config = config
        self.block_manager = block_manager
        # the three stage queues, oldest first
        self.waiting_encode: deque[AsrRequest] = deque()
        self.waiting_prefill: deque[AsrRequest] = deque()
        self.running: deque[AsrRequest] = deque()
        self.aborted: list[AsrRequest] = []  # ended without finishing; drained by the engine
        self.tracked: dict[int, AsrRequest] = {}  # every in-flight request, for cancel()
        self.stats = SchedulerStats()
        self._seq_cap = AdaptiveCap(config.max_num_seqs)
        self._frame_cap = AdaptiveCap(config.max_audio_batch_frames)

    @property
    def model_batch_limit(self) -> int:
        return self._seq_cap.value

    @property
    def audio_frame_limit(self) -> int:
        return self._frame_cap.value

    # ------------------------------------------------------------- queue access

    def add(self, request: AsrRequest) -> None:
        self.tracked[request.request_id] = request
        self.waiting_encode.append(request)

    def admit_prefill(self, requests: list[AsrRequest]) -> None:
        """Encoded requests join the prefill queue."""
        self.waiting_prefill.extend(requests)

    def drain_aborted(self) -> list[AsrRequest]:
        out = self.aborted
        self.aborted = []
        return out

    @property
    def has_work(self) -> bool:
        return self.num_in_flight > 0

    @property
    def num_in_flight(self) -> int:
        return sum(map(len, (self.waiting_encode, self.waiting_prefill, self.running)))

    def cancel(self, request_id: int) -> bool:
        """End a request wherever it waits (it is reported with reason "cancelled").
        One inside the step being executed is only flagged; the step's results end it.
        Returns whether the id was in flight."""
        request = self.tracked.get(request_id)
        if request is None:
            return False
        queue = next((q for q in (self.waiting_encode, self.waiting_prefill, self.running)
                      if request in q), None)
        if queue is None:
            request.cancel_requested = True
        else:
            queue.remove(request)
            self._retire(request, "cancelled")
        return True

    def _retire(self, request: AsrRequest, reason: str) -> None:
        """End a request that did not finish normally: free everything it holds and
        report it through ``aborted``."""
        self.block_manager.deallocate(request)
        request.num_computed_tokens = 0
        request.audio_embeds = None
        request.finish(reason)
        self.tracked.pop(request.request_id, None)
        self.aborted.append(request)

    def _release_finished(self, request: AsrRequest) -> None:
        self.block_manager.deallocate(request)
        request.audio_embeds = None
        self.tracked.pop(request.request_id, None)

    # ------------------------------------------------------------------ encode

    def schedule_audio(self) -> list[AsrRequest]:
        """The requests of the next encoder call (possibly none)."""
        room = min(self.config.max_num_seqs - len(self.waiting_prefill),
                   self.config.max_audio_batch_size)
        count, frames = 0, 0
        for request in self.waiting_encode:
            if count >= room:
                break
            frames += request.features.mel_frames
            if count > 0 and frames > self._frame_cap.value:
                break
            count += 1
        if count <= 0:
            return []
        now = time.perf_counter()
        picked = [self.waiting_encode.popleft() for _ in range(count)]
        for request in picked:
            request.timings.encode_start = now
        self.stats.num_encode_batches += 1
        self.stats.num_encoded_requests += count
        return picked

    # ------------------------------------------------------------------- model

    def _preempt(self, request: AsrRequest) -> None:
        """Send a running request back to prefill to free its blocks (its audio
        embeddings stay: only the text prefill repeats)."""
        self.block_manager.deallocate(request)
        request.num_computed_tokens = 0
        request.move_to(RequestStage.WAITING_PREFILL)
        self.waiting_prefill.appendleft(request)
        self.stats.num_preemptions += 1

    def _take_decodes(self, batch: ModelBatch) -> None:
        bm = self.block_manager
        # can_append asks for at most one free block and taking a request changes no
        # free count: with one free (or no request opening a block) all of them join
        if self.running and (bm.num_free_blocks > 0 or all(
                len(r.token_ids) % bm.block_size != 1 for r in self.running)):
            batch.decode.extend(self.running)
            self.running.clear()
            return
        while self.running:
            if bm.can_append(self.running[0]):
                batch.decode.append(self.running.popleft())
            elif len(self.running) > 1:
                self._preempt(self.running.pop())  # the newest makes room for the oldest
            else:
                self._retire(self.running.popleft(), "aborted:out_of_kv_blocks")
                return

    def _take_prefills(self, batch: ModelBatch) -> None:
        bm = self.block_manager
        tokens = self.config.max_num_batched_tokens - len(batch.decode)
        seqs = self._seq_cap.value - len(batch.decode)
        while seqs > 0 and self.waiting_prefill:
            head = self.waiting_prefill[0]
            # len(head) bounds the query length (a prefix-cache hit only shortens it):
            # checked before allocating, so blocks are never taken only to be returned
            if len(head) > tokens:
                return
            if not bm.can_ever_allocate(head):
                # no amount of waiting frees enough blocks: end it instead of stalling
                self._retire(self.waiting_prefill.popleft(), "aborted:kv_cache_too_small")
                continue
            if not bm.can_allocate(head):
                return
            self.waiting_prefill.popleft()
            bm.allocate(head)
            batch.prefill.append(head)
            tokens -= head.num_tokens_to_compute
            seqs -= 1

    def schedule_model(self) -> ModelBatch:
        """The next decoder step: running decodes first, then prefills."""
        batch = ModelBatch()
        self._take_decodes(batch)
        self._take_prefills(batch)
        if batch:
            s = self.stats
            s.num_model_steps += 1
            s.num_mixed_steps += int(bool(batch.prefill and batch.decode))
            s.num_prefilled_tokens += sum(r.num_tokens_to_compute for r in batch.prefill)
            s.num_decoded_tokens += len(batch.decode)
        return batch

    # ---------------------------------------------------------------- recovery

    def on_model_oom(self, batch: ModelBatch) -> None:
        """Undo a decoder step that ran out of memory (nothing in it was mutated: tokens
        and block growth happen in ``postprocess``) and cut the sequence cap."""
        self.stats.num_model_ooms += 1
        for request in reversed(batch.prefill):  # newest first: the free list's order
            self.block_manager.deallocate(request)
            request.num_computed_tokens = 0
        self.waiting_prefill.extendleft(reversed(batch.prefill))
        self.running.extendleft(reversed(batch.decode))
        attempted = len(batch.prefill) + len(batch.decode)
        if attempted > 1:
            self._seq_cap.cut_to(attempted // 2)
            return
        self._seq_cap.cut_to(1)  # nothing left to shrink: give one request up
        if self.running:
            self._retire(self.running.pop(), "aborted:out_of_memory")
        elif self.waiting_prefill:
            self._retire(self.waiting_prefill.popleft(), "aborted:out_of_memory")

    def on_audio_oom(self, requests: list[AsrRequest]) -> None:
        """Undo an encoder call that ran out of memory and cut the frame cap."""
        self.stats.num_audio_ooms += 1
        for request in requests:
            request.timings.encode_start = None
            request.audio_embeds = None
        self.waiting_encode.extendleft(reversed(requests))
        if len(requests) > 1:
            self._frame_cap.cut_to(sum(r.features.mel_frames for r in requests) // 2)
        else:  # one recording alone does not fit: no cap can help it
            self._retire(self.waiting_encode.popleft(), "aborted:out_of_memory")

    def relax_limits(self) -> None:
        self._seq_cap.relax()
        self._frame_cap.relax()

    # ----------------------------------------------------------------- results

    def _record(self, request: AsrRequest, token_id: int) -> bool:
        """Append one sampled token; returns whether the request ended with it."""
        request.num_computed_tokens = len(request)
        request.append_token(token_id)
        if request.stage is RequestStage.WAITING_PREFILL:
            request.mark_prefilled()
        if request.cancel_requested:
            request.finish("cancelled")
            return True
        return request.check_finished()

    def _record_run(self, request: AsrRequest, run) -> bool:
        """``_record`` of each token of ``run`` in turn, stopping at the first that ends
        the request (the rest are dropped). A decoding request that no cancel has
        reached takes them in one append: the first ending token is the first stop
        token (unless ignored) or the one that reaches the output cap, whichever
        comes first -- a stop token at the cap ends it as "stop", as
        ``check_finished`` rules."""
        if request.cancel_requested or request.stage is not RequestStage.RUNNING_DECODE:
            return any(self._record(request, token) for token in run)
        ids = request.token_ids
        sampling = request.sampling
        end = sampling.max_new_tokens - (len(ids) - request.num_prompt_tokens) - 1
        end = max(end, 0)  # index of the token that reaches the cap
        reason = "length"
        if not sampling.ignore_eos:
            stops = request.stop_token_ids
            for k, token in enumerate(run):
                if token in stops:
                    if k <= end:
                        end, reason = k, "stop"
                    break
        if end >= len(run):
            ids.extend(run)
            request.num_computed_tokens = len(ids) - 1
            return False
        ids.extend(run[:end + 1])
        request.num_computed_tokens = len(ids) - 1
        request.finish(reason)
        return True

    def postprocess(self, batch: ModelBatch, token_ids: list[int]) -> list[AsrRequest]:
        """Apply one step's sampled tokens (one per request, batch order); the requests
        that ended are returned, the others go back to ``running`` with room for
        their next token."""
        requests = batch.requests
        if len(token_ids) != len(requests):
            raise ValueError(f"sampler returned {len(token_ids)} tokens for {len(requests)} requests")
        finished: list[AsrRequest] = []
        for request, token in zip(requests, token_ids):
            if self._record_run(request, (token,)):
                self._release_finished(request)
                finished.append(request)
            else:
                self.block_manager.may_append(request)
                self.running.append(request)
        return finished

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
        lengths = []
        for r in batch.decode:
            if r.cancel_requested:
                return 1
            n = len(r.token_ids)
            lengths.append(n)
            steps = min(steps, r.sampling.max_new_tokens - (n - r.num_prompt_tokens),
                        max_model_len - n + 1)
        if steps <= 1:
            return 1
        bm = self.block_manager
        bs = bm.block_size
        # BlockManager.blocks_ahead of every request, without re-measuring them
        ahead = [(r, -(-(n + steps - 1) // bs) - len(r.block_table))
                 for r, n in zip(batch.decode, lengths)]
        ahead = [(r, k) for r, k in ahead if k > 0]
        if sum(k for _, k in ahead) > bm.num_free_blocks:
            return 1
        for r, _ in ahead:
            bm.append_ahead(r, steps)
        return steps

    def postprocess_steps(self, batch: ModelBatch, tokens: list[list[int]]) -> list[AsrRequest]:
        """``postprocess`` for several decode steps of a decode-only batch: tokens[k][i] is
        request i's token of step k; a request stops at its first ending token and its
        later tokens are dropped."""
        requests = batch.decode
        if batch.prefill or any(len(step) != len(requests) for step in tokens):
            raise ValueError("multi-step results do not match the decode batch")
        finished: list[AsrRequest] = []
        may_append = self.block_manager.may_append
        for request, run in zip(requests, zip(*tokens)):
            if self._record_run(request, run):
                self._release_finished(request)
                finished.append(request)
            else:
                may_append(request)
                self.running.append(request)
        extra = len(tokens) - 1
        self.stats.num_model_steps += extra
        self.stats.num_decoded_tokens += extra * len(requests)
        return finished
