"""AsrEngine: the public API of the ragged continuous-batching path.

Keeps the reference's interface and loop (engine/engine.py:70-627): ``add_request``
/ ``prepare_request`` / ``admit``, ``step`` (one audio-encode batch + one decoder
batch), ``transcribe`` (order-preserving, bounded admission, progress watchdog),
``cancel``, OOM rollback, stage profiling. Underneath, every hot-path operation runs
on the b200asr sm_100a kernels and decode steps replay whole-step CUDA graphs.
"""

from __future__ import annotations

import itertools
import logging
import time
from dataclasses import dataclass, field
from typing import Iterable, Sequence

import numpy as np
import torch

from voiceagent_b200 import kernels as kx
from voiceagent_b200.audio.frontend import AudioFeatures, AudioFrontend, GpuMelFrontend
from voiceagent_b200.audio.tokens import num_audio_tokens
from voiceagent_b200.checkpoint import random_state_dict
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.audio_runner import AudioRunner
from voiceagent_b200.engine.block_manager import BlockManager
from voiceagent_b200.engine.model_runner import ModelRunner
from voiceagent_b200.engine.request import AsrRequest, RequestTimings, SamplingParams
from voiceagent_b200.engine.scheduler import Scheduler
from voiceagent_b200.loader import load_tensors, load_weights
from voiceagent_b200.profiling import StageTimer
from voiceagent_b200.prompt import PromptBuilder, normalize_language
from voiceagent_b200.qwen3_asr.model import Qwen3ASRForConditionalGeneration

logger = logging.getLogger(__name__)
OutOfMemoryError = getattr(torch, "OutOfMemoryError", torch.cuda.OutOfMemoryError)


@dataclass
class AsrOutput:
    request_id: int
    text: str
    language: str
    raw_text: str
    audio_seconds: float
    num_prompt_tokens: int
    num_audio_tokens: int
    num_output_tokens: int
    finish_reason: str | None
    timings: RequestTimings = field(default_factory=RequestTimings)
    output_token_ids: list[int] = field(default_factory=list)


class AsrEngine:
    """``AsrEngine(model_dir, **engine_config_kwargs)`` or ``AsrEngine(config=...)``.

    Weights: ``weights="checkpoint"`` loads ``model_dir``'s safetensors,
    ``weights="random"`` builds the seeded random-init tensors of
    ``voiceagent_b200.checkpoint`` directly on the device (same values the checkpoint
    writer would save), ``"auto"`` picks the former when safetensors exist.
    """

    def __init__(self, model: str | None = None, config: EngineConfig | None = None, *,
                 weights: str = "auto", seed: int = 0, **kwargs):
        if (model is None) == (config is None):
            raise ValueError("pass exactly one of model or config")
        self.config = config or EngineConfig(model=model, **kwargs)
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is unavailable: the b200asr kernels need a B200 (sm_100a)")
        device = torch.device(self.config.device)
        if device.type == "cuda" and device.index is not None:
            torch.cuda.set_device(device)
        self._limit_frontend_threads()
        kx.set_pdl(self.config.pdl)  # before any graph capture
        if self.config.frontend == "gpu":
            self.frontend = GpuMelFrontend(self.config.model, device=device)
        else:
            self.frontend = AudioFrontend(self.config.model)
        self.prompt_builder = PromptBuilder(self.config.model_config.audio_token_id,
                                            self.config.model_config.stop_token_ids
                                            or (151643, 151645))
        self.model = self._build_model(weights, seed)
        self.model.model.fused_decode = self.config.fused_decode
        self.model.model.l2_prefetch = self.config.l2_prefetch
        self.model_runner = ModelRunner(self.model, self.config)
        num_blocks = self.model_runner.determine_num_blocks()
        self.model_runner.allocate_kv_cache(num_blocks)
        self.model_runner.capture_graphs()
        self.num_kvcache_blocks = num_blocks
        self.audio_runner = AudioRunner(self.model, self.config)
        self.model.audio_tower.warm_up()
        if isinstance(self.frontend, GpuMelFrontend):
            self.audio_runner.renderer = self.frontend
            self.model_runner.host_work = self._stage_upcoming_audio
        self.block_manager = BlockManager(num_blocks, self.config.kvcache_block_size,
                                          self.config.enable_prefix_cache)
        self.scheduler = Scheduler(self.config, self.block_manager)
        self.stage_seconds = {"frontend": 0.0, "audio_encode": 0.0, "model_step": 0.0}
        logger.info("engine ready: kv_blocks=%d (%.1f GiB) max_num_seqs=%d max_model_len=%d",
                    num_blocks, num_blocks * self.model_runner.kv_cache_bytes_per_block() / 2**30,
                    self.config.max_num_seqs, self.config.max_model_len)

    # ------------------------------------------------------------ set-up

    def _build_model(self, weights: str, seed: int) -> Qwen3ASRForConditionalGeneration:
        torch.set_default_dtype(self.config.dtype)
        try:
            with torch.device(self.config.device):
                model = Qwen3ASRForConditionalGeneration(self.config.model_config,
                                                         self.config.max_model_len)
        finally:
            torch.set_default_dtype(torch.float32)
        import glob
        import os

        has_ckpt = bool(glob.glob(os.path.join(self.config.model, "*.safetensors")))
        if weights == "checkpoint" or (weights == "auto" and has_ckpt):
            load_weights(model, self.config.model)
        elif weights in ("random", "auto"):
            cfg = self.config.model_config
            preset = {"audio": vars(cfg.audio), "text": vars(cfg.text)}
            load_tensors(model, random_state_dict(preset, seed).items(), prefixed=False)
        else:
            raise ValueError(f"unknown weights source {weights!r}")
        return model.eval()

    def _limit_frontend_threads(self) -> None:
        wanted = self.config.frontend_threads
        if wanted > 0 and torch.get_num_threads() > wanted:
            torch.set_num_threads(wanted)

    def enable_stage_profiling(self) -> StageTimer:
        timer = StageTimer(enabled=True)
        self.model_runner.timer = timer
        return timer

    def kv_bytes_for(self, num_tokens: int) -> int:
        t = self.config.model_config.text
        return 2 * t.num_hidden_layers * num_tokens * t.num_key_value_heads * t.head_dim * 2

    # ---------------------------------------------------------- requests

    def prepare_request(self, waveform: np.ndarray, sample_rate: int = 16000,
                        context: str | list[int] = "", language: str | None = None,
                        sampling: SamplingParams | None = None) -> AsrRequest:
        """Mel features + prompt layout; touches no engine state (thread-safe)."""
        started = time.perf_counter()
        features = self.frontend(waveform, sample_rate)
        self.stage_seconds["frontend"] += time.perf_counter() - started
        return self.prepare_request_from_features(features, context, language, sampling)

    def prepare_request_from_features(self, features: AudioFeatures,
                                      context: str | list[int] = "", language: str | None = None,
                                      sampling: SamplingParams | None = None) -> AsrRequest:
        """Build a request from precomputed mel features (which may already be on the
        GPU -- the encoder then reads them in place)."""
        lang = normalize_language(language)
        layout = self.prompt_builder.build(features.num_audio_tokens, context=context, language=lang)
        if len(layout) > self.config.max_model_len:
            raise ValueError(f"prompt needs {len(layout)} tokens but max_model_len is "
                             f"{self.config.max_model_len}")
        return AsrRequest(features=features, layout=layout, sampling=sampling or SamplingParams(),
                          block_size=self.config.kvcache_block_size,
                          stop_token_ids=self.prompt_builder.stop_token_ids, language=lang)

    def admit(self, request: AsrRequest) -> AsrRequest:
        self.scheduler.add(request)
        return request

    def add_request(self, waveform: np.ndarray, sample_rate: int = 16000,
                    context: str | list[int] = "", language: str | None = None,
                    sampling: SamplingParams | None = None) -> AsrRequest:
        return self.admit(self.prepare_request(waveform, sample_rate, context, language, sampling))

    def cancel(self, request_id: int) -> bool:
        return self.scheduler.cancel(request_id)

    def _finalize(self, request: AsrRequest) -> AsrOutput:
        ids = request.output_token_ids
        if ids and ids[-1] in request.stop_token_ids and not request.sampling.ignore_eos:
            ids = ids[:-1]
        raw = self.prompt_builder.decode(ids)
        return AsrOutput(request_id=request.request_id, text=raw, language=request.language or "",
                         raw_text=raw, audio_seconds=request.features.audio_seconds,
                         num_prompt_tokens=request.num_prompt_tokens,
                         num_audio_tokens=request.layout.audio_length, num_output_tokens=len(ids),
                         finish_reason=request.finish_reason, timings=request.timings,
                         output_token_ids=list(ids))

    def _stage_upcoming_audio(self, budget_seconds: float) -> None:
        """While a decoder call runs on the GPU: copy the waveforms of the requests at the
        head of the encode queue (the next encoder call's, at most one call's worth) into
        pinned memory, so that call's host-to-device copy needs no host copy first. Stops
        once ``budget_seconds`` of host time are spent (the rest waits for the next call)."""
        deadline = time.perf_counter() + budget_seconds
        stage = self.audio_runner.renderer.stage
        for request in itertools.islice(self.scheduler.waiting_encode,
                                        self.config.max_audio_batch_size):
            if stage(request.features) and time.perf_counter() >= deadline:
                return

    # -------------------------------------------------------------- loop

    def step(self) -> list[AsrOutput]:
        encode_batch = self.scheduler.schedule_audio()
        if encode_batch:
            started = time.perf_counter()
            try:
                # No host sync: the embeddings stay on the device and everything that
                # reads them runs later on the same stream, so the host goes on to
                # schedule and launch the next work while the encoder still runs.
                self.audio_runner.encode(encode_batch)
            except OutOfMemoryError:
                logger.warning("audio encode ran out of memory on %d requests; rolling back",
                               len(encode_batch))
                self._recover_from_oom()
                self.scheduler.on_audio_oom(encode_batch)
            else:
                self.scheduler.admit_prefill(encode_batch)
            self.stage_seconds["audio_encode"] += time.perf_counter() - started

        finished: list[AsrRequest] = []
        batch = self.scheduler.schedule_model()
        if batch:
            started = time.perf_counter()
            steps = 1
            if self.model_runner.can_use_graph(batch):
                steps = self.scheduler.decode_steps_for(batch, self.model_runner.max_decode_steps,
                                                        self.config.max_model_len)
            try:
                if steps > 1:
                    tokens = self.model_runner.run_steps(batch, steps)
                else:
                    token_ids = self.model_runner.run(batch)
            except OutOfMemoryError:
                logger.warning("decoder step ran out of memory on %d requests; rolling back",
                               len(batch.requests))
                self._recover_from_oom()
                self.scheduler.on_model_oom(batch)
            else:
                if steps > 1:
                    finished = self.scheduler.postprocess_steps(batch, tokens)
                else:
                    finished = self.scheduler.postprocess(batch, token_ids)
                self.scheduler.relax_limits()
            self.stage_seconds["model_step"] += time.perf_counter() - started
        return [self._finalize(r) for r in self.scheduler.drain_aborted() + finished]

    @staticmethod
    def _recover_from_oom() -> None:
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    def transcribe(self, audios: Sequence[np.ndarray] | Iterable[np.ndarray], sample_rate: int = 16000,
                   context: str | list[int] = "", language: str | None = None,
                   sampling: SamplingParams | None = None, features: bool = False) -> list[AsrOutput]:
        """Transcribe a batch in input order.

        Requests are admitted a few batches ahead of the scheduler (at most
        ``max(4 * max_num_seqs, max_audio_batch_size)`` in flight). With
        ``features=True`` the items are :class:`AudioFeatures` instead of waveforms.
        """
        source = iter(audios)
        limit = max(self.config.max_num_seqs * 4, self.config.max_audio_batch_size)
        order: dict[int, int] = {}
        results: dict[int, AsrOutput] = {}
        pending: set[int] = set()
        exhausted = False
        next_index = 0
        while pending or not exhausted:
            while not exhausted and self.scheduler.num_in_flight < limit:
                try:
                    item = next(source)
                except StopIteration:
                    exhausted = True
                    break
                if features:
                    request = self.admit(self.prepare_request_from_features(
                        item, context=context, language=language, sampling=sampling))
                else:
                    request = self.add_request(item, sample_rate, context, language, sampling)
                order[request.request_id] = next_index
                pending.add(request.request_id)
                next_index += 1
            if not self.scheduler.has_work:
                if pending:
                    raise RuntimeError(f"{len(pending)} requests are unaccounted for but the "
                                       "scheduler has no work left")
                continue
            before = (self.scheduler.stats.num_model_steps, self.scheduler.stats.num_encode_batches)
            outputs = self.step()
            after = (self.scheduler.stats.num_model_steps, self.scheduler.stats.num_encode_batches)
            if not outputs and before == after:
                raise RuntimeError(f"scheduler is not making progress with "
                                   f"{self.scheduler.num_in_flight} requests in flight")
            for out in outputs:
                idx = order.get(out.request_id)
                if idx is None:
                    continue
                results[idx] = out
                pending.discard(out.request_id)
        self.model_runner.check_device_errors()
        return [results[i] for i in range(next_index)]


def features_from_mel(mel: torch.Tensor, audio_seconds: float | None = None) -> AudioFeatures:
    """Wrap a (bins, frames) mel tensor (host or device) as request features."""
    frames = int(mel.shape[-1])
    return AudioFeatures(mel=mel, mel_frames=frames, num_audio_tokens=num_audio_tokens(frames),
                         audio_seconds=audio_seconds if audio_seconds is not None else frames / 100.0)
