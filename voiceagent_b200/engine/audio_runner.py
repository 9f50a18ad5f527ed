"""The audio-encode stage of a step: one packed encoder call for a batch of requests.

The scheduler picks the batch (``Scheduler.schedule_audio``); this packs the requests'
log-mel features into the encoder's ragged layout (``audio.batcher.pack_audio_batch``,
rendering deferred GPU log-mel on the way), runs the audio tower once, and hands each
request its slice of the output. Each slice must have exactly the number of audio
positions the request's prompt reserved, since prefill scatters it into those
positions. The embeddings then stay with the request until it finishes, so a preempted
request is prefilled again without being re-encoded. (Counterpart of the reference's
engine/audio_runner.py.)
"""

from __future__ import annotations

import torch

from voiceagent_b200.audio.batcher import pack_audio_batch
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.request import AsrRequest


class AudioRunner:
    def __init__(self, model, config: EngineConfig):
        self.model = model
        self.device = torch.device(config.device)
        self.window_frames = config.model_config.audio.n_window_infer
        self.renderer = None  # the GPU log-mel frontend, when features are rendered on device
        self.config = config

    @torch.inference_mode()
    def encode(self, requests: list[AsrRequest]) -> None:
        """Encode ``requests`` in one call and attach each one's embeddings."""
        if not requests:
            return
        packed = pack_audio_batch([r.features for r in requests], n_window_infer=self.window_frames,
                                  device=self.device, renderer=self.renderer)
        outputs = self.model.encode_audio(packed)
        wrong = [(r.request_id, int(e.shape[0]), r.layout.audio_length)
                 for r, e in zip(requests, outputs) if e.shape[0] != r.layout.audio_length]
        if wrong:
            rid, got, want = wrong[0]
            raise RuntimeError(f"audio encoder output does not fit the prompt: request {rid} has "
                               f"{want} audio positions, the encoder returned {got} embeddings")
        for request, embeds in zip(requests, outputs):
            request.audio_embeds = embeds
            request.mark_encoding()
