"""Audio encoding stage (engine/audio_runner.py of the reference).

One encoder call covers every request of the batch; embeddings stay with the
request until it finishes so a preempted request re-prefills without re-encoding.
"""

from __future__ import annotations

import torch

from voiceagent_b200.audio.batcher import pack_audio_batch
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.request import AsrRequest


class AudioRunner:
    def __init__(self, model, config: EngineConfig):
        self.model = model
        self.config = config
        self.device = torch.device(config.device)
        self.n_window_infer = config.model_config.audio.n_window_infer
        self.renderer = None  # GpuMelFrontend when requests defer their mel to the GPU

    @torch.inference_mode()
    def encode(self, requests: list[AsrRequest]) -> None:
        if not requests:
            return
        batch = pack_audio_batch([r.features for r in requests],
                                 n_window_infer=self.n_window_infer, device=self.device,
                                 renderer=self.renderer)
        embeddings = self.model.encode_audio(batch)
        for request, embeds in zip(requests, embeddings):
            if embeds.size(0) != request.layout.audio_length:
                raise RuntimeError(f"request {request.request_id}: encoder produced "
                                   f"{embeds.size(0)} audio tokens but the prompt reserved "
                                   f"{request.layout.audio_length}")
            request.audio_embeds = embeds
            request.mark_encoding()
