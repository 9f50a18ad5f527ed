"""Top-level Qwen3-ASR assembly (models/qwen3_asr.py of the reference).

Audio encoding is a separate pipeline stage: by the time a request reaches the text
decoder its audio embeddings exist and are written into the placeholder span,
whose offset and length were fixed when the prompt was built.
"""

from __future__ import annotations

import torch
from torch import nn

from voiceagent_b200.audio.batcher import PackedAudioBatch
from voiceagent_b200.config import Qwen3ASRConfig
from voiceagent_b200.qwen3_asr.audio_encoder import AudioEncoder
from voiceagent_b200.qwen3_asr.decoder import Qwen3Model, project


class Qwen3ASRForConditionalGeneration(nn.Module):
    def __init__(self, config: Qwen3ASRConfig, max_position: int):
        super().__init__()
        self.config = config
        self.audio_tower = AudioEncoder(config.audio)
        self.model = Qwen3Model(config.text, max_position)
        self.lm_head = nn.Linear(config.text.hidden_size, config.text.vocab_size, bias=False)
        if config.text.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight

    def encode_audio(self, batch: PackedAudioBatch) -> list[torch.Tensor]:
        return batch.split_outputs(self.audio_tower(batch))

    def embed_tokens(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.model.embed_tokens(input_ids)

    @staticmethod
    def scatter_audio_embeddings(inputs_embeds: torch.Tensor,
                                 spans: list[tuple[int, torch.Tensor]]) -> torch.Tensor:
        """Slice-write each (offset, embeddings) pair into the packed batch."""
        for offset, embeds in spans:
            inputs_embeds[offset:offset + embeds.size(0)] = embeds.to(inputs_embeds.dtype)
        return inputs_embeds

    def forward(self, input_ids, positions, inputs_embeds=None) -> torch.Tensor:
        return self.model(input_ids, positions, inputs_embeds=inputs_embeds)

    def compute_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return project(hidden_states, self.lm_head)
