"""Greedy or temperature sampling (layers/sampler.py:9-27).

The greedy result always comes from the b200asr argmax kernel; the Gumbel-max
temperature branch (rare for ASR) replaces it only for rows that asked for it.
"""

from __future__ import annotations

import torch
from torch import nn

from voiceagent_b200 import kernels as kx

GREEDY_TEMPERATURE_EPS = 1e-4


class Sampler(nn.Module):
    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        greedy = kx.greedy_argmax(logits, out=out)
        if temperatures is None or bool((temperatures < GREEDY_TEMPERATURE_EPS).all()):
            return greedy
        scaled = logits.float() / temperatures.clamp_min(GREEDY_TEMPERATURE_EPS).unsqueeze(-1)
        probs = torch.softmax(scaled, dim=-1)
        noise = torch.empty_like(probs).exponential_(1.0)
        sampled = probs.div_(noise).argmax(dim=-1)
        return torch.where(temperatures < GREEDY_TEMPERATURE_EPS, greedy, sampled)
