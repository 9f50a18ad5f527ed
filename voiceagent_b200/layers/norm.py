"""RMSNorm, SiLU-and-multiply and the RoPE table on the b200asr kernels."""

from __future__ import annotations

import torch
from torch import nn

from voiceagent_b200 import kernels as kx


class RMSNorm(nn.Module):
    """RMS norm with an optional fused residual add (layers/layernorm.py:7-43).

    ``forward(x)`` returns the norm; ``forward(x, residual)`` returns
    ``(norm(x + residual), x + residual)`` and writes the sum into ``residual``'s
    storage (the returned residual is that same tensor).
    """

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return kx.rmsnorm(x, self.weight, self.eps)
        out = kx.rmsnorm(x, self.weight, self.eps, residual=residual)
        return out, residual


class SiluAndMul(nn.Module):
    """SwiGLU over a fused ``gate_up`` projection (layers/activation.py:8-14)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return kx.silu_mul(x)


def rope_table(head_dim: int, max_position: int, base: float, device) -> torch.Tensor:
    """fp32 [max_position, head_dim] table of [cos | sin] (rotary_embedding.py:17-25),
    computed with the same torch ops on the engine's device as the reference."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float, device=device)
                               / head_dim))
    positions = torch.arange(max_position, dtype=torch.float, device=device)
    freqs = torch.einsum("i,j->ij", positions, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).contiguous()
