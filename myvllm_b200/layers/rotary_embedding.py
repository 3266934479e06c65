"""Rotary embedding (drop-in for ``myvllm.layers.rotary_embedding``, reference
``m/layers/rotary_embedding.py:6-31``): half-split rotation of the last dim given to it.
With partial rotary (Qwen3.5: 64 of 256 dims), callers rotate ``x[..., :rotary_dim]``;
``apply_partial_rotary`` does that slice."""

from __future__ import annotations

import torch
from torch import nn


class RotaryEmbedding(nn.Module):
    inv_freq: torch.Tensor

    def __init__(self, dim: int, theta: float = 10000.0) -> None:
        super().__init__()
        self.dim = dim
        self.theta = theta
        inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    def forward(self, position_ids: torch.Tensor) -> torch.Tensor:
        """angles [..., dim/2] = position * inv_freq."""
        return position_ids.to(torch.float32)[..., None] * self.inv_freq

    def cos_sin(self, position_ids: torch.Tensor):
        ang = self.forward(position_ids)
        return ang.cos(), ang.sin()


def apply_rotary_pos_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, d]; cos, sin [T, d/2]."""
    cos = cos[:, None, :].to(x.dtype)
    sin = sin[:, None, :].to(x.dtype)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


def apply_partial_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotates the first ``2 * cos.shape[-1]`` dims of the last axis, keeps the rest."""
    rd = 2 * cos.shape[-1]
    if rd == x.shape[-1]:
        return apply_rotary_pos_emb(x, cos, sin)
    return torch.cat((apply_rotary_pos_emb(x[..., :rd], cos, sin), x[..., rd:]), dim=-1)
