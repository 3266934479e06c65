"""Norms (drop-in for ``myvllm.layers.norm``, reference ``m/layers/norm.py:6-88``).

``RMSNormGated`` -- the GDN output norm, on the decode and prefill hot path -- runs the
library's fused CUDA kernel (``mvb_rmsnorm_gated``) for CUDA bf16/fp16 rows.  ``RMSNorm``
(q/k norms of full attention, pre-norms) and ``LayerNorm`` keep the reference's eager
math (the reference ``torch.compile``s them).
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _lib


class RMSNorm(nn.Module):
    def __init__(self, normalized_shape: tuple[int, ...], eps: float = 1e-5, zero_centered_gamma=False):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.eps = eps
        self.zero_centered_gamma = zero_centered_gamma

    @property
    def gamma(self):
        return self.weight

    def rms_forward(self, x: torch.Tensor) -> torch.Tensor:
        weight = self.weight.to(torch.float32)
        if self.zero_centered_gamma:
            weight = weight + 1.0
        xf = x.to(torch.float32)
        y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps) * weight
        return y.to(x.dtype)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        """Returns ``rms(x)`` (the reference returns ``(rms(x), x)`` without a residual,
        ``norm.py:40``, which no caller uses; with a residual, ``(rms(x + r), x + r)``)."""
        if residual is not None:
            x = x + residual
            return self.rms_forward(x), x
        return self.rms_forward(x)


class RMSNormGated(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight * silu(gate), over the last dim."""

    def __init__(self, normalized_shape: tuple[int, ...], eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda("RMSNormGated", x, gate, self.weight)
        d = x.shape[-1]
        xs = x.reshape(-1, d)
        gs = gate.reshape(-1, d)
        out = torch.empty(xs.shape, dtype=x.dtype, device=x.device)
        _lib.call("RMSNormGated", "mvb_rmsnorm_gated", _lib.desc(xs), _lib.desc(gs), _lib.desc(self.weight.detach()),
                  float(self.variance_epsilon), _lib.desc(out), _lib.stream_of(x))
        return out.view(x.shape)


class LayerNorm(nn.Module):
    def __init__(self, normalized_shape: tuple[int, ...], eps: float = 1e-05) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.bias = nn.Parameter(torch.zeros(normalized_shape))
        self.eps = eps

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is not None:
            x = x + residual
        xf = x.to(torch.float32)
        mu = xf.mean(-1, keepdim=True)
        var = (xf - mu).pow(2).mean(-1, keepdim=True)
        y = (xf - mu) * torch.rsqrt(var + self.eps) * self.weight.float() + self.bias.float()
        return y.to(x.dtype), x
