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


def _rows(x: torch.Tensor):
    """x [..., d] as a 2-D [rows, d] view with one row stride (no copy), or None."""
    if x.dim() < 2 or x.stride(-1) != 1:
        return None
    stride = x.stride(-2)
    for i in range(x.dim() - 2):
        if x.shape[i + 1] > 1 and x.stride(i) != x.stride(i + 1) * x.shape[i + 1]:
            return None
    rows = x.numel() // x.shape[-1]
    return torch.as_strided(x, (rows, x.shape[-1]), (stride, 1))


class RMSNorm(nn.Module):
    def __init__(self, normalized_shape: tuple[int, ...], eps: float = 1e-5, zero_centered_gamma=False):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.eps = eps
        self.zero_centered_gamma = zero_centered_gamma

    @property
    def gamma(self):
        return self.weight

    def rms_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """One fused kernel on CUDA bf16/fp16 tensors (``mvb_rmsnorm``); eager fp32 math
        otherwise (CPU tensors, fp32)."""
        d = x.shape[-1]
        xs = _rows(x)
        if xs is None and x.dim() == 3 and x.stride(-1) == 1 and residual is None:
            xs = x  # [T, H, D] with two row strides (e.g. a head view of a fused projection)
        if x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and d % 8 == 0 and d <= 2048 and \
                xs is not None and (residual is None or residual.is_contiguous()):
            out = torch.empty(xs.shape, dtype=x.dtype, device=x.device)
            res = _lib.desc(residual.view(-1, d)) if residual is not None else None
            _lib.call("RMSNorm", "mvb_rmsnorm", _lib.desc(xs), res, _lib.desc(self.weight.detach()), float(self.eps),
                      int(self.zero_centered_gamma), _lib.desc(out), _lib.stream_of(x))
            return out.view(x.shape)
        if residual is not None:
            residual.copy_(x + residual)
            x = residual
        weight = self.weight.to(torch.float32)
        if self.zero_centered_gamma:
            weight = weight + 1.0
        xf = x.to(torch.float32)
        y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps) * weight
        return y.to(x.dtype)

    def rope_forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """``apply_partial_rotary(rms(x), cos, sin)`` for x [T, H, D] -- the q/k norm and
        rotary of full attention -- in one kernel (``mvb_rmsnorm_rope``) on CUDA 16-bit
        tensors; the two reference steps otherwise."""
        rd = 2 * cos.shape[-1]
        if x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and x.dim() == 3 and x.stride(-1) == 1 and \
                x.shape[-1] % 8 == 0 and x.shape[-1] <= 256 and 16 <= rd <= x.shape[-1] and (rd & (rd - 1)) == 0:
            out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
            c32, s32 = cos.to(torch.float32).contiguous(), sin.to(torch.float32).contiguous()
            _lib.call("RMSNorm.rope", "mvb_rmsnorm_rope", _lib.desc(x), _lib.desc(self.weight.detach()),
                      float(self.eps), int(self.zero_centered_gamma), _lib.desc(c32), _lib.desc(s32), _lib.desc(out),
                      _lib.stream_of(x))
            return out
        from .rotary_embedding import apply_partial_rotary

        return apply_partial_rotary(self.rms_forward(x), cos, sin)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        """``rms(x)``; with ``residual``: ``(rms(x + residual), x + residual)``, the sum also
        written into ``residual`` (the fused pre-norm of a decoder step).  The reference
        returns ``(rms(x), x)`` without a residual (``norm.py:40``), which no caller uses."""
        if residual is not None:
            return self.rms_forward(x, residual), residual
        return self.rms_forward(x)


class RMSNormGated(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight * silu(gate), over the last dim."""

    def __init__(self, normalized_shape: tuple[int, ...], eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        """x, gate [..., D]; a [T, H, D] gate may be a strided view (e.g. a column slice of a
        fused projection) -- the kernel takes two row strides, so it is not copied."""
        _lib.require_cuda("RMSNormGated", x, gate, self.weight)
        d = x.shape[-1]
        if x.dim() == 3 and gate.dim() == 3:
            xs, gs = x, gate
        else:
            xs, gs = x.reshape(-1, d), gate.reshape(-1, d)
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
