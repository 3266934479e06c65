"""Causal depthwise conv1d ops (drop-in for ``myvllm.ops.causal_conv1d``).

Same signatures as the reference (``m/ops/causal_conv1d.py:221-227, 434-439``);
the work runs in ``mvb_causal_conv1d_fn`` / ``mvb_causal_conv1d_update``.
Layouts: x [T, dim]; weight [dim, W]; conv_state [S_max, W-1, dim], updated in place
at ``conv_state_indices``; cu_seqlens [S+1] int32.  Unlike the reference wrapper
(``:230``) there is no host synchronisation: tiles are mapped to sequences on device.
"""

from __future__ import annotations

import torch

from .. import _lib


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 else t.to(torch.int32)


def _weight(weight: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    # nn.Linear-style [dim, W] parameters may arrive as [dim, 1, W] (conv layout)
    if weight.dim() == 3 and weight.shape[1] == 1:
        weight = weight[:, 0]
    if weight.dtype not in (torch.float32, x.dtype):
        weight = weight.to(x.dtype)
    return weight


def causal_conv1d_fn(
    x: torch.Tensor,  # (total_tokens, dim)
    weight: torch.Tensor,  # (dim, kernel_size)
    conv_state: torch.Tensor,  # (max_seq_cnt, kernel_size - 1, dim)
    conv_state_indices: torch.Tensor,  # (seq_cnt,)
    cu_seqlens: torch.Tensor,  # (seq_cnt + 1,)
    activation: bool = True,
) -> torch.Tensor:
    _lib.require_cuda("causal_conv1d_fn", x, weight, conv_state, conv_state_indices, cu_seqlens)
    weight = _weight(weight, x)
    idx, cu = _i32(conv_state_indices), _i32(cu_seqlens)
    o = torch.empty_like(x, memory_format=torch.contiguous_format)
    _lib.call("causal_conv1d_fn", "mvb_causal_conv1d_fn", _lib.desc(x), _lib.desc(weight), _lib.desc(conv_state),
              _lib.desc(idx), _lib.desc(cu), _lib.desc(o), int(activation), _lib.stream_of(x))
    return o


def causal_conv1d_update(
    x: torch.Tensor,  # (seq_cnt, dim)
    weight: torch.Tensor,  # (dim, kernel_size)
    conv_state: torch.Tensor,  # (max_seq_cnt, kernel_size - 1, dim)
    conv_state_indices: torch.Tensor,  # (seq_cnt,)
    activation: bool = True,
) -> torch.Tensor:
    _lib.require_cuda("causal_conv1d_update", x, weight, conv_state, conv_state_indices)
    weight = _weight(weight, x)
    idx = _i32(conv_state_indices)
    o = torch.empty_like(x, memory_format=torch.contiguous_format)
    _lib.call("causal_conv1d_update", "mvb_causal_conv1d_update", _lib.desc(x), _lib.desc(weight),
              _lib.desc(conv_state), _lib.desc(idx), _lib.desc(o), int(activation), _lib.stream_of(x))
    return o
