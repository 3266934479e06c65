"""Gated DeltaNet layer (drop-in for ``myvllm.layers.linear_attention.GatedDeltaNet``).

Constructor and ``forward(x, cu_seqlens, conv_state_indices, recurrent_state_indices,
is_prefill)`` as in the reference (``m/layers/linear_attention.py:15-123``), with the data
flow the reference intends:

    qkv, z, a, b = in_proj_qkv(x), in_proj_z(x), in_proj_a(x), in_proj_b(x)
    beta = sigmoid(b);  g = -exp(A_log) * softplus(a + dt_bias)          (fp32)
    qkv  = causal_conv1d_fn / causal_conv1d_update (qkv)                  (+ SiLU)
    o    = chunk_gated_delta_rule / recurrent_gated_delta_rule (q, k, v)  (q, k L2-normalised
                                                                        inside the kernel)
    out  = out_proj(RMSNormGated(o, z))                                   (all_reduce at TP > 1)

The reference convolves ``x`` instead of ``qkv`` (``:93, :95``) and projects ``z`` instead of
the normalised output (``:122``); both are fixed here.  ``conv_state`` and
``recurrent_state`` are attributes the caller points at its cache, as in the reference
(``:74-75``): ``[S_max, W-1, conv_dim]`` and ``[S_max, Hv, K, V]`` (fp32) for this rank.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch
import torch.nn.functional as F
from torch import nn

from ..ops.causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from ..ops.gated_delta_rule.fused_layer import (fused_decode_supported, fused_prefill_supported,
                                                 gated_deltanet_decode, gated_deltanet_prefill)
from ..ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule, recurrent_gated_delta_rule
from .linear import ColumnParallelLinear, QKVParallelLinear, RowParallelLinear, tp_rank_size
from .norm import RMSNormGated


class GatedDeltaNet(nn.Module):
    def __init__(self, hidden_size: int, num_k_heads: int, num_v_heads: int, k_head_dim: int, v_head_dim: int,
                 conv_kernel_size: int, act_fn: Callable[[torch.Tensor], torch.Tensor] = F.silu,
                 rms_norm_eps: float = 1e-06) -> None:
        super().__init__()
        self.tp_rank, self.tp_size = tp_rank_size()
        assert num_k_heads % self.tp_size == 0 and num_v_heads % self.tp_size == 0
        self.hidden_size = hidden_size
        self.total_num_k_heads, self.total_num_v_heads = num_k_heads, num_v_heads
        self.num_k_heads = num_k_heads // self.tp_size
        self.num_v_heads = num_v_heads // self.tp_size
        self.k_head_dim, self.v_head_dim = k_head_dim, v_head_dim
        self.total_k_size, self.total_v_size = k_head_dim * num_k_heads, v_head_dim * num_v_heads
        self.k_size, self.v_size = k_head_dim * self.num_k_heads, v_head_dim * self.num_v_heads
        self.conv_kernel_size = conv_kernel_size
        self.act_fn = act_fn  # SiLU is fused into the conv kernel (the reference's kernel hardcodes it too)
        self.rms_norm_eps = rms_norm_eps
        self.conv1d = QKVParallelLinear(conv_kernel_size, k_head_dim, k_head_dim, v_head_dim, num_k_heads,
                                        num_k_heads, num_v_heads)  # weight [conv_dim (this rank), W]
        self.dt_bias = nn.Parameter(torch.ones(self.num_v_heads))
        # A_log ~ U(0, ln 16): the reference draws log(U(0, 16)) (:58), which can be -inf
        self.A_log = nn.Parameter(torch.empty(self.num_v_heads).uniform_(0, math.log(16)))
        self.norm = RMSNormGated((self.v_head_dim,), self.rms_norm_eps)
        self.out_proj = RowParallelLinear(self.total_v_size, hidden_size, bias=False)
        self.in_proj_qkv = QKVParallelLinear(hidden_size, k_head_dim, k_head_dim, v_head_dim, num_k_heads,
                                             num_k_heads, num_v_heads, bias=False)
        self.in_proj_z = ColumnParallelLinear(hidden_size, self.total_v_size, bias=False)
        self.in_proj_b = ColumnParallelLinear(hidden_size, num_v_heads, bias=False)
        self.in_proj_a = ColumnParallelLinear(hidden_size, num_v_heads, bias=False)
        self.recurrent_state: torch.Tensor = torch.empty(0)
        self.conv_state: torch.Tensor = torch.empty(0)
        # decode through the one-kernel layer step (mvb_gated_deltanet_decode) instead of the
        # conv-update, recurrence and gated-norm kernels
        self.fused_decode = False

    def gates(self, a: torch.Tensor, b: torch.Tensor):
        """The layer's gate math in torch (the kernels form the same gates in-kernel from
        ``gate_inputs``; this is kept for callers of the unfused ops)."""
        beta = b.sigmoid()
        g = -self.A_log.float().exp() * F.softplus(a.float() + self.dt_bias.float())
        return g, beta

    def fuse_projections(self) -> None:
        """Concatenate the four input projections of this rank into one weight, so a forward
        runs one GEMM instead of four.  Call after the weights are loaded (like vLLM's
        post-load weight processing); the forward then slices q|k|v, z, a, b out of one
        output without copies.  Re-run after changing the projection weights."""
        ws = [self.in_proj_qkv.weight, self.in_proj_z.weight, self.in_proj_a.weight, self.in_proj_b.weight]
        self._w_in = torch.cat([w.detach() for w in ws], 0)
        self._in_split = [w.shape[0] for w in ws]

    def forward(self, x: torch.Tensor, cu_seqlens: torch.Tensor, conv_state_indices: torch.Tensor,
                recurrent_state_indices: torch.Tensor, is_prefill: bool) -> torch.Tensor:
        T = x.shape[0]
        if getattr(self, "_w_in", None) is not None:
            qkv, z, a, b = F.linear(x, self._w_in).split(self._in_split, dim=-1)
        else:
            qkv, z = self.in_proj_qkv(x), self.in_proj_z(x)
            a, b = self.in_proj_a(x), self.in_proj_b(x)
        gate_inputs = (a, b, self.A_log, self.dt_bias)  # g, beta are formed inside the kernel
        zv = z.view(T, self.num_v_heads, self.v_head_dim)
        if not is_prefill and self.fused_decode and fused_decode_supported(qkv, self.recurrent_state,
                                                                           self.num_k_heads, self.num_v_heads, zv):
            # conv update + q/k norm + gates + recurrence + RMSNormGated in one kernel (off by
            # default: the separate kernels stream the state faster at serving batch sizes)
            o = gated_deltanet_decode(qkv, self.conv1d.weight, self.conv_state, conv_state_indices, a, b, self.A_log,
                                      self.dt_bias, self.recurrent_state, recurrent_state_indices, zv,
                                      self.norm.weight, self.norm.variance_epsilon)
            return self.out_proj(o.reshape(T, self.v_size))
        if is_prefill:
            qkv = causal_conv1d_fn(qkv, self.conv1d.weight, self.conv_state, conv_state_indices, cu_seqlens)
        else:
            qkv = causal_conv1d_update(qkv, self.conv1d.weight, self.conv_state, conv_state_indices)
        q, k, v = torch.split(qkv, [self.k_size, self.k_size, self.v_size], dim=-1)
        q = q.view(T, self.num_k_heads, self.k_head_dim)
        k = k.view(T, self.num_k_heads, self.k_head_dim)
        v = v.view(T, self.num_v_heads, self.v_head_dim)
        if is_prefill and fused_prefill_supported(q, k, v, self.recurrent_state, zv):
            # chunked GDN with the gates, the q/k norm and RMSNormGated in the kernel
            o = gated_deltanet_prefill(q, k, v, a, b, self.A_log, self.dt_bias, self.recurrent_state,
                                       recurrent_state_indices, cu_seqlens, zv, self.norm.weight,
                                       self.norm.variance_epsilon)
            return self.out_proj(o.reshape(T, self.v_size))
        if is_prefill:
            o = chunk_gated_delta_rule(q, k, v, None, None, self.recurrent_state, recurrent_state_indices, cu_seqlens,
                                       use_qk_l2norm_in_kernel=True, gate_inputs=gate_inputs)
        else:
            o = recurrent_gated_delta_rule(q, k, v, None, None, self.recurrent_state, recurrent_state_indices,
                                           use_qk_l2norm_in_kernel=True, gate_inputs=gate_inputs)
        o = self.norm(o, zv)
        return self.out_proj(o.reshape(T, self.v_size))
