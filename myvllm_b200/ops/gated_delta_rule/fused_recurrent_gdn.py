"""Recurrent gated delta rule, one token per sequence (drop-in for
``myvllm.ops.gated_delta_rule.fused_recurrent_gdn``, reference ``:105-166``)."""

from __future__ import annotations

import torch

from ... import _lib


def fused_recurrent_gdn(
    q: torch.Tensor,  # (seq_cnt, num_k_heads, k_head_dim)
    k: torch.Tensor,  # (seq_cnt, num_k_heads, k_head_dim)
    v: torch.Tensor,  # (seq_cnt, num_v_heads, v_head_dim)
    g: torch.Tensor | None,  # (seq_cnt, num_v_heads)   natural-log decay
    beta: torch.Tensor | None,  # (seq_cnt, num_v_heads)
    recurrent_state: torch.Tensor,  # (max_seq_cnt, num_v_heads, k_head_dim, v_head_dim) fp32, in place
    recurrent_state_indices: torch.Tensor,  # (seq_cnt,)
    *,
    use_qk_l2norm_in_kernel: bool = False,
    gate_inputs: tuple | None = None,
) -> torch.Tensor:
    """``gate_inputs=(a, b, A_log, dt_bias)`` (with ``g`` and ``beta`` None) forms the gates in
    the kernel the way ``GatedDeltaNet`` does (``linear_attention.py:89-90``):
    ``g = -exp(A_log) * softplus(a + dt_bias)``, ``beta = sigmoid(b)``."""
    idx = recurrent_state_indices if recurrent_state_indices.dtype == torch.int32 else recurrent_state_indices.int()
    o = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    scale = float(k.shape[-1] ** -0.5)
    if gate_inputs is not None:
        if g is not None or beta is not None:
            raise ValueError("fused_recurrent_gdn: pass either g/beta or gate_inputs, not both")
        a, b, a_log, dt_bias = gate_inputs
        _lib.require_cuda("fused_recurrent_gdn", q, k, v, a, b, a_log, dt_bias, recurrent_state,
                          recurrent_state_indices)
        _lib.call("fused_recurrent_gdn", "mvb_fused_recurrent_gdn_gated", _lib.desc(q), _lib.desc(k), _lib.desc(v),
                  _lib.desc(a), _lib.desc(b), _lib.desc(a_log), _lib.desc(dt_bias), _lib.desc(recurrent_state),
                  _lib.desc(idx), _lib.desc(o), scale, int(use_qk_l2norm_in_kernel), _lib.stream_of(q))
        return o
    _lib.require_cuda("fused_recurrent_gdn", q, k, v, g, beta, recurrent_state, recurrent_state_indices)
    _lib.call("fused_recurrent_gdn", "mvb_fused_recurrent_gdn", _lib.desc(q), _lib.desc(k), _lib.desc(v),
              _lib.desc(g), _lib.desc(beta), _lib.desc(recurrent_state), _lib.desc(idx), _lib.desc(o),
              scale, int(use_qk_l2norm_in_kernel), _lib.stream_of(q))
    return o
