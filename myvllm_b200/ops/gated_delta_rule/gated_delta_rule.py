"""Gated delta rule entry points (drop-in for
``myvllm.ops.gated_delta_rule.gated_delta_rule``, reference ``:31-92``).

``chunk_gated_delta_rule`` runs the chunked (WY, chunk 64) prefill in one kernel launch
with no host synchronisation (the reference calls ``.item()`` per sequence,
``gated_delta_rule.py:19-23, 61``).  It reads the incoming state at
``recurrent_state_indices`` (the reference starts from zero, ``h.py:61-67``; identical
for a zeroed slot) and writes the final fp32 state there.
"""

from __future__ import annotations

import torch

from ... import _lib
from .fused_recurrent_gdn import fused_recurrent_gdn

CHUNK_SIZE = 64


def prepare_chunk_indices(cu_seqlens: torch.Tensor, chunk_size: int = CHUNK_SIZE):
    """(chunk_indices [n_chunks, 2] = (seq, chunk-in-seq), cu_chunk_cnts [S+1]), computed on
    device.  Kept for callers of the reference helper (``gated_delta_rule.py:15-28``);
    the kernels do not need it."""
    seqlens = (cu_seqlens[1:] - cu_seqlens[:-1]).long()
    cnts = (seqlens + chunk_size - 1) // chunk_size
    cu_cnts = torch.zeros(cnts.numel() + 1, dtype=cu_seqlens.dtype, device=cu_seqlens.device)
    cu_cnts[1:] = cnts.cumsum(0)
    seq_ids = torch.repeat_interleave(torch.arange(cnts.numel(), device=cu_seqlens.device), cnts)
    offs = torch.arange(seq_ids.numel(), device=cu_seqlens.device) - cu_cnts[:-1].long()[seq_ids]
    return torch.stack((seq_ids, offs), dim=1).to(cu_seqlens.dtype), cu_cnts


def chunk_gated_delta_rule(
    q: torch.Tensor,  # (total_tokens, num_k_heads, k_head_dim)
    k: torch.Tensor,  # (total_tokens, num_k_heads, k_head_dim)
    v: torch.Tensor,  # (total_tokens, num_v_heads, v_head_dim)
    g: torch.Tensor | None,  # (total_tokens, num_v_heads)   natural-log decay
    beta: torch.Tensor | None,  # (total_tokens, num_v_heads)
    recurrent_state: torch.Tensor,  # (max_seq_cnt, num_v_heads, k_head_dim, v_head_dim) fp32, in place
    recurrent_state_indices: torch.Tensor,  # (seq_cnt,)
    cu_seqlens: torch.Tensor,  # (seq_cnt + 1,)
    *,
    use_qk_l2norm_in_kernel: bool = False,
    gate_inputs: tuple | None = None,
) -> torch.Tensor:
    """``use_qk_l2norm_in_kernel`` folds the layer's q/k L2 norm (``linear_attention.py:113-114``)
    into the kernel's tile load; the default keeps the reference contract (q, k normalised
    by the caller).  ``gate_inputs=(a, b, A_log, dt_bias)`` (with ``g`` and ``beta`` None)
    forms the gates in the kernel as the layer does (``linear_attention.py:89-90``)."""
    idx = recurrent_state_indices if recurrent_state_indices.dtype == torch.int32 else recurrent_state_indices.int()
    cu = cu_seqlens if cu_seqlens.dtype == torch.int32 else cu_seqlens.int()
    o = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    ws = _lib.chunk_gdn_workspace(q.device)
    scale = float(k.shape[-1] ** -0.5)
    if gate_inputs is not None:
        if g is not None or beta is not None:
            raise ValueError("chunk_gated_delta_rule: pass either g/beta or gate_inputs, not both")
        a, b, a_log, dt_bias = gate_inputs
        _lib.require_cuda("chunk_gated_delta_rule", q, k, v, a, b, a_log, dt_bias, recurrent_state,
                          recurrent_state_indices, cu_seqlens)
        _lib.call("chunk_gated_delta_rule", "mvb_chunk_gated_delta_rule_gated", _lib.desc(q), _lib.desc(k),
                  _lib.desc(v), _lib.desc(a), _lib.desc(b), _lib.desc(a_log), _lib.desc(dt_bias),
                  _lib.desc(recurrent_state), _lib.desc(idx), _lib.desc(cu), _lib.desc(o), scale,
                  int(use_qk_l2norm_in_kernel), ws.data_ptr(), ws.numel(), _lib.stream_of(q))
        return o
    _lib.require_cuda("chunk_gated_delta_rule", q, k, v, g, beta, recurrent_state, recurrent_state_indices,
                      cu_seqlens)
    _lib.call("chunk_gated_delta_rule", "mvb_chunk_gated_delta_rule", _lib.desc(q), _lib.desc(k), _lib.desc(v),
              _lib.desc(g), _lib.desc(beta), _lib.desc(recurrent_state), _lib.desc(idx), _lib.desc(cu),
              _lib.desc(o), scale, int(use_qk_l2norm_in_kernel), ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    return o


def recurrent_gated_delta_rule(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor | None,
    beta: torch.Tensor | None,
    recurrent_state: torch.Tensor,
    recurrent_state_indices: torch.Tensor,
    *,
    use_qk_l2norm_in_kernel: bool = False,
    gate_inputs: tuple | None = None,
) -> torch.Tensor:
    """Decode: one token per sequence (reference ``gated_delta_rule.py:69-92``)."""
    return fused_recurrent_gdn(q, k, v, g, beta, recurrent_state, recurrent_state_indices,
                               use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, gate_inputs=gate_inputs)
