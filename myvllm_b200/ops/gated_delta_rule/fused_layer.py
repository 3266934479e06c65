"""The decode step of a Gated DeltaNet layer as one library call (``mvb_gated_deltanet_decode``).

The reference's decode branch (``m/layers/linear_attention.py:85-123``) runs
``causal_conv1d_update`` -> q/k ``l2norm`` -> ``recurrent_gated_delta_rule`` -> ``RMSNormGated``
(``m/layers/norm.py:44-58``) as separate ops; this runs them in one kernel.  Its result is
the input of ``out_proj``.
"""

from __future__ import annotations

import torch

from ... import _lib


def fused_decode_supported(qkv: torch.Tensor, recurrent_state: torch.Tensor, num_k_heads: int, num_v_heads: int,
                           z: torch.Tensor) -> bool:
    """Layouts the fused kernel takes: 16-bit activations, K = V = 128, Hv / Hk in {1, 2, 4},
    16-byte aligned projection rows with unit channel stride (the fused input projection's
    output qualifies)."""
    return (qkv.is_cuda and qkv.dtype in (torch.bfloat16, torch.float16) and qkv.dim() == 2 and qkv.stride(1) == 1
            and qkv.stride(0) % 8 == 0 and qkv.data_ptr() % 16 == 0 and recurrent_state.dim() == 4
            and tuple(recurrent_state.shape[2:]) == (128, 128) and recurrent_state.dtype == torch.float32
            and num_v_heads % num_k_heads == 0 and num_v_heads // num_k_heads in (1, 2, 4)
            and z.stride(-1) == 1 and z.dtype == qkv.dtype)


def gated_deltanet_decode(qkv, conv_weight, conv_state, conv_state_indices, a, b, A_log, dt_bias, recurrent_state,
                          recurrent_state_indices, z, norm_weight, norm_eps: float) -> torch.Tensor:
    """qkv [S, 2 Hk K + Hv V] (the input projection's q | k | v channels, before the conv);
    conv_weight [conv_dim, W]; conv_state [S_max, W-1, conv_dim] and recurrent_state
    [S_max, Hv, K, V] (fp32), both updated in place at their index rows; a, b [S, Hv] raw
    gate projections; A_log, dt_bias [Hv]; z [S, Hv, V] the output gate; norm_weight [V].
    Returns RMSNormGated(o, z) as [S, Hv, V]."""
    _lib.require_cuda("gated_deltanet_decode", qkv, conv_weight, conv_state, conv_state_indices, a, b, A_log,
                      dt_bias, recurrent_state, recurrent_state_indices, z, norm_weight)
    S, hv, vd = qkv.shape[0], recurrent_state.shape[1], recurrent_state.shape[3]
    out = torch.empty(S, hv, vd, dtype=qkv.dtype, device=qkv.device)
    cidx = conv_state_indices if conv_state_indices.dtype == torch.int32 else conv_state_indices.int()
    ridx = recurrent_state_indices if recurrent_state_indices.dtype == torch.int32 else recurrent_state_indices.int()
    scale = float(recurrent_state.shape[2] ** -0.5)
    _lib.call("gated_deltanet_decode", "mvb_gated_deltanet_decode", _lib.desc(qkv), _lib.desc(conv_weight),
              _lib.desc(conv_state), _lib.desc(cidx), _lib.desc(a), _lib.desc(b), _lib.desc(A_log),
              _lib.desc(dt_bias), _lib.desc(recurrent_state), _lib.desc(ridx), _lib.desc(z),
              _lib.desc(norm_weight), float(norm_eps), scale, _lib.desc(out), _lib.stream_of(qkv))
    return out
