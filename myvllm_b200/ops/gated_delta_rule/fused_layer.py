"""The decode step of a Gated DeltaNet layer as one library call (``mvb_gated_deltanet_decode``).

The reference's decode branch (``m/layers/linear_attention.py:85-123``) runs
``causal_conv1d_update`` -> q/k ``l2norm`` -> ``recurrent_gated_delta_rule`` -> ``RMSNormGated``
(``m/layers/norm.py:44-58``) as separate ops; this runs them in one kernel.  Its result is
the input of ``out_proj``.
"""

from __future__ import annotations

import ctypes

import torch

from ... import _lib


def fused_decode_supported(qkv: torch.Tensor, recurrent_state: torch.Tensor, num_k_heads: int, num_v_heads: int,
                           z: torch.Tensor) -> bool:
    """Layouts the fused kernel takes: 16-bit activations, K = V = 128, 16-byte aligned
    projection rows with unit channel stride (the fused input projection's output qualifies)."""
    return (qkv.is_cuda and qkv.dtype in (torch.bfloat16, torch.float16) and qkv.dim() == 2 and qkv.stride(1) == 1
            and qkv.stride(0) % 8 == 0 and qkv.data_ptr() % 16 == 0 and recurrent_state.dim() == 4
            and tuple(recurrent_state.shape[2:]) == (128, 128) and recurrent_state.dtype == torch.float32
            and num_v_heads % num_k_heads == 0 and z.stride(-1) == 1 and z.dtype == qkv.dtype)


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
    hk = (qkv.shape[1] - hv * vd) // (2 * recurrent_state.shape[2])
    # counters (zero, and left at zero by every call) and the halves' partial outputs, in two
    # buffers so that no call's records land on another call's counters
    nc, nr = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check("gated_deltanet_decode",
               _lib.load().mvb_gated_deltanet_decode_workspace_sizes(S, hk, hv, ctypes.byref(nc), ctypes.byref(nr)))
    cnt = _lib.workspace(qkv.device, nc.value, tag="gdn_decode_counters")
    rec = _lib.workspace(qkv.device, nr.value, tag="gdn_decode_records")
    _lib.call("gated_deltanet_decode", "mvb_gated_deltanet_decode", _lib.desc(qkv), _lib.desc(conv_weight),
              _lib.desc(conv_state), _lib.desc(cidx), _lib.desc(a), _lib.desc(b), _lib.desc(A_log),
              _lib.desc(dt_bias), _lib.desc(recurrent_state), _lib.desc(ridx), _lib.desc(z),
              _lib.desc(norm_weight), float(norm_eps), scale, _lib.desc(out), cnt.data_ptr(), cnt.numel(),
              rec.data_ptr(), rec.numel(), _lib.stream_of(qkv))
    return out


def fused_prefill_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, recurrent_state: torch.Tensor,
                            z: torch.Tensor) -> bool:
    """Layouts the tensor-core chunk kernel takes (16-bit q/k/v with K = V = 128, unit inner
    strides, 16-byte aligned rows), with a 16-byte aligned z of v's shape and dtype."""
    def rows16(t):
        return t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0

    return (q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and q.shape[-1] == 128 and v.shape[-1] == 128
            and all(rows16(t) for t in (q, k, v, z)) and z.shape == v.shape and z.dtype == v.dtype
            and recurrent_state.dtype == torch.float32 and recurrent_state.stride(-1) == 1)


def gated_deltanet_prefill(q, k, v, a, b, A_log, dt_bias, recurrent_state, recurrent_state_indices, cu_seqlens, z,
                           norm_weight, norm_eps: float) -> torch.Tensor:
    """The prefill branch of GatedDeltaNet after its conv: chunked gated delta rule with the q/k
    L2 norm and the gates formed in the kernel, and RMSNormGated(o, z) applied to each output
    tile before it is stored (``mvb_gated_deltanet_prefill``).  q, k [T, Hk, K]; v, z
    [T, Hv, V]; a, b [T, Hv]; recurrent_state [S_max, Hv, K, V] fp32, read at and written back
    to recurrent_state_indices; returns [T, Hv, V]."""
    _lib.require_cuda("gated_deltanet_prefill", q, k, v, a, b, A_log, dt_bias, recurrent_state,
                      recurrent_state_indices, cu_seqlens, z, norm_weight)
    idx = recurrent_state_indices if recurrent_state_indices.dtype == torch.int32 else recurrent_state_indices.int()
    cu = cu_seqlens if cu_seqlens.dtype == torch.int32 else cu_seqlens.int()
    out = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    ws = _lib.chunk_gdn_workspace(q.device)
    _lib.call("gated_deltanet_prefill", "mvb_gated_deltanet_prefill", _lib.desc(q), _lib.desc(k), _lib.desc(v),
              _lib.desc(a), _lib.desc(b), _lib.desc(A_log), _lib.desc(dt_bias), _lib.desc(recurrent_state),
              _lib.desc(idx), _lib.desc(cu), _lib.desc(z), _lib.desc(norm_weight), float(norm_eps), _lib.desc(out),
              float(k.shape[-1] ** -0.5), ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    return out
