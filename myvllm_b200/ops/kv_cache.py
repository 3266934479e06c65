"""Paged KV-cache write (new op; the reference only sketches ``slot_mapping`` in
``m/utils/context.py:15``).  Cache layout [n_blocks, block_size, Hkv, D] as read by
``m/ops/full_attention.py:186-195``; slot = block * block_size + offset, -1 = skip."""

from __future__ import annotations

import torch

from .. import _lib


def store_kvcache(
    k: torch.Tensor,  # (total_tokens, num_kv_heads, head_dim)
    v: torch.Tensor,  # (total_tokens, num_kv_heads, head_v_dim)
    k_cache: torch.Tensor,  # (n_blocks, block_size, num_kv_heads, head_dim)
    v_cache: torch.Tensor,  # (n_blocks, block_size, num_kv_heads, head_v_dim)
    slot_mapping: torch.Tensor,  # (total_tokens,)
) -> None:
    _lib.require_cuda("store_kvcache", k, v, k_cache, v_cache, slot_mapping)
    sm = slot_mapping if slot_mapping.dtype == torch.int32 else slot_mapping.int()
    _lib.call("store_kvcache", "mvb_store_kvcache", _lib.desc(k), _lib.desc(v), _lib.desc(k_cache),
              _lib.desc(v_cache), _lib.desc(sm), _lib.stream_of(k))
