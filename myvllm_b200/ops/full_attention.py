"""Full-attention ops (drop-in for ``myvllm.ops.full_attention``).

Signatures follow the reference (``m/ops/full_attention.py:114-125, 282-290, 454-464``).
None of them synchronises the host: the reference's ``.max().item()`` (``:142``) is
replaced by device-side tile mapping, and the paged decode sizes its split-KV grid from
``block_tables.shape[1] * block_size``.
"""

from __future__ import annotations

import torch

from .. import _lib


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 else t.to(torch.int32)


def flash_attention_prefill(
    q: torch.Tensor,  # (total_seq_len, num_heads, head_dim)
    k: torch.Tensor,  # (total_seq_len, num_kv_heads, head_dim)
    v: torch.Tensor,  # (total_seq_len, num_kv_heads, head_v_dim)
    cu_seqlens: torch.Tensor,  # (num_seq + 1,)
    scale: float,
    num_heads: int,
    num_kv_heads: int,
    head_dim: int,
    head_v_dim: int,
    is_causal: bool,
) -> torch.Tensor:
    _lib.require_cuda("flash_attention_prefill", q, k, v, cu_seqlens)
    o = torch.empty(q.shape[0], q.shape[1], head_v_dim, dtype=q.dtype, device=q.device)
    _lib.call("flash_attention_prefill", "mvb_flash_attention_prefill", _lib.desc(q), _lib.desc(k), _lib.desc(v),
              _lib.desc(_i32(cu_seqlens)), float(scale), int(num_heads), int(num_kv_heads), int(head_dim),
              int(head_v_dim), int(bool(is_causal)), _lib.desc(o), _lib.stream_of(q))
    return o


def paged_flash_attention_decode(
    q: torch.Tensor,  # (seq_cnt, num_q_heads, qk_head_dim)
    k_cache: torch.Tensor,  # (max_num_cached_blocks, block_size, num_kv_heads, qk_head_dim)
    v_cache: torch.Tensor,  # (max_num_cached_blocks, block_size, num_kv_heads, v_head_dim)
    block_tables: torch.Tensor,  # (seq_cnt, max_num_blocks)
    context_lens: torch.Tensor,  # (seq_cnt,)
    scale: float,
    block_size: int,
    max_context_len: int | None = None,
    *,
    output_gate: torch.Tensor | None = None,
) -> torch.Tensor:
    """``output_gate`` [seq_cnt, num_q_heads, v_head_dim] (optional, additive to the reference
    signature): returns ``o * sigmoid(output_gate)``, the gated attention's output gate applied
    where the kernel writes o."""
    _lib.require_cuda("paged_flash_attention_decode", q, k_cache, v_cache, block_tables, context_lens)
    seq_cnt, num_q_heads, _ = q.shape
    num_kv_heads, v_head_dim = v_cache.shape[-2:]
    o = torch.empty(seq_cnt, num_q_heads, v_head_dim, dtype=q.dtype, device=q.device)
    bound = int(max_context_len) if max_context_len else int(block_tables.shape[1]) * int(block_size)
    nbytes = _lib.load().mvb_paged_attention_decode_workspace_size(seq_cnt, num_kv_heads, v_head_dim, bound)
    ws = _lib.workspace(q.device, nbytes, tag="paged_decode") if nbytes else None
    if output_gate is not None:
        _lib.require_cuda("paged_flash_attention_decode", output_gate)
        _lib.call("paged_flash_attention_decode", "mvb_paged_attention_decode_gated", _lib.desc(q),
                  _lib.desc(k_cache), _lib.desc(v_cache), _lib.desc(_i32(block_tables)), _lib.desc(_i32(context_lens)),
                  float(scale), int(block_size), bound, _lib.desc(output_gate), _lib.desc(o),
                  ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, _lib.stream_of(q))
        return o
    _lib.call("paged_flash_attention_decode", "mvb_paged_attention_decode", _lib.desc(q), _lib.desc(k_cache),
              _lib.desc(v_cache), _lib.desc(_i32(block_tables)), _lib.desc(_i32(context_lens)), float(scale),
              int(block_size), bound, _lib.desc(o), ws.data_ptr() if ws is not None else None,
              ws.numel() if ws is not None else 0, _lib.stream_of(q))
    return o


def paged_flash_attention_decode_part(
    q: torch.Tensor,  # (seq_cnt, num_q_heads, qk_head_dim): every q head of the kv heads in the cache
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    block_size: int,
    part: int,
    n_parts: int,
    max_context_len: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Context-split decode (no counterpart in the reference, which asserts TP <= Hkv): this
    rank's part of the attention over every ``n_parts``-th split of each context.  Returns
    ``(o_part [seq_cnt, num_q_heads, v_head_dim] fp32, lse_part [seq_cnt, num_q_heads] fp32)``,
    normalised within the part; :func:`merge_attention_parts` weighs it against the others."""
    _lib.require_cuda("paged_flash_attention_decode_part", q, k_cache, v_cache, block_tables, context_lens)
    seq_cnt, num_q_heads, _ = q.shape
    num_kv_heads, v_head_dim = v_cache.shape[-2:]
    o = torch.empty(seq_cnt, num_q_heads, v_head_dim, dtype=torch.float32, device=q.device)
    lse = torch.empty(seq_cnt, num_q_heads, dtype=torch.float32, device=q.device)
    bound = int(max_context_len) if max_context_len else int(block_tables.shape[1]) * int(block_size)
    nbytes = _lib.load().mvb_paged_attention_decode_part_workspace_size(seq_cnt, num_kv_heads, v_head_dim, bound,
                                                                       int(n_parts))
    ws = _lib.workspace(q.device, nbytes, tag="paged_decode_part")
    _lib.call("paged_flash_attention_decode_part", "mvb_paged_attention_decode_part", _lib.desc(q), _lib.desc(k_cache),
              _lib.desc(v_cache), _lib.desc(_i32(block_tables)), _lib.desc(_i32(context_lens)), float(scale),
              int(block_size), bound, int(part), int(n_parts), _lib.desc(o), _lib.desc(lse), ws.data_ptr(), ws.numel(),
              _lib.stream_of(q))
    return o, lse


def merge_attention_parts(o_part: torch.Tensor, lse_parts: torch.Tensor, part: int,
                          output_gate: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16
                          ) -> torch.Tensor:
    """This part's weighted share of the context-split attention (``* sigmoid(output_gate)``):
    ``lse_parts`` [n_parts, seq_cnt, num_q_heads] holds every part's log2-sum-exp.  The shares
    of all parts sum to the attention over the whole context."""
    _lib.require_cuda("merge_attention_parts", o_part, lse_parts)
    o = torch.empty(o_part.shape, dtype=output_gate.dtype if output_gate is not None else out_dtype,
                    device=o_part.device)
    _lib.call("merge_attention_parts", "mvb_attention_merge_parts", _lib.desc(o_part), _lib.desc(lse_parts), int(part),
              _lib.desc(output_gate) if output_gate is not None else None, _lib.desc(o), _lib.stream_of(o_part))
    return o


def paged_flash_attention_prefill(
    q: torch.Tensor,  # (total_tokens, num_q_heads, qk_head_dim)
    k_cache: torch.Tensor,  # (max_num_cached_blocks, block_size, num_kv_heads, qk_head_dim)
    v_cache: torch.Tensor,  # (max_num_cached_blocks, block_size, num_kv_heads, v_head_dim)
    page_block_tables: torch.Tensor,  # (seq_cnt, max_num_blocks)
    context_lens: torch.Tensor,  # (seq_cnt,)
    cu_seqlens: torch.Tensor,  # (seq_cnt + 1,)
    block_m_indices: torch.Tensor | None,  # ignored: tiles are mapped on device
    scale: float,
    page_block_size: int,
) -> torch.Tensor:
    _lib.require_cuda("paged_flash_attention_prefill", q, k_cache, v_cache, page_block_tables, context_lens,
                      cu_seqlens)
    total_tokens, num_q_heads, _ = q.shape
    v_head_dim = v_cache.shape[-1]
    o = torch.empty(total_tokens, num_q_heads, v_head_dim, dtype=q.dtype, device=q.device)
    _lib.call("paged_flash_attention_prefill", "mvb_paged_attention_prefill", _lib.desc(q), _lib.desc(k_cache),
              _lib.desc(v_cache), _lib.desc(_i32(page_block_tables)), _lib.desc(_i32(context_lens)),
              _lib.desc(_i32(cu_seqlens)), float(scale), int(page_block_size), _lib.desc(o), _lib.stream_of(q))
    return o
