"""Per-step attention metadata (drop-in for ``myvllm.utils.context``).

The reference ``Context`` (``m/utils/context.py:6-52``) carries ``is_prefill`` and the two
state-index tensors, with the full-attention fields (cu_seqlens, slot_mapping,
context_lens, block_tables) only sketched in comments (``:11-17``).  Here they are real
fields, so ``GatedAttention`` can find its paged-cache metadata the same way.  All index
tensors are int32 on the device; nothing here synchronises the host.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class Context:
    is_prefill: bool = False
    conv_state_indices: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    recurrent_state_indices: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    block_size: int = 256


_context = Context()


def get_context() -> Context:
    return _context


def reset_context():
    global _context
    _context = Context()


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0, slot_mapping=None,
                context_lens=None, block_tables=None, conv_state_indices=None, recurrent_state_indices=None,
                block_size=256):
    global _context
    _context = Context(
        is_prefill=is_prefill,
        conv_state_indices=conv_state_indices if conv_state_indices is not None else torch.empty(0),
        recurrent_state_indices=recurrent_state_indices if recurrent_state_indices is not None else torch.empty(0),
        cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k, max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k,
        slot_mapping=slot_mapping, context_lens=context_lens, block_tables=block_tables, block_size=block_size)
