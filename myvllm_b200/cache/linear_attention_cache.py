"""State caches (drop-in for ``myvllm.cache.linear_attention_cache``).

``LinearAttentionCache`` keeps the reference API (``m/cache/linear_attention_cache.py:7-88``:
constructor arguments, ``bytes_per_seq``, ``can_allocate``/``allocate``/``deallocate``)
with the layouts the ops use:
  conv_cache      [L, S_max, W-1, 2 Hk K + Hv V]   in ``dtype`` (bf16)
  recurrent_cache [L, S_max, Hv, K, V]              in ``state_dtype`` (fp32)
The reference sizes the recurrent cache by k-heads and gives both caches one dtype
(``:37-44``); the ops index the state by v-head and the model keeps it in fp32
(``mamba_ssm_dtype``), which is what is allocated here.

``PagedKVCache`` (new; the reference leaves the KV cache to the caller) owns per-layer
``[n_blocks, block_size, Hkv, D]`` K/V caches, a block allocator, and builds
``block_tables`` / ``slot_mapping`` / ``context_lens`` on the device.
"""

from __future__ import annotations

from collections import deque

import torch


class LinearAttentionCache:
    def __init__(self, layer_cnt: int, max_seq_cnt: int, conv_kernel_size: int, k_head_dim: int, v_head_dim: int,
                 num_k_heads: int, num_v_heads: int, dtype: torch.dtype, device: torch.device,
                 state_dtype: torch.dtype = torch.float32) -> None:
        self.layer_cnt = layer_cnt
        self.max_seq_cnt = max_seq_cnt
        self.conv_kernel_size = conv_kernel_size
        self.k_head_dim, self.v_head_dim = k_head_dim, v_head_dim
        self.num_k_heads, self.num_v_heads = num_k_heads, num_v_heads
        self.dtype, self.state_dtype, self.device = dtype, state_dtype, device
        dim = 2 * k_head_dim * num_k_heads + v_head_dim * num_v_heads
        self.conv_cache = torch.zeros(layer_cnt, max_seq_cnt, conv_kernel_size - 1, dim, dtype=dtype, device=device)
        self.recurrent_cache = torch.zeros(layer_cnt, max_seq_cnt, num_v_heads, k_head_dim, v_head_dim,
                                           dtype=state_dtype, device=device)
        self.free_slot_ids: deque[int] = deque(range(max_seq_cnt))
        self.used_slot_ids: set[int] = set()

    @staticmethod
    def bytes_per_seq(layer_cnt: int, conv_kernel_size: int, k_head_dim: int, v_head_dim: int, num_k_heads: int,
                      num_v_heads: int, dtype: torch.dtype, state_dtype: torch.dtype = torch.float32) -> int:
        conv = layer_cnt * (conv_kernel_size - 1) * (2 * k_head_dim * num_k_heads + v_head_dim * num_v_heads) * \
            dtype.itemsize
        rec = layer_cnt * num_v_heads * k_head_dim * v_head_dim * state_dtype.itemsize
        return conv + rec

    def layer_states(self, layer_idx: int):
        """(conv_state, recurrent_state) views of one layer, as the GDN layer expects."""
        return self.conv_cache[layer_idx], self.recurrent_cache[layer_idx]

    def can_allocate(self) -> bool:
        return len(self.free_slot_ids) > 0

    def allocate(self) -> int:
        assert len(self.free_slot_ids) > 0
        slot_id = self.free_slot_ids.popleft()
        self.used_slot_ids.add(slot_id)
        return slot_id

    def deallocate(self, slot_id: int):
        assert slot_id in self.used_slot_ids
        self.conv_cache[:, slot_id].zero_()
        self.recurrent_cache[:, slot_id].zero_()
        self.used_slot_ids.remove(slot_id)
        self.free_slot_ids.appendleft(slot_id)


class PagedKVCache:
    """Block-paged K/V caches of the full-attention layers."""

    def __init__(self, layer_cnt: int, n_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device):
        self.block_size = block_size
        self.k = torch.empty(layer_cnt, n_blocks, block_size, num_kv_heads, head_dim, dtype=dtype, device=device)
        self.v = torch.empty_like(self.k)
        self.free_blocks: deque[int] = deque(range(n_blocks))
        self.seq_blocks: dict[int, list[int]] = {}
        self.seq_lens: dict[int, int] = {}
        self.device = device

    def layer_caches(self, layer_idx: int):
        return self.k[layer_idx], self.v[layer_idx]

    def append(self, seq_id: int, n_tokens: int) -> None:
        """Reserves room for ``n_tokens`` more tokens of ``seq_id``."""
        blocks = self.seq_blocks.setdefault(seq_id, [])
        new_len = self.seq_lens.get(seq_id, 0) + n_tokens
        while len(blocks) * self.block_size < new_len:
            if not self.free_blocks:
                raise RuntimeError("PagedKVCache: out of blocks")
            blocks.append(self.free_blocks.popleft())
        self.seq_lens[seq_id] = new_len

    def free(self, seq_id: int) -> None:
        self.free_blocks.extend(self.seq_blocks.pop(seq_id, []))
        self.seq_lens.pop(seq_id, None)

    def metadata(self, seq_ids: list[int], new_tokens: list[int]):
        """block_tables [S, max_blocks], context_lens [S] and slot_mapping for the last
        ``new_tokens[s]`` positions of every sequence (all int32, on the device)."""
        max_blocks = max(len(self.seq_blocks[s]) for s in seq_ids)
        bt = torch.zeros(len(seq_ids), max_blocks, dtype=torch.int32)
        slots = []
        for i, s in enumerate(seq_ids):
            blocks = self.seq_blocks[s]
            bt[i, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
            n = self.seq_lens[s]
            pos = torch.arange(n - new_tokens[i], n)
            slots.append(bt[i, pos // self.block_size].long() * self.block_size + pos % self.block_size)
        ctx = torch.tensor([self.seq_lens[s] for s in seq_ids], dtype=torch.int32)
        return (bt.to(self.device), ctx.to(self.device),
                torch.cat(slots).to(device=self.device, dtype=torch.int32))
