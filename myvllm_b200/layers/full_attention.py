"""Gated full-attention layer (drop-in for ``myvllm.layers.full_attention.GatedAttention``).

Constructor and ``forward(x, rotary_pos_emb_cos, rotary_pos_emb_sin)`` as in the reference
(``m/layers/full_attention.py:10-64``), which stops after RoPE and returns an empty tensor.
Completed here with the Qwen3.5 gated attention the config describes
(``attn_output_gate``, partial rotary):

    q, gate = q_proj(x)           (per head: [q | gate], GatedQParallelLinear)
    q, k    = q_norm(q), k_norm(k_proj(x));  v = v_proj(x)
    q, k    = RoPE on the first 2 * cos.shape[-1] dims
    store_kvcache(k, v) at context.slot_mapping            (when a cache is attached)
    o       = varlen causal prefill | paged prefill | paged decode   (from the Context)
    out     = o_proj(o * sigmoid(gate))                    (all_reduce at TP > 1)

Attention metadata comes from ``myvllm_b200.utils.context`` (the reference sketches the
same fields there).  KV heads are split across ranks at TP <= Hkv (the reference's only
case: it asserts ``num_kv_heads % tp == 0``).  At larger TP the ``share = TP / Hkv`` ranks
of a kv head each keep a copy of its cache and, by default, split the attention over it by
context (``context_split``): every rank of the share projects q and gate for all q heads of
that kv head, attends over every share-th split of each context, weighs its part against
the others' log-sum-exps (a small all-gather) and projects its part with the o_proj rows of
those heads; the all-reduce after o_proj adds the parts.  Each rank then reads 1 / share of
the kv head's cache per decode step instead of all of it.  With ``context_split = False`` the
ranks of a share keep their own q heads and each reads the whole cache.  ``k_cache`` /
``v_cache`` are attributes the caller points at its paged cache
``[n_blocks, block_size, Hkv_rank, D]``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..ops.full_attention import (flash_attention_prefill, merge_attention_parts, paged_flash_attention_decode,
                                   paged_flash_attention_decode_part, paged_flash_attention_prefill)
from ..ops.kv_cache import store_kvcache
from ..utils.context import get_context
from . import comm
from .linear import GatedQParallelLinear, KVParallelLinear, RowParallelLinear, tensor_parallel, tp_rank_size
from .norm import RMSNorm
from .rotary_embedding import apply_partial_rotary


class GatedAttention(nn.Module):
    context_split = True  # at TP > Hkv: split each kv head's context over the ranks that share it

    def __init__(self, hidden_size: int, qk_head_dim: int, num_q_heads: int, v_head_dim: int, num_kv_heads: int,
                 attention_bias: bool, rms_norm_eps: float) -> None:
        super().__init__()
        self.tp_rank, self.tp_size = tp_rank_size()
        assert num_q_heads % self.tp_size == 0
        self.hidden_size = hidden_size
        self.qk_head_dim, self.v_head_dim = qk_head_dim, v_head_dim
        self.total_num_q_heads, self.total_num_kv_heads = num_q_heads, num_kv_heads
        self.num_q_heads = num_q_heads // self.tp_size
        self.attention_bias = attention_bias
        self.rms_norm_eps = rms_norm_eps
        self.scale = qk_head_dim ** -0.5
        # ranks per kv head past TP = Hkv, and this rank's part of the kv head's context
        self.kv_share = self.tp_size // num_kv_heads if self.tp_size > num_kv_heads else 1
        self.kv_part = self.tp_rank % self.kv_share
        split = self.kv_share > 1 and self.context_split and self.tp_size % num_kv_heads == 0
        self.kv_share, self.kv_part = (self.kv_share, self.kv_part) if split else (1, 0)
        if split:
            # q/gate and o_proj sharded by kv head: the share's ranks hold all its q heads
            with tensor_parallel(self.tp_rank // self.kv_share, num_kv_heads):
                self.q_proj = GatedQParallelLinear(hidden_size, qk_head_dim, num_q_heads, bias=attention_bias)
                self.o_proj = RowParallelLinear(num_q_heads * v_head_dim, hidden_size, bias=False)
            self.o_proj.tp_rank, self.o_proj.tp_size = self.tp_rank, self.tp_size  # all-reduce over every rank
            self.num_q_heads = num_q_heads // num_kv_heads
        else:
            self.q_proj = GatedQParallelLinear(hidden_size, qk_head_dim, num_q_heads, bias=attention_bias)
            self.o_proj = RowParallelLinear(num_q_heads * v_head_dim, hidden_size, bias=False)
        self.k_proj = KVParallelLinear(hidden_size, qk_head_dim, num_kv_heads, bias=attention_bias)
        self.v_proj = KVParallelLinear(hidden_size, v_head_dim, num_kv_heads, bias=attention_bias)
        self.num_kv_heads = self.k_proj.num_kv_heads
        self.q_norm = RMSNorm((qk_head_dim,), rms_norm_eps, True)
        self.k_norm = RMSNorm((qk_head_dim,), rms_norm_eps, True)
        self.k_cache: torch.Tensor = torch.empty(0)
        self.v_cache: torch.Tensor = torch.empty(0)

    @property
    def k_nrom(self):  # the reference's attribute name (m/layers/full_attention.py:47)
        return self.k_norm

    def fuse_projections(self) -> None:
        """Concatenate q (with its gate), k and v projections of this rank into one weight
        (and bias), so a forward runs one GEMM instead of three.  Call after the weights are
        loaded; re-run after changing them."""
        mods = [self.q_proj, self.k_proj, self.v_proj]
        self._w_qkv = torch.cat([m.weight.detach() for m in mods], 0)
        self._b_qkv = torch.cat([m.bias.detach() for m in mods], 0) if self.attention_bias else None
        self._qkv_split = [m.weight.shape[0] for m in mods]

    def forward(self, x: torch.Tensor, rotary_pos_emb_cos: torch.Tensor | None,
                rotary_pos_emb_sin: torch.Tensor | None) -> torch.Tensor:
        ctx = get_context()
        T = x.size(0)
        D, Dv = self.qk_head_dim, self.v_head_dim
        if getattr(self, "_w_qkv", None) is not None:
            qg, kp, vp = F.linear(x, self._w_qkv, self._b_qkv).split(self._qkv_split, dim=-1)
        else:
            qg, kp, vp = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        q, gate = torch.chunk(qg.view(T, self.num_q_heads, 2 * D), 2, dim=-1)
        v = vp.view(T, self.num_kv_heads, Dv)
        if rotary_pos_emb_cos is not None and rotary_pos_emb_sin is not None:
            # q/k norm and partial rotary in one kernel per tensor
            q = self.q_norm.rope_forward(q, rotary_pos_emb_cos, rotary_pos_emb_sin)
            k = self.k_norm.rope_forward(kp.view(T, self.num_kv_heads, D), rotary_pos_emb_cos, rotary_pos_emb_sin)
        else:
            q = self.q_norm(q)
            k = self.k_norm(kp.view(T, self.num_kv_heads, D))
        cached = self.k_cache.numel() > 0
        if cached and ctx.slot_mapping is not None:
            store_kvcache(k, v, self.k_cache, self.v_cache, ctx.slot_mapping)
        if ctx.is_prefill:
            # context split: this rank prefills its own q heads of the share and leaves the
            # others' rows of o at zero (they come through the all-reduce from their ranks)
            hpr = self.num_q_heads // self.kv_share
            lo = self.kv_part * hpr
            q_own = q if self.kv_share == 1 else q[:, lo:lo + hpr].contiguous()
            if cached and ctx.block_tables is not None and ctx.max_seqlen_k > ctx.max_seqlen_q:
                o = paged_flash_attention_prefill(q_own, self.k_cache, self.v_cache, ctx.block_tables,
                                                  ctx.context_lens, ctx.cu_seqlens_q, None, self.scale, ctx.block_size)
            else:
                o = flash_attention_prefill(q_own, k, v, ctx.cu_seqlens_q, self.scale, hpr, self.num_kv_heads, D, Dv,
                                            True)
            o = o * torch.sigmoid(gate[:, lo:lo + hpr])
            if self.kv_share > 1:
                o = F.pad(o, (0, 0, lo, self.num_q_heads - lo - hpr))
            return self.o_proj(o.reshape(T, self.num_q_heads * Dv))
        if self.kv_share > 1:
            # this rank's part of every context, weighed against the other parts
            o_part, lse = paged_flash_attention_decode_part(q, self.k_cache, self.v_cache, ctx.block_tables,
                                                            ctx.context_lens, self.scale, ctx.block_size,
                                                            self.kv_part, self.kv_share)
            o = merge_attention_parts(o_part, comm.all_gather_block(lse, self.kv_share), self.kv_part,
                                      output_gate=gate)
            return self.o_proj(o.reshape(T, self.num_q_heads * Dv))
        # the output gate is applied where the decode kernel writes o
        o = paged_flash_attention_decode(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens,
                                         self.scale, ctx.block_size, output_gate=gate)
        return self.o_proj(o.reshape(T, self.num_q_heads * Dv))
