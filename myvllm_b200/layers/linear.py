"""Tensor-parallel linear layers (drop-in for ``myvllm.layers.linear``).

Same classes, constructor arguments and ``weight_loader`` sharding rules as the reference
(``m/layers/linear.py:7-169``); the projections are plain ``F.linear`` (cuBLAS) and the
only collective is the ``all_reduce(SUM)`` after a row-parallel projection
(``linear.py:159-164``), which is where the attention stack exchanges data across GPUs.

Differences: with no initialised process group the layers run unsharded (tp = 1) instead
of failing in ``dist.get_rank()``, and ``KVParallelLinear`` (new) replicates KV heads when
the tensor-parallel size exceeds the number of KV heads (the reference asserts,
``m/layers/full_attention.py:35``).
"""

from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from . import comm


_tp_override: tuple[int, int] | None = None


def tp_rank_size(group=None) -> tuple[int, int]:
    if _tp_override is not None:
        return _tp_override
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


@contextlib.contextmanager
def tensor_parallel(rank: int, size: int):
    """Layers constructed inside this block are rank ``rank`` of a ``size``-way split,
    whatever the process group says; ``tensor_parallel(0, 1)`` builds unsharded layers (no
    all-reduce) inside a multi-rank job, e.g. a single-rank reference of a sharded model."""
    global _tp_override
    prev = _tp_override
    _tp_override = (int(rank), int(size))
    try:
        yield
    finally:
        _tp_override = prev


class Linear(nn.Module):
    def __init__(self, input_size: int, output_size: int, bias: bool = False, prefix: str = ""):
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.weight = nn.Parameter(torch.empty(output_size, input_size))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.zeros(output_size))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight, self.bias)

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        param.data.copy_(loaded_weights)


class ColumnParallelLinear(Linear):
    """Output dimension split across ranks (reference ``linear.py:36-51``)."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False, prefix: str = ""):
        self.tp_rank, self.tp_size = tp_rank_size()
        assert output_size % self.tp_size == 0
        super().__init__(input_size, output_size // self.tp_size, bias, prefix)

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        shard = loaded_weights.narrow(0, self.tp_rank * self.output_size, self.output_size)
        param.data.copy_(shard)


class GatedQParallelLinear(ColumnParallelLinear):
    """q and its output gate, sharded by head (reference ``linear.py:54-82``).

    Rows are per-head blocks ``[q_h (head_dim) | gate_h (head_dim)]``, the layout the
    forward reads (``q_proj(x).view(T, H, 2 * head_dim).chunk(2, -1)``,
    ``m/layers/full_attention.py:56``).  The reference loader instead writes
    ``[all q | all gate]``, which that forward would misread; here a rank takes its
    heads' contiguous blocks."""

    def __init__(self, hidden_size: int, head_dim: int, total_num_heads: int, bias: bool = False):
        self.hidden_size = hidden_size
        self.head_dim = head_dim
        self.total_num_heads = total_num_heads
        _, tp = tp_rank_size()
        assert total_num_heads % tp == 0
        self.num_heads = total_num_heads // tp
        super().__init__(input_size=hidden_size, output_size=total_num_heads * head_dim * 2, bias=bias)

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        rows = self.num_heads * self.head_dim * 2
        param.data.copy_(loaded_weights.narrow(0, self.tp_rank * rows, rows))


class QKVParallelLinear(ColumnParallelLinear):
    """q | k | v blocks, each head-sharded; rank layout [q shard | k shard | v shard]
    (reference ``linear.py:85-147``).  Also used for the GDN conv weight."""

    def __init__(self, hidden_size: int, q_head_dim: int, k_head_dim: int, v_head_dim: int, total_num_q_heads: int,
                 total_num_k_heads: int, total_num_v_heads: int, bias: bool = False,
                 params_dtype: torch.dtype | None = None):
        self.hidden_size = hidden_size
        self.q_head_dim, self.k_head_dim, self.v_head_dim = q_head_dim, k_head_dim, v_head_dim
        self.total_num_q_heads = total_num_q_heads
        self.total_num_k_heads = total_num_k_heads
        self.total_num_v_heads = total_num_v_heads
        _, tp = tp_rank_size()
        assert total_num_q_heads % tp == 0 and total_num_k_heads % tp == 0 and total_num_v_heads % tp == 0
        self.num_q_heads = total_num_q_heads // tp
        self.num_k_heads = total_num_k_heads // tp
        self.num_v_heads = total_num_v_heads // tp
        out = q_head_dim * total_num_q_heads + k_head_dim * total_num_k_heads + v_head_dim * total_num_v_heads
        super().__init__(input_size=hidden_size, output_size=out, bias=bias)

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        qs = self.q_head_dim * self.num_q_heads
        ks = self.k_head_dim * self.num_k_heads
        vs = self.v_head_dim * self.num_v_heads
        q_total = self.q_head_dim * self.total_num_q_heads
        k_total = self.k_head_dim * self.total_num_k_heads
        param.data.narrow(0, 0, qs).copy_(loaded_weights.narrow(0, self.tp_rank * qs, qs))
        param.data.narrow(0, qs, ks).copy_(loaded_weights.narrow(0, q_total + self.tp_rank * ks, ks))
        param.data.narrow(0, qs + ks, vs).copy_(loaded_weights.narrow(0, q_total + k_total + self.tp_rank * vs, vs))


class KVParallelLinear(Linear):
    """K (or V) projection of ``total_num_kv_heads`` heads.  At tp <= heads the heads are
    split like ColumnParallelLinear; at tp > heads every rank keeps one head, head
    ``rank * heads // tp`` (KV-head replication, so tp may exceed the KV head count)."""

    def __init__(self, hidden_size: int, head_dim: int, total_num_kv_heads: int, bias: bool = False):
        self.tp_rank, self.tp_size = tp_rank_size()
        self.head_dim = head_dim
        self.total_num_kv_heads = total_num_kv_heads
        if self.tp_size <= total_num_kv_heads:
            assert total_num_kv_heads % self.tp_size == 0
            self.num_kv_heads = total_num_kv_heads // self.tp_size
            self.first_head = self.tp_rank * self.num_kv_heads
        else:
            assert self.tp_size % total_num_kv_heads == 0
            self.num_kv_heads = 1
            self.first_head = self.tp_rank * total_num_kv_heads // self.tp_size
        super().__init__(hidden_size, self.num_kv_heads * head_dim, bias)

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        rows = self.num_kv_heads * self.head_dim
        param.data.copy_(loaded_weights.narrow(0, self.first_head * self.head_dim, rows))


class RowParallelLinear(Linear):
    """Input dimension split across ranks; partial products are summed with an
    ``all_reduce`` (reference ``linear.py:150-169``)."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False, prefix: str = ""):
        self.tp_rank, self.tp_size = tp_rank_size()
        assert input_size % self.tp_size == 0
        # the input slice this rank loads; tp_rank/tp_size set the all-reduce, and a layer
        # may widen that to more ranks than the slicing (context-split attention)
        self.shard_rank = self.tp_rank
        super().__init__(input_size // self.tp_size, output_size, bias, prefix)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1 and self.bias is None:
            # projection + all-reduce in one kernel over NVLink, where enabled and x qualifies
            fused = comm.fused_linear(x, self.weight)
            if fused is not None:
                return fused
        # the bias is added once (by rank 0's share) so the all-reduced sum carries it once
        bias = self.bias if (self.bias is None or self.tp_rank == 0) else None
        result = F.linear(x, self.weight, bias)
        if self.tp_size > 1:
            result = comm.all_reduce(result)
        return result

    def weight_loader(self, param: nn.Parameter, loaded_weights: torch.Tensor):
        if param.dim() == 1:  # bias: replicated
            param.data.copy_(loaded_weights)
            return
        param.data.copy_(loaded_weights.narrow(1, self.shard_rank * self.input_size, self.input_size))
