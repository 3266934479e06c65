"""The hybrid decode stack of the layer API: ``n_layers`` decoder layers in which every
fourth mixer is a gated full-attention layer (``GatedAttention``) and the others are
Gated DeltaNet layers (``GatedDeltaNet``), each a pre-norm + mixer + residual, one token
per sequence per step.  This is the attention stack of a Qwen3.5-style hybrid model (no MLP
or MoE), as the reference layers compose it (``m/layers/linear_attention.py:77-123``,
``m/layers/full_attention.py:49-64``, ``m/layers/linear.py:159-164``).

Weights, recurrent/conv states and the paged KV cache are drawn from generators keyed by
(seed, layer, tensor, head), and every rank loads its tensor-parallel shard of the same
full tensors through the layers' ``weight_loader`` rules.  So a stack built at TP = n holds
exactly the head slices of the stack built at TP = 1 with the same seed, which is what a
TP-parity check compares.  Activations are bf16, GDN states fp32, conv states and KV bf16.
"""

from __future__ import annotations

import hashlib

import torch
import torch.nn.functional as F

from .cache.linear_attention_cache import LinearAttentionCache, PagedKVCache
from .layers.full_attention import GatedAttention
from .layers.linear import tensor_parallel, tp_rank_size
from .layers.linear_attention import GatedDeltaNet
from .layers.norm import RMSNorm
from .layers.rotary_embedding import RotaryEmbedding
from .utils.context import set_context

HIDDEN, GDN_HK, GDN_HV, GDN_D, CONV_W = 2048, 16, 32, 128, 4
FA_HQ, FA_HKV, FA_D, ROTARY_DIM = 16, 2, 256, 64


def layer_kinds(n_layers: int) -> list[str]:
    return ["full" if (i + 1) % 4 == 0 else "gdn" for i in range(n_layers)]


def _gen(device, *key) -> torch.Generator:
    h = int.from_bytes(hashlib.sha256(repr(key).encode()).digest()[:8], "little") & ((1 << 63) - 1)
    return torch.Generator(device=device).manual_seed(h)


def _make_mixer(kind: str):
    if kind == "gdn":
        return GatedDeltaNet(HIDDEN, GDN_HK, GDN_HV, GDN_D, GDN_D, CONV_W)
    return GatedAttention(HIDDEN, FA_D, FA_HQ, FA_D, FA_HKV, False, 1e-6)


class HybridDecodeStack:
    """Layers, states and caches of one rank.  ``tp`` = (rank, size) overrides the process
    group (``(0, 1)``: the unsharded stack inside a multi-rank job)."""

    def __init__(self, n_layers: int, n_seqs: int, ctx_lens: list[int], max_new_tokens: int, device,
                 seed: int = 1234, tp: tuple[int, int] | None = None, block_size: int = 256):
        self.device = torch.device(device)
        self.seed = seed
        self.kinds = layer_kinds(n_layers)
        self.n_seqs = n_seqs
        self.block_size = block_size
        self.rank, self.tp = tp if tp is not None else tp_rank_size()
        with tensor_parallel(self.rank, self.tp):
            self.layers = [self._build_layer(i, kind) for i, kind in enumerate(self.kinds)]
        self.gdn = [m for k, (_, m) in zip(self.kinds, self.layers) if k == "gdn"]
        self.fa = [m for k, (_, m) in zip(self.kinds, self.layers) if k == "full"]
        self._init_states()
        self._init_kv(ctx_lens, max_new_tokens)
        self.idx = torch.arange(n_seqs, dtype=torch.int32, device=self.device)
        self.rope = RotaryEmbedding(ROTARY_DIM, 10_000_000.0).to(self.device)

    # ------------------------------------------------------------------ weights ----
    def _build_layer(self, i: int, kind: str):
        dev = self.device
        with torch.device("meta"), tensor_parallel(0, 1):
            full_shapes = {n: p.shape for n, p in _make_mixer(kind).named_parameters()}
        mixer = _make_mixer(kind).to(dev, torch.bfloat16)
        hv_r = GDN_HV // self.tp
        for name, prm in mixer.named_parameters():
            shape = full_shapes[name]
            g = _gen(dev, self.seed, "w", i, name)
            if name.endswith("A_log"):
                full = torch.empty(shape, device=dev).uniform_(0.0, 2.772588722239781, generator=g)  # U(0, ln 16)
            elif name.endswith("dt_bias"):
                full = 0.1 * torch.randn(shape, generator=g, device=dev)
            elif "norm" in name:
                full = torch.ones(shape, device=dev)
            else:
                full = 0.02 * torch.randn(shape, generator=g, device=dev)
            loader = getattr(prm, "weight_loader", None)
            if name.endswith("A_log") or name.endswith("dt_bias"):
                prm.data = full[self.rank * hv_r:(self.rank + 1) * hv_r].float().contiguous()
            elif loader is not None:
                loader(prm, full.to(prm.dtype))
            else:
                prm.data.copy_(full.to(prm.dtype))
        mixer.fuse_projections()
        return RMSNorm((HIDDEN,), 1e-6, True).to(dev, torch.bfloat16), mixer

    # ------------------------------------------------------------------- states ----
    def _init_states(self):
        dev, S = self.device, self.n_seqs
        hk_r, hv_r = GDN_HK // self.tp, GDN_HV // self.tp
        self.lac = LinearAttentionCache(len(self.gdn), S, CONV_W, GDN_D, GDN_D, hk_r, hv_r, torch.bfloat16, dev)
        qs, vs = hk_r * GDN_D, hv_r * GDN_D
        q_tot = GDN_HK * GDN_D
        for l, m in enumerate(self.gdn):
            for h in range(hv_r):
                head = self.rank * hv_r + h
                self.lac.recurrent_cache[l, :, h].copy_(
                    0.1 * torch.randn(S, GDN_D, GDN_D, generator=_gen(dev, self.seed, "rec", l, head), device=dev))
            full = torch.randn(S, CONV_W - 1, 2 * q_tot + GDN_HV * GDN_D, generator=_gen(dev, self.seed, "conv", l),
                               device=dev).to(torch.bfloat16)
            r = self.rank
            self.lac.conv_cache[l].copy_(torch.cat([full[..., r * qs:(r + 1) * qs],
                                                    full[..., q_tot + r * qs:q_tot + (r + 1) * qs],
                                                    full[..., 2 * q_tot + r * vs:2 * q_tot + (r + 1) * vs]], -1))
            m.conv_state, m.recurrent_state = self.lac.layer_states(l)

    def _init_kv(self, ctx_lens, max_new_tokens):
        dev, bs = self.device, self.block_size
        self.ctx_lens = list(ctx_lens)
        n_blocks = sum((c + max_new_tokens + bs - 1) // bs for c in ctx_lens)
        hkv_r = self.fa[0].num_kv_heads if self.fa else 1
        first = self.fa[0].k_proj.first_head if self.fa else 0
        self.kv = PagedKVCache(len(self.fa), n_blocks, bs, hkv_r, FA_D, torch.bfloat16, dev)
        for l, m in enumerate(self.fa):
            for j in range(hkv_r):
                for name, cache in (("k", self.kv.k), ("v", self.kv.v)):
                    g = _gen(dev, self.seed, name, l, first + j)
                    cache[l, :, :, j].copy_(torch.randn(n_blocks, bs, FA_D, generator=g, device=dev))
            m.k_cache, m.v_cache = self.kv.layer_caches(l)
        for s, c in enumerate(ctx_lens):
            self.kv.append(s, c)

    # ------------------------------------------------------------------ metadata ----
    def step_metadata(self, n_steps: int):
        """Per decode step: (block_tables, context_lens, slot_mapping, cos, sin), reserving one
        more cache slot per sequence each step; block tables padded to the widest step."""
        meta = []
        seqs = list(range(self.n_seqs))
        for _ in range(n_steps):
            for s in seqs:
                self.kv.append(s, 1)
            bt, cl, slots = self.kv.metadata(seqs, [1] * self.n_seqs)
            cos, sin = self.rope.cos_sin((cl - 1).long())
            meta.append((bt, cl, slots, cos, sin))
        width = max(m[0].shape[1] for m in meta)
        return [(F.pad(bt, (0, width - bt.shape[1])), cl, sl, c, s_) for bt, cl, sl, c, s_ in meta]

    # ------------------------------------------------------------------- forward ----
    def forward(self, x: torch.Tensor, bt, cl, slots, cos, sin) -> torch.Tensor:
        """One decode step: x [n_seqs, hidden] -> the stack's output; updates the states and
        writes this step's K/V into the cache."""
        set_context(False, slot_mapping=slots, context_lens=cl, block_tables=bt, block_size=self.block_size)
        res = x.clone()
        h = None
        for (norm, mixer), kind in zip(self.layers, self.kinds):
            if h is None:
                normed = norm(res)
            else:
                normed, res = norm(h, residual=res)  # res += h; normed = rms(res)
            h = mixer(normed, None, self.idx, self.idx, False) if kind == "gdn" else mixer(normed, cos, sin)
        return res + h

    def bytes_per_step(self) -> dict:
        """HBM bytes one step must move on this rank: the K/V read, the states read and
        written, and the weights read once."""
        hkv = self.fa[0].num_kv_heads if self.fa else 0
        share = self.fa[0].kv_share if self.fa else 1  # a context-split rank reads 1 / share of it
        kv = sum(self.ctx_lens) * len(self.fa) * hkv * FA_D * 2 * 2 // share
        states = 2 * self.lac.recurrent_cache.numel() * 4 + 2 * self.lac.conv_cache.numel() * 2
        weights = sum(p.numel() * p.element_size() for _, m in self.layers for p in m.parameters())
        return {"kv": kv, "states": states, "weights": weights, "total": kv + states + weights}

    def snapshot(self):
        """Copies of the mutable state (GDN/conv states and the KV cache)."""
        return (self.lac.recurrent_cache.clone(), self.lac.conv_cache.clone(), self.kv.k.clone(), self.kv.v.clone())

    def restore(self, snap):
        for dst, src in zip((self.lac.recurrent_cache, self.lac.conv_cache, self.kv.k, self.kv.v), snap):
            dst.copy_(src)


def hidden_input(n_seqs: int, device, seed: int = 7) -> torch.Tensor:
    return torch.randn(n_seqs, HIDDEN, generator=torch.Generator(device=device).manual_seed(seed),
                       device=device, dtype=torch.bfloat16)
