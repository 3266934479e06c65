"""Full-attention oracles (numpy) -- test infrastructure only.

Layouts follow ``m/ops/full_attention.py``:
  varlen:  q [T, Hq, D], k/v [T, Hkv, D], cu_seqlens [S+1]             (``:114-125``)
  paged:   k_cache/v_cache [n_blocks, block_size, Hkv, D], block_tables [S, max_blocks],
           context_lens [S]                                             (``:282-290``)
  q-head h reads kv-head h // (Hq // Hkv)                               (``:37, :211``)
"""

from __future__ import annotations

import numpy as np


def _softmax_attend(q, k, v, scale, mask):
    """q [Hq, M, D], k/v [Hq, N, D] (already GQA-expanded), mask [M, N] bool or None."""
    s = scale * (q @ k.transpose(0, 2, 1))
    if mask is not None:
        s = np.where(mask[None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    return (p @ v) / np.where(l > 0, l, 1.0)


def varlen(q, k, v, cu_seqlens, scale, causal, dtype=np.float64):
    """``flash_attention_prefill`` (``m/ops/full_attention.py:114-173``, kernel ``:86-111``):
    per sequence softmax(scale q k^T [+ causal mask]) v with online-softmax semantics."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    T, hq, _ = q.shape
    hkv = k.shape[1]
    rep = hq // hkv
    o = np.zeros((T, hq, v.shape[2]), dtype)
    cu = np.asarray(cu_seqlens).astype(np.int64)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        if b == a:
            continue
        L = b - a
        qs = q[a:b].transpose(1, 0, 2)
        ks = np.repeat(k[a:b].transpose(1, 0, 2), rep, axis=0)
        vs = np.repeat(v[a:b].transpose(1, 0, 2), rep, axis=0)
        mask = np.tril(np.ones((L, L), bool)) if causal else None
        o[a:b] = _softmax_attend(qs, ks, vs, scale, mask).transpose(1, 0, 2)
    return o


def gather_paged(cache, block_table, n_tokens):
    """Tokens [0, n_tokens) of one sequence from a paged cache -> [n_tokens, Hkv, D]."""
    bs = cache.shape[1]
    pos = np.arange(n_tokens)
    blocks = np.asarray(block_table)[pos // bs].astype(np.int64)
    return cache[blocks, pos % bs]


def paged_decode(q, k_cache, v_cache, block_tables, context_lens, scale, dtype=np.float64):
    """``paged_flash_attention_decode`` (``m/ops/full_attention.py:282-335``, kernel
    ``:208-279``): one query per sequence attends to its first ``context_lens[s]``
    cached tokens, located through ``block_tables[s, pos // block_size]``."""
    q = np.asarray(q, dtype)
    S, hq, _ = q.shape
    hkv = k_cache.shape[2]
    rep = hq // hkv
    o = np.zeros((S, hq, v_cache.shape[3]), dtype)
    for s in range(S):
        n = int(context_lens[s])
        if n == 0:
            continue
        ks = np.repeat(np.asarray(gather_paged(k_cache, block_tables[s], n), dtype).transpose(1, 0, 2), rep, 0)
        vs = np.repeat(np.asarray(gather_paged(v_cache, block_tables[s], n), dtype).transpose(1, 0, 2), rep, 0)
        o[s] = _softmax_attend(q[s][:, None, :], ks, vs, scale, None)[:, 0]
    return o


def paged_prefill(q, k_cache, v_cache, block_tables, context_lens, cu_seqlens, scale,
                  dtype=np.float64):
    """``paged_flash_attention_prefill`` (``m/ops/full_attention.py:454-512``, kernel
    ``:373-451``): the L_s new queries of sequence s sit at positions
    ``context_lens[s] - L_s + i`` (``:393``) and attend causally to cached tokens
    ``[0, context_lens[s])`` (which already include the new tokens)."""
    q = np.asarray(q, dtype)
    T, hq, _ = q.shape
    hkv = k_cache.shape[2]
    rep = hq // hkv
    o = np.zeros((T, hq, v_cache.shape[3]), dtype)
    cu = np.asarray(cu_seqlens).astype(np.int64)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        L = b - a
        n = int(context_lens[s])
        if L == 0 or n == 0:
            continue
        ks = np.repeat(np.asarray(gather_paged(k_cache, block_tables[s], n), dtype).transpose(1, 0, 2), rep, 0)
        vs = np.repeat(np.asarray(gather_paged(v_cache, block_tables[s], n), dtype).transpose(1, 0, 2), rep, 0)
        qpos = n - L + np.arange(L)
        mask = qpos[:, None] >= np.arange(n)[None, :]
        o[a:b] = _softmax_attend(q[a:b].transpose(1, 0, 2), ks, vs, scale, mask).transpose(1, 0, 2)
    return o


def varlen_flops(cu_seqlens, hq, d, dv, causal=True):
    """Algorithmic FLOPs of causal varlen attention: sum_s 2 Hq L(L+1)/2 (D + Dv)."""
    cu = np.asarray(cu_seqlens).astype(np.int64)
    L = cu[1:] - cu[:-1]
    pairs = L * (L + 1) // 2 if causal else L * L
    return int(2 * hq * (d + dv) * pairs.sum())
