"""Paged KV-cache write oracle (numpy) -- test infrastructure only.

The reference has no kernel for this; it is foreshadowed by the ``slot_mapping``
field of ``m/utils/context.py:15`` and implied by the cache layout that
``m/ops/full_attention.py:186-195`` reads: ``[n_blocks, block_size, Hkv, D]``.
Token t goes to flat slot ``slot_mapping[t] = block * block_size + offset``;
slot -1 means "do not store".
"""

from __future__ import annotations

import numpy as np


def store(k, v, k_cache, v_cache, slot_mapping):
    """Scatter k/v [T, Hkv, D] into the paged caches in place."""
    bs = k_cache.shape[1]
    slots = np.asarray(slot_mapping).astype(np.int64)
    keep = slots >= 0
    s = slots[keep]
    k_cache[s // bs, s % bs] = np.asarray(k)[keep]
    v_cache[s // bs, s % bs] = np.asarray(v)[keep]
