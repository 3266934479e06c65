"""Causal depthwise conv1d oracle (numpy) -- test infrastructure only.

Restates the intended math of ``m/ops/causal_conv1d.py`` (the Triton kernels do not
run as written, see ``causal_conv1d.py:33, 53, 202``):

  xp = concat(conv_state[idx] (W-1 rows), x_seq)                (``:39-63``)
  out[t, c] = silu(sum_{j<W} w[c, j] * xp[t + j, c])            (``:136-196``, fp32 acc)
  conv_state[idx] <- last W-1 rows of xp                        (``:199-218``)

Layouts: x [T, dim]; weight [dim, W]; conv_state [S_max, W-1, dim] (``:224``).
"""

from __future__ import annotations

import numpy as np


def _silu(a):
    return a / (1.0 + np.exp(-a))


def conv1d_fn(x, weight, conv_state, conv_state_indices, cu_seqlens, dtype=np.float64):
    """Varlen prefill (``causal_conv1d_fn``, ``m/ops/causal_conv1d.py:221-273``).

    Updates ``conv_state`` in place; returns out [T, dim] in ``dtype``.
    """
    x = np.asarray(x, dtype)
    w = np.asarray(weight, dtype)
    W = w.shape[1]
    T, dim = x.shape
    out = np.zeros((T, dim), dtype)
    cu = np.asarray(cu_seqlens).astype(np.int64)
    for s in range(len(cu) - 1):
        slot = int(conv_state_indices[s])
        L = cu[s + 1] - cu[s]
        xp = np.concatenate([np.asarray(conv_state[slot], dtype), x[cu[s]:cu[s + 1]]], axis=0)
        acc = np.zeros((L, dim), dtype)
        for j in range(W):
            acc += xp[j:j + L] * w[:, j][None, :]
        out[cu[s]:cu[s + 1]] = _silu(acc)
        conv_state[slot] = xp[L:L + W - 1].astype(conv_state.dtype)
    return out


def conv1d_update(x, weight, conv_state, conv_state_indices, dtype=np.float64):
    """One token per sequence (``causal_conv1d_update``, ``m/ops/causal_conv1d.py:434-470``,
    kernel ``:277-431``); shifts ``conv_state[idx]`` in place."""
    x = np.asarray(x, dtype)
    w = np.asarray(weight, dtype)
    W = w.shape[1]
    idx = np.asarray(conv_state_indices).astype(np.int64)
    st = np.asarray(conv_state[idx], dtype)  # [S, W-1, dim]
    xp = np.concatenate([st, x[:, None, :]], axis=1)  # [S, W, dim]
    acc = np.einsum("swc,cw->sc", xp, w)
    conv_state[idx] = xp[:, 1:].astype(conv_state.dtype)
    return _silu(acc)
