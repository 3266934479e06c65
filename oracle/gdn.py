"""Gated delta rule oracle (numpy) -- test infrastructure only, see ``oracle/__init__``.

Conventions (reference ``m/ops/gated_delta_rule/gated_delta_rule.py:31-92``):
  q, k  [T, Hk, K]      v [T, Hv, V]      g, beta [T, Hv]  (g = natural-log decay)
  state [S_max, Hv, K, V] fp32, addressed through ``state_indices`` (one row per seq)
  v-head h reads k-head ``h // (Hv // Hk)`` (``chunk_scaled_dot_kkt.py:35``,
  ``fused_recurrent_gdn.py:47``); scale = K ** -0.5 (``fused_recurrent_gdn.py:117``).
"""

from __future__ import annotations

import numpy as np


def _expand_heads(x: np.ndarray, hv: int) -> np.ndarray:
    """[T, Hk, D] -> [T, Hv, D] with v-head h reading k-head h // (Hv // Hk)."""
    hk = x.shape[1]
    assert hv % hk == 0
    return np.repeat(x, hv // hk, axis=1)


def recurrent_step(q, k, v, g, beta, state, state_indices, scale=None, dtype=np.float64):
    """One decode token per sequence, in place on ``state``.

    Follows ``m/ops/gated_delta_rule/fused_recurrent_gdn.py:46-101``:
      S <- exp(g) * S                       (:49, :96)
      v' = beta * (v - k^T S)               (:50, :97)
      S <- S + k v'^T                       (:98)
      o  = (scale * q)^T S                  (:68, :99)
    Returns o [S, Hv, V] (float64 unless ``dtype`` says otherwise).
    """
    n, hk, kd = q.shape
    hv = v.shape[1]
    if scale is None:
        scale = kd ** -0.5
    qf = _expand_heads(np.asarray(q, dtype), hv) * scale
    kf = _expand_heads(np.asarray(k, dtype), hv)
    vf = np.asarray(v, dtype)
    gf = np.asarray(g, dtype)
    bf = np.asarray(beta, dtype)
    idx = np.asarray(state_indices).astype(np.int64)
    S = np.asarray(state[idx], dtype)  # [n, Hv, K, V]
    S = S * np.exp(gf)[:, :, None, None]
    kS = np.einsum("nhk,nhkv->nhv", kf, S)
    vp = bf[:, :, None] * (vf - kS)
    S = S + kf[:, :, :, None] * vp[:, :, None, :]
    o = np.einsum("nhk,nhkv->nhv", qf, S)
    state[idx] = S.astype(state.dtype)
    return o


def recurrent(q, k, v, g, beta, state, state_indices, cu_seqlens, scale=None, dtype=np.float64):
    """Token-by-token gated delta rule over packed varlen sequences.

    Applies ``recurrent_step`` (the K12 update, ``fused_recurrent_gdn.py:96-99``) to
    every token of every sequence in order, starting from ``state[state_indices[s]]``
    and writing the final state back there.  This is the sequential definition the
    chunked form (``chunked``) must reproduce.
    """
    T, hk, kd = q.shape
    hv, vd = v.shape[1], v.shape[2]
    o = np.zeros((T, hv, vd), dtype)
    cu = np.asarray(cu_seqlens).astype(np.int64)
    for s in range(len(cu) - 1):
        slot = np.asarray([state_indices[s]])
        for t in range(cu[s], cu[s + 1]):
            o[t] = recurrent_step(q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1], beta[t:t + 1],
                                  state, slot, scale, dtype)[0]
    return o


def chunked(q, k, v, g, beta, state, state_indices, cu_seqlens, chunk_size=64, scale=None,
            dtype=np.float64):
    """Chunked (WY-form) gated delta rule over packed varlen sequences.

    Restates the pipeline of ``m/ops/gated_delta_rule/gated_delta_rule.py:44-64``:
      G   = in-chunk cumsum of g                            (``cumsum.py:39``; the
            reference scales by 1/ln2 and uses exp2 -- identical math)
      A   = strict_lower(beta_i (k_i . k_j) exp(G_i - G_j))  (``chunk_scaled_dot_kkt.py:55-84``)
      Ti  = (I + A)^-1                                      (``solve_tril.py:82-83``)
      u   = Ti (beta v),  w = Ti (beta exp(G) k)            (``wu.py:94-95, 130-131``)
      per chunk, serially (``h.py:118-192``):
        v_new = u - w S
        o     = scale (exp(G) (q S) + causal(q k^T exp(G_i - G_j)) v_new)   (``o.py:89-121``)
        S     = exp(G_last) S + k^T (exp(G_last - G) v_new)
    Unlike the reference (``h.py:61-67``) the incoming state ``state[idx]`` is read;
    for a zeroed slot this is identical.  The final state is written back (``h.py:178-192``).
    """
    T, hk, kd = q.shape
    hv, vd = v.shape[1], v.shape[2]
    if scale is None:
        scale = kd ** -0.5
    qf = _expand_heads(np.asarray(q, dtype), hv)
    kf = _expand_heads(np.asarray(k, dtype), hv)
    vf = np.asarray(v, dtype)
    gf = np.asarray(g, dtype)
    bf = np.asarray(beta, dtype)
    o = np.zeros((T, hv, vd), dtype)
    cu = np.asarray(cu_seqlens).astype(np.int64)
    for s in range(len(cu) - 1):
        slot = int(state_indices[s])
        S = np.asarray(state[slot], dtype).copy()  # [Hv, K, V]
        for c0 in range(cu[s], cu[s + 1], chunk_size):
            c1 = min(c0 + chunk_size, cu[s + 1])
            n = c1 - c0
            qc = qf[c0:c1].transpose(1, 0, 2)  # [Hv, n, K]
            kc = kf[c0:c1].transpose(1, 0, 2)
            vc = vf[c0:c1].transpose(1, 0, 2)  # [Hv, n, V]
            bc = bf[c0:c1].T  # [Hv, n]
            G = np.cumsum(gf[c0:c1].T, axis=1)  # [Hv, n]
            diff = G[:, :, None] - G[:, None, :]
            strict = np.tril(np.ones((n, n), bool), -1)
            incl = np.tril(np.ones((n, n), bool), 0)
            dstrict = np.where(strict, np.exp(np.where(strict, diff, 0.0)), 0.0)
            dincl = np.where(incl, np.exp(np.where(incl, diff, 0.0)), 0.0)
            A = bc[:, :, None] * (kc @ kc.transpose(0, 2, 1)) * dstrict
            Ti = np.linalg.inv(np.eye(n)[None] + A)
            u = Ti @ (bc[:, :, None] * vc)
            w = Ti @ (bc[:, :, None] * np.exp(G)[:, :, None] * kc)
            v_new = u - w @ S
            attn = (qc @ kc.transpose(0, 2, 1)) * dincl
            oc = scale * (np.exp(G)[:, :, None] * (qc @ S) + attn @ v_new)
            o[c0:c1] = oc.transpose(1, 0, 2)
            Gl = G[:, -1]
            S = np.exp(Gl)[:, None, None] * S + kc.transpose(0, 2, 1) @ (
                np.exp(Gl[:, None] - G)[:, :, None] * v_new)
        state[slot] = S.astype(state.dtype)
    return o


def flops_per_token_per_head(chunk_size: int, kd: int, vd: int) -> int:
    """Dense algorithmic FLOPs of the chunked form per token per v-head.

    kk^T, qk^T, w = Ti(beta e^G k): 3 C^2 K MACs per chunk; u = Ti(beta v),
    attn v_new: 2 C^2 V; w S, q S, k^T v_new: 3 C K V.  Per token: 2C(3K+2V) + 6KV.
    """
    return 2 * chunk_size * (3 * kd + 2 * vd) + 6 * kd * vd
