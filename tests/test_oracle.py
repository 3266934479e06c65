"""CPU tests of the oracle itself: pinned to the golden vectors produced by the reference
(tests/golden/make_golden.py) and cross-checked against independent implementations."""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_recurrent_matches_reference_kernel_c0():
    d = np.load(os.path.join(GOLDEN, "c0_gdn.npz"))
    st = np.zeros((1, 4, 64, 64))
    o = oracle.gdn.recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"], st, np.array([0]), np.array([0, 256]))
    assert np.abs(o - d["ref_o"]).max() < 1e-6
    assert np.abs(st[0] - d["ref_state"]).max() < 1e-6


def test_reference_kernel_agrees_with_fla_naive():
    d = np.load(os.path.join(GOLDEN, "c0_gdn.npz"))
    assert np.abs(d["ref_o"] - d["fla_recurrent_o"]).max() < 1e-6
    assert np.abs(d["ref_state"] - d["fla_recurrent_state"]).max() < 1e-5


@pytest.mark.parametrize("chunk", [16, 32, 64])
def test_chunked_equals_recurrent_c0(chunk):
    d = np.load(os.path.join(GOLDEN, "c0_gdn.npz"))
    st = np.zeros((1, 4, 64, 64))
    o = oracle.gdn.chunked(d["q"], d["k"], d["v"], d["g"], d["beta"], st, np.array([0]), np.array([0, 256]), chunk)
    assert np.abs(o - d["ref_o"]).max() < 1e-6
    assert np.abs(st[0] - d["ref_state"]).max() < 1e-6
    assert np.abs(o - d["fla_chunk_o"]).max() < 1e-6


def test_chunked_varlen_gqa_nonzero_state():
    rng = np.random.default_rng(0)
    lens = [1, 63, 64, 65, 0, 130]
    cu = np.concatenate([[0], np.cumsum(lens)])
    T, hk, hv, dk, dv = cu[-1], 2, 4, 32, 16
    q = rng.standard_normal((T, hk, dk)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((T, hk, dk)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, hv, dv))
    g = -rng.uniform(0.0, 0.5, (T, hv))
    b = rng.uniform(0, 1, (T, hv))
    idx = np.array([5, 0, 3, 1, 2, 4])
    s0 = rng.standard_normal((6, hv, dk, dv)) * 0.1
    s1, s2 = s0.copy(), s0.copy()
    o1 = oracle.gdn.recurrent(q, k, v, g, b, s1, idx, cu)
    o2 = oracle.gdn.chunked(q, k, v, g, b, s2, idx, cu, 64)
    assert np.abs(o1 - o2).max() < 1e-9
    assert np.abs(s1 - s2).max() < 1e-9
    assert np.array_equal(s1[2], s0[2])  # the empty sequence leaves its slot untouched


def test_paged_decode_matches_reference_kernel():
    d = np.load(os.path.join(GOLDEN, "paged_decode.npz"))
    o = oracle.attention.paged_decode(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                      float(d["scale"]))
    assert np.abs(o - d["ref_o"]).max() < 1e-5


def test_conv_matches_torch_conv1d():
    rng = np.random.default_rng(1)
    dim, W = 24, 4
    lens = [5, 1, 0, 2, 9]
    cu = np.concatenate([[0], np.cumsum(lens)])
    x = rng.standard_normal((cu[-1], dim))
    w = rng.standard_normal((dim, W))
    state = rng.standard_normal((7, W - 1, dim))
    idx = np.array([6, 0, 2, 4, 1])
    st = state.copy()
    out = oracle.conv.conv1d_fn(x, w, st, idx, cu)
    for s, n in enumerate(lens):
        xp = np.concatenate([state[idx[s]], x[cu[s]:cu[s + 1]]], 0)
        if n == 0:
            assert np.allclose(st[idx[s]], state[idx[s]])
            continue
        ref = F.conv1d(torch.tensor(xp.T[None]), torch.tensor(w[:, None, :]), groups=dim)[0].T.numpy()
        assert np.allclose(out[cu[s]:cu[s + 1]], ref / (1 + np.exp(-ref)))
        assert np.allclose(st[idx[s]], xp[n:n + W - 1])


def test_conv_update_equals_one_token_prefill():
    rng = np.random.default_rng(2)
    dim, W, S = 16, 4, 3
    x = rng.standard_normal((S, dim))
    w = rng.standard_normal((dim, W))
    state = rng.standard_normal((S, W - 1, dim))
    a, b = state.copy(), state.copy()
    idx = np.array([2, 0, 1])
    o1 = oracle.conv.conv1d_update(x, w, a, idx)
    o2 = oracle.conv.conv1d_fn(x, w, b, idx, np.arange(S + 1))
    assert np.allclose(o1, o2) and np.allclose(a, b)


@pytest.mark.parametrize("causal", [True, False])
def test_varlen_attention_matches_sdpa(causal):
    rng = np.random.default_rng(3)
    lens = [3, 17, 1]
    cu = np.concatenate([[0], np.cumsum(lens)])
    hq, hkv, d = 4, 2, 8
    q = rng.standard_normal((cu[-1], hq, d))
    k = rng.standard_normal((cu[-1], hkv, d))
    v = rng.standard_normal((cu[-1], hkv, d))
    o = oracle.attention.varlen(q, k, v, cu, 0.3, causal)
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        qt = torch.tensor(q[a:b]).transpose(0, 1)
        kt = torch.tensor(k[a:b]).transpose(0, 1).repeat_interleave(hq // hkv, 0)
        vt = torch.tensor(v[a:b]).transpose(0, 1).repeat_interleave(hq // hkv, 0)
        ref = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, scale=0.3).transpose(0, 1).numpy()
        assert np.allclose(o[a:b], ref, atol=1e-10)


def test_paged_prefill_reduces_to_varlen_when_cache_holds_only_the_prompt():
    rng = np.random.default_rng(4)
    lens = [5, 12]
    cu = np.concatenate([[0], np.cumsum(lens)])
    hq, hkv, d, bs = 4, 1, 8, 4
    q = rng.standard_normal((cu[-1], hq, d))
    k = rng.standard_normal((cu[-1], hkv, d))
    v = rng.standard_normal((cu[-1], hkv, d))
    nb = 8
    kc = np.zeros((nb, bs, hkv, d)); vc = np.zeros((nb, bs, hkv, d))
    bt = np.array([[3, 1, 0, 0], [2, 7, 5, 4]])
    slots = np.concatenate([bt[s, np.arange(n) // bs] * bs + np.arange(n) % bs for s, n in enumerate(lens)])
    oracle.kv.store(k, v, kc, vc, slots)
    o1 = oracle.attention.paged_prefill(q, kc, vc, bt, np.array(lens), cu, 0.5)
    o2 = oracle.attention.varlen(q, k, v, cu, 0.5, True)
    assert np.allclose(o1, o2)


def test_kv_store_skips_negative_slots():
    k = np.arange(12.0).reshape(3, 1, 4)
    kc = np.zeros((2, 2, 1, 4)); vc = np.zeros((2, 2, 1, 4))
    oracle.kv.store(k, k + 100, kc, vc, np.array([3, -1, 0]))
    assert np.array_equal(kc[1, 1, 0], k[0, 0]) and np.array_equal(kc[0, 0, 0], k[2, 0])
    assert np.count_nonzero(kc) == 8 - 1  # one zero element in k[0]
