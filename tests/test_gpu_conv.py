"""GPU parity: causal conv1d (varlen prefill and decode update) vs the oracle."""

import numpy as np
import pytest
import torch

import oracle
from myvllm_b200 import workloads as W
from myvllm_b200.ops.causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from tests.util import assert_close, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"


def _case(lens, dim, width, dtype, seed, n_slots=None):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    S = len(lens)
    n_slots = n_slots or S + 2
    x = torch.randn(T, dim, generator=g).to(dtype)
    w = (0.3 * torch.randn(dim, width, generator=g)).to(dtype)
    st = torch.randn(n_slots, width - 1, dim, generator=g).to(dtype)
    idx = torch.randperm(n_slots, generator=g)[:S].to(torch.int32)
    return x, w, st, idx, W.cu_from_lengths(lens, "cpu")


@pytest.mark.parametrize("width", [2, 3, 4, 6])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_conv_fn_varlen(width, dtype):
    lens = [0, 1, 2, 3, 5, 64, 65, 200]
    x, w, st, idx, cu = _case(lens, 256, width, dtype, seed=width)
    st_g = st.to(dev)
    o = causal_conv1d_fn(x.to(dev), w.to(dev), st_g, idx.to(dev), cu.to(dev))
    st_ref = to_np(st)
    ref = oracle.conv.conv1d_fn(to_np(x), to_np(w), st_ref, idx.numpy(), cu.numpy())
    assert_close(o, ref, atol=2e-2 if dtype == torch.bfloat16 else 1e-5, rtol=1e-2 if dtype == torch.bfloat16 else 1e-5)
    assert np.array_equal(to_np(st_g), st_ref)  # the new state is a copy of inputs: exact


def test_conv_fn_strided_input_and_fp32_weight():
    lens = [7, 130]
    x, w, st, idx, cu = _case(lens, 96, 4, torch.bfloat16, seed=9)
    big = torch.zeros(sum(lens), 200, dtype=torch.bfloat16)
    big[:, 50:146] = x
    xs = big.to(dev)[:, 50:146]  # row stride 200: not 16-byte aligned -> generic path
    st_g = st.to(dev)
    o = causal_conv1d_fn(xs, w.float().to(dev), st_g, idx.to(dev), cu.to(dev))
    st_ref = to_np(st)
    ref = oracle.conv.conv1d_fn(to_np(x), to_np(w), st_ref, idx.numpy(), cu.numpy())
    assert_close(o, ref)
    assert np.array_equal(to_np(st_g), st_ref)


def test_conv_fn_c1_full_size_channel_slices():
    inp = W.c1_inputs(dev)
    st0 = torch.randn_like(inp["conv_state"], dtype=torch.float32).to(torch.bfloat16)
    st = st0.clone()
    o = causal_conv1d_fn(inp["x"], inp["conv_w"], st, inp["idx"], inp["cu"])
    torch.cuda.synchronize()
    for lo in (0, 4096, 8192 - 128):
        sl = slice(lo, lo + 128)
        st_ref = to_np(st0[:, :, sl])
        ref = oracle.conv.conv1d_fn(to_np(inp["x"][:, sl]), to_np(inp["conv_w"][sl]), st_ref, inp["idx"].cpu().numpy(),
                                    inp["cu"].cpu().numpy())
        assert_close(o[:, sl], ref, what=f"channels {lo}+")
        assert np.array_equal(to_np(st[:, :, sl]), st_ref)


@pytest.mark.parametrize("width", [2, 4])
def test_conv_update(width):
    S = 9
    x, w, st, idx, _ = _case([1] * S, 8192, width, torch.bfloat16, seed=20 + width, n_slots=12)
    st_g = st.to(dev)
    o = causal_conv1d_update(x.to(dev), w.to(dev), st_g, idx.to(dev))
    st_ref = to_np(st)
    ref = oracle.conv.conv1d_update(to_np(x), to_np(w), st_ref, idx.numpy())
    assert_close(o, ref)
    assert np.array_equal(to_np(st_g), st_ref)


def test_conv_fn_c1_channels_short_sequences_permuted_slots():
    """All 8192 config-1 channels (the conv weight distribution of config 1, non-zero
    histories) on the edge cases of the state roll (m/ops/causal_conv1d.py:199-218):
    sequences of 0, 1 and 2 tokens (shorter than W - 1 = 3, so the new state keeps part of
    the old one), 3 tokens (exactly W - 1), and longer ones, written to permuted slots of a
    larger cache whose other rows must stay untouched."""
    lens = [0, 1, 2, 3, 130, 1, 64, 2]
    g = torch.Generator().manual_seed(31)
    T, dim, n_slots = sum(lens), W.GDN_CH, 13
    x = torch.randn(T, dim, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(dim, W.GDN_W, generator=g)).to(torch.bfloat16)
    st = torch.randn(n_slots, W.GDN_W - 1, dim, generator=g).to(torch.bfloat16)
    idx = torch.randperm(n_slots, generator=g)[:len(lens)].to(torch.int32)
    cu = W.cu_from_lengths(lens, "cpu")
    st_g = st.to(dev)
    o = causal_conv1d_fn(x.to(dev), w.to(dev), st_g, idx.to(dev), cu.to(dev))
    st_ref = to_np(st)
    ref = oracle.conv.conv1d_fn(to_np(x), to_np(w), st_ref, idx.numpy(), cu.numpy())
    assert_close(o, ref, what="conv out, all channels")
    assert np.array_equal(to_np(st_g), st_ref)  # rolled rows and untouched rows, bit for bit


def test_conv_update_c2_channels_permuted_slots():
    """The decode update over all 8192 channels with permuted slots, at config-2 batch."""
    S, n_slots = 256, 300
    x, w, st, idx, _ = _case([1] * S, W.GDN_CH, W.GDN_W, torch.bfloat16, seed=77, n_slots=n_slots)
    st_g = st.to(dev)
    o = causal_conv1d_update(x.to(dev), w.to(dev), st_g, idx.to(dev))
    st_ref = to_np(st)
    ref = oracle.conv.conv1d_update(to_np(x), to_np(w), st_ref, idx.numpy())
    assert_close(o, ref, what="conv update, all channels")
    assert np.array_equal(to_np(st_g), st_ref)
