"""GPU: the hybrid decode step as the bench runs it -- a slice of the config-4 stack (3 GDN
layers + 1 gated attention layer, 32 sequences, non-zero GDN/conv states, a paged bf16 KV
cache with real contexts) -- captured as one CUDA graph and replayed.

1. Replayed steps must give the same bits as the same steps run eagerly, for the outputs
   and for everything the step mutates (recurrent and conv states, the KV cache).
2. The eager step is checked layer by layer against the layer math of the reference
   (m/layers/linear_attention.py:77-123 and m/layers/full_attention.py:49-64, as restated
   with the oracle in tests/test_gpu_layers.py)."""

import numpy as np
import pytest
import torch

from myvllm_b200 import workloads as W
from myvllm_b200.decode_stack import HybridDecodeStack, hidden_input
from myvllm_b200.utils.context import reset_context, set_context
from tests.test_gpu_layers import _attn_reference, _gdn_reference
from tests.util import assert_close, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
S = 32


@pytest.fixture(scope="module")
def stack():
    ctx = W.seq_lengths(S, 200, 3000, 21)
    st = HybridDecodeStack(4, S, ctx, 8, dev, seed=77)
    yield st
    reset_context()


def _mutable(st):
    return [st.lac.recurrent_cache, st.lac.conv_cache, st.kv.k, st.kv.v]


def test_graph_replay_matches_eager_bit_for_bit(stack):
    meta = stack.step_metadata(3)
    x = hidden_input(S, dev, seed=4)
    snap = stack.snapshot()
    with torch.no_grad():
        eager = [stack.forward(x, *m).clone() for m in meta]
        after_eager = [t.clone() for t in _mutable(stack)]
        # capture with static metadata buffers (warm-up on a side stream first)
        stack.restore(snap)
        static = [t.clone() for t in meta[0]]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            stack.forward(x, *static)
        torch.cuda.current_stream().wait_stream(side)
        stack.restore(snap)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = stack.forward(x, *static)
        stack.restore(snap)
        replayed = []
        for m in meta:
            for dst, src in zip(static, m):
                dst.copy_(src)
            graph.replay()
            replayed.append(out.clone())
        torch.cuda.synchronize()
        del graph
    for i, (a, b) in enumerate(zip(replayed, eager)):
        assert torch.equal(a, b), f"step {i}: replayed output differs from eager"
    for name, a, b in zip(("recurrent", "conv", "k_cache", "v_cache"), _mutable(stack), after_eager):
        assert torch.equal(a, b), f"{name} after replay differs from eager"
    stack.restore(snap)


def test_eager_step_layer_by_layer_vs_reference_math(stack):
    """One eager step; every layer's output is compared with the reference layer math on
    the same layer input (the GDN layers with the oracle's conv and recurrent step in
    float64, the attention layer with fp32 torch attention over the cached keys)."""
    meta = stack.step_metadata(1)[0]
    bt, cl, slots, cos, sin = meta
    x = hidden_input(S, dev, seed=6)
    idx = stack.idx
    set_context(False, slot_mapping=slots, context_lens=cl, block_tables=bt, block_size=stack.block_size)
    with torch.no_grad():
        res, h = x.clone(), None
        g = 0
        for (norm, mixer), kind in zip(stack.layers, stack.kinds):
            normed = norm(res) if h is None else norm(h, residual=res)[0]
            if kind == "gdn":
                conv_ref = to_np(mixer.conv_state)
                rec_ref = to_np(mixer.recurrent_state)
                h = mixer(normed, None, idx, idx, False)
                ref = _gdn_reference(mixer, normed, conv_ref, rec_ref, idx.cpu().numpy(), None, False)
                assert_close(h, ref, what=f"GDN layer {g}")
                rel = np.linalg.norm(to_np(mixer.recurrent_state) - rec_ref) / np.linalg.norm(rec_ref)
                assert rel < 1e-3, f"GDN layer {g} state rel err {rel:.2e}"
                g += 1
            else:
                # cached keys/values of every sequence before this step's write, in fp32
                hist = []
                cl_h, bt_h = cl.cpu().tolist(), bt.cpu()
                for s in range(S):
                    pos = torch.arange(cl_h[s] - 1)
                    blk = bt_h[s, pos // stack.block_size].long()
                    off = pos % stack.block_size
                    hist.append((mixer.k_cache[blk, off].float(), mixer.v_cache[blk, off].float()))
                h = mixer(normed, cos, sin)
                for s in range(S):
                    ref, _, _ = _attn_reference(mixer, normed[s:s + 1], cos[s:s + 1], sin[s:s + 1], *hist[s])
                    assert_close(h[s:s + 1], ref, what=f"attention layer, seq {s}")
    reset_context()
