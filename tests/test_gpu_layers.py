"""GPU parity of the layer modules (single rank): GatedDeltaNet prefill + decode steps and
GatedAttention prefill + decode over a paged cache, against reference forwards built from
torch fp32 math and the numpy oracle (m/layers/linear_attention.py:77-123 with the data flow
fixed; m/layers/full_attention.py:49-64 completed)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from myvllm_b200 import workloads as W
from myvllm_b200.cache.linear_attention_cache import LinearAttentionCache, PagedKVCache
from myvllm_b200.layers.full_attention import GatedAttention
from myvllm_b200.layers.linear_attention import GatedDeltaNet
from myvllm_b200.layers.rotary_embedding import RotaryEmbedding, apply_partial_rotary
from myvllm_b200.utils.context import reset_context, set_context
from tests.util import assert_close, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"


def _init(module, seed):
    g = torch.Generator().manual_seed(seed)
    for name, p in module.named_parameters():
        if name.endswith("A_log") or name.endswith("dt_bias") or "norm" in name:
            continue
        p.data.copy_(0.02 * torch.randn(p.shape, generator=g))
    return module


def _gdn_reference(layer, x, conv_state, rec_state, idx, cu, prefill):
    """Layer math around the oracle: the layer's own bf16 projections (the same cuBLAS
    calls), the oracle's conv (rounded to bf16, the activation dtype the conv writes) and
    GDN in float64, the gated norm and out_proj in fp32."""
    f = lambda t: t.detach().float()  # noqa: E731
    with torch.no_grad():
        qkv, z = layer.in_proj_qkv(x), f(layer.in_proj_z(x))
        a, b = f(layer.in_proj_a(x)), layer.in_proj_b(x)
    beta = f(torch.sigmoid(b))
    g = -f(layer.A_log).exp() * F.softplus(a + f(layer.dt_bias))
    w = to_np(layer.conv1d.weight)
    if prefill:
        qkv = oracle.conv.conv1d_fn(to_np(qkv), w, conv_state, idx, cu)
    else:
        qkv = oracle.conv.conv1d_update(to_np(qkv), w, conv_state, idx)
    qkv = torch.tensor(qkv).to(torch.bfloat16).double().numpy()
    T = x.shape[0]
    q = qkv[:, :2048].reshape(T, 16, 128)
    k = qkv[:, 2048:4096].reshape(T, 16, 128)
    v = qkv[:, 4096:].reshape(T, 32, 128)
    q = q / np.sqrt((q ** 2).sum(-1, keepdims=True) + 1e-6)
    k = k / np.sqrt((k ** 2).sum(-1, keepdims=True) + 1e-6)
    if prefill:
        o = oracle.gdn.chunked(q, k, v, to_np(g), to_np(beta), rec_state, idx, cu, 64)
    else:
        o = oracle.gdn.recurrent_step(q, k, v, to_np(g), to_np(beta), rec_state, idx)
    o = torch.tensor(o, dtype=torch.float32, device=dev)
    zz = z.view(T, 32, 128)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + 1e-6) * f(layer.norm.weight) * F.silu(zz)
    return o.reshape(T, 4096) @ f(layer.out_proj.weight).T


def test_gated_deltanet_prefill_then_decode():
    torch.manual_seed(0)
    layer = _init(GatedDeltaNet(2048, 16, 32, 128, 128, 4), 1).to(dev, torch.bfloat16)
    layer.A_log.data = layer.A_log.data.float()
    layer.dt_bias.data = layer.dt_bias.data.float()
    cache = LinearAttentionCache(1, 4, 4, 128, 128, 16, 32, torch.bfloat16, torch.device(dev))
    layer.conv_state, layer.recurrent_state = cache.layer_states(0)
    slots = [cache.allocate() for _ in range(2)]
    idx = torch.tensor(slots, dtype=torch.int32, device=dev)
    conv_ref = cache.conv_cache[0].float().cpu().numpy().astype(np.float64)
    rec_ref = cache.recurrent_cache[0].cpu().numpy().astype(np.float64)
    lens = [100, 37]
    cu = W.cu_from_lengths(lens, dev)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(sum(lens), 2048, generator=g).to(dev, torch.bfloat16)
    out = layer(x, cu, idx, idx, True)
    ref = _gdn_reference(layer, x, conv_ref, rec_ref, idx.cpu().numpy(), cu.cpu().numpy(), True)
    assert_close(out, ref, what="prefill output")
    for step in range(3):
        xd = torch.randn(2, 2048, generator=g).to(dev, torch.bfloat16)
        out = layer(xd, None, idx, idx, False)
        ref = _gdn_reference(layer, xd, conv_ref, rec_ref, idx.cpu().numpy(), None, False)
        assert_close(out, ref, what=f"decode step {step}")
    rel = np.linalg.norm(cache.recurrent_cache[0, slots].cpu().numpy() - rec_ref[slots]) / np.linalg.norm(rec_ref[slots])
    assert rel < 1e-3


def _attn_reference(layer, x, cos, sin, k_hist, v_hist):
    """One sequence: x [L, hidden] new tokens; k_hist/v_hist: fp32 [n_prev, Hkv, D] earlier keys."""
    f = lambda t: t.detach().float()  # noqa: E731
    L = x.shape[0]
    qg = (f(x) @ f(layer.q_proj.weight).T).view(L, 16, 512)
    q, gate = qg[..., :256], qg[..., 256:]
    rms = lambda t, w: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * (f(w) + 1.0)  # noqa: E731
    q = rms(q, layer.q_norm.weight)
    k = rms((f(x) @ f(layer.k_proj.weight).T).view(L, 2, 256), layer.k_norm.weight)
    v = (f(x) @ f(layer.v_proj.weight).T).view(L, 2, 256)
    q, k = apply_partial_rotary(q, cos, sin), apply_partial_rotary(k, cos, sin)
    K = torch.cat([k_hist, k]) if k_hist is not None else k
    V = torch.cat([v_hist, v]) if v_hist is not None else v
    n = K.shape[0]
    qpos = torch.arange(n - L, n, device=dev)
    mask = qpos[:, None] >= torch.arange(n, device=dev)[None, :]
    s = torch.einsum("lhd,nhd->hln", q.view(L, 2, 8, 256).reshape(L, 16, 256),
                     K.repeat_interleave(8, 1)) / 16
    p = torch.softmax(s.masked_fill(~mask[None], float("-inf")), -1)
    o = torch.einsum("hln,nhd->lhd", p, V.repeat_interleave(8, 1)) * torch.sigmoid(gate)
    return o.reshape(L, 4096) @ f(layer.o_proj.weight).T, K, V


def test_gated_attention_prefill_then_decode_paged():
    torch.manual_seed(0)
    layer = _init(GatedAttention(2048, 256, 16, 256, 2, False, 1e-6), 3).to(dev, torch.bfloat16)
    kv = PagedKVCache(1, 16, 256, 2, 256, torch.bfloat16, torch.device(dev))
    layer.k_cache, layer.v_cache = kv.layer_caches(0)
    rope = RotaryEmbedding(64, 10_000_000.0).to(dev)
    lens = [300, 41]
    g = torch.Generator().manual_seed(4)
    x = torch.randn(sum(lens), 2048, generator=g).to(dev, torch.bfloat16)
    for s, n in enumerate(lens):
        kv.append(s, n)
    bt, ctx, slots = kv.metadata([0, 1], lens)
    pos = torch.cat([torch.arange(n) for n in lens]).to(dev)
    cos, sin = rope.cos_sin(pos)
    cu = W.cu_from_lengths(lens, dev)
    set_context(True, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(lens), max_seqlen_k=max(lens),
                slot_mapping=slots, context_lens=ctx, block_tables=bt, block_size=256)
    out = layer(x, cos, sin)
    hist = []
    a = 0
    for s, n in enumerate(lens):
        ref, K, V = _attn_reference(layer, x[a:a + n], cos[a:a + n], sin[a:a + n], None, None)
        assert_close(out[a:a + n], ref, what=f"prefill seq {s}")
        hist.append((K, V))
        a += n
    for step in range(2):
        xd = torch.randn(2, 2048, generator=g).to(dev, torch.bfloat16)
        for s in range(2):
            kv.append(s, 1)
        bt, ctx, slots = kv.metadata([0, 1], [1, 1])
        posd = torch.tensor([lens[0] + step, lens[1] + step], device=dev)
        cosd, sind = rope.cos_sin(posd)
        set_context(False, slot_mapping=slots, context_lens=ctx, block_tables=bt, block_size=256)
        out = layer(xd, cosd, sind)
        for s in range(2):
            ref, K, V = _attn_reference(layer, xd[s:s + 1], cosd[s:s + 1], sind[s:s + 1], *hist[s])
            hist[s] = (K, V)
            assert_close(out[s:s + 1], ref, what=f"decode step {step} seq {s}")
    reset_context()


def test_fused_projections_match_unfused():
    """fuse_projections(): one GEMM over the concatenated input projections must give the
    same layer outputs (prefill + decode for GatedDeltaNet, prefill for GatedAttention)."""
    torch.manual_seed(0)
    layer = _init(GatedDeltaNet(2048, 16, 32, 128, 128, 4), 7).to(dev, torch.bfloat16)
    layer.A_log.data = layer.A_log.data.float()
    layer.dt_bias.data = layer.dt_bias.data.float()
    outs = []
    for fused in (False, True):
        cache = LinearAttentionCache(1, 2, 4, 128, 128, 16, 32, torch.bfloat16, torch.device(dev))
        layer.conv_state, layer.recurrent_state = cache.layer_states(0)
        slots = [cache.allocate() for _ in range(2)]
        idx = torch.tensor(slots, dtype=torch.int32, device=dev)
        if fused:
            layer.fuse_projections()
        g = torch.Generator().manual_seed(8)
        x = torch.randn(150, 2048, generator=g).to(dev, torch.bfloat16)
        xd = torch.randn(2, 2048, generator=g).to(dev, torch.bfloat16)
        cu = W.cu_from_lengths([90, 60], dev)
        outs.append((layer(x, cu, idx, idx, True), layer(xd, None, idx, idx, False),
                     cache.recurrent_cache[0, slots].clone()))
    for a, b in zip(outs[0][:2], outs[1][:2]):
        assert_close(b, a)
    assert ((outs[1][2] - outs[0][2]).norm() / outs[0][2].norm()).item() < 1e-3

    attn = _init(GatedAttention(2048, 256, 16, 256, 2, False, 1e-6), 9).to(dev, torch.bfloat16)
    lens = [200, 33]
    g = torch.Generator().manual_seed(10)
    x = torch.randn(sum(lens), 2048, generator=g).to(dev, torch.bfloat16)
    rope = RotaryEmbedding(64, 10_000_000.0).to(dev)
    cos, sin = rope.cos_sin(torch.cat([torch.arange(n) for n in lens]).to(dev))
    cu = W.cu_from_lengths(lens, dev)
    set_context(True, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(lens), max_seqlen_k=max(lens))
    o1 = attn(x, cos, sin)
    attn.fuse_projections()
    o2 = attn(x, cos, sin)
    reset_context()
    assert_close(o2, o1)
