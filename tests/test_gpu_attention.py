"""GPU parity: varlen flash-attention prefill, paged decode, paged prefill and the
paged KV write vs the oracle (and torch fp32 attention at full sizes)."""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from myvllm_b200 import workloads as W
from myvllm_b200.ops.full_attention import (flash_attention_prefill, paged_flash_attention_decode,
                                            paged_flash_attention_prefill)
from myvllm_b200.ops.kv_cache import store_kvcache
from tests.util import assert_close, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
dev = "cuda"


def _qkv(lens, hq, hkv, d, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    return (torch.randn(T, hq, d, generator=g).to(dtype), torch.randn(T, hkv, d, generator=g).to(dtype),
            torch.randn(T, hkv, d, generator=g).to(dtype))


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("causal", [True, False])
def test_varlen_prefill_vs_oracle(d, causal):
    lens = [1, 17, 128, 129, 300, 0, 64]
    q, k, v = _qkv(lens, 16, 2, d, seed=d)
    cu = W.cu_from_lengths(lens, "cpu")
    scale = d ** -0.5
    o = flash_attention_prefill(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), scale, 16, 2, d, d, causal)
    ref = oracle.attention.varlen(to_np(q), to_np(k), to_np(v), cu.numpy(), scale, causal)
    assert_close(o, ref)


def test_varlen_prefill_c3_full_size_vs_torch_fp32():
    inp = W.c3_inputs(dev)
    o = flash_attention_prefill(inp["q"], inp["k"], inp["v"], inp["cu"], inp["scale"], 16, 2, 256, 256, True)
    from myvllm_b200 import _lib

    assert _lib.last_path(_lib.OP_FA_PREFILL)[0] == "tensor_core"  # config 3 runs the tcgen05 kernel
    cu = inp["cu"].tolist()
    for s in (0, len(cu) - 2):
        a, b = cu[s], cu[s + 1]
        for h in (0, 9):
            qf = inp["q"][a:b, h].float()[None]
            kf = inp["k"][a:b, h // 8].float()[None]
            vf = inp["v"][a:b, h // 8].float()[None]
            ref = F.scaled_dot_product_attention(qf, kf, vf, is_causal=True, scale=inp["scale"])[0]
            assert_close(o[a:b, h], ref, what=f"seq {s} head {h}")


def _paged(lens_ctx, hkv, d, bs, seed, dtype=torch.bfloat16, extra_blocks=3, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    nb_per = [max(1, (n + bs - 1) // bs) for n in lens_ctx]
    n_blocks = sum(nb_per) + extra_blocks
    perm = torch.randperm(n_blocks, generator=g)
    mb = max(nb_per)
    bt = torch.full((len(lens_ctx), mb), -1, dtype=torch.int32)  # unused entries are garbage (-1)
    o = 0
    for s, nb in enumerate(nb_per):
        bt[s, :nb] = perm[o:o + nb].to(torch.int32)
        o += nb
    if device == "cpu":
        kc = torch.randn(n_blocks, bs, hkv, d, generator=g).to(dtype)
        vc = torch.randn(n_blocks, bs, hkv, d, generator=g).to(dtype)
    else:
        gd = torch.Generator(device=device).manual_seed(seed)
        kc = torch.randn(n_blocks, bs, hkv, d, generator=gd, device=device, dtype=dtype)
        vc = torch.randn(n_blocks, bs, hkv, d, generator=gd, device=device, dtype=dtype)
    return kc, vc, bt


def test_paged_decode_golden():
    z = np.load(os.path.join(GOLDEN, "paged_decode.npz"))
    q, kc, vc = (torch.tensor(z[n]).to(torch.bfloat16) for n in ("q", "k_cache", "v_cache"))
    bt, ctx = torch.tensor(z["block_tables"]), torch.tensor(z["context_lens"])
    scale, bs = float(z["scale"]), int(z["block_size"])
    o = paged_flash_attention_decode(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), ctx.to(dev), scale, bs)
    ref = oracle.attention.paged_decode(to_np(q), to_np(kc), to_np(vc), bt.numpy(), ctx.numpy(), scale)
    assert_close(o, ref)
    # and the reference kernel's own fp32 output, within bf16 input-rounding tolerance
    assert np.abs(to_np(o) - z["ref_o"]).max() < 5e-2


@pytest.mark.parametrize("hq,hkv", [(16, 2), (4, 1), (2, 1), (8, 8), (16, 1)])
@pytest.mark.parametrize("d", [128, 256])
def test_paged_decode_vs_oracle(hq, hkv, d):
    ctx = [1, 255, 256, 257, 1000, 5000, 0, 63]
    bs = 256
    kc, vc, bt = _paged(ctx, hkv, d, bs, seed=hq + d)
    g = torch.Generator().manual_seed(1)
    q = torch.randn(len(ctx), hq, d, generator=g).to(torch.bfloat16)
    ctx_t = torch.tensor(ctx, dtype=torch.int32)
    o = paged_flash_attention_decode(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), ctx_t.to(dev), d ** -0.5, bs)
    ref = oracle.attention.paged_decode(to_np(q), to_np(kc), to_np(vc), bt.clamp_min(0).numpy(), ctx, d ** -0.5)
    assert_close(o, ref)


def test_paged_decode_small_block_and_unsplit():
    ctx = [3, 40, 17]
    kc, vc, bt = _paged(ctx, 2, 64, 16, seed=7)
    q = torch.randn(3, 8, 64).to(torch.bfloat16)
    o = paged_flash_attention_decode(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev),
                                     torch.tensor(ctx, dtype=torch.int32, device=dev), 0.125, 16)
    ref = oracle.attention.paged_decode(to_np(q), to_np(kc), to_np(vc), bt.clamp_min(0).numpy(), ctx, 0.125)
    assert_close(o, ref)


def test_paged_decode_c4_shapes_vs_torch_fp32():
    """Config-4 attention shapes: 128 seqs, ctx ~U[1024, 32768], Hq=16, Hkv=2, D=256, block 256."""
    ctx = W.seq_lengths(128, 1024, 32768, 4)
    kc, vc, bt = _paged(ctx, 2, 256, 256, seed=4, extra_blocks=0, device=dev)
    q = torch.randn(128, 16, 256).to(torch.bfloat16).to(dev)
    bt = bt.to(dev)
    o = paged_flash_attention_decode(q, kc, vc, bt, torch.tensor(ctx, dtype=torch.int32, device=dev), 1 / 16, 256)
    for s in (0, 77, 127):
        n = ctx[s]
        blocks = bt[s, torch.arange(n, device=dev) // 256].long()
        kk = kc[blocks, torch.arange(n, device=dev) % 256].float()  # [n, 2, 256]
        vv = vc[blocks, torch.arange(n, device=dev) % 256].float()
        qq = q[s].float().view(2, 8, 256)
        p = torch.softmax(torch.einsum("hgd,nhd->hgn", qq, kk) / 16, -1)
        ref = torch.einsum("hgn,nhd->hgd", p, vv).reshape(16, 256)
        assert_close(o[s], ref, what=f"seq {s}")


def test_store_kvcache_exact():
    T, hkv, d, bs, nb = 50, 2, 256, 16, 8
    g = torch.Generator().manual_seed(0)
    k = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    v = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * bs, generator=g)[:T].to(torch.int32)
    slots[::7] = -1
    kc = torch.zeros(nb, bs, hkv, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kc_g, vc_g = kc.to(dev), vc.to(dev)
    store_kvcache(k.to(dev), v.to(dev), kc_g, vc_g, slots.to(dev))
    kr, vr = kc.float().numpy(), vc.float().numpy()
    oracle.kv.store(k.float().numpy(), v.float().numpy(), kr, vr, slots.numpy())
    assert np.array_equal(kc_g.float().cpu().numpy(), kr)
    assert np.array_equal(vc_g.float().cpu().numpy(), vr)


def test_c3_kv_write_then_paged_prefill_equals_varlen():
    """Config-3 style: write K/V through slot_mapping into a permuted paged cache, then the
    paged prefill over that cache must equal the varlen prefill (same causal math)."""
    inp = W.c3_inputs(dev, lengths=[1000, 257, 2048, 5])
    bs = inp["block_size"]
    kc = torch.zeros(inp["n_blocks"], bs, 2, 256, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    store_kvcache(inp["k"], inp["v"], kc, vc, inp["slot_mapping"])
    ctx = torch.tensor(inp["lengths"], dtype=torch.int32, device=dev)
    o1 = paged_flash_attention_prefill(inp["q"], kc, vc, inp["block_tables"], ctx, inp["cu"], None, inp["scale"], bs)
    o2 = flash_attention_prefill(inp["q"], inp["k"], inp["v"], inp["cu"], inp["scale"], 16, 2, 256, 256, True)
    assert_close(o1, o2)


def test_paged_prefill_with_prior_context_vs_oracle():
    ctx = [300, 40, 513]
    new = [20, 40, 1]
    kc, vc, bt = _paged(ctx, 2, 128, 64, seed=13)
    g = torch.Generator().manual_seed(2)
    q = torch.randn(sum(new), 16, 128, generator=g).to(torch.bfloat16)
    cu = W.cu_from_lengths(new, "cpu")
    o = paged_flash_attention_prefill(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev),
                                      torch.tensor(ctx, dtype=torch.int32, device=dev), cu.to(dev), None,
                                      128 ** -0.5, 64)
    ref = oracle.attention.paged_prefill(to_np(q), to_np(kc), to_np(vc), bt.clamp_min(0).numpy(), ctx, cu.numpy(),
                                         128 ** -0.5)
    assert_close(o, ref)


@pytest.mark.parametrize("bs", [16, 48, 64, 128, 192, 256])
@pytest.mark.parametrize("d", [64, 256])
def test_paged_prefill_block_sizes_vs_oracle(bs, d):
    """Block sizes below, inside and above the 128-key K/V tile (16 / 64: eight / two pages
    per tile; 128 / 256: one page segment per tile; 48 and 192: pages straddle tiles,
    served by the mma.sync kernel)."""
    ctx = [700, 40, 129, 1]
    new = [300, 40, 64, 1]
    kc, vc, bt = _paged(ctx, 2, d, bs, seed=bs + d)
    g = torch.Generator().manual_seed(3)
    q = torch.randn(sum(new), 8, d, generator=g).to(torch.bfloat16)
    cu = W.cu_from_lengths(new, "cpu")
    o = paged_flash_attention_prefill(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev),
                                      torch.tensor(ctx, dtype=torch.int32, device=dev), cu.to(dev), None,
                                      d ** -0.5, bs)
    ref = oracle.attention.paged_prefill(to_np(q), to_np(kc), to_np(vc), bt.clamp_min(0).numpy(), ctx, cu.numpy(),
                                         d ** -0.5)
    assert_close(o, ref)


@pytest.mark.parametrize("d", [128, 256])
def test_varlen_prefill_fp16_and_strided_q(d):
    """fp16 operands, and q/k/v as column slices of one packed [T, (Hq + 2 Hkv) D] buffer."""
    lens = [513, 64, 1000]
    T, hq, hkv = sum(lens), 8, 2
    g = torch.Generator().manual_seed(d)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.float16)
    q = qkv[:, :hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    cu = W.cu_from_lengths(lens, "cpu")
    qkv_d = qkv.to(dev)
    o = flash_attention_prefill(qkv_d[:, :hq * d].view(T, hq, d), qkv_d[:, hq * d:(hq + hkv) * d].view(T, hkv, d),
                                qkv_d[:, (hq + hkv) * d:].view(T, hkv, d), cu.to(dev), d ** -0.5, hq, hkv, d, d, True)
    ref = oracle.attention.varlen(to_np(q), to_np(k), to_np(v), cu.numpy(), d ** -0.5, True)
    assert_close(o, ref)


@pytest.mark.parametrize("ctx_lens", [[3000, 17, 256, 8000], [1, 40]])
def test_paged_decode_output_gate(ctx_lens):
    """mvb_paged_attention_decode_gated: the gated attention's o * sigmoid(gate) applied in the
    decode kernel (split and unsplit paths) against the plain decode times a torch sigmoid;
    the gate is a strided view, as the layer slices it from its fused projection."""
    kc, vc, bt = _paged(ctx_lens, 2, 256, 256, seed=12, device=dev)
    g = torch.Generator(device=dev).manual_seed(13)
    q = torch.randn(len(ctx_lens), 16, 256, generator=g, device=dev).to(torch.bfloat16)
    qg = torch.randn(len(ctx_lens), 16, 512, generator=g, device=dev).to(torch.bfloat16)
    gate = qg[..., 256:]  # row strides 8192 / 512, as in [q | gate] per head
    ctx = torch.tensor(ctx_lens, dtype=torch.int32, device=dev)
    plain = paged_flash_attention_decode(q, kc, vc, bt.to(dev), ctx, 1 / 16, 256)
    gated = paged_flash_attention_decode(q, kc, vc, bt.to(dev), ctx, 1 / 16, 256, output_gate=gate)
    ref = plain.float() * torch.sigmoid(gate.float())
    assert_close(gated, ref, what="gated decode")


@pytest.mark.parametrize("n_parts", [2, 4])
@pytest.mark.parametrize("ctx_lens", [[3000, 17, 256, 8000, 33000], [1, 40]])
def test_paged_decode_context_parts(n_parts, ctx_lens):
    """Context-split decode (TP past the kv head count): each part attends over every
    n_parts-th split of each context; merged with the gathered log-sum-exps and the output
    gate, the parts' shares sum to the gated decode over the whole context.  Short contexts
    leave some parts without keys (their lse is -inf and their share zero)."""
    from myvllm_b200.ops.full_attention import merge_attention_parts, paged_flash_attention_decode_part

    kc, vc, bt = _paged(ctx_lens, 2, 256, 256, seed=21, device=dev)
    g = torch.Generator(device=dev).manual_seed(22)
    q = torch.randn(len(ctx_lens), 16, 256, generator=g, device=dev).to(torch.bfloat16)
    qg = torch.randn(len(ctx_lens), 16, 512, generator=g, device=dev).to(torch.bfloat16)
    gate = qg[..., 256:]
    ctx = torch.tensor(ctx_lens, dtype=torch.int32, device=dev)
    parts = [paged_flash_attention_decode_part(q, kc, vc, bt.to(dev), ctx, 1 / 16, 256, p, n_parts)
             for p in range(n_parts)]
    lse_all = torch.stack([lse for _, lse in parts])
    assert torch.isfinite(lse_all).any(0).all(), "every (sequence, head) has keys in some part"
    total = sum(merge_attention_parts(o_p, lse_all, p, output_gate=gate).float() for p, (o_p, _) in enumerate(parts))
    full = paged_flash_attention_decode(q, kc, vc, bt.to(dev), ctx, 1 / 16, 256, output_gate=gate)
    assert_close(total, full.float(), what=f"{n_parts} context parts")
    if len(ctx_lens) == 2:  # the 1-token context lies in part 0 only
        assert torch.isneginf(lse_all[1:, 0]).all()


def test_paged_decode_largest_first_order_is_bit_identical():
    """With long splits the decode orders its split work largest first (a one-block kernel
    builds the order in the workspace); the partials and their merge are the same as in grid
    order, so the output is bit-identical to a call whose workspace has no room for the
    order table.  Contexts include exact multiples of the split length (no partial split),
    a single token and a split plus one token."""
    from myvllm_b200 import _lib

    split = 6592  # the policy's split for 128 sequences x 2 kv heads and a 32768 bound
    ctx = W.seq_lengths(128, 1024, 32768, 4)
    ctx[:6] = [split, 2 * split, 1, split + 1, 32768, 64]
    kc, vc, bt = _paged(ctx, 2, 256, 256, seed=31, extra_blocks=0, device=dev)
    q = torch.randn(128, 16, 256, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16).to(dev)
    bt, cl = bt.to(dev), torch.tensor(ctx, dtype=torch.int32, device=dev)
    full = _lib.load().mvb_paged_attention_decode_workspace_size(128, 2, 256, 32768)
    partials = 128 * 2 * 5 * 16 * 257 * 4
    assert full > partials
    outs = []
    for nbytes in (full, partials):
        ws = torch.zeros(full, dtype=torch.uint8, device=dev)
        o = torch.empty(128, 16, 256, dtype=torch.bfloat16, device=dev)
        _lib.call("decode", "mvb_paged_attention_decode", _lib.desc(q), _lib.desc(kc), _lib.desc(vc), _lib.desc(bt),
                  _lib.desc(cl), 1 / 16, 256, 32768, _lib.desc(o), ws.data_ptr(), nbytes, _lib.stream_of(q))
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    for s in range(6):
        n = ctx[s]
        blocks = bt[s, torch.arange(n, device=dev) // 256].long()
        kk = kc[blocks, torch.arange(n, device=dev) % 256].float()
        vv = vc[blocks, torch.arange(n, device=dev) % 256].float()
        p = torch.softmax(torch.einsum("hgd,nhd->hgn", q[s].float().view(2, 8, 256), kk) / 16, -1)
        assert_close(outs[0][s], torch.einsum("hgn,nhd->hgd", p, vv).reshape(16, 256), what=f"seq {s}")
