"""CPU checks of the hybrid decode stack's tensor-parallel construction: a stack built as
rank r of an n-way split must hold exactly the head slices of the unsharded stack with the
same seed -- weights through the layers' weight_loader rules (q | k | v blocks, gated q per
head, row-parallel output projections, KV heads split or replicated), GDN recurrent and conv
states by head / channel, and the paged KV cache by kv head.  This is what the bench's
tensor-parallel parity check relies on.  No kernels run here."""

import pytest
import torch

from myvllm_b200.decode_stack import HybridDecodeStack

CTX = [300, 41]


def _stack(tp):
    return HybridDecodeStack(4, 2, CTX, 2, "cpu", seed=5, tp=tp)


@pytest.fixture(scope="module")
def full():
    return _stack((0, 1))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_stack_is_a_slice_of_the_full_stack(full, world):
    for r in (0, world - 1):
        part = _stack((r, world))
        # GDN layer 0: fused input projection rows [q_r | k_r | v_r | z_r | a_r | b_r]
        g_full, g_part = full.gdn[0], part.gdn[0]
        hk, hv = 16 // world, 32 // world
        qs, vs = hk * 128, hv * 128
        w = g_full.in_proj_qkv.weight
        want = torch.cat([w[r * qs:(r + 1) * qs], w[2048 + r * qs:2048 + (r + 1) * qs],
                          w[4096 + r * vs:4096 + (r + 1) * vs]])
        assert torch.equal(g_part.in_proj_qkv.weight, want)
        assert torch.equal(g_part.out_proj.weight, g_full.out_proj.weight[:, r * vs:(r + 1) * vs])
        assert torch.equal(g_part.A_log, g_full.A_log[r * hv:(r + 1) * hv])
        assert torch.equal(g_part.in_proj_a.weight, g_full.in_proj_a.weight[r * hv:(r + 1) * hv])
        # states: recurrent by v-head, conv by channel blocks
        assert torch.equal(part.lac.recurrent_cache, full.lac.recurrent_cache[:, :, r * hv:(r + 1) * hv])
        c = full.lac.conv_cache
        want_c = torch.cat([c[..., r * qs:(r + 1) * qs], c[..., 2048 + r * qs:2048 + (r + 1) * qs],
                            c[..., 4096 + r * vs:4096 + (r + 1) * vs]], -1)
        assert torch.equal(part.lac.conv_cache, want_c)
        # attention layer: KV heads split at tp <= 2 with the q heads; beyond, each kv head is
        # copied to the tp / 2 ranks of its share, which split its context and hold all its
        # q heads (q/gate rows, o_proj columns)
        a_full, a_part = full.fa[0], part.fa[0]
        h = r if world == 2 else r * 2 // world
        share = max(1, world // 2)
        assert (a_part.kv_share, a_part.kv_part) == (share, r % share)
        hq = 8 if share > 1 else 16 // world
        first_q = h * 8 if share > 1 else r * hq
        assert torch.equal(a_part.q_proj.weight, a_full.q_proj.weight[first_q * 512:(first_q + hq) * 512])
        assert a_part.num_kv_heads == 1
        assert torch.equal(a_part.k_proj.weight, a_full.k_proj.weight[h * 256:(h + 1) * 256])
        assert torch.equal(part.kv.k[..., 0, :], full.kv.k[..., h, :])
        assert torch.equal(part.kv.v[..., 0, :], full.kv.v[..., h, :])
        assert torch.equal(a_part.o_proj.weight, a_full.o_proj.weight[:, first_q * 256:(first_q + hq) * 256])
        assert (a_part.o_proj.tp_rank, a_part.o_proj.tp_size) == (r, world)  # the all-reduce spans every rank
        if share > 1:
            assert part.bytes_per_step()["kv"] * share == sum(CTX) * 1 * 1 * 256 * 2 * 2


def test_replicated_kv_heads_without_context_split():
    from myvllm_b200.layers.full_attention import GatedAttention

    GatedAttention.context_split = False
    try:
        full, part = _stack((0, 1)), _stack((3, 4))
    finally:
        GatedAttention.context_split = True
    a_full, a_part = full.fa[0], part.fa[0]
    assert (a_part.kv_share, a_part.num_q_heads) == (1, 4)
    assert torch.equal(a_part.q_proj.weight, a_full.q_proj.weight[12 * 512:16 * 512])
    assert torch.equal(a_part.o_proj.weight, a_full.o_proj.weight[:, 12 * 256:16 * 256])
    assert torch.equal(part.kv.k[..., 0, :], full.kv.k[..., 1, :])


def test_bytes_per_step_counts_kv_states_and_weights(full):
    by = full.bytes_per_step()
    assert by["kv"] == sum(CTX) * 1 * 2 * 256 * 2 * 2  # 1 attention layer, 2 kv heads, k and v
    assert by["total"] == by["kv"] + by["states"] + by["weights"]
