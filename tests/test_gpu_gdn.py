"""GPU parity: gated delta rule (chunked prefill and recurrent decode) vs the oracle."""

import os

import numpy as np
import pytest
import torch

import oracle
from myvllm_b200 import workloads as W
from myvllm_b200.ops.gated_delta_rule.fused_recurrent_gdn import fused_recurrent_gdn
from myvllm_b200.ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule, recurrent_gated_delta_rule
from tests.util import assert_close, assert_state_close, state_rel_err, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
dev = "cuda"


def _golden_c0():
    d = np.load(os.path.join(GOLDEN, "c0_gdn.npz"))
    t = {k: torch.tensor(d[k]).to(dev) for k in ["q", "k", "v", "g", "beta"]}
    return d, t


def test_c0_golden_prefill_entry_fp32():
    """Config 0 through chunk_gated_delta_rule (fp32 inputs run the exact fp32 kernel)."""
    d, t = _golden_c0()
    state = torch.zeros(1, 4, 64, 64, device=dev)
    o = chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], state,
                               torch.zeros(1, dtype=torch.int32, device=dev),
                               torch.tensor([0, 256], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert np.abs(to_np(o) - d["ref_o"]).max() < 2e-5
    assert np.abs(to_np(state[0]) - d["ref_state"]).max() < 2e-5


def test_c0_golden_decode_stepwise():
    """Config 0 as 256 decode steps of fused_recurrent_gdn (the reference's K12 op)."""
    d, t = _golden_c0()
    state = torch.zeros(1, 4, 64, 64, device=dev)
    idx = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = []
    for i in range(256):
        outs.append(recurrent_gated_delta_rule(t["q"][i:i + 1], t["k"][i:i + 1], t["v"][i:i + 1], t["g"][i:i + 1],
                                               t["beta"][i:i + 1], state, idx))
    o = torch.cat(outs)
    assert np.abs(to_np(o) - d["ref_o"]).max() < 2e-5
    assert np.abs(to_np(state[0]) - d["ref_state"]).max() < 2e-5


def _rand_gdn(lens, hk, hv, dk, dv, seed, dtype=torch.bfloat16, n_slots=None, state_scale=0.1):
    g_ = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.nn.functional.normalize(torch.randn(T, hk, dk, generator=g_), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(T, hk, dk, generator=g_), dim=-1)
    v = torch.randn(T, hv, dv, generator=g_)
    A_log = torch.empty(hv).uniform_(0, np.log(16), generator=g_)
    dt = 0.1 * torch.randn(hv, generator=g_)
    g, beta = W.gdn_gates(torch.randn(T, hv, generator=g_), torch.randn(T, hv, generator=g_), A_log, dt)
    S = len(lens)
    n_slots = n_slots or S + 3
    state = state_scale * torch.randn(n_slots, hv, dk, dv, generator=g_)
    idx = torch.randperm(n_slots, generator=g_)[:S].to(torch.int32)
    cu = W.cu_from_lengths(lens, "cpu")
    return dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), g=g, beta=beta, state=state, idx=idx, cu=cu)


def _to(d, device):
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


@pytest.mark.parametrize("lens", [[1, 63, 64, 65, 0, 200, 129], [64], [1], [513, 7]])
def test_chunk_bf16_vs_oracle(lens):
    cpu = _rand_gdn(lens, 2, 4, 128, 128, seed=len(lens))
    gpu = _to(cpu, dev)
    o = chunk_gated_delta_rule(gpu["q"], gpu["k"], gpu["v"], gpu["g"], gpu["beta"], gpu["state"], gpu["idx"],
                               gpu["cu"])
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.chunked(to_np(cpu["q"]), to_np(cpu["k"]), to_np(cpu["v"]), to_np(cpu["g"]), to_np(cpu["beta"]),
                             st, cpu["idx"].numpy(), cpu["cu"].numpy(), 64)
    assert_close(o, ref, what="o")
    assert_state_close(gpu["state"], st)


def test_chunk_continuation_equals_single_call():
    """A prefill split in two calls (state carried through the cache slot) equals one call."""
    lens = [300, 77]
    cpu = _rand_gdn(lens, 2, 4, 128, 128, seed=11)
    a, b = _to(cpu, dev), _to(cpu, dev)
    o1 = chunk_gated_delta_rule(a["q"], a["k"], a["v"], a["g"], a["beta"], a["state"], a["idx"], a["cu"])
    # second run: first 100 tokens of every sequence, then the rest
    cu = cpu["cu"].tolist()
    first = [list(range(cu[s], min(cu[s] + 100, cu[s + 1]))) for s in range(2)]
    rest = [list(range(cu[s] + len(first[s]), cu[s + 1])) for s in range(2)]
    outs = torch.empty_like(o1)
    for part in (first, rest):
        ids = torch.tensor(sum(part, []), device=dev)
        cu_p = W.cu_from_lengths([len(p) for p in part], dev)
        op = chunk_gated_delta_rule(b["q"][ids], b["k"][ids], b["v"][ids], b["g"][ids], b["beta"][ids], b["state"],
                                    b["idx"], cu_p)
        outs[ids] = op
    assert_close(outs, o1, what="o (split vs single)")
    assert_state_close(b["state"], a["state"], what="state (split vs single)")


def test_chunk_c1_shapes_vs_fp32_recurrent_kernel():
    """Config-1 head layout (16 k-heads / 32 v-heads x 128) at full config-1 lengths: the
    bf16 tensor-core chunk kernel against the exact fp32 token-serial kernel on the same
    inputs (a size-independent check: both compute the same recurrence)."""
    lens = W.seq_lengths(8, 512, 8192, 0)
    cpu = _rand_gdn(lens, 16, 32, 128, 128, seed=5, n_slots=8, state_scale=0.0)
    a = _to(cpu, dev)
    b = {k: (v.float() if isinstance(v, torch.Tensor) and v.dtype == torch.bfloat16 else v) for k, v in a.items()}
    b["state"] = a["state"].clone()
    o_fast = chunk_gated_delta_rule(a["q"], a["k"], a["v"], a["g"], a["beta"], a["state"], a["idx"], a["cu"])
    o_ref = chunk_gated_delta_rule(b["q"], b["k"], b["v"], b["g"], b["beta"], b["state"], b["idx"], b["cu"])
    assert_close(o_fast, o_ref, what="o (chunk bf16 vs recurrent fp32)")
    assert_state_close(a["state"], b["state"])


def _chunk_call(d, o, ws):
    from myvllm_b200 import _lib

    _lib.call("chunk_gated_delta_rule", "mvb_chunk_gated_delta_rule", _lib.desc(d["q"]), _lib.desc(d["k"]),
              _lib.desc(d["v"]), _lib.desc(d["g"]), _lib.desc(d["beta"]), _lib.desc(d["state"]), _lib.desc(d["idx"]),
              _lib.desc(d["cu"]), _lib.desc(o), 0.0, 0, ws.data_ptr() if ws is not None else None,
              ws.numel() if ws is not None else 0, _lib.stream_of(d["q"]))


def test_chunk_balanced_schedule_is_bit_identical_to_whole_chains():
    """The balanced schedule cuts (sequence, v-head) chains at SM span boundaries and hands
    the state over through recurrent_state (28 cuts for these lengths at 32 v-heads).  The
    fp32 state passes through memory exactly, so outputs and final states must equal those
    of whole-chain scheduling (the 8-byte dynamic counter, and round-robin without a
    workspace) bit for bit, on two balanced launches in a row (the launch generation
    advances between them)."""
    from myvllm_b200 import _lib

    cpu = _rand_gdn([1000, 700, 300], 16, 32, 128, 128, seed=21, n_slots=6)
    base = _to(cpu, dev)
    ws_bal = torch.zeros(int(_lib.load().mvb_chunk_gated_delta_rule_workspace_size()), dtype=torch.uint8, device=dev)
    ws_dyn = torch.zeros(8, dtype=torch.uint8, device=dev)
    outs = {}
    for name, ws in (("balanced", ws_bal), ("balanced again", ws_bal), ("dynamic", ws_dyn), ("round-robin", None)):
        d = dict(base, state=base["state"].clone())
        o = torch.empty_like(d["v"])
        _chunk_call(d, o, ws)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0, name
        outs[name] = (o, d["state"])
    ref_o, ref_s = outs["dynamic"]
    for name, (o, s) in outs.items():
        assert torch.equal(o, ref_o), f"o differs: {name} vs dynamic"
        assert torch.equal(s, ref_s), f"state differs: {name} vs dynamic"
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.chunked(to_np(cpu["q"]), to_np(cpu["k"]), to_np(cpu["v"]), to_np(cpu["g"]), to_np(cpu["beta"]),
                             st, cpu["idx"].numpy(), cpu["cu"].numpy(), 64)
    assert_close(outs["balanced"][0], ref, what="o (balanced schedule vs oracle)")
    assert_state_close(outs["balanced"][1], st, what="state (balanced schedule vs oracle)")
    words = ws_bal.view(torch.int32)
    assert words[1].item() == 0 and words[2].item() == 2, "done counter / launch generation"


def test_chunk_tc_full_c1_sequence_vs_oracle():
    """One full-length config-1 sequence (8192 tokens) through the tensor-core chunk kernel
    against the oracle (m/ops/gated_delta_rule/gated_delta_rule.py:44-64, restated in
    float64): q/k/v are the causal conv's bf16 output over the 8192 qkv channels, the q/k
    L2 norm is fused in the kernel, the gates have the config-1 distributions and the initial
    state is non-zero.  Five v-heads (both v-heads of k-head 0, and heads of the other k-head
    groups) are compared: outputs to the bf16 bar, the final state to 1e-3 relative."""
    from myvllm_b200 import _lib
    from myvllm_b200.ops.causal_conv1d import causal_conv1d_fn

    inp = W.c1_inputs(dev, seed=0, lengths=[8192])
    qkv = causal_conv1d_fn(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"], inp["cu"])
    q, k, v = W.split_qkv(qkv)
    g_ = torch.Generator(device=dev).manual_seed(9)
    state0 = 0.1 * torch.randn(inp["state"].shape, generator=g_, device=dev)
    state = state0.clone()
    o = chunk_gated_delta_rule(q, k, v, inp["g"], inp["beta"], state, inp["idx"], inp["cu"],
                               use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert _lib.last_path(_lib.OP_CHUNK_GDN)[0] == "tensor_core"
    heads = [0, 1, 9, 22, 31]
    qn, kn = to_np(q), to_np(k)
    qn = qn / np.sqrt((qn * qn).sum(-1, keepdims=True) + 1e-6)
    kn = kn / np.sqrt((kn * kn).sum(-1, keepdims=True) + 1e-6)
    kh = [h // 2 for h in heads]
    st = to_np(state0)[:, heads]
    ref = oracle.gdn.chunked(qn[:, kh], kn[:, kh], to_np(v)[:, heads], to_np(inp["g"])[:, heads],
                             to_np(inp["beta"])[:, heads], st, np.array([0]), inp["cu"].cpu().numpy(), 64)
    assert_close(o[:, heads], ref, what="o (full C1 sequence)")
    assert_state_close(state[:, heads], st, what="state (full C1 sequence)")


def test_decode_bf16_vs_oracle():
    S, hk, hv = 24, 16, 32
    cpu = _rand_gdn([1] * S, hk, hv, 128, 128, seed=3, n_slots=40)
    gpu = _to(cpu, dev)
    o = fused_recurrent_gdn(gpu["q"], gpu["k"], gpu["v"], gpu["g"], gpu["beta"], gpu["state"], gpu["idx"])
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.recurrent_step(to_np(cpu["q"]), to_np(cpu["k"]), to_np(cpu["v"]), to_np(cpu["g"]),
                                    to_np(cpu["beta"]), st, cpu["idx"].numpy())
    assert_close(o, ref, what="o")
    assert state_rel_err(gpu["state"], st) < 1e-5  # fp32 math throughout


def test_decode_c2_full_size_sampled():
    """Config 2 at full size (256 seqs, state [256,32,128,128]); 12 sequences are checked
    against the oracle, and untouched slots must stay bit-identical."""
    inp = W.c2_inputs(dev)
    q, k, v = W.split_qkv(inp["x"])
    q, k = W.l2norm(q), W.l2norm(k)
    extra = torch.randn(4, 32, 128, 128, device=dev)  # slots not addressed by idx
    state = torch.cat([inp["state"], extra])
    before = state.clone()
    o = fused_recurrent_gdn(q, k, v, inp["g"], inp["beta"], state, inp["idx"])
    torch.cuda.synchronize()
    assert torch.equal(state[256:], before[256:])
    pick = torch.arange(0, 256, 23)
    idx = inp["idx"][pick].cpu().numpy()
    st = before.cpu().double().numpy()
    ref = oracle.gdn.recurrent_step(to_np(q[pick]), to_np(k[pick]), to_np(v[pick]), to_np(inp["g"][pick]),
                                    to_np(inp["beta"][pick]), st, idx)
    assert_close(o[pick], ref, what="o")
    assert state_rel_err(state[idx], st[idx]) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_chunk_fused_l2norm(dtype):
    """use_qk_l2norm_in_kernel: unnormalised q/k in, same result as normalising first."""
    lens = [70, 129]
    cpu = _rand_gdn(lens, 2, 4, 128, 128, seed=21, dtype=dtype)
    g_ = torch.Generator().manual_seed(3)
    sc = 0.5 + 3 * torch.rand(sum(lens), 2, 1, generator=g_)
    qr, kr = (cpu["q"].float() * sc).to(dtype), (cpu["k"].float() * sc.flip(0)).to(dtype)
    gpu = _to(cpu, dev)
    o = chunk_gated_delta_rule(qr.to(dev), kr.to(dev), gpu["v"], gpu["g"], gpu["beta"], gpu["state"], gpu["idx"],
                               gpu["cu"], use_qk_l2norm_in_kernel=True)
    qn = to_np(qr) / np.sqrt((to_np(qr) ** 2).sum(-1, keepdims=True) + 1e-6)
    kn = to_np(kr) / np.sqrt((to_np(kr) ** 2).sum(-1, keepdims=True) + 1e-6)
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.chunked(qn, kn, to_np(cpu["v"]), to_np(cpu["g"]), to_np(cpu["beta"]), st, cpu["idx"].numpy(),
                             cpu["cu"].numpy(), 64)
    assert_close(o, ref, what="o")
    assert_state_close(gpu["state"], st)


def test_decode_fused_l2norm():
    S = 10
    cpu = _rand_gdn([1] * S, 16, 32, 128, 128, seed=8, n_slots=12)
    qr = (cpu["q"].float() * 3.0).to(torch.bfloat16)
    kr = (cpu["k"].float() * 0.25).to(torch.bfloat16)
    gpu = _to(cpu, dev)
    o = fused_recurrent_gdn(qr.to(dev), kr.to(dev), gpu["v"], gpu["g"], gpu["beta"], gpu["state"], gpu["idx"],
                            use_qk_l2norm_in_kernel=True)
    qn = to_np(qr) / np.sqrt((to_np(qr) ** 2).sum(-1, keepdims=True) + 1e-6)
    kn = to_np(kr) / np.sqrt((to_np(kr) ** 2).sum(-1, keepdims=True) + 1e-6)
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.recurrent_step(qn, kn, to_np(cpu["v"]), to_np(cpu["g"]), to_np(cpu["beta"]), st,
                                    cpu["idx"].numpy())
    assert_close(o, ref, what="o")
    assert state_rel_err(gpu["state"], st) < 1e-5


def test_chunk_mixed_gate_dtypes():
    """The reference layer hands over g in fp32 and beta in the activation dtype."""
    lens = [100, 64]
    cpu = _rand_gdn(lens, 2, 4, 128, 128, seed=31)
    cpu["beta"] = cpu["beta"].to(torch.bfloat16)
    gpu = _to(cpu, dev)
    o = chunk_gated_delta_rule(gpu["q"], gpu["k"], gpu["v"], gpu["g"], gpu["beta"], gpu["state"], gpu["idx"],
                               gpu["cu"])
    st = cpu["state"].double().numpy()
    ref = oracle.gdn.chunked(to_np(cpu["q"]), to_np(cpu["k"]), to_np(cpu["v"]), to_np(cpu["g"]), to_np(cpu["beta"]),
                             st, cpu["idx"].numpy(), cpu["cu"].numpy(), 64)
    assert_close(o, ref, what="o")
    assert_state_close(gpu["state"], st)


def test_chunk_no_device_timeouts():
    from myvllm_b200 import _lib

    assert _lib.device_status() == 0


@pytest.mark.parametrize("prefill", [True, False])
def test_gated_entry_points_match_torch_gates(prefill):
    """gate_inputs=(a, b, A_log, dt_bias) forms g and beta in the kernel; the result must equal
    the same op given the layer's torch-computed gates."""
    import torch.nn.functional as F
    from myvllm_b200.ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule, recurrent_gated_delta_rule

    lens = [130, 64, 1, 300] if prefill else [1] * 37
    T, hk, hv = sum(lens), 4, 8
    g0 = torch.Generator().manual_seed(11)
    q = torch.randn(T, hk, 128, generator=g0).to(torch.bfloat16).cuda()
    k = torch.randn(T, hk, 128, generator=g0).to(torch.bfloat16).cuda()
    v = torch.randn(T, hv, 128, generator=g0).to(torch.bfloat16).cuda()
    a = torch.randn(T, hv, generator=g0).to(torch.bfloat16).cuda()
    b = torch.randn(T, hv, generator=g0).to(torch.bfloat16).cuda()
    a_log = torch.empty(hv).uniform_(0, 2.77, generator=g0).cuda()
    dt_bias = (0.1 * torch.randn(hv, generator=g0)).cuda()
    g = -a_log.exp() * F.softplus(a.float() + dt_bias)
    beta = b.sigmoid()
    n = len(lens)
    st0 = 0.1 * torch.randn(n, hv, 128, 128, generator=g0).cuda()
    idx = torch.arange(n, dtype=torch.int32, device="cuda")
    s1, s2 = st0.clone(), st0.clone()
    if prefill:
        cu = W.cu_from_lengths(lens, "cuda")
        o1 = chunk_gated_delta_rule(q, k, v, g, beta, s1, idx, cu, use_qk_l2norm_in_kernel=True)
        o2 = chunk_gated_delta_rule(q, k, v, None, None, s2, idx, cu, use_qk_l2norm_in_kernel=True,
                                    gate_inputs=(a, b, a_log, dt_bias))
    else:
        o1 = recurrent_gated_delta_rule(q, k, v, g, beta, s1, idx, use_qk_l2norm_in_kernel=True)
        o2 = recurrent_gated_delta_rule(q, k, v, None, None, s2, idx, use_qk_l2norm_in_kernel=True,
                                        gate_inputs=(a, b, a_log, dt_bias))
    assert_close(o2, o1, what="output")
    assert ((s2 - s1).norm() / s1.norm()).item() < 1e-5


@pytest.mark.parametrize("hk,hv", [(16, 32), (4, 4), (2, 8)])
def test_fused_layer_decode_matches_the_unfused_ops(hk, hv):
    """mvb_gated_deltanet_decode (conv update + q/k norm + gates + recurrence + RMSNormGated in
    one kernel) against the same layer step run as the separate library ops the layer used
    before: the conv state bit for bit, the fp32 recurrent state to 1e-5 relative (the same
    arithmetic, reduced in another order), the normed output within the bf16 bar.  Hv / Hk = 2 (the config-2/4 layout), 1 and 4;
    permuted state slots; projection rows taken as strided views of one fused GEMM output."""
    from myvllm_b200.layers.norm import RMSNormGated
    from myvllm_b200.ops.causal_conv1d import causal_conv1d_update
    from myvllm_b200.ops.gated_delta_rule.fused_layer import gated_deltanet_decode

    S, n_slots, K = 64, 80, 128
    conv_dim = 2 * hk * K + hv * K
    g_ = torch.Generator(device=dev).manual_seed(hk * 100 + hv)
    fused_out = torch.randn(S, conv_dim + hv * K + 2 * hv, generator=g_, device=dev).to(torch.bfloat16)
    qkv = fused_out[:, :conv_dim]
    z = fused_out[:, conv_dim:conv_dim + hv * K].view(S, hv, K)
    a = fused_out[:, conv_dim + hv * K:conv_dim + hv * K + hv]
    b = fused_out[:, conv_dim + hv * K + hv:]
    w = (0.3 * torch.randn(conv_dim, 4, generator=g_, device=dev)).to(torch.bfloat16)
    conv0 = torch.randn(n_slots, 3, conv_dim, generator=g_, device=dev).to(torch.bfloat16)
    st0 = 0.1 * torch.randn(n_slots, hv, K, K, generator=g_, device=dev)
    A_log = torch.empty(hv, device=dev).uniform_(0, np.log(16), generator=g_)
    dt_bias = 0.1 * torch.randn(hv, generator=g_, device=dev)
    idx = torch.randperm(n_slots, generator=torch.Generator().manual_seed(3))[:S].to(torch.int32).to(dev)
    norm = RMSNormGated((K,), 1e-6).to(dev, torch.bfloat16)
    norm.weight.data.copy_(1 + 0.1 * torch.randn(K, generator=g_, device=dev))

    c1, s1 = conv0.clone(), st0.clone()
    out = gated_deltanet_decode(qkv, w, c1, idx, a, b, A_log, dt_bias, s1, idx, z, norm.weight, 1e-6)
    c2, s2 = conv0.clone(), st0.clone()
    xc = causal_conv1d_update(qkv, w, c2, idx)
    q, k, v = W.split_qkv(xc, hk, hv, K, K)
    o = fused_recurrent_gdn(q, k, v, None, None, s2, idx, use_qk_l2norm_in_kernel=True,
                            gate_inputs=(a, b, A_log, dt_bias))
    ref = norm(o, z)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2), "conv state differs from the unfused conv update"
    # same arithmetic; the fused kernel reduces k^T S over the full 128-column row in another
    # association order, so the fp32 states agree to rounding
    assert state_rel_err(s1, s2) < 1e-5, "recurrent state differs from the unfused recurrence"
    assert_close(out, ref, what="fused decode output")


def test_fused_layer_prefill_matches_the_unfused_ops():
    """mvb_gated_deltanet_prefill (chunk GDN with in-kernel gates and q/k norm, RMSNormGated
    applied to each output tile) against the chunk op followed by the RMSNormGated op: the
    final states bit for bit (the norm does not touch them), the normed output within the
    bf16 bar.  Ragged sequences (partial last chunks) and permuted state slots."""
    from myvllm_b200.layers.norm import RMSNormGated
    from myvllm_b200.ops.gated_delta_rule.fused_layer import gated_deltanet_prefill

    lens = [1, 63, 64, 65, 300, 129]
    hk, hv, K = 4, 8, 128
    T = sum(lens)
    g_ = torch.Generator(device=dev).manual_seed(21)
    proj = torch.randn(T, 2 * hk * K + 2 * hv * K + 2 * hv, generator=g_, device=dev).to(torch.bfloat16)
    q = proj[:, :hk * K].view(T, hk, K)
    k = proj[:, hk * K:2 * hk * K].view(T, hk, K)
    v = proj[:, 2 * hk * K:2 * hk * K + hv * K].view(T, hv, K)
    z = proj[:, 2 * hk * K + hv * K:2 * hk * K + 2 * hv * K].view(T, hv, K)
    a = proj[:, -2 * hv:-hv]
    b = proj[:, -hv:]
    A_log = torch.empty(hv, device=dev).uniform_(0, np.log(16), generator=g_)
    dt_bias = 0.1 * torch.randn(hv, generator=g_, device=dev)
    n_slots = len(lens) + 3
    st0 = 0.1 * torch.randn(n_slots, hv, K, K, generator=g_, device=dev)
    idx = torch.randperm(n_slots, generator=torch.Generator().manual_seed(4))[:len(lens)].to(torch.int32).to(dev)
    cu = W.cu_from_lengths(lens, dev)
    norm = RMSNormGated((K,), 1e-6).to(dev, torch.bfloat16)
    norm.weight.data.copy_(1 + 0.1 * torch.randn(K, generator=g_, device=dev))
    s1, s2 = st0.clone(), st0.clone()
    out = gated_deltanet_prefill(q, k, v, a, b, A_log, dt_bias, s1, idx, cu, z, norm.weight, 1e-6)
    o = chunk_gated_delta_rule(q, k, v, None, None, s2, idx, cu, use_qk_l2norm_in_kernel=True,
                               gate_inputs=(a, b, A_log, dt_bias))
    ref = norm(o, z)
    torch.cuda.synchronize()
    assert torch.equal(s1, s2), "final states differ between the fused and the unfused prefill"
    assert_close(out, ref, what="fused prefill output")
