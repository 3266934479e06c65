"""Seeded synthetic workloads with the shapes and value distributions of the benchmark
configurations (there are no public datasets for this path; every input is synthetic).

  c0  GDN operator, fp32: T=256, H=4, d=64 (CPU parity case)
  c1  GDN prefill layer: conv1d (W=4, 8192 channels) + chunked GDN, 8 seqs ~U[512, 8192]
  c2  GDN decode: 256 seqs, fp32 state [256, 32, 128, 128] ~N(0, 0.1), conv state ~N(0, 1)
  c3  full-attention varlen causal prefill: Hq=16, Hkv=2, D=256, 8 seqs ~U[1024, 16384],
      K/V also written to a paged cache (block 256) through a permuted block table
  c4  hybrid decode stack: 128 seqs, context ~U[1024, 32768] (built in ``bench.py``)

Sequence lengths are drawn once from a seeded generator and returned with the inputs.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

# Qwen3.5-style linear-attention layer shapes (m/configs/qwen3_5.py:69-74)
GDN_HK, GDN_HV, GDN_DK, GDN_DV, GDN_W = 16, 32, 128, 128, 4
GDN_CH = 2 * GDN_HK * GDN_DK + GDN_HV * GDN_DV  # 8192 conv channels (q | k | v)
# full-attention layer shapes (m/configs/qwen3_5.py:22, 80, 85)
FA_HQ, FA_HKV, FA_D = 16, 2, 256


def seq_lengths(n: int, lo: int, hi: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def cu_from_lengths(lengths, device) -> torch.Tensor:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int32, device=device)


def c0_inputs(seed: int = 0):
    """Config 0 (identical construction to ``tests/golden/make_golden.py``)."""
    torch.manual_seed(seed)
    T, H, D = 256, 4, 64
    q = F.normalize(torch.randn(T, H, D), dim=-1)
    k = F.normalize(torch.randn(T, H, D), dim=-1)
    v = torch.randn(T, H, D)
    beta = torch.sigmoid(torch.randn(T, H))
    g = F.logsigmoid(torch.randn(T, H) + 2.0)
    return q, k, v, beta, g


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias) in fp32
    (m/layers/linear_attention.py:89-90)."""
    beta = torch.sigmoid(b.float())
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, beta


def c1_inputs(device, seed: int = 0, lengths=None, dtype=torch.bfloat16, n_seqs: int = 8):
    """Config 1: one GDN prefill layer (conv1d + chunked GDN)."""
    if lengths is None:
        lengths = seq_lengths(n_seqs, 512, 8192, seed)
    g_ = torch.Generator(device="cpu").manual_seed(seed + 1)
    T = int(sum(lengths))
    S = len(lengths)
    x = torch.randn(T, GDN_CH, generator=g_).to(device=device, dtype=dtype)
    conv_w = (0.02 * torch.randn(GDN_CH, GDN_W, generator=g_)).to(device=device, dtype=dtype)
    conv_state = torch.zeros(S, GDN_W - 1, GDN_CH, device=device, dtype=dtype)
    A_log = torch.empty(GDN_HV).uniform_(0, math.log(16), generator=g_).to(device)
    dt_bias = (0.1 * torch.randn(GDN_HV, generator=g_)).to(device)
    a = torch.randn(T, GDN_HV, generator=g_).to(device)
    b = torch.randn(T, GDN_HV, generator=g_).to(device)
    g, beta = gdn_gates(a, b, A_log, dt_bias)
    state = torch.zeros(S, GDN_HV, GDN_DK, GDN_DV, device=device, dtype=torch.float32)
    idx = torch.arange(S, dtype=torch.int32, device=device)
    return dict(x=x, conv_w=conv_w, conv_state=conv_state, g=g, beta=beta, state=state, idx=idx,
                cu=cu_from_lengths(lengths, device), lengths=lengths, T=T)


def split_qkv(qkv: torch.Tensor, hk=GDN_HK, hv=GDN_HV, dk=GDN_DK, dv=GDN_DV):
    """[T, 2 Hk dk + Hv dv] -> q, k [T, Hk, dk], v [T, Hv, dv] (views, QKVParallelLinear order)."""
    T = qkv.shape[0]
    q, k, v = torch.split(qkv, [hk * dk, hk * dk, hv * dv], dim=-1)
    return q.view(T, hk, dk), k.view(T, hk, dk), v.view(T, hv, dv)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum x^2 + eps) in fp32 (m/layers/linear_attention.py:113-114)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) + eps)).to(x.dtype)


def c2_inputs(device, seed: int = 0, n_seqs: int = 256, dtype=torch.bfloat16):
    """Config 2: one GDN decode step."""
    g_ = torch.Generator(device="cpu").manual_seed(seed + 2)
    S = n_seqs
    state = (0.1 * torch.randn(S, GDN_HV, GDN_DK, GDN_DV, generator=g_)).to(device)
    conv_state = torch.randn(S, GDN_W - 1, GDN_CH, generator=g_).to(device=device, dtype=dtype)
    x = torch.randn(S, GDN_CH, generator=g_).to(device=device, dtype=dtype)
    conv_w = (0.02 * torch.randn(GDN_CH, GDN_W, generator=g_)).to(device=device, dtype=dtype)
    A_log = torch.empty(GDN_HV).uniform_(0, math.log(16), generator=g_).to(device)
    dt_bias = (0.1 * torch.randn(GDN_HV, generator=g_)).to(device)
    a = torch.randn(S, GDN_HV, generator=g_).to(device)
    b = torch.randn(S, GDN_HV, generator=g_).to(device)
    g, beta = gdn_gates(a, b, A_log, dt_bias)
    idx = torch.randperm(S, generator=g_).to(device=device, dtype=torch.int32)
    return dict(x=x, conv_w=conv_w, conv_state=conv_state, g=g, beta=beta, state=state, idx=idx, a=a, b=b,
                A_log=A_log, dt_bias=dt_bias)


def c3_inputs(device, seed: int = 0, lengths=None, dtype=torch.bfloat16, block_size: int = 256, n_seqs: int = 8):
    """Config 3: varlen causal attention prefill + paged KV write."""
    if lengths is None:
        lengths = seq_lengths(n_seqs, 1024, 16384, seed + 3)
    g_ = torch.Generator(device="cpu").manual_seed(seed + 3)
    T = int(sum(lengths))
    q = torch.randn(T, FA_HQ, FA_D, generator=g_).to(device=device, dtype=dtype)
    k = torch.randn(T, FA_HKV, FA_D, generator=g_).to(device=device, dtype=dtype)
    v = torch.randn(T, FA_HKV, FA_D, generator=g_).to(device=device, dtype=dtype)
    blocks_per_seq = [(n + block_size - 1) // block_size for n in lengths]
    n_blocks = sum(blocks_per_seq)
    perm = torch.randperm(n_blocks, generator=g_)
    max_blocks = max(blocks_per_seq) if blocks_per_seq else 1
    bt = torch.zeros(len(lengths), max_blocks, dtype=torch.int32)
    slots = torch.empty(T, dtype=torch.int64)
    o = 0
    t0 = 0
    for s, (n, nb) in enumerate(zip(lengths, blocks_per_seq)):
        bt[s, :nb] = perm[o:o + nb].to(torch.int32)
        pos = torch.arange(n)
        slots[t0:t0 + n] = bt[s, pos // block_size].long() * block_size + pos % block_size
        o += nb
        t0 += n
    return dict(q=q, k=k, v=v, cu=cu_from_lengths(lengths, device), lengths=lengths, T=T,
                block_tables=bt.to(device), slot_mapping=slots.to(device=device, dtype=torch.int32),
                n_blocks=n_blocks, block_size=block_size, scale=1.0 / 16)
