"""Benchmark of the myvllm attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
                    [--config all|c1|c2|c3|c4]

The headline line is config 1 -- one Gated-DeltaNet prefill layer: causal_conv1d_fn over
8192 qkv channels -> chunk_gated_delta_rule (q/k L2 norm fused, chunk 64), 8 sequences of
~U[512, 8192] tokens, bf16 activations, fp32 state.  Metric: prefill tokens/s.

  N = 1 (default ``--config all``): the config-1 line, timed over exactly K steps, with
    nested blocks for the other halves of the metric, each timed over about a second:
      "c2"  GDN decode step (conv update + recurrent GDN, 256 sequences), us/step
      "c3"  full-attention prefill (KV write + varlen causal FA, 8 x ~U[1024, 16384]), tokens/s
      "c4"  48-layer hybrid decode step (36 GDN + 12 gated attention, 128 sequences), us/step
  N > 1 (torchrun): the layer's heads are tensor-parallel over the N ranks.  Config 1 is one
    batch split by heads (16/N k-heads, 32/N v-heads and their conv channels per rank), so
    the total work is fixed ("strong" scaling; value = tokens / max-over-ranks step time).
    A "c4" block runs the 48-layer step at TP = N with an all-reduce after every output
    projection, and "tp_parity" checks both against a single-rank recompute on rank 0.

``--impl reference`` times the CPU restatement of the reference path (the numpy oracle; the
reference's own kernels are Triton and do not run on a CPU) on the host's cores.
``--config c1|c2|c3|c4`` prints one block alone as a line (profiler cases; ``--lengths``,
``--layers`` and ``--seqs`` shrink them).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SUSTAINED_S = 1.2  # nested blocks time this long (or longer) so that clocks settle


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profiled_traffic(kernel_key: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(kernel_key)
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling, windowed by mark_start/mark_stop."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._window = [None, None]
        self._proc = None

    def mark_start(self):
        self._window[0] = len(self.samples)

    def mark_stop(self):
        self._window[1] = len(self.samples)

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self._proc = None
        time.sleep(0.5)  # let the sampler start before the work it samples
        return self

    def _read(self):
        for line in self._proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 6:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        lo, hi = self._window
        window = self.samples[lo:hi + 1] if lo is not None and hi is not None else []
        # a timed region shorter than the 100 ms sampling period may hold no sample of its
        # own: fall back to the samples around it (warm-up included, same load)
        if len(window) < 3:
            window = self.samples[max(0, (lo or 0) - 10):]
        if not window:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [float(s[0]) for s in window if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in window if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in window for i in range(4) if s[2 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(window)}


def ev():
    return torch.cuda.Event(enable_timing=True)


def timed_region(step, n, world, clk=None):
    """n calls of step() between a barrier + synchronize on both sides, timed with CUDA events
    on the current stream; returns ms per step, max over ranks."""
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s0, s1 = ev(), ev()
    if clk is not None:
        clk.mark_start()
    s0.record()
    for i in range(n):
        step(i)
    s1.record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.mark_stop()
    ms = s0.elapsed_time(s1) / n
    return max_over_ranks(ms, world)


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.item()


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return t.item()


def steps_for(seconds: float, ms_est: float, lo: int = 3) -> int:
    return max(lo, int(math.ceil(seconds * 1e3 / max(ms_est, 1e-3))))


def check_device(what: str) -> int:
    """The kernels' device error word after a timed region; a non-zero word means a bounded
    wait gave up and outputs are invalid, so the line is not printed."""
    from myvllm_b200 import _lib

    status = _lib.device_status()
    if status != 0:
        raise RuntimeError(f"bench {what}: device status {status} (a kernel's bounded wait gave up)")
    return status


def host_threads():
    """Threads the numpy oracle's BLAS runs with right now (threadpoolctl); 1 without BLAS."""
    from threadpoolctl import threadpool_info

    return max([d["num_threads"] for d in threadpool_info()] + [1])


# --------------------------------------------------------------------- CPU baselines ----
def cpu_baseline_c1(budget_s: float = 12.0, seed: int = 0):
    """The oracle (numpy restatement of the reference path) on a bounded sample of the
    config-1 workload: whole sequences of the seeded batch, conv1d + l2norm + chunked GDN,
    all 32 heads, until ``budget_s`` of CPU time is spent.  Returns tokens/s."""
    import oracle
    from myvllm_b200 import workloads as W

    lengths = W.seq_lengths(8, 512, 8192, seed)
    rng = np.random.default_rng(seed)
    tokens, spent = 0, 0.0
    for L in lengths:
        x = rng.standard_normal((L, W.GDN_CH)).astype(np.float32)
        w = (0.02 * rng.standard_normal((W.GDN_CH, W.GDN_W))).astype(np.float32)
        cst = np.zeros((1, W.GDN_W - 1, W.GDN_CH), np.float32)
        g = -rng.uniform(0.01, 1.0, (L, W.GDN_HV)).astype(np.float32)
        beta = rng.uniform(0, 1, (L, W.GDN_HV)).astype(np.float32)
        st = np.zeros((1, W.GDN_HV, W.GDN_DK, W.GDN_DV), np.float32)
        t0 = time.perf_counter()
        qkv = oracle.conv.conv1d_fn(x, w, cst, np.array([0]), np.array([0, L]), dtype=np.float32)
        q = qkv[:, :2048].reshape(L, 16, 128)
        k = qkv[:, 2048:4096].reshape(L, 16, 128)
        v = qkv[:, 4096:].reshape(L, 32, 128)
        q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
        k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
        oracle.gdn.chunked(q, k, v, g, beta, st, np.array([0]), np.array([0, L]), 64, dtype=np.float32)
        spent += time.perf_counter() - t0
        tokens += L
        if spent >= budget_s:
            break
    return tokens / spent, tokens, spent, host_threads()


def _cpu_gdn_decode(batch, rng):
    """One oracle GDN decode layer (conv update + l2norm + recurrent step, fp32) over
    ``batch`` sequences; returns the seconds it took."""
    import oracle
    from myvllm_b200 import workloads as W

    x = rng.standard_normal((batch, W.GDN_CH)).astype(np.float32)
    w = (0.02 * rng.standard_normal((W.GDN_CH, W.GDN_W))).astype(np.float32)
    cst = rng.standard_normal((batch, W.GDN_W - 1, W.GDN_CH)).astype(np.float32)
    st = (0.1 * rng.standard_normal((batch, W.GDN_HV, W.GDN_DK, W.GDN_DV))).astype(np.float32)
    g = -rng.uniform(0.01, 1.0, (batch, W.GDN_HV)).astype(np.float32)
    beta = rng.uniform(0, 1, (batch, W.GDN_HV)).astype(np.float32)
    idx = np.arange(batch)
    t0 = time.perf_counter()
    qkv = oracle.conv.conv1d_update(x, w, cst, idx, dtype=np.float32)
    q = qkv[:, :2048].reshape(batch, 16, 128)
    k = qkv[:, 2048:4096].reshape(batch, 16, 128)
    v = qkv[:, 4096:].reshape(batch, 32, 128)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    oracle.gdn.recurrent_step(q, k, v, g, beta, st, idx, dtype=np.float32)
    return time.perf_counter() - t0


def cpu_baseline_c2(budget_s: float = 8.0, seed: int = 0):
    """The oracle of one config-2 decode step on batches of sequences until ``budget_s`` is
    spent; returns microseconds per full 256-sequence step (extrapolated), the sample size
    and the BLAS threads used."""
    rng = np.random.default_rng(seed)
    n, spent, batch = 0, 0.0, 16
    while spent < budget_s and n < 256:
        spent += _cpu_gdn_decode(batch, rng)
        n += batch
    return spent / n * 256 * 1e6, n, spent, host_threads()


def cpu_baseline_c3(budget_s: float = 8.0, seed: int = 0):
    """The oracle (numpy, fp32) of causal varlen attention with the config-3 heads on one
    sequence of growing length until ``budget_s`` is spent; returns tokens/s of the last
    (longest) sample and its length.  Per-token cost grows with the length, so the
    sample length is reported with it."""
    import oracle

    rng = np.random.default_rng(seed)
    L, best = 256, None
    total = 0.0
    while total < budget_s and L <= 16384:
        q = rng.standard_normal((L, 16, 256)).astype(np.float32)
        k = rng.standard_normal((L, 2, 256)).astype(np.float32)
        v = rng.standard_normal((L, 2, 256)).astype(np.float32)
        t0 = time.perf_counter()
        oracle.attention.varlen(q, k, v, np.array([0, L]), 1 / 16, True, dtype=np.float32)
        dt = time.perf_counter() - t0
        total += dt
        best = (L / dt, L, dt)
        L *= 2
    return best[0], best[1], best[2], host_threads()


def cpu_baseline_c4(ctx_lens, budget_s: float = 10.0, seed: int = 0):
    """The oracle of one config-4 decode step, extrapolated from a bounded sample: GDN decode
    layers over batches of 16 sequences, and single-query paged attention over the first
    sequences' full contexts (numpy, fp32), each until half the budget is spent, plus the
    projection GEMMs of one layer of each kind at the full batch.  Returns us per 48-layer
    step for 128 sequences, and the sample description."""
    import oracle

    rng = np.random.default_rng(seed)
    S, hidden = len(ctx_lens), 2048
    # GDN mixers
    n, t_gdn = 0, 0.0
    while t_gdn < budget_s / 2 and n < S:
        t_gdn += _cpu_gdn_decode(16, rng)
        n += 16
    gdn_per_seq = t_gdn / n
    # attention: one query per sequence over its context (one layer, all 16 heads)
    m, t_fa, tok = 0, 0.0, 0
    while t_fa < budget_s / 2 and m < S:
        L = ctx_lens[m]
        bs = 256
        nb = (L + bs - 1) // bs
        kc = rng.standard_normal((nb, bs, 2, 256)).astype(np.float32)
        vc = rng.standard_normal((nb, bs, 2, 256)).astype(np.float32)
        q = rng.standard_normal((1, 16, 256)).astype(np.float32)
        t0 = time.perf_counter()
        oracle.attention.paged_decode(q, kc, vc, np.arange(nb)[None].astype(np.int32), np.array([L], np.int32), 1 / 16)
        t_fa += time.perf_counter() - t0
        tok += L
        m += 1
    fa_per_token = t_fa / tok
    # projections of one layer of each kind at the full batch (fp32 GEMMs)
    x = rng.standard_normal((S, hidden)).astype(np.float32)
    o_in = rng.standard_normal((S, 4096)).astype(np.float32)

    def proj_s(n_in):  # the fused input projection and the output projection of one layer
        w_in = (0.02 * rng.standard_normal((n_in, hidden))).astype(np.float32)
        w_out = (0.02 * rng.standard_normal((hidden, 4096))).astype(np.float32)
        t0 = time.perf_counter()
        _ = x @ w_in.T
        _ = o_in @ w_out.T
        return time.perf_counter() - t0

    t_pg = proj_s(12352)  # GDN: qkv | z | a | b
    t_pf = proj_s(9216)   # attention: q + gate | k | v
    step_s = 36 * (gdn_per_seq * S + t_pg) + 12 * (fa_per_token * sum(ctx_lens) + t_pf)
    sample = (f"oracle GDN decode over {n} sequences ({t_gdn:.1f} s), paged decode over {m} contexts "
              f"({tok} tokens, {t_fa:.1f} s) and one layer's projections of each kind, extrapolated to "
              f"36 + 12 layers x {S} sequences")
    return step_s * 1e6, sample, host_threads()


# ----------------------------------------------------------------------------- c1 ----
def c1_rank_inputs(device, rank: int, world: int, lengths=None):
    """Config-1 inputs of one rank: the whole seeded batch with this rank's heads -- k-heads
    [r Hk/N, (r+1) Hk/N), v-heads [r Hv/N, (r+1) Hv/N) and their conv channels in
    QKVParallelLinear order [q_r | k_r | v_r].  Also returns the full inputs (for the
    tensor-parallel parity check on rank 0)."""
    from myvllm_b200 import workloads as W

    full = W.c1_inputs(device, seed=0, lengths=lengths)
    if world == 1:
        return dict(full, hk=W.GDN_HK, hv=W.GDN_HV), full
    hk, hv = W.GDN_HK // world, W.GDN_HV // world
    qs, vs, qt = hk * W.GDN_DK, hv * W.GDN_DV, W.GDN_HK * W.GDN_DK

    def channels(t, dim):
        parts = [t.narrow(dim, rank * qs, qs), t.narrow(dim, qt + rank * qs, qs), t.narrow(dim, 2 * qt + rank * vs, vs)]
        return torch.cat(parts, dim).contiguous()

    heads = slice(rank * hv, (rank + 1) * hv)
    mine = dict(full, x=channels(full["x"], 1), conv_w=channels(full["conv_w"], 0),
                conv_state=channels(full["conv_state"], 2), g=full["g"][:, heads].contiguous(),
                beta=full["beta"][:, heads].contiguous(), state=full["state"][:, heads].contiguous(), hk=hk, hv=hv)
    return mine, full


def c1_step(inp, events=None):
    """conv1d -> chunked GDN with the q/k L2 norm fused into its tile load; returns o.
    ``events`` brackets the GDN launch."""
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.causal_conv1d import causal_conv1d_fn
    from myvllm_b200.ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule

    qkv = causal_conv1d_fn(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"], inp["cu"])
    q, k, v = W.split_qkv(qkv, inp["hk"], inp["hv"])
    if events is not None:
        events[0].record()
    o = chunk_gated_delta_rule(q, k, v, inp["g"], inp["beta"], inp["state"], inp["idx"], inp["cu"],
                               use_qk_l2norm_in_kernel=True)
    if events is not None:
        events[1].record()
    return o


def c1_e2e(inp, world, n_steps):
    """End to end through the public op API with host buffers: every step copies its inputs
    from pinned host memory and reads its output back.  The steps are pipelined as a serving
    loop runs them: step i+1's H2D (copy stream) overlaps step i's compute and step i-1's
    D2H (second copy stream); two device input sets alternate.  Returns (ms per step, H2D
    bytes, D2H bytes)."""
    keys = ("x", "g", "beta", "cu")
    host = {k: inp[k].cpu().pin_memory() for k in keys}
    o_host = torch.empty((inp["T"], inp["hv"], 128), dtype=torch.bfloat16).pin_memory()
    dev_in = [dict(inp), dict(inp, **{k: torch.empty_like(inp[k]) for k in keys})]
    s_in, s_out, comp = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.current_stream()
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]

    def run(n, e_start=None, e_end=None):
        if e_start is not None:
            e_start.record(s_in)
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(comp_done[b])  # the step that read this input set is done
                for k_ in keys:
                    dev_in[b][k_].copy_(host[k_], non_blocking=True)
                h2d_done[b].record(s_in)
            comp.wait_event(h2d_done[b])
            o = c1_step(dev_in[b])
            comp_done[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[b])
                o_host.copy_(o, non_blocking=True)
                o.record_stream(s_out)
        if e_end is not None:
            e_end.record(s_out)

    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = ev(), ev()
    run(n_steps, e0, e1)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n_steps, world)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    return ms, h2d, o_host.numel() * o_host.element_size()


def c1_tp_parity(mine, full, rank, world):
    """After the timed region: every rank reruns one config-1 step on its heads from a zero
    state; rank 0 gathers the outputs and final states and compares them with one step over
    all heads on rank 0 alone.  The per-head math does not depend on the split, so the
    comparison is bit for bit."""
    mine = dict(mine)
    mine["state"] = torch.zeros_like(mine["state"])
    mine["conv_state"] = torch.zeros_like(mine["conv_state"])
    o = c1_step(mine)
    parts = [torch.empty_like(o) for _ in range(world)]
    torch.distributed.all_gather(parts, o.contiguous())
    sparts = [torch.empty_like(mine["state"]) for _ in range(world)]
    torch.distributed.all_gather(sparts, mine["state"])
    if rank != 0:
        return None
    from myvllm_b200 import workloads as W

    ref_in = dict(full, hk=W.GDN_HK, hv=W.GDN_HV, state=torch.zeros_like(full["state"]),
                  conv_state=torch.zeros_like(full["conv_state"]))
    ref = c1_step(ref_in)
    got, got_s = torch.cat(parts, 1), torch.cat(sparts, 1)
    torch.cuda.synchronize()
    return {"check": f"o and final states of {world}-way head-sharded config 1 vs one rank over all heads",
            "bit_exact": bool(torch.equal(got, ref) and torch.equal(got_s, ref_in["state"])),
            "max_abs_diff_o": (got.float() - ref.float()).abs().max().item(),
            "max_abs_diff_state": (got_s - ref_in["state"]).abs().max().item()}


def run_c1(args, rank, world, device):
    import oracle
    from myvllm_b200 import workloads as W

    inp, full = c1_rank_inputs(device, rank, world, args.lengths)
    T = inp["T"]
    with ClockSampler(device.index or 0) as clk:
        for _ in range(args.warmup):
            c1_step(inp)
        evs = [(ev(), ev()) for _ in range(args.steps)]
        ms = timed_region(lambda i: c1_step(inp, evs[i]), args.steps, world, clk)
        gdn_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evs), world)
        clocks = clk.summary()
        # the same loop for about a second and a half, for the settled (power-capped) figure
        n_sus = steps_for(1.5, ms, lo=args.steps)
        ms_sus = timed_region(lambda i: c1_step(inp), n_sus, world, clk)
        clocks_sus = clk.summary()
    check_device("c1")
    e2e_ms, h2d, d2h = c1_e2e(inp, world, max(8, args.steps))
    parity = c1_tp_parity(inp, full, rank, world) if world > 1 else None
    if rank != 0:
        return None
    pk, src = peaks()
    flops = T * inp["hv"] * oracle.gdn.flops_per_token_per_head(64, W.GDN_DK, W.GDN_DV)  # one rank's launch
    achieved = flops / (gdn_ms * 1e-3) / 1e12
    traffic = profiled_traffic("gdn_chunk_c1")
    cpu = None
    if world == 1:
        base_tps, base_tok, base_s, base_cores = cpu_baseline_c1()
        cpu = {"value": base_tps, "unit": "tokens/s", "cores": base_cores, "kind": "port",
               "sample": f"{base_tok} tokens of config-1 sequences (numpy oracle, fp32), {base_s:.1f} s"}
    line = {
        "metric": "prefill tokens/s (GDN layer: conv1d + chunked gated delta rule)",
        "value": T / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "c1: GDN prefill layer, 8 seqs ~U[512,8192] (seed 0), 16/32 heads x 128, "
                               "conv W=4 over 8192 ch, chunk 64",
                   "tokens": T, "lengths": inp["lengths"],
                   "parallelism": f"tp{world}: {inp['hk']} k-heads / {inp['hv']} v-heads per rank, one batch",
                   "l2": "inputs larger than L2 (x is %.0f MB)" % (full["x"].numel() * 2 / 1e6)},
        "roofline": {"bound": "tensor", "kernel": "gdn_chunk_tc_kernel", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                     "peak_source": f"{src} bf16 burst", "flops_per_launch_rank0": flops, "launch_ms": gdn_ms,
                     "traffic": traffic if world == 1 else None},
        "sustained": {"steps": n_sus, "ms_per_step": ms_sus, "value": T / (ms_sus * 1e-3), "clocks": clocks_sus},
        "cpu_baseline": cpu,
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": max(8, args.steps),
                "pipeline": "per step: H2D of x, g, beta, cu (pinned) -> conv1d + chunk GDN -> D2H of o; "
                            "H2D, compute and D2H of neighbouring steps overlap on three streams"},
        "gpu_launches": 2 * args.steps,
        "device_status": 0,
        "clocks": clocks,
    }
    if parity is not None:
        line["tp_parity"] = {"c1": parity}
    return line


def _standalone(block, args, world):
    """A nested block as a line of its own (``--config c2|c3|c4``)."""
    out = dict(block)
    out.update({"n_gpus": world, "warmup": args.warmup, "scaling": block.get("scaling", "strong"),
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic"})
    return out


def _serial_e2e(step, host_in: dict, dev_in: dict, out_host: torch.Tensor, n: int, world: int):
    """Per step: pinned host inputs -> device, the step, its output -> pinned host; steps in
    order on one stream (a decode loop).  Returns ms per step, max over ranks."""
    for _ in range(2):
        for k, v in host_in.items():
            dev_in[k].copy_(v, non_blocking=True)
        out_host.copy_(step(), non_blocking=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record()
    for _ in range(n):
        for k, v in host_in.items():
            dev_in[k].copy_(v, non_blocking=True)
        out_host.copy_(step(), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1) / n, world)


# ----------------------------------------------------------------------------- c2 ----
def run_c2(args, rank, world, device):
    """Config 2: one GDN decode step (conv update + recurrent GDN with the q/k norm fused),
    256 sequences, state [256, 32, 128, 128] fp32 read and written in place."""
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.causal_conv1d import causal_conv1d_update
    from myvllm_b200.ops.gated_delta_rule.fused_recurrent_gdn import fused_recurrent_gdn

    inp = W.c2_inputs(device, seed=0)
    evs = []

    def step(i=None):
        qkv = causal_conv1d_update(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"])
        q, k, v = W.split_qkv(qkv)
        if i is not None:
            evs[i][0].record()
        o = fused_recurrent_gdn(q, k, v, inp["g"], inp["beta"], inp["state"], inp["idx"], use_qk_l2norm_in_kernel=True)
        if i is not None:
            evs[i][1].record()
        return o

    for _ in range(args.warmup):
        step()
    est = timed_region(lambda i: step(), 3, world)
    n = steps_for(SUSTAINED_S, est, lo=args.steps)
    evs[:] = [(ev(), ev()) for _ in range(n)]
    with ClockSampler(device.index or 0) as clk:
        ms = timed_region(step, n, world, clk)
        clocks = clk.summary()
    check_device("c2")
    rec_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evs), world)
    # the same decode step as the layer runs it: one kernel for conv update + q/k norm + gates
    # + recurrence + RMSNormGated (the norm's gate z and weight added)
    from myvllm_b200.ops.gated_delta_rule.fused_layer import gated_deltanet_decode

    gz = torch.Generator(device=device).manual_seed(5)
    z = torch.randn(inp["x"].shape[0], W.GDN_HV, W.GDN_DV, generator=gz, device=device).to(torch.bfloat16)
    nw = torch.ones(W.GDN_DV, device=device, dtype=torch.bfloat16)

    def fused_step(i=None):
        return gated_deltanet_decode(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"], inp["a"], inp["b"],
                                     inp["A_log"], inp["dt_bias"], inp["state"], inp["idx"], z, nw, 1e-6)

    for _ in range(args.warmup):
        fused_step()
    fused_ms = timed_region(fused_step, n, world)
    check_device("c2 fused")
    host_in = {k: inp[k].cpu().pin_memory() for k in ("x", "g", "beta")}
    o_host = torch.empty(inp["x"].shape[0], W.GDN_HV, W.GDN_DV, dtype=torch.bfloat16).pin_memory()
    e2e_ms = _serial_e2e(step, host_in, inp, o_host, 20, world)
    if rank != 0:
        return None
    state_bytes = 2 * inp["state"].numel() * 4
    step_bytes = state_bytes + 2 * inp["conv_state"].numel() * 2 + 2 * inp["x"].numel() * 2 + o_host.numel() * 2
    pk, src = peaks()
    gbs = state_bytes / (rec_ms * 1e-3) / 1e9
    cpu = None
    if world == 1:
        us, ns, spent, cores = cpu_baseline_c2()
        cpu = {"value": us, "unit": "us", "cores": cores, "kind": "port",
               "sample": f"{ns} of 256 sequences (numpy oracle, fp32), {spent:.1f} s, extrapolated to the full step"}
    return {"metric": "decode us/step (GDN layer: conv1d update + recurrent GDN)", "value": ms * 1e3, "unit": "us",
            "ms_per_step": ms, "steps": n, "higher_is_better": False,
            "config": {"workload": "c2: 256 seqs, state [256,32,128,128] fp32 ~N(0,0.1), conv state [256,3,8192] bf16",
                       "l2": "state (512 MiB) larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "gdn_recurrent_kernel", "achieved": gbs, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "peak_source": src, "launch_us": rec_ms * 1e3,
                         "bytes_per_launch": state_bytes, "traffic": profiled_traffic("gdn_recurrent_c2"),
                         "step_frac": step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_ms * 1e3, "unit": "us", "h2d_bytes_per_step":
                    sum(v.numel() * v.element_size() for v in host_in.values()),
                    "d2h_bytes_per_step": o_host.numel() * 2, "steps": 20,
                    "pipeline": "per step: H2D of the step's qkv projection and gates (pinned) -> conv update + "
                                "recurrent GDN -> D2H of o; states stay resident"},
            "fused_layer_step": {"us": fused_ms * 1e3, "steps": n, "kernel": "gdn_decode_fused_kernel",
                                 "what": "conv update + q/k L2 norm + gates + recurrence + RMSNormGated in one "
                                         "kernel (mvb_gated_deltanet_decode), as GatedDeltaNet decodes",
                                 "hbm_frac": (step_bytes + 2 * z.numel() * 2) / (fused_ms * 1e-3) / 1e9
                                 / pk["hbm_gbs"]},
            "gpu_launches": 2 * n, "device_status": 0, "clocks": clocks}


# ----------------------------------------------------------------------------- c3 ----
def run_c3(args, rank, world, device):
    """Config 3: the KV write into a paged cache (block 256, permuted block table) and varlen
    causal flash-attention prefill, 16 q / 2 kv heads, head dim 256, 8 seqs ~U[1024, 16384].
    Timed over at least a second of back-to-back launches (the settled, power-capped rate)."""
    import oracle
    from myvllm_b200 import _lib
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.full_attention import flash_attention_prefill
    from myvllm_b200.ops.kv_cache import store_kvcache

    inp = W.c3_inputs(device, seed=0, lengths=args.lengths)
    kc = torch.zeros(inp["n_blocks"], inp["block_size"], 2, 256, dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    evs = []

    def step(i=None):
        store_kvcache(inp["k"], inp["v"], kc, vc, inp["slot_mapping"])
        if i is not None:
            evs[i][0].record()
        o = flash_attention_prefill(inp["q"], inp["k"], inp["v"], inp["cu"], inp["scale"], 16, 2, 256, 256, True)
        if i is not None:
            evs[i][1].record()
        return o

    for _ in range(args.warmup):
        step()
    path = _lib.last_path(_lib.OP_FA_PREFILL)
    est = timed_region(lambda i: step(), 3, world)
    n = steps_for(SUSTAINED_S, est, lo=args.steps)
    evs[:] = [(ev(), ev()) for _ in range(n)]
    with ClockSampler(device.index or 0) as clk:
        ms = timed_region(step, n, world, clk)
        clocks = clk.summary()
    check_device("c3")
    fa_times = [a.elapsed_time(b) for a, b in evs]
    fa_ms = max_over_ranks(statistics.mean(fa_times), world)
    host_in = {k: inp[k].cpu().pin_memory() for k in ("q", "k", "v", "cu", "slot_mapping")}
    o_host = torch.empty(inp["T"], 16, 256, dtype=torch.bfloat16).pin_memory()
    e2e_ms = _serial_e2e(step, host_in, inp, o_host, 4, world)
    if rank != 0:
        return None
    flops = oracle.attention.varlen_flops(inp["cu"].cpu().numpy(), 16, 256, 256, True)
    pk, src = peaks()
    tf = flops / (fa_ms * 1e-3) / 1e12
    first_ms = fa_times[0]
    cpu = None
    if world == 1:
        tps, ns, spent, cores = cpu_baseline_c3()
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"one {ns}-token sequence with the config-3 heads (numpy oracle, fp32), {spent:.1f} s; "
                         "per-token cost grows with length, so this understates the CPU time at config-3 lengths"}
    return {"metric": "prefill tokens/s (full attention: KV write + varlen causal FA)", "value": inp["T"] / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": n, "higher_is_better": True,
            "config": {"workload": "c3: Hq16/Hkv2/D256 causal, 8 seqs ~U[1024,16384], KV written to a paged cache "
                                   "(block 256)", "tokens": inp["T"], "lengths": inp["lengths"],
                       "l2": "q/k/v (%.0f MB) larger than L2" % ((inp["q"].numel() + 2 * inp["k"].numel()) * 2 / 1e6),
                       "timed_region_s": ms * n / 1e3},
            "roofline": {"bound": "tensor", "kernel": "fa_tc_kernel", "path": path[0], "achieved": tf,
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": tf / pk["bf16_tflops"],
                         "frac_of_sustained": tf / pk.get("bf16_tflops_sustained", pk["bf16_tflops"]),
                         "peak_source": f"{src} bf16 burst", "launch_ms": fa_ms, "first_launch_ms": first_ms,
                         "flops_per_launch": flops, "traffic": profiled_traffic("flash_prefill_c3")},
            "cpu_baseline": cpu,
            "e2e": {"value": inp["T"] / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": sum(v.numel() * v.element_size() for v in host_in.values()),
                    "d2h_bytes_per_step": o_host.numel() * 2, "steps": 4,
                    "pipeline": "per step: H2D of q, k, v, cu_seqlens, slot_mapping (pinned) -> KV write + FA -> "
                                "D2H of o, in order on one stream"},
            "gpu_launches": 2 * n, "device_status": 0, "clocks": clocks}


# ----------------------------------------------------------------------------- c4 ----
def run_c4(args, rank, world, device):
    """Config 4: one decode step of a 48-layer hybrid stack (36 GDN + 12 gated full
    attention, hidden 2048, pre-norm + mixer + residual; no MLP/MoE; each mixer's input
    projections fused into one GEMM, the GDN gates formed in-kernel), 128 sequences with
    context ~U[1024, 32768] in a paged bf16 KV cache (block 256) and fp32 GDN states.  Heads
    are tensor-parallel over the ranks with an all-reduce after every output projection (the
    one-shot NVLink kernel by default, NCCL with --allreduce nccl); KV heads are replicated
    past TP 2.  The step is captured once as a CUDA graph and replayed."""
    from myvllm_b200 import _lib
    from myvllm_b200 import workloads as W
    from myvllm_b200.decode_stack import HybridDecodeStack, hidden_input

    S, n_layers = args.seqs or 128, args.layers or 48
    oneshot = fused = None
    if world > 1 and args.allreduce in ("oneshot", "fused"):
        from myvllm_b200.layers import comm

        # the o_proj / out_proj partial sums ([128, 2048] bf16, 512 KiB) go through the
        # one-shot NVLink kernel instead of NCCL; with "fused" the projection and its
        # all-reduce run as one kernel (decode batches), the one-shot kernel covering the rest
        oneshot = comm.enable_oneshot(max_bytes=2 << 20)
        if args.allreduce == "fused":
            fused = comm.enable_fused_linear()
    ctx_lens = W.seq_lengths(S, 1024, 32768, 4)
    n_max = max(args.steps, 300)
    stack = HybridDecodeStack(n_layers, S, ctx_lens, args.warmup + n_max + 8, device, seed=1234)
    meta = stack.step_metadata(args.warmup + n_max + 8)
    st_bt, st_cl, st_sl, st_cos, st_sin = (t.clone() for t in meta[0])
    x0 = hidden_input(S, device)
    x_in = x0.clone()

    def load_meta(i):
        for dst, src in zip((st_bt, st_cl, st_sl, st_cos, st_sin), meta[i]):
            dst.copy_(src, non_blocking=True)

    with torch.no_grad():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(args.warmup):
                load_meta(i)
                stack.forward(x_in, st_bt, st_cl, st_sl, st_cos, st_sin)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        load_meta(args.warmup)
        calls0 = _lib.n_calls
        with torch.cuda.graph(graph):
            out_static = stack.forward(x_in, st_bt, st_cl, st_sl, st_cos, st_sin)
        calls_per_step = _lib.n_calls - calls0  # library entry points captured in one step
        torch.cuda.synchronize()
        base = args.warmup + 1

        def replay(i):
            load_meta(base + i)
            graph.replay()

        est = timed_region(replay, 3, world)
        base += 3
        n = min(n_max - 3, steps_for(SUSTAINED_S, est, lo=args.steps))
        with ClockSampler(device.index or 0) as clk:
            ms = timed_region(replay, n, world, clk)
            clocks = clk.summary()
        base += n
        check_device("c4")
        # end to end: hidden states in from pinned host memory, out to pinned host memory
        xh = x0.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        e0, e1 = ev(), ev()
        e0.record()
        for i in range(3):
            x_in.copy_(xh, non_blocking=True)
            load_meta(base + i % 4)
            graph.replay()
            oh.copy_(out_static, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / 3, world)
        del graph  # graphs holding NCCL work are released before the process group
    parity = c4_tp_parity(rank, world, device) if world > 1 else None
    if oneshot is not None:
        from myvllm_b200.layers import comm

        comm.disable_oneshot()  # raises if a one-shot wait gave up
        if fused is not None:
            comm.disable_fused_linear()
    by = stack.bytes_per_step()
    del stack
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    pk, src = peaks()
    gbs = by["total"] / (ms * 1e-3) / 1e9
    cpu = None
    if world == 1:
        us, sample, cores = cpu_baseline_c4(ctx_lens)
        cpu = {"value": us, "unit": "us", "cores": cores, "kind": "port", "sample": sample}
    block = {"metric": f"decode us/step ({n_layers}-layer hybrid stack, {S} seqs)", "value": ms * 1e3, "unit": "us",
             "ms_per_step": ms, "steps": n, "higher_is_better": False, "scaling": "strong",
             "config": {"workload": f"c4: {n_layers - n_layers // 4} GDN + {n_layers // 4} gated-attention layers, "
                                    f"hidden 2048, {S} seqs, ctx ~U[1024,32768]",
                        "parallelism": f"tp{world}", "l2": "KV and states far larger than L2",
                        "all_reduce": ("none" if world == 1 else
                                       "output projection + all-reduce in one kernel (mvb_linear_allreduce)"
                                       if fused is not None else
                                       "one-shot NVLink kernel (mvb_allreduce_oneshot)" if oneshot is not None
                                       else "NCCL"),
                        "execution": "one CUDA graph per decode step"},
             "roofline": {"bound": "hbm", "kernel": "whole decode step (per rank)", "achieved": gbs,
                          "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "peak_source": src,
                          "bytes_per_step_rank0": by, "traffic": None},
             "cpu_baseline": cpu,
             "e2e": {"value": e2e_ms * 1e3, "unit": "us", "h2d_bytes_per_step": xh.numel() * 2,
                     "d2h_bytes_per_step": oh.numel() * 2, "steps": 3},
             "gpu_launches": calls_per_step * n,
             "gpu_launches_note": "library entry-point calls in the captured step x steps (each launches one or "
                                  "more kernels; the GEMMs are cuBLAS)",
             "device_status": 0, "clocks": clocks}
    if parity is not None:
        block["tp_parity"] = parity
    return block


def c4_tp_parity(rank, world, device):
    """Two decode steps of a 4-layer slice of the stack (3 GDN + 1 gated attention, 8
    sequences, non-zero states, paged KV) at TP = world, against the same slice built
    unsharded on rank 0 from the same seeded full weights, states and caches.

    The two runs differ only in bf16 rounding: the sharded GEMMs reduce in another order and
    the all-reduce adds the partial sums, so single activations move by an ulp (2^-8
    relative), and a GDN decay gate g = -exp(A_log) softplus(a + dt_bias) turns an ulp of
    its projection `a` into a relative change of the whole state of up to exp(A_log) * 2^-8.
    The check is therefore normwise: ||out_tp - out_1|| / ||out_1|| <= 1e-2 per step and the
    same for rank 0's GDN states; a sharding error (a wrong head, channel or KV slice)
    gives errors of order one."""
    from myvllm_b200 import workloads as W
    from myvllm_b200.decode_stack import HybridDecodeStack, hidden_input

    ctx = W.seq_lengths(8, 100, 1500, 11)
    x = hidden_input(8, device, seed=3)
    with torch.no_grad():
        stack = HybridDecodeStack(4, 8, ctx, 4, device, seed=99)
        outs = [stack.forward(x, *m) for m in stack.step_metadata(2)]
        torch.cuda.synchronize()
        torch.distributed.barrier()
        res = None
        if rank == 0:
            ref = HybridDecodeStack(4, 8, ctx, 4, device, seed=99, tp=(0, 1))
            routs = [ref.forward(x, *m) for m in ref.step_metadata(2)]
            rel, mx = [], []
            for a, b in zip(outs, routs):
                a, b = a.float(), b.float()
                rel.append(((a - b).norm() / b.norm()).item())
                mx.append((a - b).abs().max().item())
            hv_r = stack.lac.recurrent_cache.shape[2]
            s_a, s_b = stack.lac.recurrent_cache, ref.lac.recurrent_cache[:, :, :hv_r]
            s_rel = ((s_a - s_b).norm() / s_b.norm()).item()
            res = {"check": f"2 decode steps of a 3 GDN + 1 attention slice at tp{world} vs one rank unsharded "
                            "(normwise relative error <= 1e-2)",
                   "pass": max(rel) <= 1e-2 and s_rel <= 1e-2, "out_rel_err": rel, "out_max_abs_diff": mx,
                   "state_rel_err_rank0_heads": s_rel}
            del ref
        torch.distributed.barrier()
    return res


# ------------------------------------------------------------------------ reference ----
def run_reference(args):
    """The CPU restatement of the reference path on this host's cores, on the config-1
    metric.  torchrun sets OMP_NUM_THREADS=1; the BLAS pools are widened to every host
    thread."""
    from threadpoolctl import threadpool_limits

    t_all = 0.0
    tok_all = 0
    with threadpool_limits(limits=os.cpu_count()):
        cpu_baseline_c1(budget_s=0.5, seed=1)  # warm-up: imports, BLAS thread start
        for _ in range(args.steps):
            _, tok, s, cores = cpu_baseline_c1(budget_s=max(2.0, 30.0 / max(1, args.steps)), seed=0)
            t_all += s
            tok_all += tok
    v = tok_all / t_all
    return {"metric": "prefill tokens/s (GDN layer: conv1d + chunked gated delta rule)", "value": v,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t_all / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "c1: GDN prefill layer, 8 seqs ~U[512,8192] (seed 0), bounded sample per step"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{tok_all} tokens over {args.steps} steps (numpy oracle of the reference "
                                       "path; its Triton kernels do not run on a CPU)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--config", default="all", choices=["all", "c1", "c2", "c3", "c4"])
    ap.add_argument("--layers", type=int, default=None,
                    help="c4: layers instead of 48 (a multiple of 4; smaller cases for profiler captures)")
    ap.add_argument("--seqs", type=int, default=None, help="c4: sequences instead of 128 (profiler cases)")
    ap.add_argument("--allreduce", default="oneshot", choices=["oneshot", "fused", "nccl"],
                    help="c4 at N > 1: the tensor-parallel all-reduce after each output projection (fused: the "
                         "projection and its all-reduce in one kernel)")
    ap.add_argument("--lengths", default=None,
                    help="c1/c3: sequence lengths instead of the config's seeded draw, e.g. 8x2048 or 700,1500 "
                         "(smaller cases for profiler captures)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.lengths:
        if "x" in args.lengths:
            n, length = args.lengths.split("x")
            args.lengths = [int(length)] * int(n)
        else:
            args.lengths = [int(v) for v in args.lengths.split(",")]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    from myvllm_b200 import _lib

    _lib.load()  # fail loudly if the library is missing
    if args.config == "c1":
        line = run_c1(args, rank, world, device)
    elif args.config != "all":
        fn = {"c2": run_c2, "c3": run_c3, "c4": run_c4}[args.config]
        block = fn(args, rank, world, device)
        line = _standalone(block, args, world) if block is not None else None
    else:
        line = run_c1(args, rank, world, device)
        torch.cuda.empty_cache()
        blocks = ("c2", "c3", "c4") if world == 1 else ("c4",)
        for name in blocks:
            block = {"c2": run_c2, "c3": run_c3, "c4": run_c4}[name](args, rank, world, device)
            torch.cuda.empty_cache()
            if line is not None:
                if name == "c4" and block is not None and "tp_parity" in block:
                    line.setdefault("tp_parity", {})["c4"] = block.pop("tp_parity")
                line[name] = block
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
