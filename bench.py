"""Benchmark of the myvllm attention hot path on B200.

Default (the headline line): config 1 -- one Gated-DeltaNet prefill layer, i.e.
causal_conv1d_fn over 8192 qkv channels -> l2norm(q, k) -> chunk_gated_delta_rule
(chunk 64), 8 sequences with lengths ~U[512, 8192], bf16 activations, fp32 state.
Metric: prefill tokens/s.  Multi-GPU (torchrun): every rank runs its own independent
config-1 batch (sequences are independent objects; no collective on the data path),
so scaling is weak and ``value`` = all ranks' tokens / max-over-ranks step time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
                    [--config c1|c2|c3]

``--impl reference`` times the CPU restatement of the reference path (the oracle; the
reference's own kernels are Triton and do not run on a CPU) on the host's cores.
``--config c2|c3`` prints the same kind of line for the decode / full-attention
configs (diagnostic; the headline is c1).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


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
    """nvidia-smi clock / throttle sampling during the timed region."""

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
        self.samples = window
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[2 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- c1 ----
def c1_step(inp, ops, events=None):
    """conv1d -> chunked GDN with the q/k L2 norm fused into its tile load; returns o.
    ``events`` brackets the GDN launch."""
    from myvllm_b200 import workloads as W

    qkv = ops.causal_conv1d_fn(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"], inp["cu"])
    q, k, v = W.split_qkv(qkv)
    if events is not None:
        events[0].record()
    o = ops.chunk_gated_delta_rule(q, k, v, inp["g"], inp["beta"], inp["state"], inp["idx"], inp["cu"],
                                   use_qk_l2norm_in_kernel=True)
    if events is not None:
        events[1].record()
    return o


class _C1Ops:
    def __init__(self):
        from myvllm_b200.ops.causal_conv1d import causal_conv1d_fn
        from myvllm_b200.ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule

        self.causal_conv1d_fn = causal_conv1d_fn
        self.chunk_gated_delta_rule = chunk_gated_delta_rule


def host_threads():
    """Threads the numpy oracle's BLAS runs with right now (threadpoolctl); 1 without BLAS."""
    from threadpoolctl import threadpool_info

    return max([d["num_threads"] for d in threadpool_info()] + [1])


def cpu_baseline_c1(budget_s: float = 12.0, seed: int = 0):
    """The oracle (numpy restatement of the reference path) on a bounded sample of the
    config-1 workload: whole sequences of the seeded batch, conv1d + l2norm + chunked
    GDN, all 32 heads, until ``budget_s`` of CPU time is spent.  Returns tokens/s."""
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


def cpu_baseline_c2(budget_s: float = 8.0, seed: int = 0):
    """The oracle (numpy, fp32) of one config-2 decode step -- conv update + l2norm +
    recurrent GDN over all 32 heads -- on batches of sequences until ``budget_s`` is spent;
    returns microseconds per full 256-sequence step (extrapolated), the sample size and the
    BLAS threads used."""
    import oracle
    from myvllm_b200 import workloads as W

    rng = np.random.default_rng(seed)
    n, spent, batch = 0, 0.0, 16
    while spent < budget_s and n < 256:
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
        spent += time.perf_counter() - t0
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


def run_c1(args, rank, world, device):
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.gated_delta_rule.gated_delta_rule import chunk_gated_delta_rule  # noqa: F401
    import oracle

    ops = _C1Ops()
    inp = W.c1_inputs(device, seed=rank, lengths=args.lengths)
    T = inp["T"]
    clk = ClockSampler(device.index or 0).__enter__()
    time.sleep(1.0)  # let the sampler start before the work it samples
    for _ in range(args.warmup):
        c1_step(inp, ops)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.mark_start()
    if True:
        start.record()
        for i in range(args.steps):
            c1_step(inp, ops, ev[i])
        stop.record()
        torch.cuda.synchronize()
    clk.mark_stop()
    clk.__exit__()
    ms = start.elapsed_time(stop) / args.steps
    gdn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    if world > 1:
        t = torch.tensor([ms, float(T)], device=device, dtype=torch.float64)
        mx = t.clone()
        torch.distributed.all_reduce(mx[:1], op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(t[1:], op=torch.distributed.ReduceOp.SUM)
        ms, tokens_all = mx[0].item(), t[1].item()
        torch.distributed.barrier()
    else:
        tokens_all = float(T)

    # end to end through the public op API with host buffers: every step copies its inputs
    # from pinned host memory and reads its output back.  The steps are pipelined as a
    # serving loop runs them: step i+1's H2D (copy stream) overlaps step i's compute and
    # step i-1's D2H (second copy stream); two device input sets alternate.
    keys = ("x", "g", "beta", "cu")
    host = {k: inp[k].cpu().pin_memory() for k in keys}
    o_host = torch.empty((T, W.GDN_HV, W.GDN_DV), dtype=torch.bfloat16).pin_memory()
    dev_in = [dict(inp), dict(inp, **{k: torch.empty_like(inp[k]) for k in keys})]
    s_in, s_out, comp = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.current_stream()
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_steps(n, e_start=None, e_end=None):
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
            o = c1_step(dev_in[b], ops)
            comp_done[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[b])
                o_host.copy_(o, non_blocking=True)
                o.record_stream(s_out)
        if e_end is not None:
            e_end.record(s_out)

    e2e_steps(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(8, args.steps)
    e2e_steps(n_e2e, e0, e1)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / n_e2e
    if world > 1:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = o_host.numel() * o_host.element_size()

    if rank != 0:
        return None
    pk, src = peaks()
    flops = T * W.GDN_HV * oracle.gdn.flops_per_token_per_head(64, W.GDN_DK, W.GDN_DV)
    achieved = flops / (gdn_ms * 1e-3) / 1e12
    traffic = profiled_traffic("gdn_chunk_c1")
    # the CPU baseline is timed on rank 0 of a single-GPU run only (it is a reported
    # baseline, not part of the job)
    cpu = None
    if world == 1:
        base_tps, base_tok, base_s, base_cores = cpu_baseline_c1()
        cpu = {"value": base_tps, "unit": "tokens/s", "cores": base_cores, "kind": "port",
               "sample": f"{base_tok} tokens of config-1 sequences (numpy oracle, fp32), {base_s:.1f} s"}
    line = {
        "metric": "prefill tokens/s (GDN layer: conv1d + chunked gated delta rule)",
        "value": tokens_all / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "c1: GDN prefill layer, 8 seqs ~U[512,8192] (seed 0+rank), 16/32 heads x 128, "
                               "conv W=4 over 8192 ch, chunk 64",
                   "tokens_per_rank": T, "lengths_rank0": inp["lengths"], "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2 (x is %.0f MB)" % (inp["x"].numel() * 2 / 1e6)},
        "roofline": {"bound": "tensor", "kernel": "gdn_chunk_tc_kernel", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                     "peak_source": f"{src} bf16 burst", "flops_per_launch": flops, "launch_ms": gdn_ms,
                     "traffic": traffic},
        "cpu_baseline": cpu,
        "e2e": {"value": tokens_all / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "pipeline": "per step: H2D of x, g, beta, cu (pinned) -> conv1d + chunk GDN -> D2H of o; "
                            "H2D, compute and D2H of neighbouring steps overlap on three streams"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    return line


# ----------------------------------------------------------------------------- c2 ----
def run_c2(args, rank, world, device):
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.causal_conv1d import causal_conv1d_update
    from myvllm_b200.ops.gated_delta_rule.fused_recurrent_gdn import fused_recurrent_gdn

    inp = W.c2_inputs(device, seed=rank)

    def step(ev=None):
        qkv = causal_conv1d_update(inp["x"], inp["conv_w"], inp["conv_state"], inp["idx"])
        q, k, v = W.split_qkv(qkv)
        if ev:
            ev[0].record()
        o = fused_recurrent_gdn(q, k, v, inp["g"], inp["beta"], inp["state"], inp["idx"], use_qk_l2norm_in_kernel=True)
        if ev:
            ev[1].record()
        return o

    for _ in range(args.warmup):
        step()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        s0.record()
        for i in range(args.steps):
            step(evs[i])
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / args.steps
    rec_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    state_bytes = 2 * inp["state"].numel() * 4
    pk, src = peaks()
    gbs = state_bytes / (rec_ms * 1e-3) / 1e9
    cpu = None
    if world == 1 and rank == 0:
        us, n, spent, cores = cpu_baseline_c2()
        cpu = {"value": us, "unit": "us", "cores": cores, "kind": "port",
               "sample": f"{n} of 256 sequences (numpy oracle, fp32), {spent:.1f} s, extrapolated to the full step"}
    return {"metric": "decode us/step (GDN layer: conv1d update + recurrent GDN)", "value": ms * 1e3, "unit": "us",
            "cpu_baseline": cpu,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "c2: 256 seqs, state [256,32,128,128] fp32"},
            "roofline": {"bound": "hbm", "kernel": "gdn_recurrent_kernel", "achieved": gbs, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "peak_source": src, "launch_us": rec_ms * 1e3,
                         "traffic": profiled_traffic("gdn_recurrent_c2")},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary()}


# ----------------------------------------------------------------------------- c3 ----
def run_c3(args, rank, world, device):
    import oracle
    from myvllm_b200 import workloads as W
    from myvllm_b200.ops.full_attention import flash_attention_prefill
    from myvllm_b200.ops.kv_cache import store_kvcache

    inp = W.c3_inputs(device, seed=rank, lengths=args.lengths)
    kc = torch.zeros(inp["n_blocks"], inp["block_size"], 2, 256, dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)

    def step(ev=None):
        store_kvcache(inp["k"], inp["v"], kc, vc, inp["slot_mapping"])
        if ev:
            ev[0].record()
        o = flash_attention_prefill(inp["q"], inp["k"], inp["v"], inp["cu"], inp["scale"], 16, 2, 256, 256, True)
        if ev:
            ev[1].record()
        return o

    for _ in range(args.warmup):
        step()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        s0.record()
        for i in range(args.steps):
            step(evs[i])
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / args.steps
    fa_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    flops = oracle.attention.varlen_flops(inp["cu"].cpu().numpy(), 16, 256, 256, True)
    pk, src = peaks()
    tf = flops / (fa_ms * 1e-3) / 1e12
    cpu = None
    if world == 1 and rank == 0:
        tps, n, spent, cores = cpu_baseline_c3()
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"one {n}-token sequence with the config-3 heads (numpy oracle, fp32), {spent:.1f} s; "
                         "per-token cost grows with length, so this understates the CPU time at config-3 lengths"}
    return {"metric": "prefill tokens/s (full attention: KV write + varlen causal FA)", "cpu_baseline": cpu,
            "value": inp["T"] / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "c3: Hq16/Hkv2/D256 causal, 8 seqs ~U[1024,16384]", "tokens": inp["T"]},
            "roofline": {"bound": "tensor", "kernel": "fa_tc_kernel", "achieved": tf,
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": tf / pk["bf16_tflops"],
                         "peak_source": src, "launch_ms": fa_ms, "flops_per_launch": flops,
                         "traffic": profiled_traffic("flash_prefill_c3")},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary()}


# ----------------------------------------------------------------------------- c4 ----
def run_c4(args, rank, world, device):
    """Config 4: one decode step of a 48-layer hybrid stack (36 GDN + 12 gated full
    attention, hidden 2048, pre-norm + mixer + residual; no MLP/MoE; each mixer's input
    projections fused into one GEMM, the GDN gates formed in-kernel), 128 sequences with
    context ~U[1024, 32768] in a paged bf16 KV cache (block 256) and fp32 GDN states.
    Heads are tensor-parallel over the ranks with an all-reduce after every output
    projection (the one-shot NVLink kernel by default, NCCL with --allreduce nccl); KV heads
    are replicated past TP 2."""
    from myvllm_b200 import _lib
    from myvllm_b200 import workloads as W
    from myvllm_b200.cache.linear_attention_cache import LinearAttentionCache, PagedKVCache
    from myvllm_b200.layers.full_attention import GatedAttention
    from myvllm_b200.layers.linear_attention import GatedDeltaNet
    from myvllm_b200.layers.norm import RMSNorm
    from myvllm_b200.layers.rotary_embedding import RotaryEmbedding
    from myvllm_b200.utils.context import set_context

    torch.manual_seed(1234)  # identical weights on every rank (each loads its shard)
    S, hidden, n_layers, bs = args.seqs or 128, 2048, args.layers or 48, 256
    oneshot = None
    if world > 1 and args.allreduce == "oneshot":
        from myvllm_b200.layers import comm

        # the o_proj / out_proj partial sums ([128, 2048] bf16, 512 KiB) go through the
        # one-shot NVLink kernel instead of NCCL
        oneshot = comm.enable_oneshot(max_bytes=2 << 20)
    kinds = ["full" if (i + 1) % 4 == 0 else "gdn" for i in range(n_layers)]
    layers = []
    for kind in kinds:
        mixer = GatedDeltaNet(hidden, 16, 32, 128, 128, 4) if kind == "gdn" else \
            GatedAttention(hidden, 256, 16, 256, 2, False, 1e-6)
        for name, prm in mixer.named_parameters():
            if not (name.endswith("A_log") or name.endswith("dt_bias") or "norm" in name):
                prm.data.normal_(0.0, 0.02)
        mixer = mixer.to(device, torch.bfloat16)
        if kind == "gdn":
            mixer.A_log.data = mixer.A_log.data.float()
            mixer.dt_bias.data = mixer.dt_bias.data.float()
        mixer.fuse_projections()  # weights are final: one input GEMM per layer
        layers.append((RMSNorm((hidden,), 1e-6, True).to(device, torch.bfloat16), mixer))
    gdn = [m for k, (_, m) in zip(kinds, layers) if k == "gdn"]
    fa = [m for k, (_, m) in zip(kinds, layers) if k == "full"]
    lac = LinearAttentionCache(len(gdn), S, 4, 128, 128, gdn[0].num_k_heads, gdn[0].num_v_heads, torch.bfloat16,
                               device)
    lac.recurrent_cache.normal_(0.0, 0.1)
    lac.conv_cache.normal_(0.0, 1.0)
    for i, m in enumerate(gdn):
        m.conv_state, m.recurrent_state = lac.layer_states(i)
    ctx_lens = W.seq_lengths(S, 1024, 32768, 4)
    steps_total = args.warmup + args.steps + 4
    n_blocks = sum((c + steps_total + bs - 1) // bs for c in ctx_lens)
    kv = PagedKVCache(len(fa), n_blocks, bs, fa[0].num_kv_heads, 256, torch.bfloat16, device)
    for i in range(len(fa)):  # fill the caches layer by layer (bounded temporaries)
        kv.k[i].normal_()
        kv.v[i].normal_()
    for i, m in enumerate(fa):
        m.k_cache, m.v_cache = kv.layer_caches(i)
    seq_ids = list(range(S))
    for s, c in enumerate(ctx_lens):
        kv.append(s, c)
    idx = torch.arange(S, dtype=torch.int32, device=device)
    rope = RotaryEmbedding(64, 10_000_000.0).to(device)
    meta = []  # per-step metadata, built before timing
    for step in range(steps_total):
        for s in seq_ids:
            kv.append(s, 1)
        bt, cl, slots = kv.metadata(seq_ids, [1] * S)
        cos, sin = rope.cos_sin((cl - 1).long())
        meta.append((bt, cl, slots, cos, sin))
    g_ = torch.Generator(device=device).manual_seed(7)
    x0 = torch.randn(S, hidden, generator=g_, device=device, dtype=torch.bfloat16)

    # static buffers: the whole step is captured once as a CUDA graph and replayed with each
    # step's metadata copied in (block tables padded to the widest step)
    width = max(m[0].shape[1] for m in meta)
    meta = [(F.pad(bt, (0, width - bt.shape[1])), cl, sl, c, s_) for bt, cl, sl, c, s_ in meta]
    st_bt, st_cl, st_sl, st_cos, st_sin = (t.clone() for t in meta[0])
    x_in = x0.clone()

    def load_meta(i):
        for dst, src in zip((st_bt, st_cl, st_sl, st_cos, st_sin), meta[i]):
            dst.copy_(src, non_blocking=True)

    def step_static():
        set_context(False, slot_mapping=st_sl, context_lens=st_cl, block_tables=st_bt, block_size=bs)
        res = x_in.clone()
        h = None
        for (norm, mixer), kind in zip(layers, kinds):
            if h is None:
                normed = norm(res)
            else:
                normed, res = norm(h, residual=res)  # res += h; normed = rms(res)
            h = mixer(normed, None, idx, idx, False) if kind == "gdn" else mixer(normed, st_cos, st_sin)
        return res + h

    with torch.no_grad():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(args.warmup):
                load_meta(i)
                step_static()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        load_meta(args.warmup)
        calls0 = _lib.n_calls
        with torch.cuda.graph(graph):
            out_static = step_static()
        calls_per_step = _lib.n_calls - calls0  # library entry points captured in one step
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        clk = ClockSampler(device.index or 0).__enter__()
        time.sleep(0.5)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk.mark_start()
        s0.record()
        for i in range(args.steps):
            load_meta(args.warmup + i)
            graph.replay()
        s1.record()
        torch.cuda.synchronize()
        clk.mark_stop()
        clk.__exit__()
        ms = s0.elapsed_time(s1) / args.steps
        # end to end: hidden states in from pinned host memory, out to pinned host memory
        xh = x0.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(3):
            x_in.copy_(xh, non_blocking=True)
            load_meta(args.warmup + args.steps + i % 4)
            graph.replay()
            oh.copy_(out_static, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / 3
        del graph  # graphs holding NCCL work are released before the process group
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = t[0].item(), t[1].item()
    if oneshot is not None:
        comm.disable_oneshot()
    if rank != 0:
        return None
    hkv_rank = fa[0].num_kv_heads
    kv_bytes = sum(ctx_lens) * len(fa) * hkv_rank * 256 * 2 * 2
    state_bytes = 2 * lac.recurrent_cache.numel() * 4 + 2 * lac.conv_cache.numel() * 2
    w_bytes = sum(p.numel() * p.element_size() for _, m in layers for p in m.parameters())
    step_bytes = kv_bytes + state_bytes + w_bytes
    pk, src = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {"metric": "decode us/step (48-layer hybrid stack, 128 seqs)", "value": ms * 1e3, "unit": "us",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"c4: {n_layers - n_layers // 4} GDN + {n_layers // 4} gated-attention layers, hidden 2048, "
                                   f"{S} seqs, ctx ~U[1024,32768]",
                       "parallelism": f"tp{world}", "l2": "KV and states far larger than L2",
                       "all_reduce": ("none" if world == 1 else
                                      "one-shot NVLink kernel (mvb_allreduce_oneshot)" if oneshot is not None else "NCCL"),
                       "execution": "one CUDA graph per decode step"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (per rank)", "achieved": gbs,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "peak_source": src,
                         "bytes_per_step_rank0": step_bytes, "traffic": None},
            "e2e": {"value": e2e_ms * 1e3, "unit": "us", "h2d_bytes_per_step": xh.numel() * 2,
                    "d2h_bytes_per_step": oh.numel() * 2},
            "gpu_launches": calls_per_step * args.steps,
            "gpu_launches_note": "library entry-point calls in the captured step x steps (each launches one or more "
                                 "kernels; the GEMMs are cuBLAS)",
            "clocks": clk.summary()}


# ------------------------------------------------------------------------ reference ----
def run_reference(args):
    """The CPU restatement of the reference path on this host's cores, on the c1 metric.
    torchrun sets OMP_NUM_THREADS=1; the BLAS pools are widened to every host thread."""
    from threadpoolctl import threadpool_limits

    t_all = 0.0
    tok_all = 0
    with threadpool_limits(limits=os.cpu_count()):
        cpu_baseline_c1(budget_s=0.5, seed=1)  # warm-up: imports, BLAS thread start
        for i in range(args.steps):
            _, tok, s, cores = cpu_baseline_c1(budget_s=max(2.0, 30.0 / max(1, args.steps)), seed=0)
            t_all += s
            tok_all += tok
    v = tok_all / t_all
    return {"metric": "prefill tokens/s (GDN layer: conv1d + chunked gated delta rule)", "value": v,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t_all / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "c1: GDN prefill layer, 8 seqs ~U[512,8192] (seed 0), bounded sample per step"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{tok_all} tokens over {args.steps} steps (numpy oracle of the reference "
                                       "path; its Triton kernels do not run on a CPU)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--config", default="c1", choices=["c1", "c2", "c3", "c4"])
    ap.add_argument("--layers", type=int, default=None,
                    help="c4: layers instead of 48 (a multiple of 4; smaller cases for profiler captures)")
    ap.add_argument("--seqs", type=int, default=None, help="c4: sequences instead of 128 (profiler cases)")
    ap.add_argument("--allreduce", default="oneshot", choices=["oneshot", "nccl"],
                    help="c4 at N > 1: the tensor-parallel all-reduce after each output projection")
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
    fn = {"c1": run_c1, "c2": run_c2, "c3": run_c3, "c4": run_c4}[args.config]
    line = fn(args, rank, world, device)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
