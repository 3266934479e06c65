"""GPU: the one-shot NVLink all-reduce (mvb_allreduce_oneshot, used by RowParallelLinear
through myvllm_b200.layers.comm) on every GPU of the box up to 8 (skipped with fewer than 2).
One process per GPU, NVLS off.

The kernel adds the ranks' inputs in fp32 in rank order and rounds once, so its output is
compared bit for bit with that sum formed by torch from the all-gathered inputs.  NCCL's
all_reduce is a cross-check within a relative tolerance: past two ranks it rounds its
partial sums to 16 bits, so it differs from the exact sum by an ulp or so."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_GPUS = min(8, torch.cuda.device_count()) if torch.cuda.is_available() else 0
needs_two = pytest.mark.skipif(N_GPUS < 2, reason="needs 2 or more GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from myvllm_b200 import _lib
        from myvllm_b200.layers import comm

        ar = comm.enable_oneshot(max_bytes=2 << 20)
        g = torch.Generator(device=dev).manual_seed(100 + rank)

        def exact_sum(x):
            # every rank's input, added in fp32 in rank order, rounded once
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)
            acc = torch.zeros(x.shape, dtype=torch.float32, device=dev)
            for part in parts:
                acc += part.float()
            return acc.to(x.dtype)

        def rel_err(y, ref):
            return (y.float() - ref.float()).abs().max().item() / max(1.0, ref.float().abs().max().item())
        # element counts: one block, ragged block split, decode size (128 x 2048), the limit
        for n in (8, 4096 + 8, 3 * 8192 + 56, 128 * 2048, 1 << 20):
            for dtype in (torch.bfloat16, torch.float16):
                x = torch.randn(n, generator=g, device=dev).to(dtype)
                y = comm.all_reduce(x.clone())
                exact = exact_sum(x)
                assert torch.equal(y.view(torch.int16), exact.view(torch.int16)), (n, dtype, rel_err(y, exact))
                ref = x.clone()
                dist.all_reduce(ref)
                assert rel_err(y, ref) <= 2e-2, (n, dtype, rel_err(y, ref))
                # every rank holds the same bits
                peer = y.clone()
                dist.broadcast(peer, 0)
                assert torch.equal(y.view(torch.int16), peer.view(torch.int16)), (n, dtype)
        # back-to-back calls of changing sizes with no host or collective synchronisation
        # between them, while the ranks drift apart (a spin kernel on a different rank at each
        # call): a slot overwritten while a lagging peer still reads it would mix two calls
        sizes = [4096, 6144, 8, 131072, 4104, 262144, 16, 65536 + 8, 8, 128 * 2048, 4096, 6144]
        ins, outs = [], []
        for i, n in enumerate(sizes):
            if i % world == rank:
                torch.cuda._sleep(2_000_000)
            x = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
            ins.append(x)
            outs.append(comm.all_reduce(x))
        torch.cuda.synchronize()
        for i, (x, y) in enumerate(zip(ins, outs)):
            exact = exact_sum(x)
            assert torch.equal(y.view(torch.int16), exact.view(torch.int16)), ("unsynchronised", i, sizes[i],
                                                                               rel_err(y, exact))
        # too large for the buffer: NCCL takes it
        big = torch.ones(2 << 20, device=dev, dtype=torch.bfloat16)
        assert not ar.eligible(big), "a 4 MiB message must not fit the 2 MiB slots"
        assert comm.all_reduce(big) is big and big[0].item() == world, big[0].item()
        # a CUDA graph replays the kernel with fresh call counters each time
        x = torch.randn(128, 2048, generator=g, device=dev).to(torch.bfloat16)
        out = [None, None]
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            comm.all_reduce(x)  # warm-up outside capture
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out[0] = comm.all_reduce(x)
            out[1] = comm.all_reduce(out[0])
        for it in range(3):
            x.copy_(torch.randn(128, 2048, generator=g, device=dev).to(torch.bfloat16))
            graph.replay()
            torch.cuda.synchronize()
            ref0 = exact_sum(x)
            ref1 = exact_sum(ref0)  # every rank holds the same ref0, as it holds the same out[0]
            assert torch.equal(out[0].view(torch.int16), ref0.view(torch.int16)), (it, rel_err(out[0], ref0))
            assert torch.equal(out[1].view(torch.int16), ref1.view(torch.int16)), (it, rel_err(out[1], ref1))
        torch.cuda.synchronize()
        del graph
        status = _lib.device_status()
        assert status == 0, f"device error word {status}"
        comm.disable_oneshot()
        dist.barrier()
        dist.destroy_process_group()
        results[rank] = "ok"
    except Exception as e:  # noqa: BLE001
        results[rank] = f"{type(e).__name__}: {e}"


@needs_two
def test_oneshot_allreduce_matches_nccl():
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, N_GPUS, port, results)) for r in range(N_GPUS)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(results.get(r) == "ok" for r in range(N_GPUS)), dict(results)


def _worker_fused(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from myvllm_b200 import _lib
        from myvllm_b200.layers import comm

        f = comm.enable_fused_linear()
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        K, N = 4096 // world, 2048

        def reference(x, w):
            xs = [torch.empty_like(x) for _ in range(world)]
            ws = [torch.empty_like(w) for _ in range(world)]
            dist.all_gather(xs, x)
            dist.all_gather(ws, w)
            return sum(a.float() @ b.float().T for a, b in zip(xs, ws))

        def same_on_all_ranks(y):
            peer = y.clone()
            dist.broadcast(peer, 0)
            return torch.equal(y.view(torch.int16), peer.view(torch.int16))

        def close(y, ref):
            return bool(((y.float() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all().item())

        w = (0.02 * torch.randn(N, K, generator=g, device=dev)).to(torch.bfloat16)
        # row counts: a full decode batch, ragged, one row
        for m in (128, 37, 1):
            x = torch.randn(m, K, generator=g, device=dev).to(torch.bfloat16)
            assert f.eligible(x, w)
            y = comm.fused_linear(x, w)
            torch.cuda.synchronize()
            assert close(y, reference(x, w)), ("fused linear", m)
            assert same_on_all_ranks(y), ("bits differ across ranks", m)
        # back-to-back calls of changing row counts with no synchronisation between them, the
        # ranks drifting apart
        ms = [128, 5, 64, 128, 1, 100]
        ins, outs = [], []
        for i, m in enumerate(ms):
            if i % world == rank:
                torch.cuda._sleep(2_000_000)
            x = torch.randn(m, K, generator=g, device=dev).to(torch.bfloat16)
            ins.append(x)
            outs.append(comm.fused_linear(x, w))
        torch.cuda.synchronize()
        for i, (x, y) in enumerate(zip(ins, outs)):
            assert close(y, reference(x, w)), ("unsynchronised fused linear", i)
        # CUDA graph replay
        x = torch.randn(128, K, generator=g, device=dev).to(torch.bfloat16)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            comm.fused_linear(x, w)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = comm.fused_linear(x, w)
        for it in range(3):
            x.copy_(torch.randn(128, K, generator=g, device=dev).to(torch.bfloat16))
            graph.replay()
            torch.cuda.synchronize()
            assert close(out, reference(x, w)), ("graph replay", it)
        del graph
        # the layer: RowParallelLinear takes the fused path and matches F.linear + NCCL
        from myvllm_b200.layers.linear import RowParallelLinear

        lin = RowParallelLinear(K * world, N, bias=False).to(dev, torch.bfloat16)
        lin.weight.data.copy_(w)
        x = torch.randn(16, K, generator=g, device=dev).to(torch.bfloat16)
        y = lin(x)
        ref = torch.nn.functional.linear(x, w)
        dist.all_reduce(ref)
        assert close(y, ref.float()), "RowParallelLinear fused path"
        assert _lib.device_status() == 0
        comm.disable_fused_linear()
        dist.barrier()
        dist.destroy_process_group()
        results[rank] = "ok"
    except Exception as e:  # noqa: BLE001
        results[rank] = f"{type(e).__name__}: {e}"


@needs_two
def test_fused_linear_allreduce():
    """mvb_linear_allreduce: each rank's x W^T (tcgen05 GEMM) and the sum over ranks in one
    kernel, against the fp32 sum of the all-gathered partial products (bf16 bar), identical
    bits on every rank, unsynchronised back-to-back calls, graph replay, and the
    RowParallelLinear path."""
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fused, args=(r, N_GPUS, port, results)) for r in range(N_GPUS)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(results.get(r) == "ok" for r in range(N_GPUS)), dict(results)


def test_fused_linear_single_rank():
    """mvb_linear_allreduce with one rank (the kernel's GEMM tiles, the split-K partials in its
    buffer and their reduction, without peers) against torch fp32 x W^T, on one GPU; two calls
    in a row exercise the slot alternation."""
    import ctypes

    from myvllm_b200 import _lib

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    buf = torch.zeros(int(lib.mvb_linear_allreduce_buffer_bytes()) + 256, dtype=torch.uint8, device=dev)
    base = (buf.data_ptr() + 255) // 256 * 256
    peers = _lib.MvbAllReducePeers()
    peers.world, peers.rank, peers.buf_bytes = 1, 0, int(lib.mvb_linear_allreduce_buffer_bytes())
    peers.bufs[0] = base
    g = torch.Generator(device=dev).manual_seed(7)
    for m, k, n in ((128, 4096, 2048), (37, 1024, 2048), (1, 512, 4096)):
        x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
        w = (0.02 * torch.randn(n, k, generator=g, device=dev)).to(torch.bfloat16)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        _lib.call("linear_allreduce", "mvb_linear_allreduce", ctypes.byref(peers), _lib.desc(x), _lib.desc(w),
                  _lib.desc(out), _lib.stream_of(x))
        ref = x.float() @ w.float().T
        torch.cuda.synchronize()
        assert bool(((out.float() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all().item()), (m, k, n)
    assert _lib.device_status() == 0
