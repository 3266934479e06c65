"""GPU: the one-shot NVLink all-reduce (mvb_allreduce_oneshot, used by RowParallelLinear
through myvllm_b200.layers.comm) against NCCL's all_reduce on the same inputs, on every GPU
of the box up to 8 (skipped with fewer than 2).  One process per GPU, NVLS off."""

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
        # element counts: one block, ragged block split, decode size (128 x 2048), the limit
        for n in (8, 4096 + 8, 3 * 8192 + 56, 128 * 2048, 1 << 20):
            for dtype in (torch.bfloat16, torch.float16):
                x = torch.randn(n, generator=g, device=dev).to(dtype)
                y = comm.all_reduce(x.clone())
                ref = x.clone()
                dist.all_reduce(ref)
                tol = 0 if world == 2 else 2e-2
                err = (y.float() - ref.float()).abs().max().item()
                assert err <= tol * max(1.0, ref.float().abs().max().item()), (n, dtype, err)
                # every rank holds the same bits
                peer = y.clone()
                dist.broadcast(peer, 0)
                assert torch.equal(y.view(torch.int16), peer.view(torch.int16)), (n, dtype)
        # too large for the buffer: NCCL takes it
        big = torch.ones(2 << 20, device=dev, dtype=torch.bfloat16)
        assert not ar.eligible(big) and comm.all_reduce(big) is big and big[0].item() == world
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
            ref0 = x.clone()
            dist.all_reduce(ref0)
            ref1 = ref0.clone()
            dist.all_reduce(ref1)
            assert (out[0].float() - ref0.float()).abs().max().item() <= (0 if world == 2 else 0.05)
            assert (out[1].float() - ref1.float()).abs().max().item() <= 0.05 * max(1.0, ref1.float().abs().max().item())
        torch.cuda.synchronize()
        del graph
        assert _lib.device_status() == 0
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
