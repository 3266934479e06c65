"""Tensor-parallel host logic on CPU with world_size-2 gloo ranks: the weight loaders
shard full checkpoints the way the forwards read them, and row-parallel partial products
summed by all_reduce reproduce the unsharded projections (reference m/layers/linear.py)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, results):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.manual_seed(0)
        from myvllm_b200.layers import linear as L

        hidden = 32
        x = torch.randn(5, hidden)
        if case == "column_row":
            col = L.ColumnParallelLinear(hidden, 48, bias=True)
            row = L.RowParallelLinear(48, hidden, bias=True)
            w1, b1 = torch.randn(48, hidden), torch.randn(48)
            w2, b2 = torch.randn(hidden, 48), torch.randn(hidden)
            col.weight_loader(col.weight, w1)
            col.weight_loader(col.bias, b1)
            row.weight_loader(row.weight, w2)
            row.weight_loader(row.bias, b2)
            y = row(col(x))
            ref = (x @ w1.T + b1) @ w2.T + b2
            assert torch.allclose(y, ref, atol=1e-4), (y - ref).abs().max()
        # shard GEMMs and full GEMMs may take different BLAS kernels: fp32 rounding-level
        # differences (~1e-6) are expected, hence the absolute tolerances below
        elif case == "qkv":
            m = L.QKVParallelLinear(hidden, 4, 4, 8, 4, 4, 6)
            w = torch.randn(4 * 4 + 4 * 4 + 8 * 6, hidden)
            m.weight_loader(m.weight, w)
            full = x @ w.T
            q, k, v = full[:, :16], full[:, 16:32], full[:, 32:]
            mine = m(x)
            qs, ks, vs = 4 * 2, 4 * 2, 8 * 3
            assert torch.allclose(mine[:, :qs], q[:, rank * qs:(rank + 1) * qs], atol=1e-5)
            assert torch.allclose(mine[:, qs:qs + ks], k[:, rank * ks:(rank + 1) * ks], atol=1e-5)
            assert torch.allclose(mine[:, qs + ks:], v[:, rank * vs:(rank + 1) * vs], atol=1e-5)
        elif case == "gated_q":
            m = L.GatedQParallelLinear(hidden, 8, 4)
            w = torch.randn(4 * 16, hidden)
            m.weight_loader(m.weight, w)
            full = (x @ w.T).view(5, 4, 16)
            mine = m(x).view(5, 2, 16)
            assert torch.allclose(mine, full[:, rank * 2:(rank + 1) * 2], atol=1e-5)
        elif case == "kv_replicated":
            for heads in (2, 1):  # split at tp <= heads, replicated at tp > heads
                m = L.KVParallelLinear(hidden, 8, heads)
                w = torch.randn(heads * 8, hidden)
                m.weight_loader(m.weight, w)
                full = (x @ w.T).view(5, heads, 8)
                head = rank if heads == 2 else 0
                assert m.num_kv_heads == 1
                assert torch.allclose(m(x).view(5, 8), full[:, head], atol=1e-5)
        elif case == "layers":
            from myvllm_b200.layers.full_attention import GatedAttention
            from myvllm_b200.layers.linear_attention import GatedDeltaNet

            gdn = GatedDeltaNet(64, 16, 32, 8, 8, 4)
            assert gdn.num_k_heads == 8 and gdn.num_v_heads == 16
            assert gdn.conv1d.weight.shape == (2 * 8 * 8 + 16 * 8, 4)
            assert gdn.out_proj.weight.shape == (64, 16 * 8)
            att = GatedAttention(64, 16, 16, 16, 2, False, 1e-6)
            assert att.num_q_heads == 8 and att.num_kv_heads == 1
            assert att.o_proj.weight.shape == (64, 8 * 16)
        elif case == "comm_dispatch":
            # comm.all_reduce: the collective by default; an enabled one-shot object takes the
            # tensors it calls eligible (a stand-in here: IPC buffers need GPUs)
            from myvllm_b200.layers import comm

            t = torch.full((4,), float(rank + 1))
            assert comm.all_reduce(t) is t and torch.equal(t, torch.full((4,), 3.0))

            class Fake:
                calls = 0

                def eligible(self, x):
                    return x.numel() <= 4

                def __call__(self, x):
                    Fake.calls += 1
                    return x * 10

            comm._oneshot[None] = Fake()
            try:
                small = comm.all_reduce(torch.ones(4))
                assert Fake.calls == 1 and torch.equal(small, torch.full((4,), 10.0))
                big = torch.ones(8)
                assert comm.all_reduce(big) is big and torch.equal(big, torch.full((8,), 2.0)) and Fake.calls == 1
                # the row-parallel layer routes its partial sums through the same function
                row = L.RowParallelLinear(8, 4)
                row.weight.data.fill_(1.0)
                y = row(torch.ones(1, 4))  # this rank's half of the 8 input features
                assert Fake.calls == 2 and torch.equal(y, torch.full((1, 4), 40.0))
            finally:
                comm._oneshot.pop(None, None)
        results.put((rank, None))
    except Exception as e:  # report to the parent instead of hanging it
        results.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("case", ["column_row", "qkv", "gated_q", "kv_replicated", "layers", "comm_dispatch"])
def test_tp2_gloo(case):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    errors = [f"rank {r}: {e}" for r, e in results if e is not None]
    assert not errors, "; ".join(errors)
