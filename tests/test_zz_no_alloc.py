"""GPU test of the allocation-free paged decode entry point.

`mvb_paged_attention_decode_noalloc` serves callers that may not allocate device memory
when they decode: its split-KV partial results live in a fixed array inside the library
instead of a caller workspace.  Here it is called through the C ABI twice in a row, on two
different problems, and each result must match the workspace entry point
(`paged_flash_attention_decode`) within the bf16 tolerance; the second call also shows
that what the first call left in the shared array does not leak into the next result.

This file is named to be collected last: a failure here leaves every other test run.
"""

import pytest
import torch

from myvllm_b200 import _lib
from myvllm_b200.ops.full_attention import paged_flash_attention_decode
from tests.util import assert_close

pytestmark = pytest.mark.gpu


def _problem(seed, ctx, hq, hkv, d, bs):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nb_per = [(n + bs - 1) // bs for n in ctx]
    n_blocks = sum(nb_per) + 2
    perm = torch.randperm(n_blocks, generator=torch.Generator().manual_seed(seed))
    bt = torch.zeros(len(ctx), max(nb_per), dtype=torch.int32)
    o = 0
    for s, nb in enumerate(nb_per):
        bt[s, :nb] = perm[o:o + nb].to(torch.int32)
        o += nb
    kc = torch.randn(n_blocks, bs, hkv, d, generator=g, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn(n_blocks, bs, hkv, d, generator=g, device="cuda", dtype=torch.bfloat16)
    q = torch.randn(len(ctx), hq, d, generator=g, device="cuda", dtype=torch.bfloat16)
    return q, kc, vc, bt.cuda(), torch.tensor(ctx, dtype=torch.int32, device="cuda")


def _decode_noalloc(q, kc, vc, bt, ctx, scale, bs):
    o = torch.empty(q.shape[0], q.shape[1], vc.shape[-1], dtype=q.dtype, device=q.device)
    _lib.call("paged_attention_decode_noalloc", "mvb_paged_attention_decode_noalloc", _lib.desc(q), _lib.desc(kc),
              _lib.desc(vc), _lib.desc(bt), _lib.desc(ctx), float(scale), int(bs), int(bt.shape[1]) * int(bs),
              _lib.desc(o), _lib.stream_of(q))
    return o


def test_noalloc_decode_matches_workspace_entry_on_two_calls():
    problems = [
        # config-4 attention shapes, long enough contexts to split
        (dict(seed=0, ctx=[8000, 1, 257, 4096, 6000, 31, 512, 7777] * 2, hq=16, hkv=2, d=256, bs=256), 1 / 16),
        # a different shape on the second call (reduced heads as at 8-way tensor parallelism)
        (dict(seed=1, ctx=[3000, 700, 5, 2048, 1500], hq=2, hkv=1, d=128, bs=64), 128 ** -0.5),
    ]
    for kw, scale in problems:
        q, kc, vc, bt, ctx = _problem(**kw)
        ref = paged_flash_attention_decode(q, kc, vc, bt, ctx, scale, kw["bs"])
        out = _decode_noalloc(q, kc, vc, bt, ctx, scale, kw["bs"])
        torch.cuda.synchronize()
        assert_close(out, ref, what=f"noalloc decode (seed {kw['seed']})")


def test_noalloc_decode_runs_unsplit_when_two_splits_do_not_fit():
    # 256 sequences x 2 kv heads x head dim 256: the partials of two splits (2 x 8.4 MB) do
    # not fit the 16 MiB array, so this entry point decodes every context in one split while
    # the workspace entry point splits them (3 splits here); the results must still agree
    rng = torch.Generator().manual_seed(5)
    ctx = torch.randint(1, 3001, (256,), generator=rng).tolist()
    q, kc, vc, bt, ctx_t = _problem(seed=5, ctx=ctx, hq=16, hkv=2, d=256, bs=256)
    ref = paged_flash_attention_decode(q, kc, vc, bt, ctx_t, 1 / 16, 256)
    out = _decode_noalloc(q, kc, vc, bt, ctx_t, 1 / 16, 256)
    torch.cuda.synchronize()
    assert_close(out, ref, what="noalloc decode, unsplit")
