"""Generate the golden fixtures in this directory from the reference itself.

Run once, in a container that has the reference checkout and Triton (CPU is enough):

    REF_SRC=<reference>/src python tests/golden/make_golden.py

It imports the reference package ``myvllm`` with ``TRITON_INTERPRET=1`` and runs the
two reference kernels that work as written:

* ``_fused_recurrent_gdn`` (``src/myvllm/ops/gated_delta_rule/fused_recurrent_gdn.py:6-102``),
  stepped once per token over config 0 (T=256, H=4, d=64, fp32, zero initial state).
  The wrapper ``fused_recurrent_gdn`` (``:105-166``) passes its grid as a list, which
  the interpreter rejects, so this script launches the reference's own kernel object
  with the same arguments and the grid as a tuple.
* ``paged_flash_attention_decode`` (``src/myvllm/ops/full_attention.py:282-335``), as is.

It also records fla 0.5.1's naive recurrent and chunk (chunk 64) gated delta rule on
the same config-0 inputs as an independent cross-check.  Nothing at test time reads
the reference; the tests read only the ``.npz`` files written here.
"""

from __future__ import annotations

import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
if not os.environ.get("REF_SRC"):
    sys.exit("make_golden.py: set REF_SRC to the reference checkout's src/ directory")
sys.path.insert(0, os.environ["REF_SRC"])


def c0_inputs(seed: int = 0):
    """Config 0: T=256, H=4, d_k=d_v=64, fp32; q,k ~N(0,1) L2-normalised per head;
    v ~N(0,1); beta = sigmoid(N(0,1)); g = logsigmoid(N(2,1))."""
    torch.manual_seed(seed)
    T, H, D = 256, 4, 64
    q = F.normalize(torch.randn(T, H, D), dim=-1)
    k = F.normalize(torch.randn(T, H, D), dim=-1)
    v = torch.randn(T, H, D)
    beta = torch.sigmoid(torch.randn(T, H))
    g = F.logsigmoid(torch.randn(T, H) + 2.0)
    return q, k, v, beta, g


def run_reference_recurrent(q, k, v, beta, g):
    from myvllm.ops.gated_delta_rule.fused_recurrent_gdn import _fused_recurrent_gdn

    T, H, D = q.shape
    state = torch.zeros(1, H, D, D)
    idx = torch.zeros(1, dtype=torch.int32)
    o_all = torch.zeros(T, H, D)
    for t in range(T):
        qt, kt, vt = q[t:t + 1].contiguous(), k[t:t + 1].contiguous(), v[t:t + 1].contiguous()
        gt, bt = g[t:t + 1].contiguous(), beta[t:t + 1].contiguous()
        o = torch.zeros_like(vt)
        BLOCK_V = 8
        grid = (1, H, triton_cdiv(D, BLOCK_V))
        _fused_recurrent_gdn[grid](
            qt, *qt.stride(), kt, *kt.stride(), vt, *vt.stride(), o, *o.stride(),
            gt, *gt.stride(), bt, *bt.stride(), state, *state.stride(), idx,
            D ** -0.5, H, D, H, D, BLOCK_V,
        )
        o_all[t] = o[0]
    return o_all, state[0]


def triton_cdiv(a, b):
    return (a + b - 1) // b


def paged_decode_case(seed: int = 1):
    """Small paged decode case: 3 seqs, Hq=4, Hkv=2, D=64, block 16, ctx [1, 37, 100]."""
    g = torch.Generator().manual_seed(seed)
    S, Hq, Hkv, D, bs = 3, 4, 2, 64, 16
    ctx = torch.tensor([1, 37, 100], dtype=torch.int32)
    max_blocks = 8
    n_blocks = 24
    perm = torch.randperm(n_blocks, generator=g)[: S * max_blocks].view(S, max_blocks).to(torch.int32)
    q = torch.randn(S, Hq, D, generator=g)
    kc = torch.randn(n_blocks, bs, Hkv, D, generator=g)
    vc = torch.randn(n_blocks, bs, Hkv, D, generator=g)
    return q, kc, vc, perm, ctx, D ** -0.5, bs


def main():
    q, k, v, beta, g = c0_inputs()
    ref_o, ref_state = run_reference_recurrent(q, k, v, beta, g)
    from fla.ops.gated_delta_rule.naive import naive_chunk_gated_delta_rule, naive_recurrent_gated_delta_rule

    fo, fs = naive_recurrent_gated_delta_rule(q[None], k[None], v[None], beta[None], g[None],
                                              output_final_state=True)
    co, cs = naive_chunk_gated_delta_rule(q[None], k[None], v[None], g[None], beta[None], chunk_size=64,
                                          output_final_state=True)
    np.savez_compressed(
        os.path.join(HERE, "c0_gdn.npz"),
        q=q.numpy(), k=k.numpy(), v=v.numpy(), beta=beta.numpy(), g=g.numpy(),
        ref_o=ref_o.numpy(), ref_state=ref_state.numpy(),
        fla_recurrent_o=fo[0].numpy(), fla_recurrent_state=fs[0].numpy(),
        fla_chunk_o=co[0].numpy(), fla_chunk_state=cs[0].numpy(),
    )
    print("c0: ref vs fla recurrent o", (ref_o - fo[0]).abs().max().item(),
          "state", (ref_state - fs[0]).abs().max().item())

    from myvllm.ops.full_attention import paged_flash_attention_decode

    qd, kc, vc, bt, ctx, scale, bs = paged_decode_case()
    od = paged_flash_attention_decode(qd, kc, vc, bt, ctx, scale, bs)
    np.savez_compressed(os.path.join(HERE, "paged_decode.npz"), q=qd.numpy(), k_cache=kc.numpy(),
                        v_cache=vc.numpy(), block_tables=bt.numpy(), context_lens=ctx.numpy(),
                        scale=np.float64(scale), block_size=np.int64(bs), ref_o=od.numpy())
    print("paged decode done", od.shape)


if __name__ == "__main__":
    main()
