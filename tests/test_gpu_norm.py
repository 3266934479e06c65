"""GPU parity: gated RMSNorm vs a torch fp32 reference (m/layers/norm.py:50-58)."""

import pytest
import torch

from myvllm_b200 import _lib
from tests.util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d", [128, 256, 1024])
def test_rmsnorm_gated(d):
    g = torch.Generator().manual_seed(d)
    x = torch.randn(333, d, generator=g).to(torch.bfloat16).cuda()
    z = torch.randn(333, d, generator=g).to(torch.bfloat16).cuda()
    w = torch.randn(d, generator=g).cuda()
    out = torch.empty_like(x)
    _lib.call("rmsnorm_gated", "mvb_rmsnorm_gated", _lib.desc(x), _lib.desc(z), _lib.desc(w), 1e-6, _lib.desc(out),
              _lib.stream_of(x))
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w * torch.nn.functional.silu(z.float())
    assert_close(out, ref)


@pytest.mark.parametrize("d", [256, 2048])
@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm_zero_centered_and_residual(d, residual):
    from myvllm_b200.layers.norm import RMSNorm

    g = torch.Generator().manual_seed(d + residual)
    norm = RMSNorm((d,), 1e-6, True).cuda()
    norm.weight.data.normal_(0, 0.1, generator=None)
    x = torch.randn(77, d, generator=g).to(torch.bfloat16).cuda()
    r = torch.randn(77, d, generator=g).to(torch.bfloat16).cuda()
    r0 = r.clone()
    if residual:
        out, s = norm(x, residual=r)
        base = (x.float() + r0.float())
        assert_close(s, base)
    else:
        out = norm(x)
        base = x.float()
    ref = base * torch.rsqrt(base.pow(2).mean(-1, keepdim=True) + 1e-6) * (norm.weight.float() + 1)
    assert_close(out, ref)


def test_rmsnorm_strided_head_rows():
    from myvllm_b200.layers.norm import RMSNorm

    norm = RMSNorm((256,), 1e-6, True).cuda()
    qg = torch.randn(9, 16, 512, device="cuda").to(torch.bfloat16)
    q = qg[..., :256]  # strided head rows, as q of the gated q projection
    out = norm(q)
    qf = q.float()
    assert_close(out, qf * torch.rsqrt(qf.pow(2).mean(-1, keepdim=True) + 1e-6) * 2.0)


def test_norms_on_two_stride_head_views():
    """q/k head views and the z gate of a fused projection: [T, H, D] slices whose rows sit
    at two strides; the kernels index them directly."""
    from myvllm_b200.layers.norm import RMSNorm, RMSNormGated

    g = torch.Generator().manual_seed(5)
    y = torch.randn(37, 12352, generator=g).to(torch.bfloat16).cuda()  # a fused projection output
    k = y[:, 8192:8704].view(37, 2, 256)  # k heads of the fused projection
    norm = RMSNorm((256,), 1e-6, True).cuda()
    kf = k.float()
    assert_close(norm(k), kf * torch.rsqrt(kf.pow(2).mean(-1, keepdim=True) + 1e-6) * 2.0)
    z = y[:, 9216:12288].view(37, 24, 128)
    x = torch.randn(37, 24, 128, generator=g).to(torch.bfloat16).cuda()
    gated = RMSNormGated((128,), 1e-6).cuda()
    gated.weight.data.uniform_(0.5, 1.5)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * gated.weight.float() * \
        torch.nn.functional.silu(z.float())
    assert_close(gated(x, z), ref)


@pytest.mark.parametrize("d,rd,heads", [(256, 64, 16), (128, 128, 4), (256, 16, 2)])
def test_rmsnorm_rope_matches_norm_then_rotary(d, rd, heads):
    """Fused q/k norm + partial rotary (mvb_rmsnorm_rope) against the layer's two steps in
    fp32 (m/layers/full_attention.py:49-64, m/layers/rotary_embedding.py:6-31), on a strided
    head view like the fused projection's q."""
    from myvllm_b200.layers.norm import RMSNorm
    from myvllm_b200.layers.rotary_embedding import RotaryEmbedding, apply_partial_rotary

    g = torch.Generator().manual_seed(d + rd)
    T = 37
    norm = RMSNorm((d,), 1e-6, True).cuda()
    norm.weight.data = (0.1 * torch.randn(d, generator=g)).cuda()
    base = torch.randn(T, heads, 2 * d, generator=g).to(torch.bfloat16).cuda()
    x = base[:, :, :d]  # strided rows, as q out of the fused q|gate projection
    pos = torch.randint(0, 30000, (T,), generator=g).cuda()
    cos, sin = RotaryEmbedding(rd, 10_000_000.0).cuda().cos_sin(pos)
    out = norm.rope_forward(x, cos, sin)
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * (norm.weight.float() + 1.0)
    ref = apply_partial_rotary(y, cos.float(), sin.float())
    assert_close(out, ref)
