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
