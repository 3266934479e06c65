"""GPU self-test of the tensor-core layer (descriptors, swizzled layouts, negation,
accumulation) against torch fp32 matmul."""

import pytest
import torch

from myvllm_b200 import _lib
from tests.util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [64, 128])
@pytest.mark.parametrize("k", [64, 128])
@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("negate", [0, 1])
def test_umma_layouts(n, k, a_mn, b_mn, negate):
    g = torch.Generator().manual_seed(n + k + 2 * a_mn + 4 * b_mn + 8 * negate)
    A = torch.randn(128, k, generator=g).half()
    B1 = torch.randn(k, n, generator=g).half()
    B2 = torch.randn(k, n, generator=g).half()
    a_store = (A.t() if a_mn else A).contiguous().cuda()
    b1_store = (B1 if b_mn else B1.t()).contiguous().cuda()
    b2_store = (B2 if b_mn else B2.t()).contiguous().cuda()
    d = torch.full((128, n), float("nan"), device="cuda")
    _lib.call("selftest_umma", "mvb_selftest_umma", a_store.data_ptr(), b1_store.data_ptr(), b2_store.data_ptr(),
              d.data_ptr(), n, k, a_mn, b_mn, negate, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = A.float() @ B1.float() + (-1 if negate else 1) * (A.float() @ B2.float())
    assert_close(d, ref, atol=1e-3, rtol=1e-3)
