"""Tolerances and comparison helpers shared by the parity tests.

Tolerances are the ones the port is held to: outputs in bf16 within 2e-2 max-abs /
1e-2 relative (elementwise |a - b| <= 2e-2 + 1e-2 |b|); final fp32 recurrent states
within 1e-3 relative (Frobenius norm of the error over that of the oracle, per
(sequence, head)).
"""

import numpy as np
import torch

BF16_ATOL = 2e-2
BF16_RTOL = 1e-2
STATE_RTOL = 1e-3


def to_np(t):
    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy().astype(np.float64)
    return np.asarray(t, dtype=np.float64)


def assert_close(out, ref, atol=BF16_ATOL, rtol=BF16_RTOL, what="output"):
    o, r = to_np(out), to_np(ref)
    assert o.shape == r.shape, f"{what}: shape {o.shape} != {r.shape}"
    assert np.isfinite(o).all(), f"{what}: non-finite values"
    err = np.abs(o - r)
    bad = err > atol + rtol * np.abs(r)
    assert not bad.any(), (f"{what}: {bad.sum()} / {bad.size} elements out of tolerance; "
                           f"max abs err {err.max():.3e} (atol {atol}, rtol {rtol})")


def state_rel_err(out, ref):
    """max over leading (seq, head) of ||out - ref||_F / ||ref||_F."""
    o, r = to_np(out), to_np(ref)
    o = o.reshape(-1, o.shape[-2] * o.shape[-1])
    r = r.reshape(-1, r.shape[-2] * r.shape[-1])
    num = np.linalg.norm(o - r, axis=1)
    den = np.maximum(np.linalg.norm(r, axis=1), 1e-12)
    return float((num / den).max())


def assert_state_close(out, ref, rtol=STATE_RTOL, what="state"):
    e = state_rel_err(out, ref)
    assert e <= rtol, f"{what}: relative error {e:.3e} > {rtol}"
