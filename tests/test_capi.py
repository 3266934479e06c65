"""CPU tests of the C ABI boundary: the library loads, exports every entry point that
include/myvllm_b200.h declares, and rejects malformed arguments with the documented
status codes before touching the device (no kernel runs here)."""

import ctypes
import os
import re

import pytest

from myvllm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "myvllm_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(mvb_\w+)\s*\(", text, re.M)))


def test_header_declares_the_op_surface():
    syms = declared_symbols()
    for name in ["mvb_causal_conv1d_fn", "mvb_causal_conv1d_update", "mvb_chunk_gated_delta_rule",
                 "mvb_fused_recurrent_gdn", "mvb_flash_attention_prefill", "mvb_paged_attention_decode",
                 "mvb_paged_attention_prefill", "mvb_store_kvcache"]:
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_allreduce_rejects_bad_arguments():
    """The one-shot all-reduce validates its peers and tensors before touching a device."""
    lib = _lib.load()
    assert lib.mvb_allreduce_buffer_bytes(1 << 20) == 8192 + 2 * (1 << 20)
    x = _fake([128, 2048])
    y = _fake([128, 2048], ptr=0x200000)
    peers = _lib.MvbAllReducePeers()
    peers.world, peers.rank, peers.buf_bytes = 1, 0, lib.mvb_allreduce_buffer_bytes(1 << 20)
    peers.bufs[0] = 0x10000
    call = lambda: lib.mvb_allreduce_oneshot(ctypes.byref(peers), ctypes.byref(x), ctypes.byref(y), None)  # noqa: E731
    assert call() == _lib.MVB_ERR_ARG  # one rank
    peers.world = 2
    assert call() == _lib.MVB_ERR_ARG  # rank 1's buffer is NULL
    peers.bufs[1] = 0x20000
    peers.buf_bytes = lib.mvb_allreduce_buffer_bytes(4096)
    assert call() == _lib.MVB_ERR_ARG  # 512 KiB message, 4 KiB slots
    peers.buf_bytes = lib.mvb_allreduce_buffer_bytes(1 << 20)
    z = _fake([128, 2048], dtype=_lib.MVB_F32, ptr=0x200000)
    assert lib.mvb_allreduce_oneshot(ctypes.byref(peers), ctypes.byref(z), ctypes.byref(z), None) == \
        _lib.MVB_ERR_UNSUPPORTED  # fp32


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.mvb_version() >= 100
    assert isinstance(lib.mvb_last_error(), bytes)


def _fake(shape, dtype=_lib.MVB_BF16, stride=None, ptr=0x1000):
    t = _lib.MvbTensor()
    t.data = ptr
    t.dtype = dtype
    t.ndim = len(shape)
    if stride is None:
        stride, acc = [], 1
        for s in reversed(shape):
            stride.insert(0, acc)
            acc *= s
    for i, (s, st) in enumerate(zip(shape, stride)):
        t.shape[i] = s
        t.stride[i] = st
    return t


def _status(fn, *args):
    lib = _lib.load()
    wrapped = [ctypes.byref(a) if isinstance(a, _lib.MvbTensor) else a for a in args]
    rc = getattr(lib, fn)(*wrapped)
    return rc, lib.mvb_last_error().decode()


def test_rejects_wrong_rank():
    q = _fake([4, 2, 128])
    bad = _fake([4, 2])
    rc, msg = _status("mvb_fused_recurrent_gdn", q, q, bad, _fake([4, 2], _lib.MVB_F32),
                      _fake([4, 2], _lib.MVB_F32), _fake([4, 2, 128, 128], _lib.MVB_F32),
                      _fake([4], _lib.MVB_I32), _fake([4, 2, 128]), ctypes.c_float(0.0), 0, None)
    assert rc == 1 and "v must have 3 dims" in msg


def test_rejects_head_mismatch_and_state_dtype():
    q = _fake([4, 3, 128])
    v = _fake([4, 4, 128])
    g = _fake([4, 4], _lib.MVB_F32)
    st = _fake([4, 4, 128, 128], _lib.MVB_F32)
    idx = _fake([4], _lib.MVB_I32)
    rc, msg = _status("mvb_fused_recurrent_gdn", q, q, v, g, g, st, idx, v, ctypes.c_float(0.0), 0, None)
    assert rc == 1 and "multiple of Hk" in msg
    q = _fake([4, 2, 128])
    st16 = _fake([4, 4, 128, 128], _lib.MVB_BF16)
    rc, msg = _status("mvb_fused_recurrent_gdn", q, q, v, g, g, st16, idx, v, ctypes.c_float(0.0), 0, None)
    assert rc == 1 and "float32" in msg


def test_conv_width_out_of_range_is_unsupported():
    x = _fake([8, 64])
    w = _fake([64, 9])
    st = _fake([2, 8, 64])
    rc, msg = _status("mvb_causal_conv1d_update", x, w, st, _fake([8], _lib.MVB_I32), x, 1, None)
    assert rc == 2 and "width" in msg


def test_attention_rejects_fp32_and_bad_gqa():
    q = _fake([16, 16, 256], _lib.MVB_F32)
    k = _fake([16, 2, 256], _lib.MVB_F32)
    cu = _fake([2], _lib.MVB_I32)
    rc, msg = _status("mvb_flash_attention_prefill", q, k, k, cu, ctypes.c_float(0.0625), 16, 2, 256, 256, 1, q, None)
    assert rc == 2 and "bf16" in msg
    q = _fake([16, 6, 256])
    k = _fake([16, 4, 256])
    rc, msg = _status("mvb_flash_attention_prefill", q, k, k, cu, ctypes.c_float(0.0625), 6, 4, 256, 256, 1, q, None)
    assert rc == 1


def test_null_data_pointer_is_rejected():
    x = _fake([8, 64], ptr=None)
    w = _fake([64, 4])
    st = _fake([2, 3, 64])
    rc, msg = _status("mvb_causal_conv1d_update", x, w, st, _fake([8], _lib.MVB_I32), _fake([8, 64]), 1, None)
    assert rc == 1 and "no data pointer" in msg


def test_decode_workspace_size_policy():
    lib = _lib.load()
    assert lib.mvb_paged_attention_decode_workspace_size(0, 2, 256, 1024) == 0
    small = lib.mvb_paged_attention_decode_workspace_size(128, 2, 256, 512)
    big = lib.mvb_paged_attention_decode_workspace_size(128, 2, 256, 32768)
    assert big >= small
    # split results [S, Hkv, splits, 16, Dv + 1] fp32, then the largest-first order table
    # int32 [2 S + 2] padded to 16 bytes
    order = (2 * 128 + 2) * 4 // 16 * 16 + (16 if (2 * 128 + 2) * 4 % 16 else 0)
    assert (big - order) % (128 * 2 * 16 * 257 * 4) == 0
    assert lib.mvb_paged_attention_decode_part_workspace_size(128, 1, 256, 32768, 2) > 0


def test_ops_refuse_cpu_tensors():
    import torch

    from myvllm_b200.ops.causal_conv1d import causal_conv1d_update

    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        causal_conv1d_update(x, torch.zeros(8, 4), torch.zeros(2, 3, 8, dtype=torch.bfloat16),
                             torch.zeros(2, dtype=torch.int32))


def test_last_path_query():
    """mvb_last_path answers without a GPU: no call yet on this thread -> "none"; an op id
    outside the table is rejected."""
    import threading

    res = {}

    def fresh_thread():  # the record is per host thread, so a new thread starts empty
        res["paths"] = [_lib.last_path(op) for op in (_lib.OP_CHUNK_GDN, _lib.OP_FA_PREFILL, _lib.OP_PAGED_PREFILL)]

    t = threading.Thread(target=fresh_thread)
    t.start()
    t.join()
    assert res["paths"] == [("none", "")] * 3
    with pytest.raises(ValueError):
        _lib.last_path(7)
