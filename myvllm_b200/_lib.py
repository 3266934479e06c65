"""ctypes binding of ``libmyvllm_b200.so`` (declared in ``include/myvllm_b200.h``).

The library is the only compute path: there is no CPU or eager-PyTorch fallback.
If the shared object is missing, importing an op raises immediately; if a kernel
rejects its arguments, the op raises ``RuntimeError`` naming the op and the reason.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MYVLLM_B200_LIB", os.path.join(_HERE, "_lib", "libmyvllm_b200.so"))

MAX_DIMS = 6
MVB_F32, MVB_BF16, MVB_F16, MVB_I32 = 0, 1, 2, 3
MVB_OK, MVB_ERR_ARG, MVB_ERR_UNSUPPORTED, MVB_ERR_CUDA = 0, 1, 2, 3
_DTYPES = {torch.float32: MVB_F32, torch.bfloat16: MVB_BF16, torch.float16: MVB_F16, torch.int32: MVB_I32}
_STATUS = {1: "bad argument", 2: "unsupported", 3: "CUDA error"}


class MvbTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


AR_MAX_RANKS = 8


class MvbAllReducePeers(ctypes.Structure):
    """Mirror of ``mvb_allreduce_peers`` (include/myvllm_b200.h)."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("bufs", ctypes.c_void_p * AR_MAX_RANKS),
        ("buf_bytes", ctypes.c_size_t),
    ]


_T = ctypes.POINTER(MvbTensor)
_P = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/myvllm_b200.h
SIGNATURES = {
    "mvb_version": (ctypes.c_int, []),
    "mvb_last_error": (ctypes.c_char_p, []),
    "mvb_causal_conv1d_fn": (ctypes.c_int, [_T, _T, _T, _T, _T, _T, ctypes.c_int, _P]),
    "mvb_causal_conv1d_update": (ctypes.c_int, [_T, _T, _T, _T, _T, ctypes.c_int, _P]),
    "mvb_chunk_gated_delta_rule_workspace_size": (ctypes.c_size_t, []),
    "mvb_chunk_gated_delta_rule": (ctypes.c_int, [_T, _T, _T, _T, _T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int,
                                                  _P, ctypes.c_size_t, _P]),
    "mvb_fused_recurrent_gdn": (ctypes.c_int, [_T, _T, _T, _T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int, _P]),
    "mvb_chunk_gated_delta_rule_gated": (ctypes.c_int, [_T] * 11 + [ctypes.c_float, ctypes.c_int, _P, ctypes.c_size_t,
                                                                    _P]),
    "mvb_fused_recurrent_gdn_gated": (ctypes.c_int, [_T] * 10 + [ctypes.c_float, ctypes.c_int, _P]),
    "mvb_gated_deltanet_decode_workspace_sizes": (ctypes.c_int, [ctypes.c_int64] * 3 +
                                                  [ctypes.POINTER(ctypes.c_size_t)] * 2),
    "mvb_gated_deltanet_decode": (ctypes.c_int, [_T] * 12 + [ctypes.c_float, ctypes.c_float, _T, _P, ctypes.c_size_t,
                                                             _P, ctypes.c_size_t, _P]),
    "mvb_gated_deltanet_prefill": (ctypes.c_int, [_T] * 12 + [ctypes.c_float, _T, ctypes.c_float, _P, ctypes.c_size_t,
                                                              _P]),
    "mvb_flash_attention_prefill": (ctypes.c_int, [_T, _T, _T, _T, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, _T, _P]),
    "mvb_paged_attention_decode_workspace_size": (ctypes.c_size_t, [ctypes.c_int64] * 4),
    "mvb_paged_attention_decode": (ctypes.c_int, [_T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int, ctypes.c_int64,
                                                  _T, _P, ctypes.c_size_t, _P]),
    "mvb_paged_attention_decode_gated": (ctypes.c_int, [_T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int,
                                                        ctypes.c_int64, _T, _T, _P, ctypes.c_size_t, _P]),
    "mvb_paged_attention_decode_noalloc": (ctypes.c_int, [_T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int,
                                                          ctypes.c_int64, _T, _P]),
    "mvb_paged_attention_decode_part_workspace_size": (ctypes.c_size_t, [ctypes.c_int64] * 4 + [ctypes.c_int]),
    "mvb_paged_attention_decode_part": (ctypes.c_int, [_T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int,
                                                       ctypes.c_int64, ctypes.c_int, ctypes.c_int, _T, _T, _P,
                                                       ctypes.c_size_t, _P]),
    "mvb_attention_merge_parts": (ctypes.c_int, [_T, _T, ctypes.c_int, _T, _T, _P]),
    "mvb_paged_attention_prefill": (ctypes.c_int, [_T, _T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_int, _T, _P]),
    "mvb_store_kvcache": (ctypes.c_int, [_T, _T, _T, _T, _T, _P]),
    "mvb_rmsnorm_gated": (ctypes.c_int, [_T, _T, _T, ctypes.c_float, _T, _P]),
    "mvb_rmsnorm": (ctypes.c_int, [_T, _T, _T, ctypes.c_float, ctypes.c_int, _T, _P]),
    "mvb_rmsnorm_rope": (ctypes.c_int, [_T, _T, ctypes.c_float, ctypes.c_int, _T, _T, _T, _P]),
    "mvb_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "mvb_last_path": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]),
    "mvb_allreduce_buffer_bytes": (ctypes.c_size_t, [ctypes.c_size_t]),
    "mvb_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "mvb_ipc_free": (ctypes.c_int, [_P]),
    "mvb_ipc_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mvb_ipc_close": (ctypes.c_int, [_P]),
    "mvb_allreduce_oneshot": (ctypes.c_int, [ctypes.POINTER(MvbAllReducePeers), _T, _T, _P]),
    "mvb_linear_allreduce_buffer_bytes": (ctypes.c_size_t, []),
    "mvb_linear_allreduce": (ctypes.c_int, [ctypes.POINTER(MvbAllReducePeers), _T, _T, _T, _P]),
    "mvb_selftest_umma": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, _P]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads the library once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"myvllm_b200: {LIB_PATH} is missing; build it with `python -m myvllm_b200.build` "
                    "(there is no fallback implementation)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def desc(t: torch.Tensor) -> MvbTensor:
    """Descriptor of a device tensor (shape/strides in elements)."""
    if t.dim() > MAX_DIMS:
        raise ValueError(f"myvllm_b200: tensors of rank > {MAX_DIMS} are not supported")
    d = MvbTensor()
    d.data = t.data_ptr() if t.numel() > 0 else None
    try:
        d.dtype = _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"myvllm_b200: unsupported dtype {t.dtype}") from None
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = s
        d.stride[i] = st
    return d


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(op: str, *tensors: torch.Tensor) -> None:
    dev = None
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(f"{op}: all tensors must be CUDA tensors (this library has no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{op}: tensors are on different devices ({dev} vs {t.device})")


def check(op: str, status: int) -> None:
    if status != 0:
        msg = load().mvb_last_error().decode(errors="replace")
        raise RuntimeError(f"{op}: {_STATUS.get(status, status)}: {msg}")


n_calls = 0  # entry-point calls made through call(): each launches one or more kernels

# MYVLLM_B200_STRICT=1: after every entry point, wait for the device and raise if a kernel
# reported a device-side failure (a bounded wait that gave up).  Debugging aid: it
# synchronises after each op, so it is off by default and must stay off during graph capture.
STRICT = os.environ.get("MYVLLM_B200_STRICT", "0") not in ("", "0")


def call(op: str, fn_name: str, *args) -> None:
    """Calls an int-returning entry point and raises on a non-zero status."""
    global n_calls
    n_calls += 1
    lib = load()
    wrapped = [ctypes.byref(a) if isinstance(a, MvbTensor) else a for a in args]
    check(op, getattr(lib, fn_name)(*wrapped))
    if STRICT:
        status = device_status()
        if status != 0:
            raise RuntimeError(f"{op}: a kernel reported device status {status} (a bounded wait gave up; "
                               "the output is not valid)")


OP_CHUNK_GDN, OP_FA_PREFILL, OP_PAGED_PREFILL = 0, 1, 2
PATHS = {0: "none", 1: "tensor_core", 2: "serial", 3: "mma_sync"}


def last_path(op: int) -> tuple[str, str]:
    """(kernel family, fallback reason) of the last call of ``op`` on this thread:
    "tensor_core" is the tcgen05 kernel; "serial" / "mma_sync" are the fallbacks for layouts
    it does not take, with the reason."""
    reason = ctypes.c_char_p()
    code = load().mvb_last_path(int(op), ctypes.byref(reason))
    if code < 0:
        raise ValueError(f"last_path: unknown op {op}")
    return PATHS.get(code, str(code)), (reason.value or b"").decode(errors="replace")


_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int, tag: str = "scratch") -> torch.Tensor:
    """A per-device, per-op scratch buffer, grown on demand, zero-initialised and reused
    across calls (kernels on one stream are ordered, so reuse is safe there; ops running
    concurrently on different streams must not share one)."""
    key = (device.type, device.index, tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def chunk_gdn_workspace(device: torch.device) -> torch.Tensor:
    """Zero-initialised workspace of the chunked GDN entry points, sized for the balanced
    schedule (the chains spread evenly over the SMs, with state hand-offs between them)."""
    return workspace(device, int(load().mvb_chunk_gated_delta_rule_workspace_size()), tag="gdn_chunk")


def device_status() -> int:
    """Reads and clears the kernels' device error word (0 = ok); synchronises."""
    v = ctypes.c_int(0)
    check("device_status", load().mvb_device_status(ctypes.byref(v)))
    return v.value
