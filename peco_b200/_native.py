"""Load libpeco_b200.so and declare its C ABI (include/peco_b200.h).

The library is built in-tree by ``peco_b200.build``; it is required.  There is
no fallback: if it cannot be loaded, or no CUDA device is present, every
entry point raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpeco_b200.so"
_LOCK = threading.Lock()
_LIB = None

P = ctypes.c_void_p
I = ctypes.c_int
LL = ctypes.c_longlong
F = ctypes.c_float

_SIGNATURES = {
    "peco_assign_tokens_to_centers": [P] * 5 + [I] * 5 + [P],
    "peco_recompute_cluster_centers": [P] * 6 + [I] * 4 + [P],
    "peco_recompute_cluster_centers_static": [P] * 6 + [I] * 4 + [P],
    "peco_recompute_cluster_centers_static_capacity": [],
    "peco_reorder_token_features": [P] * 3 + [I] * 5 + [P],
    "peco_sparse_attention": [P] * 8 + [I] * 7 + [P],
    "peco_sort_labels": [P] * 4 + [I] * 3 + [P],
    "peco_kmeans_fit": [P, LL, I, I, P, P, P, P, P, P, P, P, P, LL, I, I, P, P, P, P, P, P, P, P, I, I, I, P],
    "peco_select_cluster_connections": [P] * 5 + [I] * 4 + [F, I, P, P],
    "peco_select_text_partition": [P] * 7 + [I] * 4 + [F, I, I, I, P, P],
    "peco_base_offset": [I] + [P] * 7 + [I] * 6 + [P],
    "peco_quantize_gather": [P] * 12 + [I] * 7 + [P, I, I, P],
    "peco_attention_plan": [P] * 6 + [I] * 6 + [P],
    "peco_pack_key_blocks": [P] * 5 + [I] * 6 + [P],
    "peco_sparse_attention_restore": [P] * 5 + [I] * 6 + [P, I, P],
    "peco_prepare_qkv": [P, P, P, LL, I, P, P, P, LL, I, P, P, F, P, P, F, P, P, P, P, P, I, I, P],
    "peco_exchange_put": [P, P, P, P, LL, I, P, P, I, I, I, LL, P, P],
    "peco_exchange_wait": [P, I, I, LL, P],
    "peco_attention_workspace_stride": [I, I, I, I],
    "peco_key_block_rows": [I, I],
    "peco_kmeans_work_floats": [I, I, I],
    "peco_device_status": [P, I, P],
    "peco_error_string": [I],
    "peco_cluster_error_message": [I],
    "peco_attention_error_string": [I],
    "peco_library_version": [],
    "peco_launch_count": [],
}
_RESTYPES = {
    "peco_launch_count": ctypes.c_ulonglong,
    "peco_attention_workspace_stride": LL,
    "peco_key_block_rows": LL,
    "peco_kmeans_work_floats": LL,
    "peco_recompute_cluster_centers_static_capacity": LL,
    "peco_error_string": ctypes.c_char_p,
    "peco_cluster_error_message": ctypes.c_char_p,
    "peco_attention_error_string": ctypes.c_char_p,
}


def load(path: Path | str | None = None):
    """Load the shared library once per process (thread-safe) and return it."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    with _LOCK:
        if _LIB is not None and path is None:
            return _LIB
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(f"{p} is missing; build it with `python -m peco_b200.build`")
        lib = ctypes.CDLL(str(p))
        for name, args in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, I)
        if path is None:
            _LIB = lib
        return lib


def error_text(code: int) -> str:
    return load().peco_error_string(int(code)).decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    """Raise for a non-zero status returned by an entry point."""
    if status:
        raise RuntimeError(f"{what} failed: {error_text(status)} (status {status})")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device; raise otherwise (no CPU fallback)."""
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError("peco_b200 runs on CUDA devices only; got a tensor on " + str(dev))
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    return dev


def stream_of(device: torch.device, *tensors: torch.Tensor) -> P:
    """Current stream of ``device`` as a void*; keeps the tensors' memory alive
    until the stream has consumed them (ctypes bypasses the allocator's tracking)."""
    s = torch.cuda.current_stream(device)
    for t in tensors:
        if t is not None:
            t.record_stream(s)
    return P(s.cuda_stream)


def ptr(t: torch.Tensor | None) -> P:
    return P(t.data_ptr() if t is not None else 0)


def device_status(clear: bool = True, device=None) -> int:
    """Return (and optionally clear) the device status word (PECO_STATUS_* bits)."""
    lib = load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_uint(0)
    with torch.cuda.device(dev):
        check(lib.peco_device_status(ctypes.byref(out), int(clear), P(torch.cuda.current_stream(dev).cuda_stream)),
              "peco_device_status")
    return out.value


DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
