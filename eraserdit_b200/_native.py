"""ctypes binding of ``liberaserdit_b200.so`` (declared in ``include/eraserdit_b200.h``).

The library is the only compute path: if it is missing or cannot be loaded,
every entry point raises.  There is no CPU or PyTorch fallback.

Tensors are passed as raw device pointers with element strides, on the
caller's current CUDA stream, in the style of the reference's mask-STA ctypes
binding (``layers/attention/backends/mask_sta.py:108-131``): a nonzero return
code raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "liberaserdit_b200.so"
ABI_VERSION = 5

_c_int, _c_i64, _c_float, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> argument types, in header order.
SIGNATURES = {
    "erd_abi_version": [],
    "erd_error_string": [_c_int],
    "erd_rope_axis_table": [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_float,
                            _c_float, _c_float, _c_float, _c_float, _c_float, _c_float, _vp, _vp],
    "erd_qk_norm_rope": [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp, _vp,
                         _c_float, _c_int, _vp, _vp, _c_i64, _c_i64, _vp, _c_int, _c_int, _c_int,
                         _c_int, _c_int, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int,
                         _c_i64, _vp],
    "erd_attn_fwd_bf16": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4 + [_vp, _c_int, _c_float,
                                                                            _vp] + [_c_i64] * 4
                         + [_vp, _vp],
    "erd_attn_fwd_sparse_bf16": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                                + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 4
                                + [_vp, _c_int, _vp, _c_i64, _vp, _vp, _vp],
    "erd_gather_tokens": [_vp, _c_i64, _c_i64, _c_int, _vp, _c_i64, _c_i64, _vp, _c_int, _c_int,
                          _c_int, _vp],
    "erd_qk_norm_rope_peer": [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp, _vp,
                              _c_float, _c_int, _vp, _vp, _c_i64, _c_i64, _vp, _c_int, _c_int,
                              _c_int, _c_int, _c_int, _vp, _vp, _c_int, _c_i64, _c_i64, _c_i64,
                              _c_i64, _c_i64, _c_int, _vp],
    "erd_attn_fwd_bf16_peer": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                              + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 3 + [_vp, _vp],
    "erd_attn_fwd_sparse_bf16_peer": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                                     + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 3
                                     + [_vp, _c_int, _vp, _c_i64, _vp, _vp],
    "erd_attn_fwd_fp8_peer": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                             + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 3
                             + [_vp, ctypes.c_size_t, _vp, _vp],
    "erd_quantize_e4m3": [_vp, _vp, _c_i64, _c_float, _vp],
    "erd_linear_bf16": [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _c_i64, _c_int, _c_int, _c_int, _vp,
                        _vp],
    "erd_linear_bf16_scatter": [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _c_i64, _c_int, _c_int,
                                _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                _vp, _vp],
    "erd_linear_fp8": [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _c_i64, _c_int, _c_int, _c_int,
                       _vp, _vp],
    "erd_attn_fwd_cross_bf16": [_vp, _vp, _vp] + [_c_i64] * 9 + [_c_int] * 4
                               + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 3 + [_vp, _vp],
    "erd_ring_state_bytes": [_c_int, _c_int, _c_int, _c_int],
    "erd_attn_fwd_ring_bf16": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                              + [_vp, _c_int, _c_int, _vp, _c_int, _c_float, _vp] + [_c_i64] * 4
                              + [_vp, _vp, ctypes.c_size_t, _c_int, _vp, _vp],
    "erd_peer_alloc": [ctypes.c_size_t, ctypes.POINTER(_vp)],
    "erd_peer_free": [_vp],
    "erd_peer_ipc_handle": [_vp, _vp],
    "erd_peer_ipc_open": [_vp, ctypes.POINTER(_vp)],
    "erd_peer_ipc_close": [_vp],
    "erd_peer_signal": [_vp, _c_int, ctypes.c_int32, _vp],
    "erd_peer_wait": [_vp, _c_int, ctypes.c_int32, _c_i64, _vp, _vp],
    "erd_attn_fp8_workspace_bytes": [_c_int, _c_int, _c_int, _c_int],
    "erd_attn_fwd_fp8": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4 + [_vp, _c_int, _c_float,
                                                                           _vp] + [_c_i64] * 4
                        + [_vp, ctypes.c_size_t, _vp, _vp],
    "erd_attn_fwd_fp8_static_scratch": [_vp, _vp, _vp] + [_c_i64] * 12 + [_c_int] * 4
                                       + [_vp, _c_int, _c_float, _vp] + [_c_i64] * 4 + [_vp, _vp],
}
RESTYPES = {"erd_error_string": ctypes.c_char_p, "erd_attn_fp8_workspace_bytes": ctypes.c_size_t,
            "erd_ring_state_bytes": ctypes.c_size_t}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is absent or of another ABI version."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("ERASERDIT_B200_LIBRARY", LIBRARY_PATH))
        if not path.exists():
            raise RuntimeError(
                f"eraserdit_b200 CUDA library not found at {path}; build it with "
                "`python -m eraserdit_b200.csrc.build` (no fallback path exists)")
        lib = ctypes.CDLL(str(path))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        if lib.erd_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"eraserdit_b200 ABI mismatch: library {lib.erd_abi_version()}, "
                f"binding {ABI_VERSION}")
        _lib = lib
    return _lib


def check(code: int, what: str) -> None:
    if code != 0:
        message = load().erd_error_string(code).decode()
        raise RuntimeError(f"{what} failed ({code}): {message}")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels set when a bounded wait gives up."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _status.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _status[index] = word
    return word


def read_status(device: torch.device, reset: bool = True) -> int:
    """Synchronise and return the device status bits (0 = no kernel timed out)."""
    word = status_word(device)
    value = int(word.item())
    if reset and value:
        word.zero_()
    return value


_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> int:
    """Address of a caller-owned, 1024-byte aligned device buffer of at least
    ``nbytes`` for work enqueued on the current stream of ``device`` (one buffer
    per stream, grown on demand, reused in that stream's order)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, stream_handle(torch.device("cuda", index)))
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes + 1024:
        buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=torch.device("cuda", index))
        _workspaces[key] = buf
    base = buf.data_ptr()
    return (base + 1023) // 1024 * 1024


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
