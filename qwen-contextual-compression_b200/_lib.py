"""ctypes binding of the C ABI in ``include/qcc_b200.h`` (``libqcc_b200.so``).

This module only turns tensors into pointers and status codes into
exceptions.  The library is loaded on first use; a missing library is an
error (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_PACKAGE_DIR = Path(__file__).resolve().parent
_LIBRARY_PATH = _PACKAGE_DIR / "libqcc_b200.so"

DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
INDEX_I32, INDEX_I64 = 0, 1
IDS_READY = 0x100  # OR-ed into the index type: the ids are not written by an earlier qcc launch on the stream


def mask_shift(s: int) -> int:
    """QCC_MASK_SHIFT(s): OR-ed into the index type, token b of the call reads bit s + b of the token mask."""
    return (s & 7) << 12

OK = 0
ERR_INVALID_ARGUMENT, ERR_SHAPE, ERR_DTYPE, ERR_ALIGNMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = range(1, 8)
DEV_ID_RANGE, DEV_TIMEOUT = 1, 2

TORCH_DTYPES = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16, torch.float32: DTYPE_F32}
INDEX_DTYPES = {torch.int32: INDEX_I32, torch.int64: INDEX_I64}

_c_void_p, _c_int, _c_int64, _c_size_t = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/qcc_b200.h
SIGNATURES = {
    "qcc_version": (_c_int, []),
    "qcc_status_string": (ctypes.c_char_p, [_c_int]),
    "qcc_last_cuda_error_string": (ctypes.c_char_p, []),
    "qcc_hidden_pad": (_c_int, [_c_int, _c_int]),
    "qcc_record_bytes": (_c_int64, [_c_int, _c_int]),
    "qcc_pack_records": (_c_int, [_c_void_p, _c_void_p, _c_int64, _c_void_p, _c_int64, _c_int64, _c_int64, _c_int,
                                  _c_int, _c_void_p, _c_void_p]),
    "qcc_decode_max_batch": (_c_int, [_c_int, _c_int]),
    "qcc_decode_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int]),
    "qcc_workspace_status_offset": (_c_size_t, []),
    "qcc_workspace_init": (_c_int, [_c_void_p, _c_size_t, _c_void_p]),
    "qcc_indexed_ffn_decode": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int64, _c_int, _c_void_p,
                                        _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p,
                                        _c_int64, _c_int, _c_void_p, _c_int64, _c_void_p, _c_int64, _c_void_p]),
    "qcc_indexed_ffn_decode_static": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int64, _c_int,
                                               _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int64,
                                               _c_int, _c_void_p, _c_int64, _c_void_p]),
    "qcc_select_topk": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_void_p, _c_int64, _c_void_p]),
    "qcc_activation_topk": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p,
                                     _c_int64, _c_void_p, _c_int64, _c_void_p]),
    "qcc_block_topk": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_int64, _c_void_p,
                                _c_int64, _c_void_p]),
    "qcc_tile_block_union": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                      _c_void_p, _c_void_p]),
    "qcc_ffn_activations": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int64, _c_int, _c_void_p,
                                     _c_void_p, _c_int64, _c_void_p, _c_int64, _c_void_p, _c_size_t, _c_void_p]),
    "qcc_indexed_ffn_down": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_void_p, _c_int64, _c_int,
                                      _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_size_t,
                                      _c_void_p, _c_int64, _c_int, _c_void_p, _c_int64, _c_void_p]),
    "qcc_build_union": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, ctypes.c_int32, ctypes.c_int32, _c_void_p,
                                 _c_void_p, _c_void_p, _c_void_p]),
    "qcc_cast_f32": (_c_int, [_c_void_p, _c_void_p, _c_int64, _c_int, _c_void_p]),
    "qcc_column_norms": (_c_int, [_c_void_p, _c_int64, _c_int64, _c_int64, _c_int, _c_void_p, _c_void_p]),
    "qcc_cache_resolve": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p,
                                   _c_void_p, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                   _c_void_p]),
    "qcc_gather_records": (_c_int, [_c_void_p, _c_int64, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p,
                                    _c_void_p]),
    "qcc_exchange_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "qcc_exchange_alloc": (_c_int, [_c_size_t, ctypes.POINTER(_c_void_p)]),
    "qcc_exchange_init": (_c_int, [_c_void_p, _c_size_t]),
    "qcc_exchange_free": (_c_int, [_c_void_p]),
    "qcc_ipc_handle": (_c_int, [_c_void_p, _c_void_p]),
    "qcc_ipc_open": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "qcc_ipc_close": (_c_int, [_c_void_p]),
    "qcc_exchange_set_wait_limit": (_c_int, [_c_void_p, ctypes.c_uint64]),
    "qcc_indexed_ffn_decode_allreduce": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int64, _c_int,
                                                  _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
                                                  _c_size_t, _c_void_p, _c_int64, _c_int, _c_void_p, _c_int64,
                                                  _c_int64, _c_int64, _c_void_p, _c_size_t, _c_int, _c_int,
                                                  _c_void_p]),
    "qcc_selector_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "qcc_selector_scores_topk": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                          _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                          _c_void_p, _c_void_p, ctypes.c_float, _c_void_p, _c_void_p, _c_int,
                                          _c_void_p, _c_int64, _c_void_p, _c_int64, _c_void_p, _c_size_t,
                                          _c_void_p]),
    "qcc_prefill_workspace_bytes": (_c_size_t, [_c_int64, _c_int]),
    "qcc_prefill_workspace_status_offset": (_c_size_t, []),
    "qcc_indexed_ffn_prefill": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int64, _c_int,
                                         _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p, _c_int64, _c_int,
                                         _c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class QCCError(RuntimeError):
    """A qcc_b200 C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def library_path() -> Path:
    return _LIBRARY_PATH


def library() -> ctypes.CDLL:
    """Load ``libqcc_b200.so`` once and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIBRARY_PATH.exists():
                raise RuntimeError(f"qcc_b200 CUDA library missing at {_LIBRARY_PATH}; build it with "
                                   "`python qwen-contextual-compression_b200/build.py` (there is no CPU fallback)")
            lib = ctypes.CDLL(str(_LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    lib = library()
    text = lib.qcc_status_string(status).decode()
    if status == ERR_CUDA:
        text += ": " + lib.qcc_last_cuda_error_string().decode()
    raise QCCError(status, f"{what} failed: {text}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return TORCH_DTYPES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected bfloat16, float16 or float32") from None


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device (the product path has no CPU fallback)."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError("qcc_b200 runs on CUDA tensors only (no CPU fallback); got a tensor on "
                               f"{t.device}")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError("all tensors must share a device")
    if device is None:
        raise RuntimeError("no CUDA tensor given")
    return device
