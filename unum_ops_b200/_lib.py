"""ctypes binding of the C ABI in include/unum_ops_b200.h.

The product path has no CPU fallback: when the CUDA library is missing or a
tensor is not on a CUDA device, the wrappers raise.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _build

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_p = ctypes.c_void_p

UNUM_OK = 0
UNUM_ERR_INVALID = -1
UNUM_ERR_UNSUPPORTED = -2
UNUM_ERR_CUDA = -3
UNUM_ERR_WORKSPACE = -4

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

# symbol -> (argtypes, restype); the complete list of entry points of the header
SIGNATURES = {
    "unum_last_error": ([], ctypes.c_char_p),
    "unum_abi_version": ([], _int),
    "unum_get_block_table": ([_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p,
                              _int, _p, _int, _i32, _p, _p], _int),
    "unum_get_block_table_shard": ([_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p,
                                    _p, _int, _p, _int, _i32, _i64, _i64, _p, _p], _int),
    "unum_max_pooling_1d_varlen": ([_p, _int, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _p, _p], _int),
    "unum_topk_blocks": ([_p, _int, _i64, _i64, _i64, _i64, _p, _p], _int),
    "unum_topk_blocks_to_peers": ([_p, _int, _i64, _i64, _i64, _i64, _p, _p, _i32, _i64, _p], _int),
    "unum_peer_signal_wait": ([_p, _i32, _i32, _i32, _p, _p], _int),
    "unum_compress_keys": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _p, _p],
                           _int),
    "unum_stage1_workspace_size": ([_i64], ctypes.c_size_t),
    "unum_infllmv2_attn_stage1": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p,
                                   _p, _i64, ctypes.c_float, _int, _p, _i64, _p, ctypes.c_size_t, _p],
                                  _int),
    "unum_stage1_status": ([_p, _p, ctypes.POINTER(_i32)], _int),
    "unum_stage1_noalloc_status": ([_p, ctypes.POINTER(_i32)], _int),
    "unum_infllmv2_attn_stage1_pooled": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                          _i64, _p, _p, _i64, ctypes.c_float, _int, _p, _i64, _p,
                                          _i64, _i64, _i64, _p, ctypes.c_size_t, _p], _int),
    "unum_block_select_decode": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _p,
                                  _i64, ctypes.c_float, _int, _p, _i64, _p, _i64, _i64, _i64, _p, _i64,
                                  _p, _p, _i64, _i64, _i64, _p, _p, _int, _p, _int, _i32, _p,
                                  ctypes.c_size_t, _p], _int),
    "unum_infllmv2_attn_stage1_window": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                          _i64, _p, _p, _i64, ctypes.c_float, _int, _p, _i64, _p,
                                          _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_size_t, _p],
                                         _int),
    "unum_sparse_attn_blocks": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                 _p, _i64, _i64, _i64, _p, _p, _int, _p, _int, _i32, ctypes.c_float, _p,
                                 _p, _p], _int),
    "unum_infllmv2_attn_stage1_noalloc": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                           _i64, _p, _p, _i64, ctypes.c_float, _int, _p, _i64, _p],
                                          _int),
}

_lib = None


def library_path() -> str:
    return _build.LIB


def load() -> ctypes.CDLL:
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"unum_ops_b200 CUDA library not found at {path}; build it with "
                "`python -m unum_ops_b200._build` (there is no CPU fallback)")
        L = ctypes.CDLL(path)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc == UNUM_OK:
        return
    msg = load().unum_last_error().decode(errors="replace")
    if rc == UNUM_ERR_INVALID:
        raise ValueError(msg)
    if rc == UNUM_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"unum_ops_b200 error {rc}: {msg}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            continue
        if t.device.type != "cuda":
            raise ValueError(f"unum_ops_b200 runs on CUDA tensors only; got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def ptr(t) -> int:
    return t.data_ptr() if t is not None else 0
