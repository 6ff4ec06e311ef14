"""CPU oracle for the InfLLM-v2 block-selection path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this package, and only as the
checker (or as the timed CPU baseline).  The product package ``unum_ops_b200``
never imports it and has no CPU fallback.

The arithmetic lives in ``oracle.c`` (plain C, pthreads), a restatement of the
reference's torch/Triton semantics with file:line citations.  This module is a
numpy front end over it through ctypes.  ``build()`` compiles the shared
library with gcc.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_ptr = ctypes.c_void_p


def build(force: bool = False) -> str:
    """Compile liboracle.so from oracle.c (gcc, via the Makefile)."""
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_stage1.argtypes = [_ptr, _ptr, _i64, _i64, _i64, _i64, _ptr, _ptr, _i64,
                                    ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _ptr]
        L.oracle_stage1.restype = None
        L.oracle_stage1_visible.argtypes = [_i64, _i64, _i64, ctypes.c_int]
        L.oracle_stage1_visible.restype = _i64
        L.oracle_max_pool.argtypes = [_ptr, _i64, _i64, _i64, _i64, _ptr, _ptr, _ptr, _i64,
                                      _i64, _i64, _i64, _i64, _i64, _ptr]
        L.oracle_max_pool.restype = None
        L.oracle_topk.argtypes = [_ptr, _i64, _i64, _i64, _ptr]
        L.oracle_topk.restype = None
        L.oracle_get_block_table.argtypes = [_ptr, _i64, _i64, _i64, _ptr, _i64, _i64, _ptr,
                                             _ptr, ctypes.c_int, _ptr, ctypes.c_int, _i32, _ptr]
        L.oracle_get_block_table.restype = None
        L.oracle_compress_keys.argtypes = [_ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, _ptr]
        L.oracle_compress_keys.restype = None
        L.oracle_sparse_attn.argtypes = [_ptr, _i64, _i64, _i64, _ptr, _ptr, _i64, _i64, _ptr, _i64,
                                         _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i32, ctypes.c_float, _ptr]
        L.oracle_sparse_attn.restype = None
        L.oracle_set_num_threads.argtypes = [ctypes.c_int]
        L.oracle_num_threads.restype = ctypes.c_int
        _lib = L
        L.oracle_set_num_threads(0)  # default: every online core
    return _lib


def set_num_threads(n: int) -> int:
    """Set the worker count (n <= 0: all online cores); returns the count in use."""
    L = lib()
    L.oracle_set_num_threads(int(n))
    return L.oracle_num_threads()


def num_threads() -> int:
    return lib().oracle_num_threads()


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def stage1_visible(local_q: int, q_len: int, k_len: int, causal: bool) -> int:
    return int(lib().oracle_stage1_visible(local_q, q_len, k_len, int(bool(causal))))


def stage1(q, k, cu_q, cu_k, causal, scale=None, out_stride=None, t_range=None):
    """Stage-1 scores, fp32 [Hk, T, out_stride].

    q: [T, Hq, D], k: [Tk, Hk, D] (float32 values; bf16 inputs widened).
    out_stride defaults to round-up-128 of the longest compressed sequence,
    like infllmv2_attn_stage1_triton_v2.py:199-225.  t_range=(a, b) computes
    only the rows of tokens a..b-1 and returns [Hk, b-a, out_stride].
    """
    q = _c(q, np.float32)
    k = _c(k, np.float32)
    cu_q = _c(cu_q, np.int32)
    cu_k = _c(cu_k, np.int32)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    n_seq = cu_q.shape[0] - 1
    if scale is None:
        scale = D ** -0.5
    if out_stride is None:
        mk = int(np.max(cu_k[1:] - cu_k[:-1])) if n_seq > 0 else 0
        out_stride = (mk + 127) // 128 * 128 if mk > 0 else 0
    a, b = (0, T) if t_range is None else (max(0, t_range[0]), min(T, t_range[1]))
    out = np.zeros((Hk, max(0, b - a), out_stride), np.float32)
    if out_stride == 0 or b <= a:
        return out
    lib().oracle_stage1(_p(q), _p(k), T, Hq, Hk, D, _p(cu_q), _p(cu_k), n_seq, float(scale),
                        int(bool(causal)), out_stride, a, b, _p(out))
    return out


def max_pool(inp, cu_q, cu_k, cache_lens, max_seqlen_q, max_context_len, local_blocks,
             init_blocks, block_size=64, stride=16):
    """max_pooling_1d_varlen semantics (max_pooling_1d_varlen.py:127-183), fp32 out."""
    inp = _c(inp, np.float32)
    cu_q = _c(cu_q, np.int32)
    cu_k = _c(cu_k, np.int32)
    cache_lens = _c(cache_lens, np.int32)
    H, T = inp.shape[0], inp.shape[1]
    NB = -(-int(max_context_len) // int(block_size))
    fs = int(max_seqlen_q) // int(stride)
    out = np.empty((H, T, NB), np.float32)
    if out.size:
        lib().oracle_max_pool(_p(inp), inp.size, H, T, fs, _p(cu_q), _p(cu_k), _p(cache_lens),
                              cu_q.shape[0] - 1, NB, int(block_size), int(stride),
                              int(init_blocks), int(local_blocks), _p(out))
    return out


def topk(scores, K):
    """Top-K block indices per row of scores [..., NB]: ascending, -1 padded."""
    s = _c(scores, np.float32)
    NB = s.shape[-1]
    rows = int(np.prod(s.shape[:-1]))
    out = np.empty(s.shape[:-1] + (K,), np.int32)
    if rows and K:
        lib().oracle_topk(_p(s), rows, NB, K, _p(out))
    return out


def get_block_table(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q,
                    head_group=2):
    """get_block_table_ref_torch semantics (get_table_torch.py:4-44): int32 [T, H, K*64]."""
    tk = _c(topk_idx, np.int32)
    bt = _c(block_table, np.int32)
    tb = _c(token_to_bs, np.int32)
    pb = _c(np.atleast_1d(token_pos_in_bs), np.int32)
    sq = _c(np.atleast_1d(seqlen_q), np.int32)
    H, T, K = tk.shape
    B, L = bt.shape
    out = np.empty((T, H, K * 64), np.int32)
    if out.size:
        lib().oracle_get_block_table(_p(tk), H, T, K, _p(bt), B, L, _p(tb), _p(pb),
                                     int(pb.size == 1), _p(sq), int(sq.size == 1),
                                     int(head_group), _p(out))
    return out


def sparse_attn(q, k_cache, v_cache, topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q,
                head_group=2, softmax_scale=None):
    """Stage-2 sparse attention over the selected blocks (oracle.c: oracle_sparse_attn):
    q [T, Hq, D], k_cache / v_cache [n_slots, D] (slot = head_group * physical token + kv
    head), topk_idx int32 [Hk, T, K]; returns float32 [T, Hq, D]."""
    qf = _c(q, np.float32)
    kc = _c(k_cache, np.float32).reshape(-1, qf.shape[-1])
    vc = _c(v_cache, np.float32).reshape(-1, qf.shape[-1])
    tk = _c(topk_idx, np.int32)
    bt = _c(block_table, np.int32)
    tb = _c(token_to_bs, np.int32)
    T, Hq, D = qf.shape
    pb = _c(np.broadcast_to(np.asarray(token_pos_in_bs, np.int32), (T,)), np.int32)
    sq = _c(np.atleast_1d(seqlen_q), np.int32)
    if sq.size == 1:
        sq = np.full(bt.shape[0], sq[0], np.int32)
    Hk, _, K = tk.shape
    B, L = bt.shape
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    out = np.empty((T, Hq, D), np.float32)
    if out.size:
        lib().oracle_sparse_attn(_p(qf), T, Hq, D, _p(kc), _p(vc), kc.shape[0], Hk, _p(tk), K, _p(bt), B,
                                 L, _p(tb), _p(pb), _p(sq), int(head_group), float(scale), _p(out))
    return out


def compressed_counts(seqlens, kernel=32, stride=16):
    """Compressed keys per sequence: (L - kernel) // stride + 1, 0 when L < kernel."""
    L = np.asarray(seqlens, np.int64)
    return np.where(L >= kernel, (L - kernel) // stride + 1, 0)


def compress_keys(k, cu_seqlens, kernel=32, stride=16):
    """Mean-pooled keys (the stage-1 input k_cmp): k [T, Hk, 128] (float values, bf16
    inputs widened) -> (bf16 bits uint16 [N, Hk, 128], cu_out int32 [B+1])."""
    k = _c(k, np.float32)
    cu = _c(cu_seqlens, np.int32)
    n = compressed_counts(np.diff(cu), kernel, stride)
    cu_out = np.concatenate([[0], np.cumsum(n)]).astype(np.int32)
    out = np.zeros((int(cu_out[-1]), k.shape[1], 128), np.uint16)
    if out.size:
        lib().oracle_compress_keys(_p(k), k.shape[1], _p(cu), _p(cu_out), len(cu) - 1, int(kernel),
                                   int(stride), _p(out))
    return out, cu_out
