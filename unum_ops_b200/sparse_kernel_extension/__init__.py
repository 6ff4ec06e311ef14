"""Logical top-k block ids -> physical paged-KV slot ids on B200.

Drop-in for ``unum_ops.sparse_kernel_extension`` (reference:
src/unum_ops/sparse_kernel_extension/__init__.py:1-21): the same six public
names and the signature (topk_idx, block_table, token_to_bs, token_pos_in_bs,
seqlen_q, topk=None), computed by the sm_100a kernel of libunum_ops_b200.so.

The torch reference multiplies the table entry by a constant 2
(get_table_torch.py:12) and the Triton kernels by H (get_table_triton.py:252);
each name keeps its own convention (identical for the 2-kv-head model).  Table
columns are clamped to L-1 like the torch reference (:35) for every name; the
Triton kernels read past the row there instead.
"""
from __future__ import annotations

import torch

from .. import _lib

__all__ = [
    "get_block_table_ref_torch",
    "get_block_table_ref_triton",
    "get_block_table_ref_triton_v2",
    "get_block_table_ref_triton_v3",
    "get_block_table_v2",
    "get_block_table_v3",
]

_BLOCK = 64  # kSparseBlockSize


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t


def _get_block_table(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q, head_group):
    dev = _lib.require_cuda(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q)
    H, T, K = topk_idx.shape
    B, L = block_table.shape
    out = torch.empty(T, H, K * _BLOCK, dtype=torch.int32, device=dev)
    if out.numel() == 0:
        return out
    tk = _i32(topk_idx)
    bt = _i32(block_table)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    tb = _i32(token_to_bs).contiguous()
    pos = _i32(token_pos_in_bs).contiguous()
    sq = _i32(seqlen_q).contiguous()
    with torch.cuda.device(dev):
        rc = _lib.load().unum_get_block_table(
            tk.data_ptr(), H, T, K, tk.stride(0), tk.stride(1), tk.stride(2), bt.data_ptr(), B, L,
            bt.stride(0), tb.data_ptr(), pos.data_ptr(), int(pos.numel() == 1), sq.data_ptr(),
            int(sq.numel() == 1), int(head_group), out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return out


def get_block_table_ref_torch(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q,
                              topk=None):
    """get_block_table_ref_torch semantics (get_table_torch.py:4-44): 2 * table + h."""
    return _get_block_table(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q, 2)


def get_block_table_ref_triton(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q,
                               topk=None):
    """get_block_table_ref_triton semantics (get_table_triton.py:218-262): H * table + h."""
    H, _, K = topk_idx.shape
    if topk is not None:
        assert topk == K, f"topk={topk} != K={K}"
    return _get_block_table(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q, H)


get_block_table_ref_triton_v2 = get_block_table_ref_triton
get_block_table_ref_triton_v3 = get_block_table_ref_triton
get_block_table_v2 = get_block_table_ref_triton
get_block_table_v3 = get_block_table_ref_triton
