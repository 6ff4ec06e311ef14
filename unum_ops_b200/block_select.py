"""Top-k block selection and the full InfLLM-v2 block-selection pipeline.

The reference leaves top-k to its caller (torch.topk on the pooled scores);
``topk_blocks`` is the B200 kernel for that step, and ``block_select`` chains
the four steps the way the reference's caller does:
stage 1 -> max_pooling_1d_varlen -> top-k -> get_block_table.
"""
from __future__ import annotations

import torch

import math

from . import _lib
from .infllm_v2 import _as_i32, _round_multiple, _workspace, infllmv2_attn_stage1, max_pooling_1d_varlen
from .sparse_kernel_extension import get_block_table_ref_torch

__all__ = ["topk_blocks", "block_select", "stage1_pooled"]


def stage1_pooled(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, max_context_len,
                  local_blocks, init_blocks, causal=True, softmax_scale=None):
    """Stage 1 and block max-pooling in one kernel launch.

    Returns (scores, pooled), identical to
    ``infllmv2_attn_stage1(...)`` followed by ``max_pooling_1d_varlen(scores, cu_q, cu_k,
    zeros, 16 * W, max_context_len, local_blocks, init_blocks)`` with W the scores' row
    length.  Needs n_heads / n_kv_heads >= 16."""
    dev = _lib.require_cuda(q, k_cmp, cu_seqlens_q, cu_seqlens_k)
    q = (q if q.stride(-1) == 1 else q.contiguous()).to(torch.bfloat16)
    k = (k_cmp if k_cmp.stride(-1) == 1 else k_cmp.contiguous()).to(torch.bfloat16)
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** (-0.5)
    T, Hq, D = q.shape
    Tk, Hk = k.shape[0], k.shape[1]
    B = cu_seqlens_q.numel() - 1
    cu_q, cu_k = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k)
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / 64)
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev)
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    if T == 0 or W == 0 or NB == 0:
        return scores.zero_(), pooled
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    with torch.cuda.device(dev):
        rc = L.unum_infllmv2_attn_stage1_pooled(
            q.data_ptr(), T, Hq, D, q.stride(0), q.stride(1), k.data_ptr(), Tk, Hk, k.stride(0),
            k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), B, float(softmax_scale), int(bool(causal)),
            scores.data_ptr(), W, pooled.data_ptr(), NB, int(init_blocks), int(local_blocks),
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return scores, pooled


def topk_blocks(scores: torch.Tensor, topk: int) -> torch.Tensor:
    """Top-``topk`` blocks per row of ``scores`` [..., NB] -> int32 [..., topk].

    Candidates are entries that are neither -inf nor NaN, ranked by (score
    desc, block index asc); the winners are returned in ascending block order,
    padded with -1."""
    dev = _lib.require_cuda(scores)
    if scores.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported score dtype {scores.dtype}")
    NB = scores.shape[-1]
    x = scores if scores.stride(-1) == 1 else scores.contiguous()
    x2 = x.reshape(-1, NB) if x.dim() != 2 else x
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    out = torch.empty(*scores.shape[:-1], topk, dtype=torch.int32, device=dev)
    if out.numel() == 0:
        return out
    with torch.cuda.device(dev):
        rc = _lib.load().unum_topk_blocks(x2.data_ptr(), _lib.DTYPE_CODES[x2.dtype], rows, NB,
                                          x2.stride(0) if rows > 1 else NB, int(topk),
                                          out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return out


def block_select(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table, token_to_bs,
                 token_pos_in_bs, seqlen_q, *, max_context_len, cache_lens=None, causal=True,
                 init_blocks=1, local_blocks=2, topk=64, block_size=64, stride=16,
                 softmax_scale=None):
    """Run the whole block-selection path; returns (scores, pooled, topk_idx, slots).

    scores  bf16 [Hk, T, W]     stage-1 output, W = round_up(max_seqlen_k, 128)
    pooled  bf16 [Hk, T, NB]    NB = ceil(max_context_len / block_size)
    topk_idx int32 [Hk, T, topk]
    slots   int32 [T, Hk, topk*64]  physical slot ids (get_block_table_ref_torch semantics)
    The pooling step reads stage-1 rows with flat stride W, i.e. it is called
    with max_seqlen_q = stride * W (the glue the reference's caller applies).
    """
    G = q.shape[1] // k_cmp.shape[1]
    if (cache_lens is None and block_size == 64 and stride == 16 and G >= 16 and k_cmp.shape[0] > 0
            and q.shape[-1] == 128):
        # one launch: the pooling is taken from the scores while they are on chip
        scores, pooled = stage1_pooled(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k,
                                       max_context_len, local_blocks, init_blocks, causal,
                                       softmax_scale)
    else:
        scores = infllmv2_attn_stage1(q, k_cmp, None, cu_seqlens_q, cu_seqlens_k,
                                      max_seqlen_k=max_seqlen_k, causal=causal,
                                      softmax_scale=softmax_scale)
        W = scores.shape[-1]
        if cache_lens is None:
            cache_lens = torch.zeros(cu_seqlens_q.numel() - 1, dtype=torch.int32, device=q.device)
        pooled = max_pooling_1d_varlen(scores, cu_seqlens_q, cu_seqlens_k, cache_lens, stride * W,
                                       max_context_len, local_blocks, init_blocks, block_size,
                                       stride)
    idx = topk_blocks(pooled, topk)
    slots = get_block_table_ref_torch(idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q)
    return scores, pooled, idx, slots
