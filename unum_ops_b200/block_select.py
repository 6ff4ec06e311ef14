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

__all__ = ["topk_blocks", "block_select", "block_select_streamed", "stage1_pooled"]


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


def block_select_streamed(q_host, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table,
                          token_to_bs, token_pos_in_bs, seqlen_q, *, max_context_len,
                          init_blocks=1, local_blocks=2, topk=64, causal=True,
                          softmax_scale=None, chunk_tokens=16384, result_host=None):
    """The block-selection path for queries that live in (pinned) host memory.

    The queries are copied to the GPU chunk by chunk on a side stream while the
    previous chunk runs stage 1 (with fused pooling, restricted to the chunk's
    tokens), top-k and get_block_table on the current stream, so the
    host-to-device copy overlaps the compute.  Results equal ``block_select``'s.
    Everything except ``q_host`` (and ``result_host``) must already be on the
    GPU.  ``result_host``, if given (pinned int32 [Hk, T, topk]), receives the
    top-k block ids chunk by chunk, also overlapped.  Returns
    (scores, pooled, topk_idx, slots) on the GPU.  Needs n_heads / n_kv_heads >= 16
    and, for full overlap, chunks that are multiples of 256 / G tokens.
    """
    dev = _lib.require_cuda(k_cmp, cu_seqlens_q, cu_seqlens_k, block_table)
    if q_host.device.type != "cpu":
        raise ValueError("q_host must be a host tensor (pinned for overlap)")
    T, Hq, D = q_host.shape
    k = (k_cmp if k_cmp.stride(-1) == 1 else k_cmp.contiguous()).to(torch.bfloat16)
    Tk, Hk = k.shape[0], k.shape[1]
    G = Hq // Hk
    if G < 16:
        raise NotImplementedError("block_select_streamed needs n_heads / n_kv_heads >= 16")
    if softmax_scale is None:
        softmax_scale = D ** (-0.5)
    B = cu_seqlens_q.numel() - 1
    cu_q, cu_k = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k)
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / 64)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev)
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(Hk, T, topk, dtype=torch.int32, device=dev)
    slots = torch.empty(T, Hk, topk * 64, dtype=torch.int32, device=dev)
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)   # host -> device: query chunks
    back = torch.cuda.Stream(dev)   # device -> host: top-k ids (PCIe is full duplex)
    tb = _as_i32(token_to_bs)
    pos = _as_i32(token_pos_in_bs)
    sq = _as_i32(seqlen_q)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    qsrc = q_host if q_host.dtype == torch.bfloat16 else q_host.to(torch.bfloat16)
    step = max(int(chunk_tokens) // 128 * 128, 128)
    # last chunks first: with causal masking the late tokens cost the most, so the
    # cheapest chunk is the one left exposed after the final copy
    bounds = [(a, min(a + step, T)) for a in range(0, T, step)][::-1]
    copied = []
    # the query buffer may reuse memory that kernels of an earlier call on the compute
    # stream still read: the copies start only after the compute stream's earlier work
    copy.wait_stream(comp)
    q.record_stream(copy)
    with torch.cuda.stream(copy):
        for a, b in bounds:
            q[a:b].copy_(qsrc[a:b], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
            copied.append(ev)
    with torch.cuda.device(dev):
        for (a, b), ev in zip(bounds, copied):
            comp.wait_event(ev)
            rc = L.unum_infllmv2_attn_stage1_window(
                q.data_ptr(), T, Hq, D, q.stride(0), q.stride(1), k.data_ptr(), Tk, Hk,
                k.stride(0), k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), B,
                float(softmax_scale), int(bool(causal)), scores.data_ptr(), W, pooled.data_ptr(),
                NB, int(init_blocks), int(local_blocks), a, b, ws.data_ptr(), ws.numel(),
                comp.cuda_stream)
            _lib.check(rc)
            for h in range(Hk):
                rows = pooled[h, a:b]
                _lib.check(L.unum_topk_blocks(rows.data_ptr(), _lib.DTYPE_CODES[rows.dtype], b - a, NB,
                                              NB, int(topk), idx[h, a:b].data_ptr(), comp.cuda_stream))
            iv = idx[:, a:b]
            _lib.check(L.unum_get_block_table(
                iv.data_ptr(), Hk, b - a, topk, iv.stride(0), iv.stride(1), iv.stride(2),
                bt.data_ptr(), bt.shape[0], bt.shape[1], bt.stride(0), tb[a:b].data_ptr(),
                pos.data_ptr() if pos.numel() == 1 else pos[a:b].data_ptr(), int(pos.numel() == 1),
                sq.data_ptr(), int(sq.numel() == 1), 2, slots[a:b].data_ptr(), comp.cuda_stream))
            if result_host is not None:
                done = torch.cuda.Event()
                done.record(comp)
                back.wait_event(done)
                idx.record_stream(back)
                with torch.cuda.stream(back):
                    for h in range(Hk):
                        result_host[h, a:b].copy_(idx[h, a:b], non_blocking=True)
    if result_host is not None:
        comp.wait_stream(back)
    return scores, pooled, idx, slots
