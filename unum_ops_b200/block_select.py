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

__all__ = ["topk_blocks", "block_select", "BlockSelectGraph", "block_select_rows", "block_select_streamed",
           "get_block_table_shard", "stage1_pooled"]


def stage1_pooled(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, max_context_len,
                  local_blocks, init_blocks, causal=True, softmax_scale=None, write_scores=True):
    """Stage 1 and block max-pooling in one kernel launch.

    Returns (scores, pooled), identical to
    ``infllmv2_attn_stage1(...)`` followed by ``max_pooling_1d_varlen(scores, cu_q, cu_k,
    zeros, 16 * W, max_context_len, local_blocks, init_blocks)`` with W the scores' row
    length.  Needs n_heads / n_kv_heads >= 16.  With ``write_scores=False`` the scores
    stay on chip (returned as None) and only the pooled blocks reach memory."""
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
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev) if write_scores else None
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    if T == 0 or W == 0 or NB == 0:
        return (scores.zero_() if scores is not None else None), pooled
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    with torch.cuda.device(dev):
        rc = L.unum_infllmv2_attn_stage1_pooled(
            q.data_ptr(), T, Hq, D, q.stride(0), q.stride(1), k.data_ptr(), Tk, Hk, k.stride(0),
            k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), B, float(softmax_scale), int(bool(causal)),
            scores.data_ptr() if scores is not None else None, W, pooled.data_ptr(), NB, int(init_blocks),
            int(local_blocks), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
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
                 softmax_scale=None, return_scores=True):
    """Run the whole block-selection path; returns (scores, pooled, topk_idx, slots).

    scores  bf16 [Hk, T, W]     stage-1 output, W = round_up(max_seqlen_k, 128)
    pooled  bf16 [Hk, T, NB]    NB = ceil(max_context_len / block_size)
    topk_idx int32 [Hk, T, topk]
    slots   int32 [T, Hk, topk*64]  physical slot ids (get_block_table_ref_torch semantics)
    The pooling step reads stage-1 rows with flat stride W, i.e. it is called
    with max_seqlen_q = stride * W (the glue the reference's caller applies).
    ``return_scores=False``: on the fused path (G >= 16, no cache) the stage-1 scores are
    never written to memory and None is returned in their place.
    """
    G = q.shape[1] // k_cmp.shape[1]
    if _decode_fusable(q, k_cmp, cu_seqlens_q, max_seqlen_k, max_context_len, topk, block_size, stride):
        return _block_select_decode(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table,
                                    token_to_bs, token_pos_in_bs, seqlen_q, max_context_len, cache_lens,
                                    causal, init_blocks, local_blocks, topk, softmax_scale, return_scores)
    if (cache_lens is None and block_size == 64 and stride == 16 and G >= 16 and k_cmp.shape[0] > 0
            and q.shape[-1] == 128):
        # one launch: the pooling is taken from the scores while they are on chip
        scores, pooled = stage1_pooled(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k,
                                       max_context_len, local_blocks, init_blocks, causal,
                                       softmax_scale, write_scores=return_scores)
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


def _decode_fusable(q, k_cmp, cu_seqlens_q, max_seqlen_k, max_context_len, topk, block_size, stride):
    """Whether block_select can run as one fused decode launch: one or a few query
    tokens per sequence, a head group of 16 or 32, each token's score row within tensor
    memory (W <= 128 * 512 / G) and every pooling window inside the row (4 * NB <= W)."""
    T, Hq, D = q.shape
    Hk = k_cmp.shape[1]
    n_seq = cu_seqlens_q.numel() - 1
    if Hk == 0 or Hq % Hk or Hq // Hk not in (16, 32) or D != 128 or block_size != 64 or stride != 16:
        return False
    if T == 0 or n_seq <= 0 or k_cmp.shape[0] == 0 or T > 4 * n_seq:
        return False
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / block_size)
    return 0 < NB and 4 * NB <= W <= 128 * 512 // (Hq // Hk) and 0 < topk <= 1024


def _block_select_decode(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table, token_to_bs,
                         token_pos_in_bs, seqlen_q, max_context_len, cache_lens, causal, init_blocks,
                         local_blocks, topk, softmax_scale, return_scores):
    """block_select as one launch (unum_block_select_decode): the decode kernel pools, selects
    and maps each token's row while it is on chip.  Same results as the four-kernel chain."""
    dev = _lib.require_cuda(q, k_cmp, cu_seqlens_q, cu_seqlens_k, block_table, token_to_bs,
                            token_pos_in_bs, seqlen_q)
    q = (q if q.stride(-1) == 1 else q.contiguous()).to(torch.bfloat16)
    k = (k_cmp if k_cmp.stride(-1) == 1 else k_cmp.contiguous()).to(torch.bfloat16)
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** (-0.5)
    T, Hq, D = q.shape
    Tk, Hk = k.shape[0], k.shape[1]
    B = cu_seqlens_q.numel() - 1
    cu_q, cu_k = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k)
    cache = _as_i32(cache_lens) if cache_lens is not None else None
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / 64)
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev) if return_scores else None
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(Hk, T, topk, dtype=torch.int32, device=dev)
    slots = torch.empty(T, Hk, topk * 64, dtype=torch.int32, device=dev)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    tb, pos, sq = _as_i32(token_to_bs), _as_i32(token_pos_in_bs), _as_i32(seqlen_q)
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    with torch.cuda.device(dev):
        rc = L.unum_block_select_decode(
            q.data_ptr(), T, Hq, D, q.stride(0), q.stride(1), k.data_ptr(), Tk, Hk, k.stride(0),
            k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), cache.data_ptr() if cache is not None else None,
            B, float(softmax_scale), int(bool(causal)), scores.data_ptr() if scores is not None else None,
            W, pooled.data_ptr(), NB, int(init_blocks), int(local_blocks), idx.data_ptr(), topk,
            slots.data_ptr(), bt.data_ptr(), bt.shape[0], bt.shape[1], bt.stride(0), tb.data_ptr(),
            pos.data_ptr(), int(pos.numel() == 1), sq.data_ptr(), int(sq.numel() == 1), 2,
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return scores, pooled, idx, slots


def get_block_table_shard(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q, *,
                          head_offset=0, head_group=2, out=None):
    """get_block_table for a shard of kv heads: ``topk_idx`` int32 [H, T, K] holds heads
    head_offset .. head_offset+H-1 of T tokens (the matching rows of token_to_bs and
    token_pos_in_bs); returns (or fills ``out``, a [T, H, K*64] int32 view whose token
    stride may be larger, e.g. a slice of the full [T, Hk, K*64] output) the values
    get_block_table_ref_torch gives those heads."""
    dev = _lib.require_cuda(topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q)
    H, T, K = topk_idx.shape
    if out is None:
        out = torch.empty(T, H, K * 64, dtype=torch.int32, device=dev)
    if out.shape != (T, H, K * 64) or out.stride(2) != 1 or out.stride(1) != K * 64:
        raise ValueError("out must be [T, H, K*64] with contiguous heads")
    if T == 0 or H == 0 or K == 0:
        return out
    tk = topk_idx if topk_idx.dtype == torch.int32 else topk_idx.to(torch.int32)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    tb, pos, sq = _as_i32(token_to_bs), _as_i32(token_pos_in_bs), _as_i32(seqlen_q)
    with torch.cuda.device(dev):
        rc = _lib.load().unum_get_block_table_shard(
            tk.data_ptr(), H, T, K, tk.stride(0), tk.stride(1), tk.stride(2), bt.data_ptr(),
            bt.shape[0], bt.shape[1], bt.stride(0), tb.data_ptr(), pos.data_ptr(), int(pos.numel() == 1),
            sq.data_ptr(), int(sq.numel() == 1), int(head_group), int(head_offset), out.stride(0),
            out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return out


def _rows_check(q, k, t_begin, t_end, T):
    G = q.shape[1] // k.shape[1]
    if G < 16 or q.shape[1] % k.shape[1]:
        raise NotImplementedError("row-window block selection needs n_heads / n_kv_heads >= 16")
    if q.shape[-1] != 128:
        raise NotImplementedError("head dim must be 128")
    if not (0 <= t_begin <= t_end <= T):
        raise ValueError(f"token window [{t_begin}, {t_end}) outside [0, {T})")


def block_select_rows(q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table, token_to_bs,
                      token_pos_in_bs, seqlen_q, *, t_begin, t_end, max_context_len, head_offset=0,
                      init_blocks=1, local_blocks=2, topk=64, causal=True, softmax_scale=None):
    """The block-selection path for query rows [t_begin, t_end) only: one shard of a long
    sequence (or of a varlen batch) for a rank that owns that token range.

    q [T, Hq, D] and k_cmp [Tk, Hk, D] may hold a subset of the model's heads (a kv-head
    shard: Hq/Hk >= 16 query heads per kv head); ``head_offset`` is the index of k_cmp's
    first kv head in the full model, used by the block-table values.  Only q rows of the
    window (rounded out to whole stage-1 tiles of 256/G tokens) are read.  Returns
    (scores, pooled, topk_idx, slots): scores [Hk, T, W] and pooled [Hk, T, NB] valid on
    the window rows, topk_idx [Hk, t_end-t_begin, topk], slots [t_end-t_begin, Hk, topk*64];
    equal to the same rows of ``block_select`` on the whole input."""
    dev = _lib.require_cuda(q, k_cmp, cu_seqlens_q, cu_seqlens_k, block_table)
    T = q.shape[0]
    _rows_check(q, k_cmp, t_begin, t_end, T)
    qq = (q if q.stride(-1) == 1 else q.contiguous()).to(torch.bfloat16)
    k = (k_cmp if k_cmp.stride(-1) == 1 else k_cmp.contiguous()).to(torch.bfloat16)
    Hq, D = qq.shape[1], qq.shape[2]
    Tk, Hk = k.shape[0], k.shape[1]
    if softmax_scale is None:
        softmax_scale = D ** (-0.5)
    B = cu_seqlens_q.numel() - 1
    cu_q, cu_k = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k)
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / 64)
    n = t_end - t_begin
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev)
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(Hk, n, topk, dtype=torch.int32, device=dev)
    slots = torch.empty(n, Hk, topk * 64, dtype=torch.int32, device=dev)
    if n == 0:
        return scores, pooled, idx, slots
    if Tk == 0 or W == 0:
        raise NotImplementedError("row-window block selection needs at least one compressed key")
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    with torch.cuda.device(dev):
        _lib.check(L.unum_infllmv2_attn_stage1_window(
            qq.data_ptr(), T, Hq, D, qq.stride(0), qq.stride(1), k.data_ptr(), Tk, Hk, k.stride(0),
            k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), B, float(softmax_scale), int(bool(causal)),
            scores.data_ptr(), W, pooled.data_ptr(), NB, int(init_blocks), int(local_blocks), t_begin,
            t_end, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)))
        for h in range(Hk):
            rows = pooled[h, t_begin:t_end]
            _lib.check(L.unum_topk_blocks(rows.data_ptr(), _lib.DTYPE_CODES[rows.dtype], n, NB, NB,
                                          int(topk), idx[h].data_ptr(), _lib.stream_ptr(dev)))
    pos = token_pos_in_bs if token_pos_in_bs.numel() == 1 else token_pos_in_bs[t_begin:t_end]
    get_block_table_shard(idx, block_table, token_to_bs[t_begin:t_end], pos, seqlen_q,
                          head_offset=head_offset, out=slots)
    return scores, pooled, idx, slots


def block_select_streamed(q_host, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table,
                          token_to_bs, token_pos_in_bs, seqlen_q, *, max_context_len,
                          init_blocks=1, local_blocks=2, topk=64, causal=True,
                          softmax_scale=None, chunk_tokens=16384, result_host=None, t_begin=0,
                          head_offset=0):
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

    Sharded use (one rank of several): ``q_host`` may hold only the rows
    [t_begin, t_begin + q_host.shape[0]) of the T = token_to_bs.numel() tokens, and
    q_host / k_cmp only a kv-head shard whose first kv head is ``head_offset`` of the
    model; topk_idx / slots / result_host then cover the window rows only, as in
    ``block_select_rows``.
    """
    dev = _lib.require_cuda(k_cmp, cu_seqlens_q, cu_seqlens_k, block_table)
    if q_host.device.type != "cpu":
        raise ValueError("q_host must be a host tensor (pinned for overlap)")
    n, Hq, D = q_host.shape
    T = token_to_bs.numel()
    t_end = t_begin + n
    k = (k_cmp if k_cmp.stride(-1) == 1 else k_cmp.contiguous()).to(torch.bfloat16)
    Tk, Hk = k.shape[0], k.shape[1]
    G = Hq // Hk
    if G < 16:
        raise NotImplementedError("block_select_streamed needs n_heads / n_kv_heads >= 16")
    if not (0 <= t_begin <= t_end <= T):
        raise ValueError(f"q_host rows [{t_begin}, {t_end}) outside the {T} tokens")
    if softmax_scale is None:
        softmax_scale = D ** (-0.5)
    B = cu_seqlens_q.numel() - 1
    cu_q, cu_k = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k)
    W = _round_multiple(int(max_seqlen_k), 128)
    NB = math.ceil(max_context_len / 64)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    scores = torch.empty(Hk, T, W, dtype=torch.bfloat16, device=dev)
    pooled = torch.empty(Hk, T, NB, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(Hk, n, topk, dtype=torch.int32, device=dev)
    slots = torch.empty(n, Hk, topk * 64, dtype=torch.int32, device=dev)
    if n == 0:
        return scores, pooled, idx, slots
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
    # chunk edges at multiples of `step` in token coordinates; last chunks first: with
    # causal masking the late tokens cost the most, so the cheapest chunk is the one
    # left exposed after the final copy
    cuts = [t_begin] + list(range((t_begin // step + 1) * step, t_end, step)) + [t_end]
    # the chunk processed last (the window's first) is split once more, so the compute and
    # the id copy-back left after the final host-to-device copy are short
    tail = max(step // 4 // 128 * 128, 128)
    if len(cuts) > 2 and cuts[1] - cuts[0] > 2 * tail:
        cuts.insert(1, cuts[0] + tail)
    bounds = [(cuts[i], cuts[i + 1]) for i in range(len(cuts) - 1)][::-1]
    copied = []
    # the query buffer may reuse memory that kernels of an earlier call on the compute
    # stream still read: the copies start only after the compute stream's earlier work
    copy.wait_stream(comp)
    q.record_stream(copy)
    with torch.cuda.stream(copy):
        for a, b in bounds:
            q[a:b].copy_(qsrc[a - t_begin:b - t_begin], non_blocking=True)
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
            ra, rb = a - t_begin, b - t_begin  # the chunk's rows in the outputs
            for h in range(Hk):
                rows = pooled[h, a:b]
                _lib.check(L.unum_topk_blocks(rows.data_ptr(), _lib.DTYPE_CODES[rows.dtype], b - a, NB,
                                              NB, int(topk), idx[h, ra:rb].data_ptr(), comp.cuda_stream))
            iv = idx[:, ra:rb]
            _lib.check(L.unum_get_block_table_shard(
                iv.data_ptr(), Hk, b - a, topk, iv.stride(0), iv.stride(1), iv.stride(2),
                bt.data_ptr(), bt.shape[0], bt.shape[1], bt.stride(0), tb[a:b].data_ptr(),
                pos.data_ptr() if pos.numel() == 1 else pos[a:b].data_ptr(), int(pos.numel() == 1),
                sq.data_ptr(), int(sq.numel() == 1), 2, int(head_offset), slots.stride(0),
                slots[ra:rb].data_ptr(), comp.cuda_stream))
            if result_host is not None:
                done = torch.cuda.Event()
                done.record(comp)
                back.wait_event(done)
                idx.record_stream(back)
                with torch.cuda.stream(back):
                    for h in range(Hk):
                        result_host[h, ra:rb].copy_(idx[h, ra:rb], non_blocking=True)
    if result_host is not None:
        comp.wait_stream(back)
    return scores, pooled, idx, slots


class BlockSelectGraph:
    """``block_select`` captured once in a CUDA graph and replayed per step.

    For decode loops, where one step's kernels run for tens of microseconds and the
    host-side launch work of the eager call would dominate.  The tensors passed here
    are the graph's static inputs: write the next step's values into them in place
    (same shapes, same devices) and call the object; it returns the same
    (scores, pooled, topk_idx, slots) tensors every time, overwritten by the replay.
    Keyword arguments are those of ``block_select``.  The capture runs the path
    three times on a side stream first (allocations, tensor-map setup), as CUDA
    graph capture requires.
    """

    def __init__(self, q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table, token_to_bs,
                 token_pos_in_bs, seqlen_q, **kwargs):
        dev = _lib.require_cuda(q, k_cmp, cu_seqlens_q, cu_seqlens_k, block_table, token_to_bs)
        args = (q, k_cmp, cu_seqlens_q, cu_seqlens_k, max_seqlen_k, block_table, token_to_bs,
                token_pos_in_bs, seqlen_q)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                block_select(*args, **kwargs)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = block_select(*args, **kwargs)

    def __call__(self):
        self.graph.replay()
        return self.outputs
