"""Stage-2 sparse attention over the selected blocks (the consumer of the path).

No reference function: the reference's get_block_table
(src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44) turns the top-k
block ids into per-(token, kv head) physical slot ids for an attention kernel
that lives outside the repository.  ``sparse_attention`` is that consumer with
the gather fused into its loader: it reads the top-k ids and the block table
directly, so the [T, Hk, K*64] slot tensor is never written.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .infllm_v2 import _as_i32


def sparse_attention(q, k_cache, v_cache, topk_idx, block_table, token_to_bs, token_pos_in_bs, seqlen_q,
                     softmax_scale=None, head_group=2, status=None):
    """Attention of each token over the positions of its selected 64-token blocks.

    q            [T, Hq, 128] (bf16; other float types are cast), Hq = 16 * Hk
    k_cache,
    v_cache      [n_slots, 128] bf16 rows (any shape whose last dim is 128, rows
                 contiguous): row ``head_group * physical_token + kv_head``, the slot
                 numbering of get_block_table
    topk_idx     int32 [Hk, T, K], K <= 64, -1 = no block
    block_table, token_to_bs, token_pos_in_bs, seqlen_q: as for get_block_table
    Returns bf16 [T, Hq, 128]:
        out[t, h] = sum_p softmax_p(q[t,h] . k_cache[slot_p] * scale) v_cache[slot_p]
    over the positions p = topk*64 + i that get_block_table marks valid (topk >= 0,
    p < seqlen_q[bs], p < token_pos_in_bs[t]), with slot_p = head_group *
    block_table[bs, min(p, L-1)] + kv_head; rows with no valid position are 0.
    ``status``: optional int32 CUDA tensor of one element, set nonzero when a bounded
    wait inside the kernel gave up (the output is then invalid)."""
    dev = _lib.require_cuda(q, k_cache, v_cache, topk_idx, block_table, token_to_bs, token_pos_in_bs,
                            seqlen_q)
    if q.dtype != torch.bfloat16:
        q = q.to(torch.bfloat16)
    if q.stride(-1) != 1:
        q = q.contiguous()
    T, Hq, D = q.shape
    kc = k_cache.to(torch.bfloat16).reshape(-1, D).contiguous()
    vc = v_cache.to(torch.bfloat16).reshape(-1, D).contiguous()
    if kc.shape[0] != vc.shape[0]:
        raise ValueError(f"k_cache and v_cache hold different slot counts: {kc.shape[0]} vs {vc.shape[0]}")
    tk = _as_i32(topk_idx)
    if tk.stride(-1) != 1:
        tk = tk.contiguous()
    Hk, Tt, K = tk.shape
    if Tt != T:
        raise ValueError(f"topk_idx covers {Tt} tokens, q {T}")
    bt = _as_i32(block_table)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    B, L = bt.shape
    tb = _as_i32(token_to_bs).contiguous()
    pos = _as_i32(token_pos_in_bs).contiguous()
    sq = _as_i32(seqlen_q).contiguous()
    if softmax_scale is None:
        softmax_scale = D ** (-0.5)
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    if T == 0:
        return out
    st = status.data_ptr() if status is not None else None
    with torch.cuda.device(dev):
        rc = _lib.load().unum_sparse_attn_blocks(
            q.data_ptr(), T, Hq, D, q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.shape[0], Hk,
            tk.data_ptr(), K, tk.stride(0), tk.stride(1), bt.data_ptr(), B, L, bt.stride(0), tb.data_ptr(),
            pos.data_ptr(), int(pos.numel() == 1), sq.data_ptr(), int(sq.numel() == 1), int(head_group),
            ctypes.c_float(float(softmax_scale)), out.data_ptr(), st, _lib.stream_ptr(dev))
    _lib.check(rc)
    return out
