"""CPU torch restatements of the reference's torch-level steps of the path.

TEST INFRASTRUCTURE ONLY (like the rest of ``oracle/``): ``bench.py`` times these
as the reference arm's top-k and get_block_table steps on the host cores, and
``tests/`` checks them against the C oracle.  The product package never imports
this module.

* ``get_block_table``: the reference's own torch implementation of the step,
  ``get_block_table_ref_torch`` (src/unum_ops/sparse_kernel_extension/
  get_table_torch.py:4-44), restated with the same tensor operations: slot ids
  pos = topk*64 + i, valid iff pos >= 0, pos < seqlen_q[bs] and
  pos < token_pos_in_bs[t]; value 2 * block_table[bs, clamp(pos, 0, L-1)] + h,
  else 0; output [T, H, K*64].
* ``topk``: what the reference's caller runs on the pooled block scores
  (torch.topk, then the ids sorted ascending with -1 for excluded blocks — the
  layout of the reference's block-table test fixtures, test/test_sparse_kernel.py:80-87).
"""
from __future__ import annotations

import torch

BLOCK = 64
HEAD_GROUP = 2


def get_block_table(topk_idx: torch.Tensor, block_table: torch.Tensor, token_to_bs: torch.Tensor,
                    token_pos_in_bs: torch.Tensor, seqlen_q: torch.Tensor) -> torch.Tensor:
    H, T, K = topk_idx.shape
    L = block_table.shape[1]
    slot = (topk_idx[..., None] * BLOCK + torch.arange(BLOCK, dtype=topk_idx.dtype)).reshape(H, T, K * BLOCK)
    bs = token_to_bs.long()
    limit = seqlen_q.reshape(-1).expand(T) if seqlen_q.numel() == 1 else seqlen_q[bs]
    pos_lim = token_pos_in_bs.reshape(-1).expand(T) if token_pos_in_bs.numel() == 1 else token_pos_in_bs
    ok = (slot >= 0) & (slot < limit[None, :, None]) & (slot < pos_lim[None, :, None])
    rows = block_table[bs]                                     # [T, L]
    phys = torch.gather(rows.expand(H, T, L), 2, slot.clamp(0, L - 1).long())
    val = HEAD_GROUP * phys + torch.arange(H, dtype=phys.dtype)[:, None, None]
    return torch.where(ok, val, torch.zeros((), dtype=val.dtype)).transpose(0, 1).contiguous()


def topk(pooled: torch.Tensor, k: int) -> torch.Tensor:
    """[H, T, NB] pooled scores -> [H, T, k] int32 block ids, ascending, -1 for
    blocks that are excluded (-inf) or missing (fewer than k blocks)."""
    x = pooled.float()
    kk = min(k, x.shape[-1])
    vals, idx = torch.topk(x, kk, dim=-1)
    idx = torch.where(torch.isneginf(vals) | torch.isnan(vals), torch.full_like(idx, -1), idx)
    # ascending ids with the -1 padding last
    key = torch.where(idx < 0, torch.full_like(idx, 1 << 30), idx)
    idx = torch.sort(key, dim=-1).values
    idx = torch.where(idx == (1 << 30), torch.full_like(idx, -1), idx).to(torch.int32)
    if kk < k:
        pad = torch.full(idx.shape[:-1] + (k - kk,), -1, dtype=torch.int32)
        idx = torch.cat([idx, pad], dim=-1)
    return idx
