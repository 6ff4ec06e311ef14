"""Work partitioning of the block-selection path across GPUs (one process per GPU).

The path has no exchange step: sequences are independent, and so are
(kv head, query range) pieces of one long sequence.  These planners decide
which rank computes what; each rank then runs the ordinary kernels on its
shard and results are gathered only if the caller needs them in one place.

* ``plan_sequences``: longest-processing-time bin packing of whole sequences
  onto ranks by their stage-1 work (visible query/key pairs), for varlen
  prefill and decode batches.
* ``plan_query_ranges``: split one causal sequence into query ranges of equal
  stage-1 work (causal rows grow linearly, so equal row counts would be
  unbalanced by up to 2x).
"""
from __future__ import annotations

import heapq

import numpy as np
import torch


def visible_counts(q_len: int, k_len: int, causal: bool = True) -> np.ndarray:
    """Visible compressed keys per query (C integer division, like the kernels)."""
    lq = np.arange(q_len, dtype=np.int64)
    if not causal:
        return np.full(q_len, max(k_len, 0), np.int64)
    off = np.trunc((lq - 15) / 16).astype(np.int64) + k_len - int(np.trunc((q_len - 15) / 16))
    return np.clip(off, 0, max(k_len, 0))


def sequence_cost(q_lens, k_lens, causal: bool = True) -> np.ndarray:
    """Stage-1 work of each sequence: visible (query, key) pairs plus one per query."""
    return np.array([int(visible_counts(q, k, causal).sum()) + q for q, k in zip(q_lens, k_lens)],
                    np.int64)


def plan_sequences(costs, n_ranks: int) -> list[list[int]]:
    """Assign sequence indices to ranks, largest first onto the least-loaded rank.

    Returns one sorted index list per rank; every index appears exactly once.
    """
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    heap = [(0, r) for r in range(n_ranks)]
    out: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(costs[i]), r))
    return [sorted(x) for x in out]


def plan_query_ranges(q_len: int, k_len: int, n_parts: int, causal: bool = True,
                      align: int = 64, token_cost: float = 1.0) -> list[tuple[int, int]]:
    """Split [0, q_len) into n_parts contiguous ranges of near-equal work.

    A query's work is its visible compressed keys (stage 1) plus ``token_cost``, the
    per-token work of pooling, top-k and get_block_table in units of one visible key.
    Boundaries are multiples of ``align`` (a 64-token sparse block, so pooling's
    local-window rows never straddle shards) except the last.
    """
    if n_parts <= 0:
        raise ValueError("n_parts must be positive")
    w = visible_counts(q_len, k_len, causal) + float(token_cost)
    cum = np.concatenate([[0], np.cumsum(w)])
    total = cum[-1]
    bounds = [0]
    for i in range(1, n_parts):
        t = int(np.searchsorted(cum, total * i / n_parts))
        t = int(round(t / align)) * align
        bounds.append(min(max(t, bounds[-1]), q_len))
    bounds.append(q_len)
    return [(bounds[i], bounds[i + 1]) for i in range(n_parts)]


def prefill_shard(world: int, rank: int, q_len: int, k_len: int, n_kv_heads: int = 2,
                  causal: bool = True, token_cost: float = 1.0) -> tuple[int, int, int, int]:
    """The (first kv head, kv heads, t_begin, t_end) shard of one long sequence that
    rank ``rank`` of ``world`` computes: with a rank count divisible by the kv heads,
    each rank owns one kv head and one of world / n_kv_heads query ranges of equal work
    (``plan_query_ranges``); otherwise every kv head and one of ``world`` ranges.  The
    shards of all ranks cover every (kv head, query) exactly once."""
    if not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    if world % n_kv_heads == 0:
        g, nh, n_r, r = rank % n_kv_heads, 1, world // n_kv_heads, rank // n_kv_heads
    else:
        g, nh, n_r, r = 0, n_kv_heads, world, rank
    a, b = plan_query_ranges(q_len, k_len, n_r, causal, token_cost=token_cost)[r]
    return g, nh, a, b


def _as_sendable(t):
    """The same bytes as a dtype every backend transports: NCCL in torch rejects int16, so
    16-bit integer buffers travel reinterpreted as float16 (send/recv copy bytes only)."""
    return t.view(torch.float16) if t.dtype in (torch.int16, torch.uint16) else t


def exchange_shards(local, full, shards, rank, group=None, wire=None):
    """Gather every rank's shard of a [Hk, T, ...] result into ``full`` on every rank.

    ``shards[r] = (first kv head, kv heads, t_begin, t_end)`` of rank r (as from
    ``prefill_shard``); ``local`` is this rank's [kv heads, t_end - t_begin, ...] part.
    Each rank sends its exact shard to every peer (point-to-point, no padding to the
    longest shard).  A one-head shard is a contiguous slice of ``full`` and is received
    in place; a shard of several heads arrives in a contiguous buffer and is copied in.

    ``wire``: an optional [Hk, T, ...] buffer of a narrower dtype (for example int16 for
    block ids, which are below 2^15) that the shards travel in: the local shard is
    narrowed into it, the peers' shards are received into it, and ``full`` is widened
    from it once at the end, so half the bytes cross the links.  Values must fit the
    narrower type.  Works with any torch.distributed backend that has send/recv (NCCL on
    GPUs, gloo on CPU)."""
    import torch.distributed as dist

    g, nh, a, b = shards[rank]
    tgt = full if wire is None else wire
    tgt[g:g + nh, a:b].copy_(local)
    send = tgt[g:g + nh, a:b]
    if not send.is_contiguous():
        send = send.contiguous()
    ops, staged = [], []
    for r, (gr, nhr, ar, br) in enumerate(shards):
        if r == rank:
            continue
        dst = tgt[gr:gr + nhr, ar:br]
        buf = dst if dst.is_contiguous() else torch.empty(dst.shape, dtype=dst.dtype, device=dst.device)
        if buf is not dst:
            staged.append((dst, buf))
        ops.append(dist.P2POp(dist.isend, _as_sendable(send), r, group=group))
        ops.append(dist.P2POp(dist.irecv, _as_sendable(buf), r, group=group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    for dst, buf in staged:
        dst.copy_(buf)
    if wire is not None:
        full.copy_(wire)
    return full


def _rendezvous(t, group):
    """Symmetric-memory handle of ``t`` over ``group`` (peer pointers by rank)."""
    import torch.distributed._symmetric_memory as symm

    try:
        return symm.rendezvous(t, group)
    except RuntimeError:
        symm.enable_symm_mem_for_group(group.group_name)
        return symm.rendezvous(t, group)


class PeerIdExchange:
    """The top-k id exchange fused into the top-k kernel.

    Every rank's top-k kernel (``unum_topk_blocks_to_peers``) stores each row's ids,
    narrowed to int16, straight into the gathered ``[Hk, T, K]`` buffer of every rank
    over NVLink while it selects; then ``finish`` runs the bounded cross-GPU signal
    (``unum_peer_signal_wait``) and widens this rank's buffer into the int32 result.
    There is no separate collective.  The buffers are symmetric memory (the same
    allocation on every rank, peer-mapped) and alternate by step, so a rank that starts
    the next step early never writes into a buffer a slower rank is still reading.

    Per step: ``begin()``, then ``topk(...)`` for each of this rank's launches (with the
    element offset of its rows in the gathered buffer), then ``finish(full)``.
    """

    def __init__(self, shape, device, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        import torch.distributed._symmetric_memory as symm

        self.wire = [symm.empty(*shape, dtype=torch.int16, device=device) for _ in range(2)]
        self.sig = symm.empty(self.world, dtype=torch.int32, device=device)
        self.sig.zero_()
        hw = [_rendezvous(w, self.group) for w in self.wire]
        hs = _rendezvous(self.sig, self.group)
        self.ptrs = [(ctypes.c_void_p * self.world)(*h.buffer_ptrs) for h in hw]
        self.sig_ptrs = (ctypes.c_void_p * self.world)(*hs.buffer_ptrs)
        self._handles = hw + [hs]  # keep the mappings alive
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.device = device
        self.epoch = 0
        self._lib = _lib
        torch.cuda.synchronize(device)
        dist.barrier(self.group)  # every signal array is zero before anyone announces

    def begin(self):
        self.epoch += 1

    def topk(self, pooled_rows, K, out, offset):
        """Top-K of ``pooled_rows`` [rows, NB] (16-bit or fp32) into ``out`` [rows, K]
        int32 on this rank, and the same ids as int16 at element ``offset`` of every
        rank's gathered buffer."""
        L = self._lib.load()
        rows, NB = pooled_rows.shape
        with torch.cuda.device(self.device):
            rc = L.unum_topk_blocks_to_peers(
                pooled_rows.data_ptr(), self._lib.DTYPE_CODES[pooled_rows.dtype], rows, NB,
                pooled_rows.stride(0), K, out.data_ptr(), self.ptrs[self.epoch & 1], self.world,
                int(offset), self._lib.stream_ptr(self.device))
        self._lib.check(rc)

    def finish(self, full):
        """Wait (on the stream) until every rank's stores of this step have landed, then
        widen the gathered ids into ``full`` (int32, the buffer's shape)."""
        L = self._lib.load()
        with torch.cuda.device(self.device):
            rc = L.unum_peer_signal_wait(self.sig_ptrs, self.world, self.rank, self.epoch,
                                         self.status.data_ptr(), self._lib.stream_ptr(self.device))
        self._lib.check(rc)
        full.copy_(self.wire[self.epoch & 1])
        return full

    def check(self):
        """Raise if a signal wait gave up (a peer did not announce within about a second)."""
        if int(self.status.item()) != 0:
            raise RuntimeError(f"peer signal wait expired (status {int(self.status.item())})")
