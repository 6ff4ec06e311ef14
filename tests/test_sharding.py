"""Host-side multi-GPU logic: planners, and a 2-rank gloo run that shards a
small varlen batch, computes each shard with the CPU oracle and gathers it
back to the unsharded result."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from unum_ops_b200 import sharding


def test_plan_sequences_covers_each_once_and_balances():
    rng = np.random.default_rng(3)
    costs = rng.integers(1, 1000, size=101)
    for n in (1, 2, 3, 8):
        plan = sharding.plan_sequences(costs, n)
        flat = sorted(i for p in plan for i in p)
        assert flat == list(range(101))
        loads = [int(costs[p].sum()) for p in plan]
        assert max(loads) - min(loads) <= costs.max()


def test_plan_query_ranges_balances_causal_work():
    L = 131072
    k = (L - 32) // 16 + 1
    for n in (2, 4, 8):
        r = sharding.plan_query_ranges(L, k, n)
        assert r[0][0] == 0 and r[-1][1] == L
        assert all(a < b for a, b in r)
        assert all(r[i][1] == r[i + 1][0] for i in range(n - 1))
        assert all(a % 64 == 0 for a, _ in r)
        vis = sharding.visible_counts(L, k) + 1
        work = [vis[a:b].sum() for a, b in r]
        assert max(work) / min(work) < 1.01


def test_visible_counts_matches_oracle(oracle_lib):
    for q, k in ((1, 300), (64, 40), (1024, 63), (17, 1)):
        v = sharding.visible_counts(q, k)
        assert [oracle_lib.stage1_visible(i, q, k, True) for i in range(q)] == v.tolist()


def _worker(rank, world, port, q_lens, k_lens, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle

    c = cases.stage1_case("shard", 5, q_lens, k_lens, 16, 2, True)
    costs = sharding.sequence_cost(q_lens, k_lens)
    mine = sharding.plan_sequences(costs, world)[rank]
    W = (max(k_lens) + 127) // 128 * 128
    parts = {}
    for b in mine:
        qs, qe = int(c["cu_q"][b]), int(c["cu_q"][b + 1])
        ks, ke = int(c["cu_k"][b]), int(c["cu_k"][b + 1])
        s = oracle.stage1(c["q"][qs:qe], c["k"][ks:ke], np.array([0, qe - qs], np.int32),
                          np.array([0, ke - ks], np.int32), True, out_stride=W)
        parts[b] = s
    gathered = [None] * world
    dist.all_gather_object(gathered, parts)
    if rank == 0:
        full = np.zeros((2, int(c["cu_q"][-1]), W), np.float32)
        for d in gathered:
            for b, s in d.items():
                full[:, int(c["cu_q"][b]):int(c["cu_q"][b + 1]), :] = s
        ref = oracle.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], True, out_stride=W)
        ret.put(float(np.abs(full - ref).max()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_shard_and_gather(oracle_lib):
    q_lens = [300, 40, 129, 1, 77]
    k_lens = [cases.compressed_len(x) for x in q_lens[:3]] + [50, 3]
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_lens, k_lens, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert ret.get(timeout=5) == 0.0


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_prefill_shards_cover_each_head_and_token_once(world):
    from unum_ops_b200 import sharding

    L = 131072
    nk = (L - 32) // 16 + 1
    cover = np.zeros((2, L), np.int32)
    work = []
    for r in range(world):
        g, nh, a, b = sharding.prefill_shard(world, r, L, nk, 2, token_cost=560.0)
        cover[g:g + nh, a:b] += 1
        work.append((sharding.visible_counts(L, nk)[a:b] + 560.0).sum() * nh)
    assert (cover == 1).all()
    assert max(work) / min(work) < 1.05  # ranges of near-equal work


def _exchange_worker(rank, world, port, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    L, K = 4096, 8
    nk = (L - 32) // 16 + 1
    ref = torch.arange(2 * L * K, dtype=torch.int32).reshape(2, L, K)
    shards = [sharding.prefill_shard(world, r, L, nk, 2, token_cost=560.0) for r in range(world)]
    g, nh, a, b = shards[rank]
    full = torch.full((2, L, K), -7, dtype=torch.int32)
    sharding.exchange_shards(ref[g:g + nh, a:b].clone(), full, shards, rank)
    ok = bool(torch.equal(full, ref))
    # block ids on an int16 wire (ids < 2^15, -1 padding kept)
    ids = (ref % 2048) - (ref % 7 == 0).to(torch.int32) * ((ref % 2048) + 1)
    full2 = torch.full((2, L, K), -7, dtype=torch.int32)
    wire = torch.empty((2, L, K), dtype=torch.int16)
    sharding.exchange_shards(ids[g:g + nh, a:b].clone(), full2, shards, rank, wire=wire)
    ok = ok and bool(torch.equal(full2, ids)) and bool((ids == -1).any())
    ret.put((rank, ok))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_exchange_shards_gloo(world):
    """Every rank ends up with the whole [Hk, T, K] result from the exact-size shards of
    the others (kv head x query range shards for even rank counts, query ranges else)."""
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = 30500 + (os.getpid() + world) % 1000
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    got = dict(ret.get(timeout=5) for _ in range(world))
    assert all(got[r] for r in range(world))
