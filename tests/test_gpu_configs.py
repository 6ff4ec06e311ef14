"""The BASELINE configurations C0-C4 at full size on the GPU.

Where the CPU oracle finishes in seconds the whole output is compared; at
128k tokens the stage-1 output is checked with a size-independent property
(each token's row sums to G, the number of heads in the group, when any key is
visible, else 0 — every head's softmax sums to one) plus oracle comparison on
sampled token ranges, and the downstream steps are checked exactly against
the oracle applied to the GPU's own upstream outputs.
"""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200

    unum_ops_b200.load()
    return torch.device("cuda", 0)


def _inputs(seed, q_lens, k_lens, hq, hk, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    T, Tk = sum(q_lens), sum(k_lens)
    q = torch.randn(T, hq, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(Tk, hk, 128, generator=g, device=dev).to(torch.bfloat16)
    cu_q = torch.from_numpy(cases.cu(q_lens)).to(dev)
    cu_k = torch.from_numpy(cases.cu(k_lens)).to(dev)
    return q, k, cu_q, cu_k


def _row_sum_property(scores, cu_q, cu_k, G, causal=True):
    from unum_ops_b200 import sharding

    sums = scores.float().sum(-1).cpu().numpy()  # [Hk, T]
    cq, ck = cu_q.cpu().numpy(), cu_k.cpu().numpy()
    expect = np.zeros(sums.shape[1], np.float32)
    for b in range(len(cq) - 1):
        vis = sharding.visible_counts(int(cq[b + 1] - cq[b]), int(ck[b + 1] - ck[b]), causal)
        expect[cq[b]:cq[b + 1]] = np.where(vis > 0, G, 0)
    for h in range(sums.shape[0]):
        np.testing.assert_allclose(sums[h], expect, rtol=2e-2, atol=1e-3)


def _oracle_rows(oracle_lib, q, k, cu_q, cu_k, a, b, W, causal=True):
    return oracle_lib.stage1(q.float().cpu().numpy(), k.float().cpu().numpy(), cu_q.cpu().numpy(),
                             cu_k.cpu().numpy(), causal, out_stride=W, t_range=(a, b))


def test_c0_full_pipeline(dev, oracle_lib):
    from unum_ops_b200 import block_select

    L = 1024
    q, k, cu_q, cu_k = _inputs(0, [L], [63], 16, 2, dev)
    table = torch.randperm(L, device=dev, dtype=torch.int64).to(torch.int32).reshape(1, L)
    tb = torch.zeros(L, dtype=torch.int32, device=dev)
    pos = torch.arange(1, L + 1, dtype=torch.int32, device=dev)
    sl = torch.tensor([L], dtype=torch.int32, device=dev)
    scores, pooled, idx, slots = block_select(q, k, cu_q, cu_k, 63, table, tb, pos, sl,
                                              max_context_len=L, init_blocks=1, local_blocks=2)
    torch.cuda.synchronize()
    sc = scores.float().cpu().numpy()
    ref = _oracle_rows(oracle_lib, q, k, cu_q, cu_k, 0, L, 128)
    np.testing.assert_allclose(sc, ref, atol=ATOL, rtol=RTOL)
    pr = oracle_lib.max_pool(sc, cu_q.cpu().numpy(), cu_k.cpu().numpy(), np.zeros(1, np.int32),
                             16 * 128, L, 2, 1)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), pr)
    ir = oracle_lib.topk(pr, 64)
    np.testing.assert_array_equal(idx.cpu().numpy(), ir)
    np.testing.assert_array_equal(slots.cpu().numpy(), oracle_lib.get_block_table(
        ir, table.cpu().numpy(), tb.cpu().numpy(), pos.cpu().numpy(), sl.cpu().numpy()))


def test_c1_varlen_prefill(dev, oracle_lib):
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, max_pooling_1d_varlen

    q_lens = [8192, 24576]
    k_lens = [cases.compressed_len(x) for x in q_lens]
    q, k, cu_q, cu_k = _inputs(1, q_lens, k_lens, 32, 2, dev)
    scores = infllmv2_attn_stage1(q, k, None, cu_q, cu_k, max_seqlen_k=max(k_lens), causal=True)
    torch.cuda.synchronize()
    W = scores.shape[-1]
    _row_sum_property(scores, cu_q, cu_k, 16)
    for a in (0, 8176, 8192, 20000, 32752):  # both sequences, their boundary, the last rows
        ref = _oracle_rows(oracle_lib, q, k, cu_q, cu_k, a, a + 16, W)
        np.testing.assert_allclose(scores[:, a:a + 16].float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
    pooled = max_pooling_1d_varlen(scores, cu_q, cu_k, torch.zeros(2, dtype=torch.int32, device=dev),
                                   16 * W, 24576, 2, 1)
    pr = oracle_lib.max_pool(scores.float().cpu().numpy(), cu_q.cpu().numpy(), cu_k.cpu().numpy(),
                             np.zeros(2, np.int32), 16 * W, 24576, 2, 1)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), pr)


def test_c2_block_table_full(dev, oracle_lib):
    from unum_ops_b200.sparse_kernel_extension import get_block_table_ref_torch

    rng = np.random.default_rng(2)
    lens = rng.integers(512, 4097, size=16)
    T = int(lens.sum())
    tb = np.repeat(np.arange(16, dtype=np.int32), lens)
    pos = np.concatenate([np.arange(1, n + 1) for n in lens]).astype(np.int32)
    topk = np.empty((2, T, 64), np.int32)
    nblk = (pos + 63) // 64
    topk[:] = (rng.random((2, T, 64)) * nblk[None, :, None]).astype(np.int32)
    topk[rng.random(topk.shape) < 0.1] = -1
    for width in (4096, 2048):  # per-token table, and BASELINE's [16, 2048] (clamp path)
        table = rng.permutation(16 * width).astype(np.int32).reshape(16, width)
        out = get_block_table_ref_torch(*[torch.from_numpy(x).to(dev) for x in
                                          (topk, table, tb, pos, lens.astype(np.int32))])
        ref = oracle_lib.get_block_table(topk, table, tb, pos, lens.astype(np.int32))
        np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_c3_128k_prefill(dev, oracle_lib):
    from unum_ops_b200 import block_select

    L = 131072
    nk = cases.compressed_len(L)
    q, k, cu_q, cu_k = _inputs(3, [L], [nk], 32, 2, dev)
    table = torch.randperm(L, device=dev, dtype=torch.int64).to(torch.int32).reshape(1, L)
    tb = torch.zeros(L, dtype=torch.int32, device=dev)
    pos = torch.arange(1, L + 1, dtype=torch.int32, device=dev)
    sl = torch.tensor([L], dtype=torch.int32, device=dev)
    scores, pooled, idx, slots = block_select(q, k, cu_q, cu_k, nk, table, tb, pos, sl,
                                              max_context_len=L)
    torch.cuda.synchronize()
    W = scores.shape[-1]
    _row_sum_property(scores, cu_q, cu_k, 16)
    # windows from the kernel's schedule as well as round numbers: work items are 16-token
    # tiles dealt last-tile-first to the 148 persistent CTAs, so L-16 is the first item
    # (most key tiles), L-75*16 the first CTA's second item (a persistent-CTA item
    # boundary near the diagonal), and 129016 / 63*2048-8 straddle two tiles where the
    # causal key count crosses a 128-key tile boundary (last key tile partly masked)
    for a in (0, 4096, 65536, L - 16, L - 75 * 16, 129016, 63 * 2048 - 8):
        ref = _oracle_rows(oracle_lib, q, k, cu_q, cu_k, a, a + 16, W)
        np.testing.assert_allclose(scores[:, a:a + 16].float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
    # downstream steps, exact, on sampled token ranges of the GPU's own outputs
    cuk = cu_k.cpu().numpy()
    for a in (0, 70000, L - 512):
        rows = scores[:, a:a + 512].float().cpu().numpy()
        pr = oracle_lib.max_pool(rows, np.array([-a, 512], np.int32), cuk, np.zeros(1, np.int32),
                                 16 * W, L, 2, 1)
        np.testing.assert_array_equal(pooled[:, a:a + 512].float().cpu().numpy(), pr)
        ir = oracle_lib.topk(pooled[:, a:a + 512].float().cpu().numpy(), 64)
        np.testing.assert_array_equal(idx[:, a:a + 512].cpu().numpy(), ir)
        sr = oracle_lib.get_block_table(ir, table.cpu().numpy(), tb[a:a + 512].cpu().numpy(),
                                        pos[a:a + 512].cpu().numpy(), sl.cpu().numpy())
        np.testing.assert_array_equal(slots[a:a + 512].cpu().numpy(), sr)


def test_c4_decode_batch(dev, oracle_lib):
    from unum_ops_b200 import block_select

    rng = np.random.default_rng(4)
    ctx = rng.integers(4096, 65537, size=512)
    k_lens = [cases.compressed_len(int(x)) for x in ctx]
    q, k, cu_q, cu_k = _inputs(4, [1] * 512, k_lens, 32, 2, dev)
    table = torch.from_numpy(rng.integers(0, 1 << 20, size=(512, 1024)).astype(np.int32)).to(dev)
    tb = torch.arange(512, dtype=torch.int32, device=dev)
    pos = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    cache = torch.from_numpy((ctx - 1).astype(np.int32)).to(dev)  # cached tokens behind each query
    scores, pooled, idx, slots = block_select(q, k, cu_q, cu_k, max(k_lens), table, tb, pos, pos,
                                              max_context_len=65536, cache_lens=cache)
    torch.cuda.synchronize()
    sc = scores.float().cpu().numpy()
    ref = _oracle_rows(oracle_lib, q, k, cu_q, cu_k, 0, 512, sc.shape[-1])
    np.testing.assert_allclose(sc, ref, atol=ATOL, rtol=RTOL)
    W = sc.shape[-1]
    pr = oracle_lib.max_pool(sc, cu_q.cpu().numpy(), cu_k.cpu().numpy(), cache.cpu().numpy(),
                             16 * W, 65536, 2, 1)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), pr)
    ir = oracle_lib.topk(pr, 64)
    np.testing.assert_array_equal(idx.cpu().numpy(), ir)
    np.testing.assert_array_equal(slots.cpu().numpy(), oracle_lib.get_block_table(
        ir, table.cpu().numpy(), tb.cpu().numpy(), pos.cpu().numpy(), pos.cpu().numpy()))
