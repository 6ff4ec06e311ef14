"""Parity of the B200 kernels with the reference (golden fixtures) and the CPU oracle.

Every test here runs the product path (libunum_ops_b200.so through the
drop-in Python API) on cuda:0 and compares with
  * the outputs of the reference implementation itself (tests/golden/*.npz), and
  * the C oracle on the same seeded inputs at sizes it finishes in seconds.
Bars: bit-exact for get_block_table, pooling and top-k; stage 1 within
atol 1e-3 / rtol 1e-2 of the fp32 oracle (bf16 inputs, fp32 accumulation).
"""
import os

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-2
GOLDEN = os.path.dirname(cases.__file__)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200

    unum_ops_b200.build()
    unum_ops_b200.load()
    return torch.device("cuda", 0)


def _npz(name):
    return np.load(os.path.join(GOLDEN, name))


def _bf16_to_f32(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


# ---------------------------------------------------------------- get_block_table
@pytest.mark.parametrize("c", cases.gbt_cases(), ids=lambda c: c["name"])
def test_gbt_matches_reference(c, dev):
    from unum_ops_b200 import sparse_kernel_extension as ske

    g = _npz("gbt.npz")[c["name"] + "/out"]
    args = [_t(c[k], dev) for k in ("topk", "table", "token_to_bs", "pos", "seqlen")]
    for fn in (ske.get_block_table_ref_torch, ske.get_block_table_ref_triton, ske.get_block_table_v2,
               ske.get_block_table_v3):
        out = fn(*args, topk=c["K"])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), g, err_msg=fn.__name__)


def test_gbt_random_vs_oracle(dev, oracle_lib):
    from unum_ops_b200 import sparse_kernel_extension as ske

    rng = np.random.default_rng(11)
    for (T, B, L, K, H) in [(1000, 7, 4096, 64, 2), (513, 3, 777, 17, 2), (64, 2, 2048, 96, 4)]:
        topk = rng.integers(-3, (L + 200) // 64, size=(H, T, K)).astype(np.int32)
        table = rng.integers(0, 1 << 20, size=(B, L)).astype(np.int32)
        tb = rng.integers(0, B, size=T).astype(np.int32)
        pos = rng.integers(0, L + 100, size=T).astype(np.int32)
        sl = rng.integers(0, L + 100, size=B).astype(np.int32)
        out = ske.get_block_table_ref_torch(*[_t(x, dev) for x in (topk, table, tb, pos, sl)])
        ref = oracle_lib.get_block_table(topk, table, tb, pos, sl, head_group=2)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
        out = ske.get_block_table_ref_triton(*[_t(x, dev) for x in (topk, table, tb, pos, sl)])
        ref = oracle_lib.get_block_table(topk, table, tb, pos, sl, head_group=H)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_gbt_noncontiguous_topk_and_empty(dev, oracle_lib):
    from unum_ops_b200 import sparse_kernel_extension as ske

    rng = np.random.default_rng(12)
    T, K, L = 33, 16, 2048
    base = rng.integers(-1, L // 64, size=(T, 2, K)).astype(np.int32)
    topk_t = _t(base, dev).permute(1, 0, 2)  # [2, T, K], non-contiguous
    table = rng.integers(1, 10000, size=(1, L)).astype(np.int32)
    tb = np.zeros(T, np.int32)
    pos = np.array([L], np.int32)
    sl = np.array([L], np.int32)
    out = ske.get_block_table_ref_torch(topk_t, _t(table, dev), _t(tb, dev), _t(pos, dev), _t(sl, dev))
    ref = oracle_lib.get_block_table(np.ascontiguousarray(base.transpose(1, 0, 2)), table, tb, pos, sl)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    empty = ske.get_block_table_ref_torch(topk_t[:, :0], _t(table, dev), _t(tb[:0], dev), _t(pos, dev),
                                          _t(sl, dev))
    assert tuple(empty.shape) == (0, 2, K * 64)


# ---------------------------------------------------------------- pooling
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("c", cases.pool_cases(), ids=lambda c: c["name"])
def test_pool_matches_reference(c, dtype, dev):
    from unum_ops_b200.infllm_v2 import max_pooling_1d_varlen

    g = _npz("pool.npz")[c["name"] + "/out"]
    x = _t(c["x"], dev, dtype)
    out = max_pooling_1d_varlen(x, _t(c["cu_q"], dev), _t(c["cu_k"], dev), _t(c["cache_lens"], dev),
                                c["max_seqlen_q"], c["max_context_len"], c["local_blocks"],
                                c["init_blocks"], c["block_size"], c["stride"])
    assert out.dtype == dtype
    np.testing.assert_array_equal(out.float().cpu().numpy(), g)


@pytest.mark.parametrize("layout", ["aligned", "odd_stride"])
def test_pool_random_vs_oracle(layout, dev, oracle_lib):
    from unum_ops_b200.infllm_v2 import max_pooling_1d_varlen

    rng = np.random.default_rng(21)
    q_lens = [700, 1, 300, 1500]
    k_lens = [43, 250, 17, 92]
    W = 256 if layout == "aligned" else 250
    T = sum(q_lens)
    x = cases.bf16_round(rng.standard_normal((2, T, W), dtype=np.float32))
    x[rng.random(x.shape) < 0.01] = -np.inf
    cache = np.array([0, 5, 100, 0], np.int32)
    cu_q, cu_k = cases.cu(q_lens), cases.cu(k_lens)
    for dtype in (torch.bfloat16, torch.float32, torch.float16):
        out = max_pooling_1d_varlen(_t(x, dev, dtype), _t(cu_q, dev), _t(cu_k, dev), _t(cache, dev),
                                    16 * W, 4096, 2, 1)
        ref = oracle_lib.max_pool(_t(x, dev, dtype).float().cpu().numpy(), cu_q, cu_k, cache, 16 * W,
                                  4096, 2, 1)
        np.testing.assert_array_equal(out.float().cpu().numpy(), ref)


# ---------------------------------------------------------------- top-k
@pytest.mark.parametrize("kw", [
    dict(rows=300, NB=16, K=64), dict(rows=300, NB=384, K=64), dict(rows=97, NB=2048, K=64, ties=True),
    dict(rows=64, NB=4096, K=64, inf_frac=0.01, neginf_frac=0.5), dict(rows=33, NB=100, K=7, ties=True),
    dict(rows=64, NB=64, K=64, neginf_frac=0.3), dict(rows=40, NB=1024, K=1024, ties=True),
], ids=lambda kw: "-".join(f"{k}{v}" for k, v in kw.items()))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_topk_vs_oracle(kw, dtype, dev, oracle_lib):
    from unum_ops_b200 import topk_blocks

    c = cases.topk_case("t", 31, **kw)
    x = _t(c["x"], dev, dtype)
    out = topk_blocks(x, c["K"])
    ref = oracle_lib.topk(x.float().cpu().numpy(), c["K"])
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def _similar_rows(seed, rows, NB, kind):
    """Runs of neighbouring rows that differ a little, like pooled scores of
    consecutive tokens: each warp of the top-k kernel then reuses the previous
    row's threshold (the candidate path), with shifts that force the fallback."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal(NB).astype(np.float32)
    drift = np.cumsum(rng.standard_normal((rows, 1)).astype(np.float32) * 0.01, axis=0)
    x = base[None, :] + 0.05 * rng.standard_normal((rows, NB)).astype(np.float32) + drift
    if kind == "ties":
        x = np.round(x * 4) / 4
    if kind == "jumps":  # the distribution moves every 500 rows
        x += (np.arange(rows) // 500 % 3)[:, None].astype(np.float32) * 2.0
    if kind == "cluster":  # winners concentrated in the positions one lane loads
        hot = (np.arange(NB) % 256) < 8
        x[:, hot] += 3.0
    if kind == "masks":
        x[rng.random(x.shape) < 0.002] = np.inf
        x[rng.random(x.shape) < 0.001] = np.nan
        cut = rng.integers(NB // 2, NB + 1, size=rows)
        x[np.arange(NB)[None, :] >= cut[:, None]] = -np.inf
    return x


@pytest.mark.parametrize("NB,K,kind", [
    (2048, 64, "plain"), (2048, 64, "masks"), (2048, 64, "ties"), (2048, 64, "jumps"),
    (2048, 64, "cluster"), (4096, 128, "ties"), (1000, 64, "masks"), (300, 7, "plain"),
], ids=lambda v: str(v))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_topk_runs_of_similar_rows(NB, K, kind, dtype, dev, oracle_lib):
    from unum_ops_b200 import topk_blocks

    rows = 24000 if NB <= 2048 else 12000
    x = _t(_similar_rows(7, rows, NB, kind), dev, dtype)
    out = topk_blocks(x, K)
    ref = oracle_lib.topk(x.float().cpu().numpy(), K)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


# ---------------------------------------------------------------- stage 1
def _stage1(c, dev):
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1

    q = _t(c["q"], dev, torch.bfloat16)
    k = _t(c["k"], dev, torch.bfloat16)
    out = infllmv2_attn_stage1(q, k, k, _t(c["cu_q"], dev), _t(c["cu_k"], dev),
                               max_seqlen_q=c["max_seqlen_q"], max_seqlen_k=c["max_seqlen_k"],
                               causal=c["causal"])
    torch.cuda.synchronize()
    from unum_ops_b200.infllm_v2 import stage1_status

    assert stage1_status(dev) == 0
    return out


@pytest.mark.parametrize("c", cases.stage1_cases(), ids=lambda c: c["name"])
def test_stage1_matches_reference(c, dev, oracle_lib):
    out = _stage1(c, dev).float().cpu().numpy()
    ref = _bf16_to_f32(_npz("stage1.npz")[c["name"] + "/out_bf16"])
    orc = oracle_lib.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], c["causal"])
    assert out.shape == ref.shape
    np.testing.assert_allclose(out, orc, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(out, ref, atol=2 * ATOL, rtol=RTOL)
    np.testing.assert_array_equal(out == 0, orc == 0)


def _synthetic_stage1(seed, q_lens, k_lens, hq, hk, causal):
    return cases.stage1_case("s", seed, q_lens, k_lens, hq, hk, causal)


@pytest.mark.parametrize("spec", [
    ("c0_L1024_g8", [1024], [63], 16, 2, True),
    ("varlen_g16", [512, 1536, 17], [31, 95, 1], 32, 2, True),
    ("noncausal_g4", [300, 45], [200, 700], 8, 2, False),
    ("g32_hk1", [256], [300], 32, 1, True),
    ("g2", [130, 3], [20, 300], 4, 2, True),
    ("decode_64", [1] * 64, list(range(1, 2000, 31)) + [3000], 32, 2, True),
], ids=lambda s: s[0])
def test_stage1_random_vs_oracle(spec, dev, oracle_lib):
    name, ql, kl, hq, hk, causal = spec
    kl = kl[:len(ql)]
    c = _synthetic_stage1(sum(map(ord, name)), ql, kl, hq, hk, causal)
    out = _stage1(c, dev).float().cpu().numpy()
    orc = oracle_lib.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], c["causal"])
    np.testing.assert_allclose(out, orc, atol=ATOL, rtol=RTOL)
    np.testing.assert_array_equal(out == 0, orc == 0)


def test_stage1_repeat_is_deterministic(dev):
    c = _synthetic_stage1(5, [700, 300], [42, 17], 32, 2, True)
    a = _stage1(c, dev)
    b = _stage1(c, dev)
    assert torch.equal(a, b)


# ---------------------------------------------------------------- pipeline
def test_pipeline_small_vs_oracle(dev, oracle_lib):
    from unum_ops_b200 import block_select

    L = 4096
    q_lens = [L, 2048]
    k_lens = [cases.compressed_len(x) for x in q_lens]
    c = cases.stage1_case("pipe", 77, q_lens, k_lens, 32, 2, True)
    T = sum(q_lens)
    rng = np.random.default_rng(78)
    table = rng.permutation(2 * L).astype(np.int32).reshape(2, L)
    tb = np.repeat(np.arange(2, dtype=np.int32), q_lens)
    pos = np.concatenate([np.arange(1, n + 1) for n in q_lens]).astype(np.int32)
    seqlen = np.array(q_lens, np.int32)
    scores, pooled, idx, slots = block_select(
        _t(c["q"], dev, torch.bfloat16), _t(c["k"], dev, torch.bfloat16), _t(c["cu_q"], dev),
        _t(c["cu_k"], dev), max(k_lens), _t(table, dev), _t(tb, dev), _t(pos, dev), _t(seqlen, dev),
        max_context_len=L)
    torch.cuda.synchronize()
    sc = scores.float().cpu().numpy()
    orc = oracle_lib.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], True)
    np.testing.assert_allclose(sc, orc, atol=ATOL, rtol=RTOL)
    # downstream steps are exact functions of the GPU's own upstream outputs
    W = sc.shape[-1]
    pr = oracle_lib.max_pool(sc, c["cu_q"], c["cu_k"], np.zeros(2, np.int32), 16 * W, L, 2, 1)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), pr)
    ir = oracle_lib.topk(pr, 64)
    np.testing.assert_array_equal(idx.cpu().numpy(), ir)
    sr = oracle_lib.get_block_table(ir, table, tb, pos, seqlen)
    np.testing.assert_array_equal(slots.cpu().numpy(), sr)


# ---------------------------------------------------------------- fused stage 1 + pooling
@pytest.mark.parametrize("spec", [
    ("single_causal", [1000], None, True, 1000, 1, 2),
    ("varlen_partial_tiles", [37, 512, 300, 1], None, True, 700, 1, 2),
    ("noncausal", [130, 70], [40, 9], False, 4096, 2, 3),
    ("ctx_shorter_than_keys", [2048], None, True, 512, 0, 0),
    ("g32", [333, 64], None, True, 2000, 1, 32),
], ids=lambda s: s[0])
def test_stage1_pooled_equals_stage1_then_pool(spec, dev):
    from unum_ops_b200.block_select import stage1_pooled
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, max_pooling_1d_varlen

    name, q_lens, k_lens, causal, ctx, init_b, local_b = spec
    if k_lens is None:
        k_lens = [max(cases.compressed_len(x), 1) for x in q_lens]
    hq = 64 if name == "g32" else 32
    c = cases.stage1_case(name, sum(map(ord, name)), q_lens, k_lens, hq, 2, causal)
    q, k = _t(c["q"], dev, torch.bfloat16), _t(c["k"], dev, torch.bfloat16)
    cq, ck = _t(c["cu_q"], dev), _t(c["cu_k"], dev)
    s_f, p_f = stage1_pooled(q, k, cq, ck, max(k_lens), ctx, local_b, init_b, causal=causal)
    s_r = infllmv2_attn_stage1(q, k, k, cq, ck, max_seqlen_k=max(k_lens), causal=causal)
    W = s_r.shape[-1]
    p_r = max_pooling_1d_varlen(s_r, cq, ck, torch.zeros(len(q_lens), dtype=torch.int32, device=dev),
                                16 * W, ctx, local_b, init_b)
    torch.cuda.synchronize()
    assert torch.equal(s_f, s_r)
    np.testing.assert_array_equal(p_f.float().cpu().numpy(), p_r.float().cpu().numpy())


def test_rows_outside_every_sequence(dev, oracle_lib):
    """Token rows before cu_seqlens_q[0] and after cu_seqlens_q[-1] get the reference's
    values: zero scores (stage 1) and a pooled row with k_len 0 (pooling)."""
    from unum_ops_b200.block_select import stage1_pooled
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, max_pooling_1d_varlen

    rng = np.random.default_rng(91)
    T, hq, hk = 300, 32, 2
    q = cases.bf16_round(rng.standard_normal((T, hq, 128), dtype=np.float32))
    k = cases.bf16_round(rng.standard_normal((40, hk, 128), dtype=np.float32))
    cu_q = np.array([20, 200, 280], np.int32)
    cu_k = np.array([0, 11, 40], np.int32)
    qd, kd = _t(q, dev, torch.bfloat16), _t(k, dev, torch.bfloat16)
    s = infllmv2_attn_stage1(qd, kd, kd, _t(cu_q, dev), _t(cu_k, dev), max_seqlen_k=29, causal=True)
    sf, pf = stage1_pooled(qd, kd, _t(cu_q, dev), _t(cu_k, dev), 29, 512, 2, 1)
    torch.cuda.synchronize()
    ref = oracle_lib.stage1(q, k, cu_q, cu_k, True, out_stride=128)
    np.testing.assert_allclose(s.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
    np.testing.assert_array_equal(s.float().cpu().numpy() == 0, ref == 0)
    assert torch.equal(s, sf)
    pr = max_pooling_1d_varlen(s, _t(cu_q, dev), _t(cu_k, dev), torch.zeros(2, dtype=torch.int32, device=dev),
                               16 * 128, 512, 2, 1)
    np.testing.assert_array_equal(pf.float().cpu().numpy(), pr.float().cpu().numpy())
    po = oracle_lib.max_pool(s.float().cpu().numpy(), cu_q, cu_k, np.zeros(2, np.int32), 16 * 128, 512, 2, 1)
    np.testing.assert_array_equal(pf.float().cpu().numpy(), po)


@pytest.mark.parametrize("q_lens,chunk", [([8192], 2048), ([3000, 5000, 17], 1000)],
                         ids=["single_8k", "varlen_unaligned_chunks"])
def test_block_select_streamed_equals_block_select(q_lens, chunk, dev):
    from unum_ops_b200 import block_select, block_select_streamed

    k_lens = [cases.compressed_len(x) for x in q_lens]
    c = cases.stage1_case("stream", 123, q_lens, k_lens, 32, 2, True)
    T = sum(q_lens)
    rng = np.random.default_rng(5)
    L = max(q_lens)
    table = rng.permutation(len(q_lens) * L).astype(np.int32).reshape(len(q_lens), L)
    tb = np.repeat(np.arange(len(q_lens), dtype=np.int32), q_lens)
    pos = np.concatenate([np.arange(1, n + 1) for n in q_lens]).astype(np.int32)
    sl = np.array(q_lens, np.int32)
    q_host = torch.from_numpy(c["q"]).to(torch.bfloat16).pin_memory()
    k = _t(c["k"], dev, torch.bfloat16)
    args = [_t(x, dev) for x in (c["cu_q"], c["cu_k"])]
    rest = [_t(x, dev) for x in (table, tb, pos, sl)]
    ref = block_select(q_host.to(dev), k, *args, max(k_lens), *rest, max_context_len=L)
    res_host = torch.empty(2, T, 64, dtype=torch.int32).pin_memory()
    got = block_select_streamed(q_host, k, *args, max(k_lens), *rest, max_context_len=L,
                                chunk_tokens=chunk, result_host=res_host)
    torch.cuda.synchronize()
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    assert torch.equal(res_host, ref[2].cpu())


def test_block_select_streamed_back_to_back(dev):
    """Several streamed calls issued without synchronising in between must each return
    the same results (buffers reused across calls are ordered by the streams)."""
    from unum_ops_b200 import block_select, block_select_streamed

    q_lens = [4096]
    k_lens = [cases.compressed_len(4096)]
    c = cases.stage1_case("stream2", 321, q_lens, k_lens, 32, 2, True)
    table = np.arange(4096, dtype=np.int32).reshape(1, 4096)
    tb = np.zeros(4096, np.int32)
    pos = np.arange(1, 4097, dtype=np.int32)
    sl = np.array([4096], np.int32)
    k = _t(c["k"], dev, torch.bfloat16)
    args = [_t(x, dev) for x in (c["cu_q"], c["cu_k"])]
    rest = [_t(x, dev) for x in (table, tb, pos, sl)]
    hosts = [torch.from_numpy(c["q"]).to(torch.bfloat16).pin_memory(),
             (torch.from_numpy(c["q"]) * -1).to(torch.bfloat16).pin_memory()]
    refs = [block_select(h.to(dev), k, *args, k_lens[0], *rest, max_context_len=4096)[2] for h in hosts]
    torch.cuda.synchronize()
    outs = [block_select_streamed(hosts[i % 2], k, *args, k_lens[0], *rest, max_context_len=4096,
                                  chunk_tokens=512)[2] for i in range(6)]
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, refs[i % 2]), i


# ---------------------------------------------------------------- sharded rows
def _c3_like(L, seed, dev):
    nk = cases.compressed_len(L)
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(L, 32, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(nk, 2, 128, generator=g, device=dev).to(torch.bfloat16)
    cu_q = torch.tensor([0, L], dtype=torch.int32, device=dev)
    cu_k = torch.tensor([0, nk], dtype=torch.int32, device=dev)
    table = torch.randperm(L, device=dev, dtype=torch.int64).to(torch.int32).reshape(1, L)
    tb = torch.zeros(L, dtype=torch.int32, device=dev)
    pos = torch.arange(1, L + 1, dtype=torch.int32, device=dev)
    sl = torch.tensor([L], dtype=torch.int32, device=dev)
    return q, k, cu_q, cu_k, nk, table, tb, pos, sl


@pytest.mark.parametrize("n_ranges", [1, 3])
def test_rows_shards_equal_full(n_ranges, dev):
    """Every (kv head, query range) shard of one causal sequence reproduces the
    unsharded path's rows bit for bit: scores, pooled scores, top-k ids, slots."""
    from unum_ops_b200 import block_select, block_select_rows, sharding

    L = 16384
    q, k, cu_q, cu_k, nk, table, tb, pos, sl = _c3_like(L, 11, dev)
    full = block_select(q, k, cu_q, cu_k, nk, table, tb, pos, sl, max_context_len=L)
    for g in range(2):
        qg, kg = q[:, 16 * g:16 * (g + 1)], k[:, g:g + 1]  # strided views of one kv group
        for a, b in sharding.plan_query_ranges(L, nk, n_ranges, token_cost=600.0):
            sc, po, idx, slots = block_select_rows(qg, kg, cu_q, cu_k, nk, table, tb, pos, sl,
                                                   t_begin=a, t_end=b, max_context_len=L,
                                                   head_offset=g)
            assert torch.equal(sc[0, a:b], full[0][g, a:b])
            assert torch.equal(po[0, a:b], full[1][g, a:b])
            assert torch.equal(idx[0], full[2][g, a:b])
            assert torch.equal(slots[:, 0], full[3][a:b, g])


def test_streamed_shard_equals_full(dev):
    """The streamed path on one rank's shard (host rows of one kv group, a token
    window that does not start at a chunk edge) equals the same rows of the full path."""
    from unum_ops_b200 import block_select, block_select_streamed

    L = 16384
    q, k, cu_q, cu_k, nk, table, tb, pos, sl = _c3_like(L, 12, dev)
    full = block_select(q, k, cu_q, cu_k, nk, table, tb, pos, sl, max_context_len=L)
    g, a, b = 1, 5184, 13760
    q_host = q[a:b, 16 * g:16 * (g + 1)].contiguous().cpu().pin_memory()
    res = torch.empty(1, b - a, 64, dtype=torch.int32).pin_memory()
    sc, po, idx, slots = block_select_streamed(q_host, k[:, g:g + 1], cu_q, cu_k, nk, table, tb, pos, sl,
                                               max_context_len=L, chunk_tokens=4096, result_host=res,
                                               t_begin=a, head_offset=g)
    torch.cuda.synchronize()
    assert torch.equal(sc[0, a:b], full[0][g, a:b])
    assert torch.equal(idx[0], full[2][g, a:b])
    assert torch.equal(res[0], full[2][g, a:b].cpu())
    assert torch.equal(slots[:, 0], full[3][a:b, g])


def test_block_table_shard_into_full_output(dev, oracle_lib):
    """get_block_table_shard writing one head's rows straight into the full
    [T, Hk, K*64] output equals the unsharded call."""
    from unum_ops_b200 import get_block_table_shard
    from unum_ops_b200.sparse_kernel_extension import get_block_table_ref_torch

    rng = np.random.default_rng(13)
    T, K = 3000, 64
    topk = rng.integers(-1, 40, size=(2, T, K)).astype(np.int32)
    table = rng.permutation(1 << 16).astype(np.int32).reshape(16, 4096)
    tb = rng.integers(0, 16, size=T).astype(np.int32)
    pos = rng.integers(1, 4096, size=T).astype(np.int32)
    sl = np.full(16, 4000, np.int32)
    args = [_t(x, dev) for x in (table, tb, pos, sl)]
    ref = get_block_table_ref_torch(_t(topk, dev), *args)
    out = torch.zeros_like(ref)
    for g in range(2):
        get_block_table_shard(_t(topk[g:g + 1], dev), *args, head_offset=g, out=out[:, g:g + 1])
    assert torch.equal(out, ref)


# ---------------------------------------------------------------- stage 1, decode kernel
@pytest.mark.parametrize("c", [c for c in cases.stage1_cases() if c["q"].shape[1] // c["k"].shape[1] >= 16],
                         ids=lambda c: c["name"])
def test_stage1_decode_kernel_matches_reference(c, dev, oracle_lib, monkeypatch):
    """The per-(token, kv head) decode kernel, forced on every fixture it can run (it is
    chosen by default for one or a few queries per sequence), against the reference's
    outputs and the oracle."""
    monkeypatch.setenv("UNUM_STAGE1_PATH", "decode")
    out = _stage1(c, dev).float().cpu().numpy()
    ref = _bf16_to_f32(_npz("stage1.npz")[c["name"] + "/out_bf16"])
    orc = oracle_lib.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], c["causal"])
    np.testing.assert_allclose(out, orc, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(out, ref, atol=2 * ATOL, rtol=RTOL)


@pytest.mark.parametrize("hq", [32, 64])
@pytest.mark.parametrize("causal", [True, False])
def test_stage1_decode_kernel_varlen(hq, causal, dev, oracle_lib):
    """Decode-shaped batches through the default dispatch: empty sequences, one to a
    few query tokens, contexts from one key to the most a row holds (G=32: 2048,
    G=16: 4096), and a token window."""
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, stage1_status

    rng = np.random.default_rng(21 + hq)
    B = 40
    q_lens = rng.integers(0, 3, size=B)
    q_lens[:4] = [1, 0, 2, 1]
    max_k = 4096 if hq == 32 else 2048
    k_lens = rng.integers(1, max_k + 1, size=B)
    k_lens[:4] = [1, 7, max_k, 128]
    T, Tk = int(q_lens.sum()), int(k_lens.sum())
    q = rng.standard_normal((T, hq, 128), dtype=np.float32)
    k = rng.standard_normal((Tk, 2, 128), dtype=np.float32)
    qb, kb = _t(q, dev, torch.bfloat16), _t(k, dev, torch.bfloat16)
    cu_q, cu_k = cases.cu(q_lens), cases.cu(k_lens)
    out = infllmv2_attn_stage1(qb, kb, None, _t(cu_q, dev), _t(cu_k, dev), max_seqlen_k=max_k,
                               causal=causal)
    torch.cuda.synchronize()
    assert stage1_status(dev) == 0
    orc = oracle_lib.stage1(qb.float().cpu().numpy(), kb.float().cpu().numpy(), cu_q, cu_k, causal,
                            out_stride=out.shape[-1])
    np.testing.assert_allclose(out.float().cpu().numpy(), orc, atol=ATOL, rtol=RTOL)


def test_stage1_decode_rows_longer_than_tensor_memory(dev, oracle_lib, monkeypatch):
    """A decode batch whose caller passes a max_seqlen_k below a sequence's key count, so
    a token has more visible keys than the decode kernel's tensor memory holds (G=16:
    4096): the softmax still runs over every visible key (the keys past the resident
    tiles on CUDA cores) and the first out_stride columns are written — the same
    result as the tile kernel and the oracle, and status 0."""
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, stage1_status

    rng = np.random.default_rng(77)
    k_lens = np.array([5000, 300, 4096, 9000, 4097, 1], np.int64)
    q_lens = np.ones(len(k_lens), np.int64)
    T, Tk = int(q_lens.sum()), int(k_lens.sum())
    q = rng.standard_normal((T, 32, 128), dtype=np.float32)
    k = rng.standard_normal((Tk, 2, 128), dtype=np.float32)
    qb, kb = _t(q, dev, torch.bfloat16), _t(k, dev, torch.bfloat16)
    cu_q, cu_k = cases.cu(q_lens), cases.cu(k_lens)
    outs = {}
    for path in ("decode", "tile"):
        monkeypatch.setenv("UNUM_STAGE1_PATH", path)
        outs[path] = infllmv2_attn_stage1(qb, kb, None, _t(cu_q, dev), _t(cu_k, dev), max_seqlen_k=4096,
                                          causal=True)
        torch.cuda.synchronize()
        assert stage1_status(dev) == 0
    assert outs["decode"].shape[-1] == 4096
    orc = oracle_lib.stage1(qb.float().cpu().numpy(), kb.float().cpu().numpy(), cu_q, cu_k, True,
                            out_stride=4096)
    for path in ("decode", "tile"):
        np.testing.assert_allclose(outs[path].float().cpu().numpy(), orc, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(outs["decode"].float().cpu().numpy(), outs["tile"].float().cpu().numpy(),
                               atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("path", ["tile", "decode"])
def test_stage1_forced_expiry_drains_and_recovers(path, dev, oracle_lib, monkeypatch):
    """The bounded-wait expiry path, taken on purpose (UNUM_STAGE1_FORCE_EXPIRY=1 makes
    every wait report expiry before any TMA or UMMA work is issued): the kernel drains,
    frees tensor memory and returns with status 30; the next normal call on the same
    workspace returns status 0 and correct scores."""
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, stage1_status

    rng = np.random.default_rng(5)
    k_lens = np.array([700, 64, 2000], np.int64)
    q_lens = np.ones(3, np.int64) if path == "decode" else np.array([300, 17, 1024], np.int64)
    T, Tk = int(q_lens.sum()), int(k_lens.sum())
    q = rng.standard_normal((T, 32, 128), dtype=np.float32)
    k = rng.standard_normal((Tk, 2, 128), dtype=np.float32)
    qb, kb = _t(q, dev, torch.bfloat16), _t(k, dev, torch.bfloat16)
    cu_q, cu_k = cases.cu(q_lens), cases.cu(k_lens)
    monkeypatch.setenv("UNUM_STAGE1_PATH", path)
    monkeypatch.setenv("UNUM_STAGE1_FORCE_EXPIRY", "1")
    infllmv2_attn_stage1(qb, kb, None, _t(cu_q, dev), _t(cu_k, dev), causal=path == "tile")
    torch.cuda.synchronize()
    assert stage1_status(dev) == 30
    monkeypatch.delenv("UNUM_STAGE1_FORCE_EXPIRY")
    out = infllmv2_attn_stage1(qb, kb, None, _t(cu_q, dev), _t(cu_k, dev), causal=path == "tile")
    torch.cuda.synchronize()
    assert stage1_status(dev) == 0
    orc = oracle_lib.stage1(qb.float().cpu().numpy(), kb.float().cpu().numpy(), cu_q, cu_k, path == "tile",
                            out_stride=out.shape[-1])
    np.testing.assert_allclose(out.float().cpu().numpy(), orc, atol=ATOL, rtol=RTOL)


def test_block_select_without_scores_matches(dev):
    """block_select(return_scores=False): the stage-1 scores stay on chip; pooled blocks,
    top-k ids and slots are identical to the call that writes the scores."""
    from unum_ops_b200 import block_select

    rng = np.random.default_rng(12)
    q_lens = np.array([3000, 17, 1200], np.int64)
    k_lens = np.array([(n - 32) // 16 + 1 if n >= 32 else 1 for n in q_lens], np.int64)
    T, Tk = int(q_lens.sum()), int(k_lens.sum())
    q = _t(rng.standard_normal((T, 32, 128), dtype=np.float32), dev, torch.bfloat16)
    k = _t(rng.standard_normal((Tk, 2, 128), dtype=np.float32), dev, torch.bfloat16)
    cu_q, cu_k = _t(cases.cu(q_lens), dev), _t(cases.cu(k_lens), dev)
    table = _t(rng.permutation(3 * 4096).astype(np.int32).reshape(3, 4096), dev)
    tb = _t(np.repeat(np.arange(3, dtype=np.int32), q_lens), dev)
    pos = _t(np.concatenate([np.arange(1, n + 1) for n in q_lens]).astype(np.int32), dev)
    sl = _t(q_lens.astype(np.int32), dev)
    args = (q, k, cu_q, cu_k, int(k_lens.max()), table, tb, pos, sl)
    full = block_select(*args, max_context_len=4096)
    part = block_select(*args, max_context_len=4096, return_scores=False)
    torch.cuda.synchronize()
    assert part[0] is None
    for a, b in zip(full[1:], part[1:]):
        assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                           b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


def test_block_select_graph_replays_new_inputs(dev):
    """BlockSelectGraph: a replay after writing new values into the static inputs gives
    what the eager block_select gives on those values (decode-shaped batch)."""
    from unum_ops_b200 import BlockSelectGraph, block_select

    rng = np.random.default_rng(31)
    B = 24
    ctx = rng.integers(300, 9000, size=B)
    k_lens = (ctx - 32) // 16 + 1
    q = torch.randn(B, 32, 128, device=dev).to(torch.bfloat16)
    k = torch.randn(int(k_lens.sum()), 2, 128, device=dev).to(torch.bfloat16)
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
    cu_k = _t(cases.cu(k_lens), dev)
    table = _t(rng.integers(0, 1 << 20, size=(B, 256)).astype(np.int32), dev)
    tb = torch.arange(B, dtype=torch.int32, device=dev)
    pos = _t(ctx.astype(np.int32), dev)
    cache = _t((ctx - 1).astype(np.int32), dev)
    args = (q, k, cu_q, cu_k, int(k_lens.max()), table, tb, pos, pos)
    kw = dict(max_context_len=16384, cache_lens=cache)
    gr = BlockSelectGraph(*args, **kw)
    for _ in range(2):
        q.copy_(torch.randn_like(q, dtype=torch.float32).to(torch.bfloat16))
        k.copy_(torch.randn_like(k, dtype=torch.float32).to(torch.bfloat16))
        got = [x.clone() for x in gr()]
        ref = block_select(*args, **kw)
        for a, b in zip(got, ref):
            assert torch.equal(a, b)


def test_decode_kernel_token_windows_equal_full(dev):
    """Stage 1 on token windows of a decode batch (the decode kernel's t_begin/t_end
    path: the window entry point without fused pooling) writes exactly the window's
    rows, equal to the same rows of the whole-batch call."""
    from unum_ops_b200 import _lib
    from unum_ops_b200.infllm_v2 import _workspace, infllmv2_attn_stage1, stage1_status

    rng = np.random.default_rng(51)
    B = 40
    ctx = rng.integers(200, 8000, size=B)
    k_lens = (ctx - 32) // 16 + 1
    q = torch.randn(B, 32, 128, device=dev).to(torch.bfloat16)
    k = torch.randn(int(k_lens.sum()), 2, 128, device=dev).to(torch.bfloat16)
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
    cu_k = _t(cases.cu(k_lens), dev)
    full = infllmv2_attn_stage1(q, k, None, cu_q, cu_k, max_seqlen_k=int(k_lens.max()), causal=True)
    W = full.shape[-1]
    out = torch.full_like(full, float("nan"))
    L = _lib.load()
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(B)))
    for a, b in ((0, 13), (13, 14), (14, 40)):
        _lib.check(L.unum_infllmv2_attn_stage1_window(
            q.data_ptr(), B, 32, 128, q.stride(0), q.stride(1), k.data_ptr(), k.shape[0], 2, k.stride(0),
            k.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), B, 128 ** -0.5, 1, out.data_ptr(), W, None, 0,
            0, 0, a, b, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)))
        torch.cuda.synchronize()
        assert stage1_status(dev) == 0
        assert torch.equal(out[:, a:b], full[:, a:b])
        assert torch.isnan(out[:, b:].float()).all()  # rows past the window untouched
