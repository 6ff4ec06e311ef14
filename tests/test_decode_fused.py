"""The fused decode selection (unum_block_select_decode, block_select's one-launch path
for decode batches) against the four-kernel chain it replaces and against the oracle.

Bar: bit-exact on every output (scores, pooled blocks, top-k ids, slot ids) against
stage 1 -> max_pooling_1d_varlen -> topk_blocks -> get_block_table_ref_torch run as
separate kernels on the same inputs, and the downstream steps bit-exact against the
C oracle applied to the GPU's own stage-1 scores."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200

    unum_ops_b200.build()
    unum_ops_b200.load()
    return torch.device("cuda", 0)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _round128(max_k):
    return (max_k + 127) // 128 * 128


def _batch(seed, dev, B=24, hq=32, hk=2, ctx_lo=300, ctx_hi=9000, q_per_seq=None, extra_tokens=0,
           same_keys=False, table_w=256):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi, size=B)
    k_lens = np.maximum((ctx - 32) // 16 + 1, 0)
    q_lens = np.ones(B, np.int64) if q_per_seq is None else np.asarray(q_per_seq)
    T = int(q_lens.sum()) + extra_tokens
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(T, hq, 128, generator=g, device=dev).to(torch.bfloat16)
    if same_keys:  # every key of a head equal: equal scores, ties broken by block index
        row = torch.randn(1, hk, 128, generator=g, device=dev)
        k = row.expand(int(k_lens.sum()), hk, 128).contiguous().to(torch.bfloat16)
    else:
        k = torch.randn(int(k_lens.sum()), hk, 128, generator=g, device=dev).to(torch.bfloat16)
    table = rng.integers(0, 1 << 20, size=(B, table_w)).astype(np.int32)
    tb = np.concatenate([np.repeat(np.arange(B), q_lens), np.zeros(extra_tokens, np.int64)]).astype(np.int32)
    pos = np.concatenate([np.repeat(ctx, q_lens), np.full(extra_tokens, 5)]).astype(np.int32)
    return dict(q=q, k=k, cu_q=_t(cases.cu(q_lens), dev), cu_k=_t(cases.cu(k_lens), dev),
                max_k=int(max(k_lens.max(), 1)), table=_t(table, dev), tb=_t(tb, dev), pos=_t(pos, dev),
                seqlen=_t(ctx.astype(np.int32), dev), cache=_t((ctx - 1).astype(np.int32), dev),
                k_lens=k_lens, np_table=table, np_tb=tb, np_pos=pos, np_ctx=ctx)


def _chain(b, max_context_len, cache, init_blocks, local_blocks, K, seqlen=None, pos=None):
    """The unfused path: four separate kernels."""
    from unum_ops_b200 import topk_blocks
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1, max_pooling_1d_varlen
    from unum_ops_b200.sparse_kernel_extension import get_block_table_ref_torch

    scores = infllmv2_attn_stage1(b["q"], b["k"], None, b["cu_q"], b["cu_k"], max_seqlen_k=b["max_k"],
                                  causal=True)
    W = scores.shape[-1]
    n = b["cu_q"].numel() - 1
    cl = cache if cache is not None else torch.zeros(n, dtype=torch.int32, device=scores.device)
    pooled = max_pooling_1d_varlen(scores, b["cu_q"], b["cu_k"], cl, 16 * W, max_context_len,
                                   local_blocks, init_blocks, 64, 16)
    idx = topk_blocks(pooled, K)
    slots = get_block_table_ref_torch(idx, b["table"], b["tb"], b["pos"] if pos is None else pos,
                                      b["seqlen"] if seqlen is None else seqlen)
    return scores, pooled, idx, slots


def _fused(b, max_context_len, cache, init_blocks, local_blocks, K, return_scores=True, seqlen=None,
           pos=None):
    from unum_ops_b200.block_select import _block_select_decode, _decode_fusable

    assert _decode_fusable(b["q"], b["k"], b["cu_q"], b["max_k"], max_context_len, K, 64, 16)
    return _block_select_decode(b["q"], b["k"], b["cu_q"], b["cu_k"], b["max_k"], b["table"], b["tb"],
                                b["pos"] if pos is None else pos, b["seqlen"] if seqlen is None else seqlen,
                                max_context_len, cache, True, init_blocks, local_blocks, K, None,
                                return_scores)


def _assert_same(got, ref, scores=True):
    names = ["scores", "pooled", "topk_idx", "slots"]
    for name, a, r in zip(names, got, ref):
        if a is None:
            assert name == "scores" and not scores
            continue
        assert a.shape == r.shape, name
        assert torch.equal(a, r), f"{name} differs at {int((a != r).sum())} positions"


@pytest.fixture(params=["pairs", "hybrid", "single"])
def cta_mode(request, monkeypatch):
    """Every form of the decode kernel: items shared by CTA pairs (a cluster of two), pairs
    that share the first 5 items and give later ones to one CTA each, and one CTA per item
    (UNUM_DECODE_PAIRS / UNUM_DECODE_JOINT_ITEMS force the choice, read at every launch)."""
    monkeypatch.setenv("UNUM_DECODE_PAIRS", "0" if request.param == "single" else "1")
    if request.param == "hybrid":
        monkeypatch.setenv("UNUM_DECODE_JOINT_ITEMS", "5")
    else:
        monkeypatch.delenv("UNUM_DECODE_JOINT_ITEMS", raising=False)
    return request.param


@pytest.mark.parametrize("hq", [32, 64])
@pytest.mark.parametrize("with_cache", [True, False])
@pytest.mark.parametrize("K", [64, 16])
def test_fused_decode_equals_chain(hq, with_cache, K, dev, cta_mode):
    b = _batch(100 + hq + K, dev, hq=hq)
    W = _round128(b["max_k"])
    ctx_max = min(16384 if hq == 32 else 8192, 16 * W)  # 4 * NB <= W
    cache = b["cache"] if with_cache else None
    got = _fused(b, ctx_max, cache, 1, 2, K)
    ref = _chain(b, ctx_max, cache, 1, 2, K)
    _assert_same(got, ref)


def test_fused_decode_without_scores(dev):
    b = _batch(7, dev)
    W = _round128(b["max_k"])
    got = _fused(b, 16 * W, b["cache"], 1, 2, 64, return_scores=False)
    ref = _chain(b, 16 * W, b["cache"], 1, 2, 64)
    assert got[0] is None
    _assert_same(got, ref, scores=False)


def test_fused_decode_edge_rows(dev, cta_mode):
    """Tokens outside every sequence, empty sequences, two-token sequences, sequences
    with no compressed key, fewer candidates than K (-1 padding), K above NB."""
    q_per = np.array([1, 0, 2, 1, 1, 0, 2, 1, 1, 1, 2, 1])
    b = _batch(11, dev, B=12, q_per_seq=q_per, extra_tokens=3, ctx_lo=20, ctx_hi=3000)
    W = _round128(b["max_k"])
    for init_blocks, local_blocks, K, ctx_max in [(1, 2, 64, 16 * W), (0, -1, 64, 16 * W), (3, 0, 200, 4 * W),
                                                    (1, 2, 7, 64 * (W // 4))]:
        for cache in (b["cache"], None):
            got = _fused(b, ctx_max, cache, init_blocks, local_blocks, K)
            ref = _chain(b, ctx_max, cache, init_blocks, local_blocks, K)
            _assert_same(got, ref)


def test_fused_decode_ties_and_scalar_maps(dev, cta_mode):
    """Equal keys give equal scores inside a row (ties ranked by block index), and a
    scalar token_pos_in_bs / seqlen_q broadcast like the reference's numel()==1 case."""
    b = _batch(13, dev, same_keys=True)
    W = _round128(b["max_k"])
    pos = torch.tensor([2000], dtype=torch.int32, device=dev)
    sl = torch.tensor([4000], dtype=torch.int32, device=dev)
    got = _fused(b, 16 * W, b["cache"], 1, 2, 64, seqlen=sl, pos=pos)
    ref = _chain(b, 16 * W, b["cache"], 1, 2, 64, seqlen=sl, pos=pos)
    _assert_same(got, ref)


def test_fused_decode_vs_oracle(dev, oracle_lib, cta_mode):
    """Downstream of the GPU's own stage-1 scores, the fused pooled blocks, ids and slots
    equal the C oracle's pooling, top-k and get_block_table; the scores themselves are
    within the fp32 oracle's tolerance."""
    b = _batch(17, dev, B=16, q_per_seq=[1, 2, 1, 1, 1, 1, 2, 1, 1, 1, 1, 1, 1, 2, 1, 1])
    W = _round128(b["max_k"])
    ctx_max = 16 * W
    scores, pooled, idx, slots = _fused(b, ctx_max, b["cache"], 1, 2, 64)
    torch.cuda.synchronize()
    sc = scores.float().cpu().numpy()
    cu_q = b["cu_q"].cpu().numpy()
    cu_k = b["cu_k"].cpu().numpy()
    pr = oracle_lib.max_pool(sc, cu_q, cu_k, b["cache"].cpu().numpy(), 16 * W, ctx_max, 2, 1)
    np.testing.assert_array_equal(pooled.float().cpu().numpy(), pr)
    ir = oracle_lib.topk(pr, 64)
    np.testing.assert_array_equal(idx.cpu().numpy(), ir)
    sr = oracle_lib.get_block_table(ir, b["np_table"], b["np_tb"], b["np_pos"], b["np_ctx"].astype(np.int32))
    np.testing.assert_array_equal(slots.cpu().numpy(), sr)
    orc = oracle_lib.stage1(b["q"].float().cpu().numpy(), b["k"].float().cpu().numpy(), cu_q, cu_k, True,
                            out_stride=W)
    np.testing.assert_allclose(sc, orc, atol=1e-3, rtol=1e-2)


def test_block_select_routes_decode_batches(dev):
    """block_select on a decode batch takes the fused path and gives the chain's results."""
    from unum_ops_b200 import block_select

    b = _batch(19, dev)
    W = _round128(b["max_k"])
    got = block_select(b["q"], b["k"], b["cu_q"], b["cu_k"], b["max_k"], b["table"], b["tb"], b["pos"],
                       b["seqlen"], max_context_len=16 * W, cache_lens=b["cache"])
    ref = _chain(b, 16 * W, b["cache"], 1, 2, 64)
    _assert_same(got, ref)


def test_pairs_match_single_cta_within_tolerance(dev, oracle_lib, monkeypatch):
    """The CTA-pair kernel sums each head's statistics in two halves, so its scores may
    differ from the one-CTA kernel's in the last bits only: both within the oracle's
    tolerance, and close to each other.  Covers items with one tile (the peer holds none)
    and rows longer than one CTA's tensor memory holds (out_stride below the keys)."""
    from unum_ops_b200.infllm_v2 import infllmv2_attn_stage1

    b = _batch(23, dev, B=20, ctx_lo=20, ctx_hi=60000)
    for mk in (b["max_k"], 1024):
        outs = {}
        for mode, jt in (("1", "999"), ("1", "8"), ("0", "0")):
            monkeypatch.setenv("UNUM_DECODE_PAIRS", mode)
            monkeypatch.setenv("UNUM_DECODE_JOINT_ITEMS", jt)
            outs[mode + jt] = infllmv2_attn_stage1(b["q"], b["k"], None, b["cu_q"], b["cu_k"],
                                                   max_seqlen_k=mk, causal=True).float()
        torch.cuda.synchronize()
        torch.testing.assert_close(outs["1999"], outs["00"], atol=1e-3, rtol=1e-2)
        torch.testing.assert_close(outs["18"], outs["00"], atol=1e-3, rtol=1e-2)
        orc = oracle_lib.stage1(b["q"].float().cpu().numpy(), b["k"].float().cpu().numpy(),
                                b["cu_q"].cpu().numpy(), b["cu_k"].cpu().numpy(), True,
                                out_stride=outs["1999"].shape[-1])
        for key in ("1999", "18"):
            np.testing.assert_allclose(outs[key].cpu().numpy(), orc, atol=1e-3, rtol=1e-2)
