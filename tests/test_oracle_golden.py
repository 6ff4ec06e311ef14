"""Pin the CPU oracle against outputs of the reference implementation.

The fixtures under tests/golden/ were produced by make_golden.py, which runs
the reference's own torch functions and Triton kernels (interpreter) on the
inputs that cases.py regenerates here.
"""
import numpy as np
import pytest

import cases

ATOL, RTOL = 1e-3, 1e-2  # stage-1 tolerance for bf16 inputs (fp32 accumulation)


def _npz(name):
    import os

    return np.load(os.path.join(os.path.dirname(cases.__file__), name))


def _bf16_to_f32(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("c", cases.gbt_cases(), ids=lambda c: c["name"])
def test_gbt_oracle_matches_reference(c, oracle_lib):
    g = _npz("gbt.npz")
    assert str(g[c["name"] + "/digest"]) == cases.digest(c["topk"], c["table"], c["token_to_bs"],
                                                         c["pos"], c["seqlen"])
    out = oracle_lib.get_block_table(c["topk"], c["table"], c["token_to_bs"], c["pos"], c["seqlen"])
    np.testing.assert_array_equal(out, g[c["name"] + "/out"])


@pytest.mark.parametrize("c", cases.pool_cases(), ids=lambda c: c["name"])
def test_pool_oracle_matches_reference(c, oracle_lib):
    g = _npz("pool.npz")
    assert str(g[c["name"] + "/digest"]) == cases.digest(c["x"], c["cu_q"], c["cu_k"], c["cache_lens"])
    out = oracle_lib.max_pool(c["x"], c["cu_q"], c["cu_k"], c["cache_lens"], c["max_seqlen_q"],
                              c["max_context_len"], c["local_blocks"], c["init_blocks"],
                              c["block_size"], c["stride"])
    np.testing.assert_array_equal(out, g[c["name"] + "/out"])


@pytest.mark.parametrize("c", cases.stage1_cases(), ids=lambda c: c["name"])
def test_stage1_oracle_matches_reference(c, oracle_lib):
    g = _npz("stage1.npz")
    assert str(g[c["name"] + "/digest"]) == cases.digest(c["q"], c["k"], c["cu_q"], c["cu_k"])
    ref = _bf16_to_f32(g[c["name"] + "/out_bf16"])
    out = oracle_lib.stage1(c["q"], c["k"], c["cu_q"], c["cu_k"], c["causal"])
    assert out.shape == ref.shape
    # the reference stores bf16: compare the oracle rounded the same way, and
    # the unrounded oracle within the stage-1 tolerance
    np.testing.assert_allclose(cases.bf16_round(out), ref, atol=2e-3, rtol=8e-3)
    np.testing.assert_allclose(ref, out, atol=ATOL, rtol=RTOL)
    # zero pattern (masked / out-of-range / empty rows) is identical
    np.testing.assert_array_equal(out == 0, ref == 0)
    key = c["name"] + "/torchref_bf16"
    if key in g:
        np.testing.assert_allclose(_bf16_to_f32(g[key]), out, atol=ATOL, rtol=RTOL)


def _topk_numpy(x, K):
    out = np.full(x.shape[:-1] + (K,), -1, np.int32)
    flat = x.reshape(-1, x.shape[-1])
    of = out.reshape(-1, K)
    for r in range(flat.shape[0]):
        row = flat[r]
        cand = np.nonzero(~(np.isnan(row) | (row == -np.inf)))[0]
        order = cand[np.lexsort((cand, -row[cand]))]
        keep = np.sort(order[:K])
        of[r, :len(keep)] = keep
    return out


@pytest.mark.parametrize("kw", [
    dict(rows=64, NB=16, K=64), dict(rows=64, NB=300, K=64), dict(rows=32, NB=2048, K=64, ties=True),
    dict(rows=32, NB=1024, K=64, inf_frac=0.01, neginf_frac=0.5), dict(rows=8, NB=100, K=7, ties=True),
    dict(rows=8, NB=64, K=64, neginf_frac=0.3),
], ids=lambda kw: "-".join(f"{k}{v}" for k, v in kw.items()))
def test_topk_oracle_definition(kw, oracle_lib):
    c = cases.topk_case("t", 7, **kw)
    np.testing.assert_array_equal(oracle_lib.topk(c["x"], c["K"]), _topk_numpy(c["x"], c["K"]))


def test_causal_visible_rule(oracle_lib):
    # prefill with k_len = (L-32)/16+1: key j visible iff 16 j + 31 <= local_q
    for L in (32, 48, 1024):
        k_len = cases.compressed_len(L)
        for lq in range(L):
            vis = oracle_lib.stage1_visible(lq, L, k_len, True)
            expect = sum(1 for j in range(k_len) if 16 * j + 31 <= lq)
            assert vis == expect, (L, lq)
    # decode: everything visible
    assert oracle_lib.stage1_visible(0, 1, 777, True) == 777
    # truncating division: chunked prefill q_len=64, k_len=40, local_q=0
    assert oracle_lib.stage1_visible(0, 64, 40, True) == 37


@pytest.mark.parametrize("c", cases.gbt_cases(), ids=lambda c: c["name"])
def test_gbt_torch_restatement_matches_reference(c):
    """The torch restatement the reference arm of bench.py times (oracle/torch_ref.py)
    equals the reference's get_block_table_ref_torch outputs."""
    import torch

    from oracle import torch_ref

    g = _npz("gbt.npz")
    args = [torch.from_numpy(np.ascontiguousarray(x)) for x in
            (c["topk"], c["table"], c["token_to_bs"], c["pos"], c["seqlen"])]
    np.testing.assert_array_equal(torch_ref.get_block_table(*args).numpy(), g[c["name"] + "/out"])


def test_topk_torch_restatement_matches_oracle(oracle_lib):
    """torch.topk + ascending sort (the reference caller's step, as bench.py's reference arm
    times it) selects the same blocks as the oracle rule on rows without ties."""
    import torch

    from oracle import torch_ref

    rng = np.random.default_rng(3)
    p = rng.standard_normal((2, 64, 512)).astype(np.float32)
    p[:, :, 400:] = -np.inf
    p[0, :3, 10:] = -np.inf  # rows with fewer candidates than K
    np.testing.assert_array_equal(torch_ref.topk(torch.from_numpy(p), 64).numpy(), oracle_lib.topk(p, 64))
