"""Stage-2 sparse attention over the selected blocks (the consumer of the path).

There is no reference implementation; the kernel is checked against the fp32
restatement in the oracle (oracle_sparse_attn), whose slot rule is the one of
the reference's get_block_table (get_table_torch.py:29-44) and which is checked
here against get_block_table's own slot ids.  Parity is unpinned beyond that rule.
"""
import numpy as np
import pytest
import torch

ATOL, RTOL = 4e-3, 2e-2  # bf16 inputs, bf16 probabilities and output


def _case(seed, B, ctx_lo, ctx_hi, tokens_per_seq, K, neg_frac=0.1, Hk=2):
    """Paged KV caches with a random permutation of physical tokens per sequence, top-K
    block ids (ascending, -1 padded) per (kv head, token), causal token limits."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=B)
    L = int(ctx.max())
    n_phys = int(ctx.sum()) + 64
    perm = rng.permutation(n_phys).astype(np.int32)
    table = np.zeros((B, L), np.int32)
    off = 0
    for b in range(B):
        n = int(ctx[b])
        table[b, :n] = perm[off:off + n]
        table[b, n:] = perm[rng.integers(0, n_phys, size=L - n)]
        off += n
    T = B * tokens_per_seq
    tb = np.repeat(np.arange(B, dtype=np.int32), tokens_per_seq)
    pos = np.concatenate([ctx[b] - np.arange(tokens_per_seq)[::-1] for b in range(B)]).astype(np.int32)
    topk = np.full((Hk, T, K), -1, np.int32)
    for g in range(Hk):
        for t in range(T):
            nblk = (int(pos[t]) + 63) // 64
            kk = min(K, nblk)
            sel = np.sort(rng.permutation(nblk)[:kk]).astype(np.int32)
            drop = rng.random(kk) < neg_frac
            topk[g, t, :kk] = np.concatenate([sel[~drop], np.full(int(drop.sum()), -1, np.int32)])
    q = rng.standard_normal((T, 16 * Hk, 128)).astype(np.float32)
    kc = rng.standard_normal((n_phys * 2, 128)).astype(np.float32)
    vc = rng.standard_normal((n_phys * 2, 128)).astype(np.float32)
    return q, kc, vc, topk, table, tb, pos, ctx.astype(np.int32)


@pytest.mark.gpu
@pytest.mark.parametrize("B,lo,hi,tps,K", [(6, 200, 5000, 1, 64), (3, 64, 700, 4, 16), (40, 4096, 9000, 1, 64),
                                           (2, 3000, 3000, 5, 7), (5, 1, 90, 2, 64)])
def test_sparse_attention_vs_oracle(B, lo, hi, tps, K, oracle_lib):
    from unum_ops_b200 import sparse_attention

    dev = torch.device("cuda", 0)
    q, kc, vc, topk, table, tb, pos, sl = _case(100 + B + K, B, lo, hi, tps, K)
    bf = lambda a: torch.from_numpy(a).to(dev, torch.bfloat16)  # noqa: E731
    i32 = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    out = sparse_attention(bf(q), bf(kc), bf(vc), i32(topk), i32(table), i32(tb), i32(pos), i32(sl), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    rnd = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy()  # noqa: E731
    ref = oracle_lib.sparse_attn(rnd(q), rnd(kc), rnd(vc), topk, table, tb, pos, sl)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_sparse_attention_oracle_uses_get_block_table_slots(oracle_lib):
    """The oracle's slot rule is get_block_table's: attending over the slot ids that
    oracle.get_block_table writes (where the rule marks them valid) gives the same output."""
    q, kc, vc, topk, table, tb, pos, sl = _case(7, 3, 100, 900, 2, 8)
    ref = oracle_lib.sparse_attn(q, kc, vc, topk, table, tb, pos, sl)
    slots = oracle_lib.get_block_table(topk, table, tb, pos, sl)  # [T, Hk, K*64]
    T, Hk, _ = slots.shape
    for t in range(T):
        for g in range(Hk):
            p = (topk[g, t][:, None] * 64 + np.arange(64)[None, :]).reshape(-1)
            valid = (np.repeat(topk[g, t], 64) >= 0) & (p < sl[tb[t]]) & (p < pos[t])
            sel = slots[t, g][valid]
            for hh in range(16):
                h = g * 16 + hh
                if sel.size == 0:
                    assert not ref[t, h].any()
                    continue
                s = kc[sel] @ q[t, h] / np.sqrt(128.0)
                w = np.exp(s - s.max())
                w /= w.sum()
                np.testing.assert_allclose(ref[t, h], w @ vc[sel], atol=1e-5, rtol=1e-4)
