"""Seeded input generators shared by the golden-fixture script and the tests.

Every case is a plain dict of numpy arrays plus scalar parameters, built from
``np.random.default_rng(seed)``.  The fixture files store the reference's
outputs together with a SHA-256 of the generated inputs, so a test can rebuild
the inputs here and detect any drift of the generator.

bf16 tensors are carried as float32 arrays whose values are exactly
representable in bf16 (round-to-nearest-even), so the same arrays feed the
fp32 oracle and, cast with ``torch.bfloat16``, the GPU kernels.
"""
from __future__ import annotations

import hashlib

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def cu(lens) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(np.asarray(lens, dtype=np.int64))]).astype(np.int32)


# --------------------------------------------------------------------------
# stage 1
# --------------------------------------------------------------------------
def stage1_case(name, seed, q_lens, k_lens, hq, hk, causal, d=128):
    rng = np.random.default_rng(seed)
    T, Tk = int(sum(q_lens)), int(sum(k_lens))
    q = bf16_round(rng.standard_normal((T, hq, d), dtype=np.float32))
    k = bf16_round(rng.standard_normal((Tk, hk, d), dtype=np.float32))
    return dict(name=name, q=q, k=k, cu_q=cu(q_lens), cu_k=cu(k_lens), causal=bool(causal),
                max_seqlen_q=int(max(q_lens)), max_seqlen_k=int(max(k_lens)))


def compressed_len(L: int) -> int:
    """Compressed keys of an L-token prefix: kernel 32, stride 16."""
    return max(0, (L - 32) // 16 + 1)


def stage1_cases():
    c = []
    # The reference's own non-causal comparison grid (32 q-heads / 2 kv-heads).
    for sq in (64, 256):
        for sk in (15, 16, 128):
            c.append(stage1_case(f"nc_q{sq}_k{sk}", 100 + sq + sk, [sq], [sk], 32, 2, False))
    # Causal prefill, k_len = compressed_len(L).
    for L in (48, 160, 512):
        c.append(stage1_case(f"causal_L{L}", 200 + L, [L], [compressed_len(L)], 32, 2, True))
    # Varlen causal prefill with the BASELINE C0 head layout (16/2, group 8).
    c.append(stage1_case("causal_varlen_g8", 301, [96, 200, 33], [compressed_len(96),
                         compressed_len(200), compressed_len(33)], 16, 2, True))
    # Chunked prefill: fewer queries than the context behind them.
    c.append(stage1_case("causal_chunk_q64_k40", 302, [64], [40], 32, 2, True))
    c.append(stage1_case("causal_chunk_q7_k300", 303, [7, 50], [300, 9], 32, 2, True))
    # Decode: one query per sequence, every key visible.
    c.append(stage1_case("decode_b5", 304, [1] * 5, [3, 129, 256, 1, 70], 32, 2, True))
    # A sequence with no compressed keys at all.
    c.append(stage1_case("empty_k", 305, [20, 40], [0, 5], 32, 2, True))
    return c


# --------------------------------------------------------------------------
# max_pooling_1d_varlen
# --------------------------------------------------------------------------
def pool_case(name, seed, H, q_lens, k_lens, row_len, max_seqlen_q, max_context_len,
              local_blocks, init_blocks, cache=None, block_size=64, stride=16, inf_frac=0.0):
    rng = np.random.default_rng(seed)
    T = int(sum(q_lens))
    x = bf16_round(rng.standard_normal((H, T, row_len), dtype=np.float32))
    if inf_frac:
        m = rng.random(x.shape) < inf_frac
        x[m] = -np.inf
    cache = np.zeros(len(q_lens), np.int32) if cache is None else np.asarray(cache, np.int32)
    return dict(name=name, x=x, cu_q=cu(q_lens), cu_k=cu(k_lens), cache_lens=cache,
                max_seqlen_q=int(max_seqlen_q), max_context_len=int(max_context_len),
                local_blocks=int(local_blocks), init_blocks=int(init_blocks),
                block_size=int(block_size), stride=int(stride))


def pool_cases():
    c = []
    # The reference's test grid shape: seqlen_q = 8+8i, seqlen_k = 16+8i, input
    # [H, total_q, max_k], max_seqlen_q = max(q lens), local 32, init 1.
    for H in (4, 8):
        for B in (1, 2, 4):
            ql = [8 + 8 * i for i in range(B)]
            kl = [16 + 8 * i for i in range(B)]
            c.append(pool_case(f"reftest_h{H}_b{B}", 400 + 10 * H + B, H, ql, kl, max(kl),
                               max(ql), max(ql), 32, 1))
    # The reference's correctness shape (local 4, max_context_len = max k).
    c.append(pool_case("refcorrect", 420, 4, [8, 12], [16, 20], 20, 12, 20, 4, 1))
    # Pipeline layout: stage-1 rows of width W, max_seqlen_q = 16 * W so the
    # flat stride equals the real row length.
    for (ql, kl, W, ctx, loc, ini, cache) in [
        ([300], [17], 128, 300, 2, 1, None),
        ([200, 333, 64], [11, 19, 3], 128, 333, 2, 1, None),
        ([130, 70], [40, 70], 128, 1400, 3, 2, [600, 10]),
        ([1, 1, 1, 1], [100, 255, 7, 256], 256, 4096, 2, 1, None),
    ]:
        c.append(pool_case(f"pipe_{len(ql)}seq_w{W}", 430 + len(c), 2, ql, kl, W, 16 * W,
                           ctx, loc, ini, cache))
    c.append(pool_case("pipe_neginf", 450, 2, [256], [120], 128, 16 * 128, 256 * 8, 1, 1,
                       inf_frac=0.2))
    return c


# --------------------------------------------------------------------------
# get_block_table
# --------------------------------------------------------------------------
def gbt_case(name, seed, B, seq, K, H=2, width=None, neg_frac=0.0, pos_mode="seqlen",
             scalar_seqlen=False, tokens_per_seq=1):
    """Decode-style inputs shaped like the reference's own test grid
    (sorted unique top-k block ids, table values in [1, 10000), seqlen_q a
    random multiple of 64), widened with padding, per-token limits and a
    table narrower than the positions (the clamp path)."""
    rng = np.random.default_rng(seed)
    nblk = seq // 64
    T = B * tokens_per_seq
    topk = np.zeros((H, T, K), np.int32)
    kk = min(K, nblk)
    for h in range(H):
        for t in range(T):
            sel = np.sort(rng.permutation(nblk)[:kk])
            topk[h, t, :kk] = sel
    if neg_frac:
        topk[rng.random(topk.shape) < neg_frac] = -1
    L = seq if width is None else width
    table = rng.integers(1, 10000, size=(B, L), dtype=np.int32)
    token_to_bs = np.repeat(np.arange(B, dtype=np.int32), tokens_per_seq)
    seqlen = (rng.integers(max(1, nblk // 4), nblk + 1, size=B) * 64).astype(np.int32)
    if scalar_seqlen:
        seqlen = np.array([seq], np.int32)
    if pos_mode == "seqlen":
        pos = seqlen[token_to_bs] if seqlen.size > 1 else np.full(T, seqlen[0], np.int32)
    elif pos_mode == "causal":
        pos = rng.integers(1, seq + 1, size=T).astype(np.int32)
    else:  # scalar
        pos = np.array([seq // 2 + 5], np.int32)
    return dict(name=name, topk=topk, table=table, token_to_bs=token_to_bs,
                pos=np.ascontiguousarray(pos, np.int32), seqlen=seqlen, K=K)


def gbt_cases():
    c = []
    for i, (B, seq, K) in enumerate([(1, 256, 4), (2, 512, 8), (4, 1024, 16), (8, 2048, 32),
                                     (4, 4096, 64), (2, 8192, 96)]):
        c.append(gbt_case(f"reftest_b{B}_s{seq}_k{K}", 500 + i, B, seq, K))
    c.append(gbt_case("neg_pad", 510, 4, 2048, 64, neg_frac=0.1))
    c.append(gbt_case("causal_pos", 511, 3, 1024, 16, pos_mode="causal", tokens_per_seq=5))
    c.append(gbt_case("scalar_pos_seqlen", 512, 3, 1024, 16, pos_mode="scalar",
                      scalar_seqlen=True))
    c.append(gbt_case("clamp_width", 513, 2, 4096, 64, width=2048, scalar_seqlen=True,
                      neg_frac=0.1))
    c.append(gbt_case("odd_width", 514, 3, 1024, 8, width=1021, neg_frac=0.05))
    return c


# --------------------------------------------------------------------------
# top-k (no reference implementation; cases for the oracle and the kernel)
# --------------------------------------------------------------------------
def topk_case(name, seed, rows, NB, K, ties=False, inf_frac=0.0, neginf_frac=0.0):
    rng = np.random.default_rng(seed)
    if ties:
        x = rng.integers(0, 8, size=(rows, NB)).astype(np.float32) / 4
    else:
        x = bf16_round(rng.standard_normal((rows, NB), dtype=np.float32))
    if inf_frac:
        x[rng.random(x.shape) < inf_frac] = np.inf
    if neginf_frac:
        x[rng.random(x.shape) < neginf_frac] = -np.inf
    return dict(name=name, x=x, K=K)
