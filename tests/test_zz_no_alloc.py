"""The allocation-free stage-1 entry point (unum_infllmv2_attn_stage1_noalloc).

Callers such as an engine whose allocator already owns all of HBM, or a plugin
host that forbids cudaMalloc inside its callbacks, cannot hand stage 1 a
workspace.  This entry point keeps its schedule scratch in a fixed array
inside the library instead.  The test calls it through the C ABI, twice in a
row with different batches (so the second call runs on scratch the first one
left behind), and checks each result against the workspace entry point on the
same inputs, and that the status word it leaves in the library's scratch
(read with unum_stage1_noalloc_status) is 0.  The batches cover the tile
kernel, the decode kernel (whose work counter also lives in the scratch) and
the largest accepted batch, whose schedule fills the scratch array to its
last word.  It lives in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases

ATOL, RTOL = 1e-3, 1e-2


def _inputs(dev, seed, q_lens, hq=32, hk=2):
    k_lens = [cases.compressed_len(n) for n in q_lens]
    c = cases.stage1_case("noalloc", seed, q_lens, k_lens, hq, hk, True)
    q = torch.from_numpy(c["q"]).to(dev, torch.bfloat16)
    k = torch.from_numpy(c["k"]).to(dev, torch.bfloat16)
    cu_q = torch.from_numpy(c["cu_q"]).to(dev)
    cu_k = torch.from_numpy(c["cu_k"]).to(dev)
    W = (max(k_lens) + 127) // 128 * 128
    return q, k, cu_q, cu_k, len(q_lens), W


def _args(q, k, cu_q, cu_k, n_seq, out, W):
    return (q.data_ptr(), q.shape[0], q.shape[1], q.shape[2], q.stride(0), q.stride(1),
            k.data_ptr(), k.shape[0], k.shape[1], k.stride(0), k.stride(1),
            cu_q.data_ptr(), cu_k.data_ptr(), n_seq, ctypes.c_float(q.shape[2] ** -0.5), 1,
            out.data_ptr(), W)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200
    from unum_ops_b200 import _lib

    unum_ops_b200.build()
    L = unum_ops_b200.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed, q_lens in ((901, [700, 1300, 48]), (902, [2048])):
        q, k, cu_q, cu_k, n_seq, W = _inputs(dev, seed, q_lens)
        ref = torch.empty(2, q.shape[0], W, dtype=torch.bfloat16, device=dev)
        ws = torch.empty(L.unum_stage1_workspace_size(n_seq), dtype=torch.uint8, device=dev)
        _lib.check(L.unum_infllmv2_attn_stage1(*_args(q, k, cu_q, cu_k, n_seq, ref, W),
                                               ws.data_ptr(), ws.numel(), stream))
        got = torch.full_like(ref, float("nan"))
        _lib.check(L.unum_infllmv2_attn_stage1_noalloc(*_args(q, k, cu_q, cu_k, n_seq, got, W),
                                                       stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(),
                                   atol=ATOL, rtol=RTOL)
        assert _noalloc_status(L, stream) == 0


def _noalloc_status(L, stream):
    from unum_ops_b200 import _lib

    st = ctypes.c_int32(-1)
    _lib.check(L.unum_stage1_noalloc_status(stream, ctypes.byref(st)))
    return st.value


def _decode_batch(dev, seed, n_seq, ctx_lo, ctx_hi):
    """n_seq sequences of one query token each; contexts uniform in [ctx_lo, ctx_hi]."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (n_seq,), generator=g)
    k_lens = (ctx - 32) // 16 + 1
    cu_k = torch.zeros(n_seq + 1, dtype=torch.int32)
    cu_k[1:] = torch.cumsum(k_lens, 0)
    q = torch.randn(n_seq, 32, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(int(cu_k[-1]), 2, 128, generator=g).to(torch.bfloat16)
    cu_q = torch.arange(n_seq + 1, dtype=torch.int32)
    W = (int(k_lens.max()) + 127) // 128 * 128
    return q.to(dev), k.to(dev), cu_q.to(dev), cu_k.to(dev), n_seq, W


@pytest.mark.gpu
def test_noalloc_decode_and_largest_batch_back_to_back():
    """Decode-shaped batches (the decode kernel, whose work counter is scratch word 1)
    and a batch of exactly the largest accepted sequence count, back to back."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200
    from unum_ops_b200 import _lib

    L = unum_ops_b200.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed, n_seq, lo, hi in ((911, 2000, 64, 8192), (912, 1500, 1024, 4096), (913, 16379, 32, 600)):
        q, k, cu_q, cu_k, n, W = _decode_batch(dev, seed, n_seq, lo, hi)
        ref = torch.empty(2, q.shape[0], W, dtype=torch.bfloat16, device=dev)
        ws = torch.empty(L.unum_stage1_workspace_size(n), dtype=torch.uint8, device=dev)
        _lib.check(L.unum_infllmv2_attn_stage1(*_args(q, k, cu_q, cu_k, n, ref, W),
                                               ws.data_ptr(), ws.numel(), stream))
        got = torch.full_like(ref, float("nan"))
        _lib.check(L.unum_infllmv2_attn_stage1_noalloc(*_args(q, k, cu_q, cu_k, n, got, W), stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(),
                                   atol=ATOL, rtol=RTOL)
        assert _noalloc_status(L, stream) == 0


@pytest.mark.gpu
def test_noalloc_rejects_too_many_sequences():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200

    L = unum_ops_b200.load()
    rc = L.unum_infllmv2_attn_stage1_noalloc(None, 1, 32, 128, 4096, 128, None, 1, 2, 256, 128,
                                             None, None, 100000, ctypes.c_float(0.1), 1, None,
                                             128, None)
    assert rc == -1
    assert b"at most 16379 sequences" in L.unum_last_error()
