"""The allocation-free stage-1 entry point (unum_infllmv2_attn_stage1_noalloc).

Callers such as an engine whose allocator already owns all of HBM, or a plugin
host that forbids cudaMalloc inside its callbacks, cannot hand stage 1 a
workspace.  This entry point keeps its schedule scratch in a fixed array
inside the library instead.  The test calls it through the C ABI, twice in a
row with different batches (so the second call runs on scratch the first one
left behind), and checks each result against the workspace entry point on the
same inputs.  It lives in its own file, collected last.
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
