"""CPU-side checks of the C ABI: the library builds, loads and exports every
entry point the public header declares; argument errors come back as codes
and messages without touching a GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "unum_ops_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(unum_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    import unum_ops_b200

    unum_ops_b200.build()
    return unum_ops_b200.load()


def test_header_symbols_exported(lib):
    names = _header_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), n


def test_binding_covers_header():
    from unum_ops_b200 import _lib

    assert sorted(_lib.SIGNATURES) == _header_functions()


def test_abi_and_workspace(lib):
    assert lib.unum_abi_version() == 102
    assert lib.unum_stage1_workspace_size(0) >= 20
    assert lib.unum_stage1_workspace_size(1000) >= 4 * 1005
    assert lib.unum_stage1_workspace_size(1000) % 16 == 0


def test_invalid_arguments_report_errors(lib):
    rc = lib.unum_get_block_table(None, -1, 1, 1, 1, 1, 1, None, 1, 1, 1, None, None, 0, None, 0, 2,
                                  None, None)
    assert rc == -1
    assert b"negative" in lib.unum_last_error()
    rc = lib.unum_max_pooling_1d_varlen(None, 1, 1, 1, 1, None, None, None, 1, 16, 64, 2, 1, 0, 16,
                                        None, None)
    assert rc == -1
    rc = lib.unum_topk_blocks(None, 1, 4, 5000, 5000, 64, ctypes.c_void_p(256), None)
    assert rc == -1 and b"NB" in lib.unum_last_error()
    # stage 1: unsupported head_dim and head group are reported before any launch
    rc = lib.unum_infllmv2_attn_stage1(None, 8, 32, 64, 0, 0, None, 8, 2, 0, 0, None, None, 1,
                                       ctypes.c_float(0.1), 1, None, 128, None, 0, None)
    assert rc == -2
    rc = lib.unum_infllmv2_attn_stage1(None, 8, 48, 128, 0, 0, None, 8, 1, 0, 0, None, None, 1,
                                       ctypes.c_float(0.1), 1, None, 128, None, 0, None)
    assert rc == -2 and b"group" in lib.unum_last_error()
    # zero-size work is a no-op
    assert lib.unum_get_block_table(None, 2, 0, 64, 1, 1, 1, None, 1, 1, 1, None, None, 0, None, 0,
                                    2, None, None) == 0


def test_python_api_rejects_cpu_tensors():
    import torch

    from unum_ops_b200 import sparse_kernel_extension as ske

    t = torch.zeros(2, 3, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        ske.get_block_table_ref_torch(t, torch.zeros(1, 8, dtype=torch.int32),
                                      torch.zeros(3, dtype=torch.int32),
                                      torch.zeros(3, dtype=torch.int32), torch.zeros(1, dtype=torch.int32))


def test_public_names_match_reference():
    import unum_ops_b200.infllm_v2 as iv
    import unum_ops_b200.sparse_kernel_extension as ske

    assert set(iv.__all__) == {"infllmv2_attn_stage1", "infllmv2_attn_stage1_triton",
                               "infllmv2_attn_stage1_triton_v2", "max_pooling_1d_varlen",
                               "max_pooling_1d_varlen_ref_triton"}
    assert set(ske.__all__) == {"get_block_table_ref_torch", "get_block_table_ref_triton",
                                "get_block_table_ref_triton_v2", "get_block_table_ref_triton_v3",
                                "get_block_table_v2", "get_block_table_v3"}


def test_decode_fusion_routing():
    """block_select takes the one-launch decode path exactly for the shapes the fused
    kernel supports: a head group of 16 or 32, head_dim 128, 64-token blocks of stride-16
    compressed keys, at most 4 query tokens per sequence, each row within tensor memory
    (W <= 128*512/G) and every pooling window inside the row (4*NB <= W)."""
    import torch

    from unum_ops_b200.block_select import _decode_fusable

    def case(T=8, hq=32, hk=2, d=128, n_seq=8, tk=100, max_k=1000, ctx=16000, topk=64, bs=64, st=16):
        q = torch.empty(T, hq, d)
        k = torch.empty(tk, hk, d)
        cu_q = torch.zeros(n_seq + 1, dtype=torch.int32)
        return _decode_fusable(q, k, cu_q, max_k, ctx, topk, bs, st)

    assert case()                               # W = 1024, NB = 250: 4*NB <= W
    assert case(hq=64, max_k=2000, ctx=32000)   # G = 32: W = 2048 is the largest row
    assert not case(hq=64, max_k=2100, ctx=32000)  # W = 2176 > 128*512/32
    assert not case(hq=16)                      # G = 8
    assert not case(d=64)
    assert not case(T=40, n_seq=8)              # 5 query tokens per sequence: prefill-like
    assert not case(ctx=17000)                  # NB = 266: a window past the 1024-wide row
    assert not case(tk=0)
    assert not case(topk=1025)
    assert not case(bs=32)
    assert not case(T=0)
