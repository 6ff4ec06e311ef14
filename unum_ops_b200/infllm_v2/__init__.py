"""InfLLM-v2 stage-1 scores and block max-pooling on B200.

Drop-in for ``unum_ops.infllm_v2`` (reference: src/unum_ops/infllm_v2/__init__.py:1-17):
the same public names and signatures, computed by the sm_100a kernels of
``libunum_ops_b200.so``.
"""
from __future__ import annotations

import math

import torch

from .. import _lib

__all__ = [
    "infllmv2_attn_stage1",
    "infllmv2_attn_stage1_triton",
    "infllmv2_attn_stage1_triton_v2",
    "max_pooling_1d_varlen",
    "max_pooling_1d_varlen_ref_triton",
]


def _round_multiple(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _as_i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


_WORKSPACES: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device, per-stream scratch for the stage-1 tile schedule (grows, never shrinks)."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def infllmv2_attn_stage1(
    q,
    k,
    v,
    cu_seqlens_q,
    cu_seqlens_k,
    cu_seqlens_v=None,
    max_seqlen_q=None,
    max_seqlen_k=None,
    dropout_p=0.0,
    softmax_scale=None,
    causal=False,
    window_size=(-1, -1),
    softcap=0.0,
    alibi_slopes=None,
    deterministic=False,
    return_attn_probs=True,
    block_table=None,
):
    """Stage-1 compressed attention scores summed per kv-head group.

    Mirrors infllmv2_attn_stage1_triton_v2 (infllmv2_attn_stage1_triton_v2.py:153-228):
    q [total_q, n_heads, head_dim], k [total_k, n_kv_heads, head_dim] (cast to bf16
    like the reference kernel's loads), int32 cu_seqlens; returns bf16
    [n_kv_heads, total_q, round_up(max_seqlen_k, 128)].  ``v`` and the
    flash-attn-style extra arguments are accepted and ignored, as in the reference.

    The call is asynchronous.  Every row is written by the kernels; the one failure
    they can report is a bounded wait inside the kernel that gave up (about a second
    without progress), which leaves the output invalid: callers that must detect it
    read ``stage1_status()`` (nonzero) after the call, which synchronises the stream.
    """
    dev = _lib.require_cuda(q, k, cu_seqlens_q, cu_seqlens_k)
    q, k = [x.contiguous() if x.stride(-1) != 1 else x for x in (q, k)]
    if q.dtype != torch.bfloat16:
        q = q.to(torch.bfloat16)
    if k.dtype != torch.bfloat16:
        k = k.to(torch.bfloat16)
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** (-0.5)
    total_q, n_heads, head_dim = q.shape
    total_k, n_kv_heads = k.shape[0], k.shape[1]
    if k.shape[2] != head_dim:
        raise ValueError(f"q and k head_dim differ: {head_dim} vs {k.shape[2]}")
    batch_size = cu_seqlens_q.numel() - 1
    cu_q = _as_i32(cu_seqlens_q)
    cu_k = _as_i32(cu_seqlens_k)
    if max_seqlen_k is None or max_seqlen_k == 0:
        # one device->host read (the reference loops over int(tensor) per sequence, :199-200)
        max_seqlen_k = int((cu_k[1:] - cu_k[:-1]).max().item()) if batch_size > 0 else 0
    max_k_rounded = _round_multiple(int(max_seqlen_k), 128) if max_seqlen_k > 0 else 0
    out = torch.empty(n_kv_heads, total_q, max_k_rounded, device=dev, dtype=torch.bfloat16)
    if max_k_rounded == 0 or total_q == 0:
        return out
    L = _lib.load()
    nbytes = int(L.unum_stage1_workspace_size(batch_size))
    ws = _workspace(dev, nbytes)
    with torch.cuda.device(dev):
        rc = L.unum_infllmv2_attn_stage1(
            q.data_ptr(), total_q, n_heads, head_dim, q.stride(0), q.stride(1),
            k.data_ptr(), total_k, n_kv_heads, k.stride(0), k.stride(1),
            cu_q.data_ptr(), cu_k.data_ptr(), batch_size, float(softmax_scale), int(bool(causal)),
            out.data_ptr(), max_k_rounded, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return out


# The reference exports three names for the same computation (__init__.py:1-5).
infllmv2_attn_stage1_triton = infllmv2_attn_stage1
infllmv2_attn_stage1_triton_v2 = infllmv2_attn_stage1


def stage1_status(device=None) -> int:
    """Status word of the last stage-1 launch on the current stream (0 = ok)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None:
        return 0
    import ctypes

    st = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().unum_stage1_status(ws.data_ptr(), _lib.stream_ptr(dev), ctypes.byref(st)))
    return int(st.value)


def max_pooling_1d_varlen(
    input: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    cache_lens: torch.Tensor,
    max_seqlen_q: int,
    max_context_len: int,
    local_blocks: int,
    init_blocks: int,
    block_size: int = 64,
    stride: int = 16,
    total_q: int = -1,
) -> torch.Tensor:
    """Compressed scores -> block scores, as max_pooling_1d_varlen_ref_triton
    (max_pooling_1d_varlen.py:127-183): input [H, total_q, *] read as a flat buffer with
    row stride max_seqlen_q // stride; returns input.dtype [H, total_q, ceil(max_context_len/block_size)].
    ``total_q`` is accepted and ignored, as in the reference (which uses input.shape[1])."""
    dev = _lib.require_cuda(input, cu_seqlens_q, cu_seqlens_k, cache_lens)
    if input.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported score dtype {input.dtype}")
    x = input.contiguous()
    num_heads, T = x.shape[0], x.shape[1]
    batch_size = cu_seqlens_q.shape[0] - 1
    max_blocks = math.ceil(max_context_len / block_size)
    out = torch.empty(num_heads, T, max_blocks, dtype=x.dtype, device=dev)
    if out.numel() == 0:
        return out
    cu_q, cu_k, cl = _as_i32(cu_seqlens_q), _as_i32(cu_seqlens_k), _as_i32(cache_lens)
    with torch.cuda.device(dev):
        rc = _lib.load().unum_max_pooling_1d_varlen(
            x.data_ptr(), _lib.DTYPE_CODES[x.dtype], num_heads, T, x.numel(), cu_q.data_ptr(),
            cu_k.data_ptr(), cl.data_ptr(), batch_size, int(max_seqlen_q), int(max_context_len),
            int(local_blocks), int(init_blocks), int(block_size), int(stride), out.data_ptr(),
            _lib.stream_ptr(dev))
    _lib.check(rc)
    return out


max_pooling_1d_varlen_ref_triton = max_pooling_1d_varlen
