"""Key compression: the producer of stage 1's compressed keys (k_cmp).

The reference consumes k_cmp and leaves building it to its caller; its stage-1
kernel assumes one compressed key per 16 tokens, compressed key j covering
tokens [16j, 16j+32) (src/unum_ops/infllm_v2/infllmv2_attn_stage1_triton_v2.py:70).
``compress_keys`` makes it on the GPU: the mean of each 32-token window, fp32
sums in token order, rounded to bf16.
"""
from __future__ import annotations

import torch

from . import _lib
from .infllm_v2 import _as_i32

__all__ = ["compress_keys"]


def compress_keys(k, cu_seqlens, kernel_size=32, stride=16, cu_seqlens_host=None):
    """k bf16 [T, Hk, 128] (varlen, cu_seqlens [B+1]) -> (k_cmp bf16 [N, Hk, 128],
    cu_seqlens_k int32 [B+1]) with (L_b - kernel_size) // stride + 1 compressed keys per
    sequence (0 when L_b < kernel_size): the inputs ``infllmv2_attn_stage1`` takes.

    The output sizes come from the sequence lengths, read on the host: pass
    ``cu_seqlens_host`` (a CPU copy) to avoid a device-to-host read."""
    dev = _lib.require_cuda(k, cu_seqlens)
    kk = (k if k.stride(-1) == 1 else k.contiguous()).to(torch.bfloat16)
    T, Hk, D = kk.shape
    cu_h = (cu_seqlens_host if cu_seqlens_host is not None else cu_seqlens).to("cpu", torch.int64)
    L = cu_h[1:] - cu_h[:-1]
    n = torch.where(L >= kernel_size, (L - kernel_size) // stride + 1, torch.zeros_like(L))
    cu_out_h = torch.zeros(len(cu_h), dtype=torch.int32)
    cu_out_h[1:] = torch.cumsum(n, 0).to(torch.int32)
    cu_out = cu_out_h.to(dev, non_blocking=True)
    n_out = int(cu_out_h[-1])
    out = torch.empty(n_out, Hk, D, dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().unum_compress_keys(kk.data_ptr(), T, Hk, D, kk.stride(0), kk.stride(1),
                                            _as_i32(cu_seqlens).data_ptr(), cu_out.data_ptr(),
                                            len(cu_h) - 1, n_out, int(kernel_size), int(stride),
                                            out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc)
    return out, cu_out
