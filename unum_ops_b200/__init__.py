"""unum_ops_b200: B200-native (sm_100a) InfLLM-v2 block selection.

Drop-in for the hot path of Yanguan619/unum_ops:
  unum_ops_b200.infllm_v2               <- unum_ops.infllm_v2
  unum_ops_b200.sparse_kernel_extension <- unum_ops.sparse_kernel_extension
plus unum_ops_b200.block_select (top-k and the chained pipeline) and
unum_ops_b200.sparse_attention (the stage-2 consumer, gather fused in).
Kernels live in libunum_ops_b200.so (C ABI: include/unum_ops_b200.h).
"""
from . import infllm_v2, sparse_kernel_extension  # noqa: F401
from .compress import compress_keys  # noqa: F401
from .sparse_attention import sparse_attention  # noqa: F401
from .block_select import (BlockSelectGraph, block_select, block_select_rows, block_select_streamed,  # noqa: F401
                           get_block_table_shard, topk_blocks)
from ._build import build  # noqa: F401
from ._lib import library_path, load  # noqa: F401

__all__ = ["infllm_v2", "sparse_kernel_extension", "compress_keys", "sparse_attention", "block_select", "BlockSelectGraph", "block_select_rows",
           "block_select_streamed", "get_block_table_shard", "topk_blocks", "build",
           "load", "library_path"]
