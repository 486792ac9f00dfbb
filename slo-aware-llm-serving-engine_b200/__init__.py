"""B200-native (sm_100a) KV-cache hot path for the SLO-aware serving engine.

Drop-in replacements for the reference engine's paged KV append
(`store_kvcache`), paged decode / varlen attention (the two flash-attn entry
points), the `Attention` module with its `Context` metadata, the mixed
prefill/decode forward, and block-pool page copies.  All compute runs in the
hand-written kernels of libslokv.so (C ABI: include/slokv.h); nothing here falls
back to a CPU or library implementation.

The package directory name contains dashes, so import it with
`importlib.import_module("slo-aware-llm-serving-engine_b200")`.
"""
from . import _lib
from ._lib import SlokvError, read_device_errors
from .kvcache import (decode_workspace, e4m3_decode, e4m3_encode, flash_attn_varlen_func,
                      flash_attn_varlen_func_fp8, flash_attn_with_kvcache, flash_attn_with_kvcache_fp8, kv_block_copy,
                      kv_block_gather, kv_block_scatter, qk_norm_rope_append, store_kvcache,
                      store_kvcache_fp8)
from .layers.attention import Attention
from .layers.linear import RowParallelAllReduce, RowParallelLinear, row_parallel_buffer_bytes
from .pool import KVPool, block_bytes, plan_num_blocks, tp_shard
from .layers.mixed_attention import MixedAttentionContext, forward_mixed, forward_mixed_fp8
from .utils.context import Context, get_context, reset_context, set_context

__all__ = [
    "Attention", "Context", "KVPool", "block_bytes", "plan_num_blocks", "tp_shard",
    "MixedAttentionContext", "SlokvError", "decode_workspace",
    "e4m3_decode", "e4m3_encode", "flash_attn_varlen_func", "flash_attn_varlen_func_fp8",
    "flash_attn_with_kvcache", "flash_attn_with_kvcache_fp8", "forward_mixed",
    "forward_mixed_fp8", "get_context", "store_kvcache_fp8",
    "kv_block_copy", "kv_block_gather", "kv_block_scatter", "qk_norm_rope_append",
    "read_device_errors", "reset_context", "set_context", "store_kvcache",
    "RowParallelAllReduce", "RowParallelLinear", "row_parallel_buffer_bytes",
]
