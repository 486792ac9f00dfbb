"""Mixed prefill/decode attention over one flat decode-first token layout.

Same `MixedAttentionContext` fields and `forward_mixed` signature as the
reference (nanovllm/layers/mixed_attention.py:15-57): one store over all T rows
through `store_fn`, decode attention for rows [:num_decode] and varlen prefill
for the rest (paged through `prefill_tables` when any row has history, else on
the contiguous k/v of the chunk).  Both kernels write straight into one [T, Hq,
D] output, so no concatenation copy is made.  `forward_mixed_fp8` is the same
step over an FP8-E4M3 pool: quantising store, FP8 decode, and prefill rows with
history attended through pages dequantised for the step.
"""
from dataclasses import dataclass

import torch

from ..kvcache import (flash_attn_varlen_func, flash_attn_varlen_func_fp8,
                       flash_attn_with_kvcache, flash_attn_with_kvcache_fp8, store_kvcache_fp8)


@dataclass
class MixedAttentionContext:
    num_decode: int
    num_prefill_tokens: int
    decode_lens: torch.Tensor | None
    decode_tables: torch.Tensor | None
    prefill_cu_q: torch.Tensor | None
    prefill_cu_k: torch.Tensor | None
    prefill_tables: torch.Tensor | None
    max_q: int
    max_k: int
    prefill_has_history: bool = True


def forward_mixed(q, k, v, k_cache, v_cache, context, scale, store_fn):
    meta = context.mixed
    if not k_cache.numel() or not v_cache.numel():
        raise RuntimeError("mixed forward requires an allocated BF16 KV pool")
    store_fn(k, v, k_cache, v_cache, context.slot_mapping)
    d = meta.num_decode
    n = d + meta.num_prefill_tokens
    out = torch.empty((n,) + tuple(q.shape[1:]), dtype=q.dtype, device=q.device)
    if d:
        flash_attn_with_kvcache(q[:d].unsqueeze(1), k_cache, v_cache,
                                cache_seqlens=meta.decode_lens, block_table=meta.decode_tables,
                                softmax_scale=scale, causal=True, out=out[:d].unsqueeze(1))
    if meta.num_prefill_tokens:
        history = meta.prefill_has_history
        flash_attn_varlen_func(q[d:n], k_cache if history else k[d:n],
                               v_cache if history else v[d:n],
                               cu_seqlens_q=meta.prefill_cu_q, cu_seqlens_k=meta.prefill_cu_k,
                               max_seqlen_q=meta.max_q, max_seqlen_k=meta.max_k,
                               softmax_scale=scale, causal=True,
                               block_table=meta.prefill_tables if history else None,
                               out=out[d:n])
    return out


def forward_mixed_fp8(q, k, v, k_codes, v_codes, k_scale, v_scale, context, scale):
    """forward_mixed over an FP8 pool (codes + per-(block, kv-head) scales)."""
    meta = context.mixed
    if not k_codes.numel() or not v_codes.numel():
        raise RuntimeError("mixed forward requires an allocated FP8 KV pool")
    store_kvcache_fp8(k, v, k_codes, v_codes, k_scale, v_scale, context.slot_mapping)
    d = meta.num_decode
    n = d + meta.num_prefill_tokens
    out = torch.empty((n,) + tuple(q.shape[1:]), dtype=q.dtype, device=q.device)
    if d:
        flash_attn_with_kvcache_fp8(q[:d].unsqueeze(1), k_codes, v_codes, k_scale, v_scale,
                                    cache_seqlens=meta.decode_lens,
                                    block_table=meta.decode_tables, softmax_scale=scale,
                                    causal=True, out=out[:d].unsqueeze(1))
    if meta.num_prefill_tokens:
        if meta.prefill_has_history:
            flash_attn_varlen_func_fp8(q[d:n], k_codes, v_codes, k_scale, v_scale,
                                       meta.prefill_cu_q, meta.prefill_cu_k, meta.max_q,
                                       meta.max_k, softmax_scale=scale, causal=True,
                                       block_table=meta.prefill_tables, out=out[d:n])
        else:
            flash_attn_varlen_func(q[d:n], k[d:n], v[d:n], cu_seqlens_q=meta.prefill_cu_q,
                                   cu_seqlens_k=meta.prefill_cu_k, max_seqlen_q=meta.max_q,
                                   max_seqlen_k=meta.max_k, softmax_scale=scale, causal=True,
                                   out=out[d:n])
    return out
