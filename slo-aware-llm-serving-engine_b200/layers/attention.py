"""Drop-in `Attention` module and `store_kvcache` for the reference engine.

Same constructor, `.k_cache`/`.v_cache` attributes (bound by the model runner to
kv_cache[0, layer] / kv_cache[1, layer]) and forward(q, k, v) dispatch as the
reference (nanovllm/layers/attention.py:43-79): store the step's K/V, then run
prefill varlen attention (paged when the context carries block tables), decode
attention over the paged cache, or the mixed prefill/decode path -- over a
bf16/f16 pool or an FP8-E4M3 one (codes plus k_scale / v_scale).
"""
import torch
from torch import nn

from ..kvcache import (flash_attn_varlen_func, flash_attn_varlen_func_fp8,
                       flash_attn_with_kvcache, flash_attn_with_kvcache_fp8, store_kvcache,
                       store_kvcache_fp8)
from ..utils.context import get_context

__all__ = ["Attention", "store_kvcache"]


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        # FP8-E4M3 pool: k_cache/v_cache hold uint8 codes and these hold the fp32
        # per-(block, kv-head) scales; None for a bf16/f16 pool.
        self.k_scale = self.v_scale = None

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if self.k_scale is not None:
            return self._forward_fp8(q, k, v, context)
        if context.mixed is not None:
            from .mixed_attention import forward_mixed
            return forward_mixed(q, k, v, k_cache, v_cache, context, self.scale, store_kvcache)
        if k_cache.numel() and v_cache.numel():
            store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        return self._attend(q, k, v, context)

    def attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """forward() without the store, for callers whose K/V rows already went
        into the pool (qk_norm_rope_append); bf16/f16 pools, prefill or decode."""
        context = get_context()
        if self.k_scale is not None or context.mixed is not None:
            raise RuntimeError("attend() covers the bf16/f16 prefill and decode paths")
        return self._attend(q, k, v, context)

    def _attend(self, q, k, v, context):
        if context.is_prefill:
            if context.block_tables is not None:    # prefix cache: keys come from the pool
                k, v = self.k_cache, self.v_cache
            return flash_attn_varlen_func(q, k, v,
                                          max_seqlen_q=context.max_seqlen_q,
                                          cu_seqlens_q=context.cu_seqlens_q,
                                          max_seqlen_k=context.max_seqlen_k,
                                          cu_seqlens_k=context.cu_seqlens_k,
                                          softmax_scale=self.scale, causal=True,
                                          block_table=context.block_tables)
        return flash_attn_with_kvcache(q.unsqueeze(1), self.k_cache, self.v_cache,
                                       cache_seqlens=context.context_lens,
                                       block_table=context.block_tables,
                                       softmax_scale=self.scale, causal=True)

    def _forward_fp8(self, q, k, v, context):
        if context.mixed is not None:
            from .mixed_attention import forward_mixed_fp8
            return forward_mixed_fp8(q, k, v, self.k_cache, self.v_cache, self.k_scale,
                                     self.v_scale, context, self.scale)
        store_kvcache_fp8(k, v, self.k_cache, self.v_cache, self.k_scale, self.v_scale,
                          context.slot_mapping)
        if context.is_prefill:
            if context.block_tables is None:   # cold prompt: keys are the step's own rows
                return flash_attn_varlen_func(q, k, v,
                                              max_seqlen_q=context.max_seqlen_q,
                                              cu_seqlens_q=context.cu_seqlens_q,
                                              max_seqlen_k=context.max_seqlen_k,
                                              cu_seqlens_k=context.cu_seqlens_k,
                                              softmax_scale=self.scale, causal=True)
            return flash_attn_varlen_func_fp8(q, self.k_cache, self.v_cache, self.k_scale,
                                              self.v_scale, context.cu_seqlens_q,
                                              context.cu_seqlens_k, context.max_seqlen_q,
                                              context.max_seqlen_k, softmax_scale=self.scale,
                                              causal=True, block_table=context.block_tables)
        return flash_attn_with_kvcache_fp8(q.unsqueeze(1), self.k_cache, self.v_cache,
                                           self.k_scale, self.v_scale,
                                           cache_seqlens=context.context_lens,
                                           block_table=context.block_tables,
                                           softmax_scale=self.scale, causal=True)
