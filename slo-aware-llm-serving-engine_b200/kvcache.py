"""Host-side mirror of the reference engine's KV-cache hot path.

Each function keeps the name, argument meaning and error behaviour of the
reference symbol it replaces, and calls the sm_100a kernels through the C ABI
(include/slokv.h) on the current CUDA stream.  Everything is asynchronous, does
no host synchronisation and allocates nothing per call (workspaces are
per-device and fixed), so it can be captured in a CUDA graph once it has been
called eagerly at the largest geometry.

  store_kvcache            nanovllm/layers/attention.py:33-40
  flash_attn_with_kvcache  call sites nanovllm/layers/attention.py:76-78,
                           nanovllm/layers/mixed_attention.py:117-121
  kv_block_copy / gather / scatter
                           page copy of diagnostics/online_token_replay/tensors.py:34-43
  store_kvcache_fp8 / flash_attn_with_kvcache_fp8
                           the same two calls over an FP8-E4M3 pool with per-(block,
                           kv-head) scales (the reference's E4M3 codec,
                           benchmarks/v0/probe_quant_support.py:24-56, applied to KV)
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import SlokvError, buffers, check, lib, require_cuda, stream_ptr


def _i32_contig(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise SlokvError(f"{name} must be int32, got {t.dtype}")
    if not t.is_contiguous():
        raise SlokvError(f"{name} must be contiguous")
    return t


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Scatter key/value rows into the paged pool: cache row slot_mapping[i] <- row i.

    slot == -1 skips the token (padding rows of captured decode graphs).  The
    assertions are the reference wrapper's own (nanovllm/layers/attention.py:36-39).
    """
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    dev = require_cuda(key, value, k_cache, v_cache, slot_mapping)
    if key.dtype != k_cache.dtype or value.dtype != v_cache.dtype or key.dtype != value.dtype:
        raise SlokvError("key/value/cache dtypes differ")
    if value.shape != key.shape:
        raise SlokvError("key and value shapes differ")
    # The kernel addresses cache row `slot` at slot * D elements, as the reference does.
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if c.stride(0) != c.shape[1] * D or c.shape[-2] * c.shape[-1] != D:
            raise SlokvError(f"{name} must be [num_blocks, block_size, {num_heads}, {head_dim}] "
                             "with contiguous blocks")
    _i32_contig("slot_mapping", slot_mapping)
    num_slots = k_cache.shape[0] * k_cache.shape[1]
    err = buffers.error_word(dev)
    check(lib().slokv_kv_append(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
        k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), N, D,
        key.element_size(), num_slots, err.data_ptr(), stream_ptr(dev)), "kv_append")


def qk_norm_rope_append(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                        q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float,
                        positions: torch.Tensor, cos_sin: torch.Tensor, slot_mapping: torch.Tensor,
                        k_cache: torch.Tensor, v_cache: torch.Tensor, k_out: bool = False):
    """Fused q_norm / k_norm + rotary embedding + store_kvcache of one layer.

    qkv: [T, (Hq + 2 Hkv) * 128] (the qkv projection output, last dim
    contiguous); q_weight / k_weight: [128]; positions: [T] int64; cos_sin: fp32
    [max_position, 128] (cos | sin halves, the reference's cos_sin_cache
    squeezed); k_cache / v_cache: [num_blocks, block_size, Hkv, 128].  Writes the
    normed, rotated k and the raw v to cache row slot_mapping[t] (slot -1 skips)
    and returns q [T, Hq, 128] (and k [T, Hkv, 128] when k_out is set, for cold
    prefill attention on the step's own rows).
    """
    T = qkv.shape[0]
    D = 128
    dev = require_cuda(qkv, q_weight, k_weight, positions, cos_sin, slot_mapping, k_cache, v_cache)
    if qkv.dim() != 2 or qkv.shape[1] != (num_q_heads + 2 * num_kv_heads) * D or qkv.stride(1) != 1:
        raise SlokvError("qkv must be [tokens, (Hq + 2 Hkv) * 128] with a contiguous last dim")
    if (q_weight.numel() != D or k_weight.numel() != D or not q_weight.is_contiguous()
            or not k_weight.is_contiguous()):
        raise SlokvError("q_weight / k_weight must be contiguous [128]")
    if q_weight.dtype != qkv.dtype or k_weight.dtype != qkv.dtype or k_cache.dtype != qkv.dtype:
        raise SlokvError("qkv, norm weights and cache dtypes differ")
    if positions.dtype != torch.int64 or not positions.is_contiguous() or positions.numel() != T:
        raise SlokvError("positions must be contiguous int64 [tokens]")
    if cos_sin.dtype != torch.float32 or cos_sin.shape[-1] != D or not cos_sin.is_contiguous():
        raise SlokvError("cos_sin must be contiguous fp32 [max_position, 128]")
    _i32_contig("slot_mapping", slot_mapping)
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if (c.shape[-1] != D or c.shape[-2] != num_kv_heads
                or c.stride(0) != c.shape[1] * num_kv_heads * D):
            raise SlokvError(f"{name} must be [num_blocks, block_size, {num_kv_heads}, 128] "
                             "with contiguous blocks")
    q = torch.empty(T, num_q_heads, D, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty(T, num_kv_heads, D, dtype=qkv.dtype, device=qkv.device) if k_out else None
    if T:
        err = buffers.error_word(dev)
        check(lib().slokv_qk_norm_rope_append(
            qkv.data_ptr(), qkv.stride(0), T, num_q_heads, num_kv_heads, D, q_weight.data_ptr(),
            k_weight.data_ptr(), float(eps), positions.data_ptr(), cos_sin.data_ptr(),
            cos_sin.numel() // D, slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.shape[0] * k_cache.shape[1], q.data_ptr(), q.stride(0),
            k.data_ptr() if k is not None else None, k.stride(0) if k is not None else 0,
            _lib.dtype_code(qkv.dtype), err.data_ptr(), stream_ptr(dev)), "qk_norm_rope_append")
    return (q, k) if k_out else q


def decode_workspace(device: torch.device, num_q_heads: int, num_kv_heads: int,
                     head_dim: int) -> torch.Tensor:
    """The fixed per-device split-K workspace used by paged decode."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    nbytes = lib().slokv_paged_decode_workspace_bytes(idx, num_q_heads, num_kv_heads, head_dim)
    if nbytes == 0:
        raise SlokvError(f"unsupported decode geometry Hq={num_q_heads} Hkv={num_kv_heads} "
                         f"D={head_dim}")
    return buffers.workspace(device, f"decode/{num_q_heads // num_kv_heads}/{head_dim}", nbytes)


def flash_attn_with_kvcache(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                            softmax_scale: float | None = None, causal: bool = True,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Paged decode attention with the flash_attn_with_kvcache calling convention.

    q: [B, 1, Hq, D]; k_cache/v_cache: [num_blocks, block_size, Hkv, D];
    cache_seqlens: [B] int32 (length including the token stored this step);
    block_table: [B, W] int32.  Returns [B, 1, Hq, D].  `causal` is accepted for
    signature compatibility (one query at the last position sees every key).
    """
    if q.dim() != 4 or q.shape[1] != 1:
        raise SlokvError("paged decode expects q of shape [batch, 1, heads, head_dim]")
    B, _, Hq, D = q.shape
    NB, block_size, Hkv, Dk = k_cache.shape
    if v_cache.shape != k_cache.shape or Dk != D:
        raise SlokvError("k_cache/v_cache shape mismatch with q")
    if q.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise SlokvError("q and cache dtypes differ")
    if q.stride(-1) != 1:
        raise SlokvError("q must have a contiguous last dimension")
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if c.stride(3) != 1 or c.stride(2) != D or c.stride(1) != Hkv * D:
            raise SlokvError(f"{name} blocks must be contiguous [block_size, Hkv, D]")
    dev = require_cuda(q, k_cache, v_cache, cache_seqlens, block_table)
    _i32_contig("cache_seqlens", cache_seqlens)
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise SlokvError("block_table must be int32 with a contiguous last dimension")
    if block_table.shape[0] < B or cache_seqlens.numel() < B:
        raise SlokvError("block_table / cache_seqlens have fewer rows than q")
    scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
    if out is None:
        out = torch.empty(B, 1, Hq, D, dtype=q.dtype, device=q.device)
    ws = decode_workspace(dev, Hq, Hkv, D)
    err = buffers.error_word(dev)
    check(lib().slokv_paged_decode(
        out.data_ptr(), out.stride(0), out.stride(2),
        q.data_ptr(), q.stride(0), q.stride(2),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), v_cache.stride(0),
        NB, block_size, Hq, Hkv, D,
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        cache_seqlens.data_ptr(), B, scale, _lib.dtype_code(q.dtype),
        ws.data_ptr(), ws.numel(), err.data_ptr(), stream_ptr(dev)), "paged_decode")
    return out


# ---------------------------------------------------------------------------
# FP8-E4M3 KV cache (per-(block, kv-head) fp32 scales; contract in include/slokv.h)
# ---------------------------------------------------------------------------

FP8_DTYPES = (torch.uint8,) + ((torch.float8_e4m3fn,) if hasattr(torch, "float8_e4m3fn") else ())


def is_fp8_cache(cache: torch.Tensor) -> bool:
    return cache.dtype in FP8_DTYPES


# Calls with at least this many tokens (prefill-sized: runs of up to a block
# per (block, head)) take the three-launch append, which works token-parallel.
_FP8_RUNS_MIN_TOKENS = 512


def store_kvcache_fp8(key: torch.Tensor, value: torch.Tensor, k_codes: torch.Tensor,
                      v_codes: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                      slot_mapping: torch.Tensor, *, runs: bool | None = None) -> None:
    """Quantising store into the FP8 pool (store_kvcache's counterpart).

    k_codes/v_codes: [num_blocks, block_size, Hkv, D] uint8 (or float8_e4m3fn);
    k_scale/v_scale: [num_blocks, Hkv] fp32, zero for freshly assigned blocks.
    The new tokens of one block must be adjacent in slot_mapping with
    consecutive offsets (the engine's decode and prefill layouts are).
    `runs`: force the token-parallel three-launch append (True) or the one-launch
    kernel (False); by default calls of >= 512 tokens take the former once its
    zeroed per-device word array exists (it is never grown during graph
    capture).  Both write identical codes and scales.
    """
    N, num_heads, head_dim = key.shape
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert slot_mapping.numel() == N
    dev = require_cuda(key, value, k_codes, v_codes, k_scale, v_scale, slot_mapping)
    NB, bs, Hkv, D = k_codes.shape
    if (Hkv, D) != (num_heads, head_dim) or v_codes.shape != k_codes.shape:
        raise SlokvError("FP8 pool geometry differs from key/value")
    for name, c in (("k_codes", k_codes), ("v_codes", v_codes)):
        if not is_fp8_cache(c) or not c.is_contiguous():
            raise SlokvError(f"{name} must be a contiguous uint8/float8_e4m3fn pool")
    for name, sc in (("k_scale", k_scale), ("v_scale", v_scale)):
        if sc.dtype != torch.float32 or tuple(sc.shape) != (NB, Hkv) or not sc.is_contiguous():
            raise SlokvError(f"{name} must be contiguous fp32 [num_blocks, num_kv_heads]")
    _i32_contig("slot_mapping", slot_mapping)
    err = buffers.error_word(dev)
    use_runs = runs if runs is not None else N >= _FP8_RUNS_MIN_TOKENS
    if use_runs:
        nbytes = lib().slokv_kv_append_fp8_runs_workspace_bytes(NB, Hkv)
        if (runs is None and torch.cuda.is_current_stream_capturing()
                and not buffers.workspace_fits(dev, "fp8_append_amax", nbytes)):
            use_runs = False
    if use_runs:
        ws = buffers.workspace(dev, "fp8_append_amax", nbytes, zero=True)
        check(lib().slokv_kv_append_fp8_runs(
            key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
            k_codes.data_ptr(), v_codes.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(),
            slot_mapping.data_ptr(), N, Hkv, D, bs, NB, _lib.dtype_code(key.dtype),
            ws.data_ptr(), ws.numel(), err.data_ptr(), stream_ptr(dev)), "kv_append_fp8_runs")
        return
    check(lib().slokv_kv_append_fp8(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
        k_codes.data_ptr(), v_codes.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(),
        slot_mapping.data_ptr(), N, Hkv, D, bs, NB, _lib.dtype_code(key.dtype),
        err.data_ptr(), stream_ptr(dev)), "kv_append_fp8")


def flash_attn_with_kvcache_fp8(q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                                k_scale: torch.Tensor, v_scale: torch.Tensor,
                                cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                                softmax_scale: float | None = None, causal: bool = True,
                                out: torch.Tensor | None = None) -> torch.Tensor:
    """Paged decode over the FP8 pool, dequantisation fused into the tile load."""
    if q.dim() != 4 or q.shape[1] != 1:
        raise SlokvError("paged decode expects q of shape [batch, 1, heads, head_dim]")
    B, _, Hq, D = q.shape
    NB, block_size, Hkv, Dk = k_codes.shape
    if v_codes.shape != k_codes.shape or Dk != D:
        raise SlokvError("FP8 pool shape mismatch with q")
    for name, c in (("k_codes", k_codes), ("v_codes", v_codes)):
        if not is_fp8_cache(c) or c.stride(3) != 1 or c.stride(2) != D or c.stride(1) != Hkv * D:
            raise SlokvError(f"{name} must be an FP8 pool with contiguous blocks")
    for name, sc in (("k_scale", k_scale), ("v_scale", v_scale)):
        if sc.dtype != torch.float32 or tuple(sc.shape) != (NB, Hkv) or not sc.is_contiguous():
            raise SlokvError(f"{name} must be contiguous fp32 [num_blocks, num_kv_heads]")
    if q.stride(-1) != 1:
        raise SlokvError("q must have a contiguous last dimension")
    dev = require_cuda(q, k_codes, v_codes, k_scale, v_scale, cache_seqlens, block_table)
    _i32_contig("cache_seqlens", cache_seqlens)
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise SlokvError("block_table must be int32 with a contiguous last dimension")
    scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
    if out is None:
        out = torch.empty(B, 1, Hq, D, dtype=q.dtype, device=q.device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    nbytes = lib().slokv_paged_decode_fp8_workspace_bytes(idx, Hq, Hkv, D)
    if nbytes == 0:
        raise SlokvError("unsupported FP8 decode geometry")
    ws = buffers.workspace(dev, f"decode_fp8/{Hq // Hkv}/{D}", nbytes)
    err = buffers.error_word(dev)
    check(lib().slokv_paged_decode_fp8(
        out.data_ptr(), out.stride(0), out.stride(2), q.data_ptr(), q.stride(0), q.stride(2),
        k_codes.data_ptr(), v_codes.data_ptr(), k_codes.stride(0), v_codes.stride(0),
        k_scale.data_ptr(), v_scale.data_ptr(), NB, block_size, Hq, Hkv, D,
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        cache_seqlens.data_ptr(), B, scale, _lib.dtype_code(q.dtype),
        ws.data_ptr(), ws.numel(), err.data_ptr(), stream_ptr(dev)), "paged_decode_fp8")
    return out


def e4m3_encode(x: torch.Tensor) -> torch.Tensor:
    """E4M3FN codes (uint8) of a CUDA fp32 tensor: RNE, ties to even, saturate at 448."""
    dev = require_cuda(x)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise SlokvError("e4m3_encode expects a contiguous fp32 tensor")
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    check(lib().slokv_fp8_e4m3_encode(x.data_ptr(), codes.data_ptr(), x.numel(),
                                      buffers.error_word(dev).data_ptr(), stream_ptr(dev)),
          "fp8_e4m3_encode")
    return codes


def e4m3_decode(codes: torch.Tensor) -> torch.Tensor:
    """fp32 values of E4M3FN codes (uint8 CUDA tensor)."""
    dev = require_cuda(codes)
    if codes.dtype not in FP8_DTYPES or not codes.is_contiguous():
        raise SlokvError("e4m3_decode expects a contiguous uint8 tensor")
    x = torch.empty(codes.shape, dtype=torch.float32, device=codes.device)
    check(lib().slokv_fp8_e4m3_decode(codes.data_ptr(), x.data_ptr(), codes.numel(),
                                      stream_ptr(dev)), "fp8_e4m3_decode")
    return x


def _pool_planes(pool: torch.Tensor):
    """View a [2, L, NB, ...] pool (or any [P0, P1, NB, ...]) as planes x pages."""
    if pool.dim() < 4:
        raise SlokvError("pool must be [2, num_layers, num_blocks, ...]")
    inner = pool[0, 0, 0]
    if not inner.is_contiguous():
        raise SlokvError("pool pages must be contiguous")
    if pool.stride(0) != pool.shape[1] * pool.stride(1):
        raise SlokvError("pool planes (K|V x layer) must be evenly strided")
    es = pool.element_size()
    return (pool.shape[0] * pool.shape[1], pool.stride(1) * es, pool.stride(2) * es,
            inner.numel() * es, pool.shape[2])


def kv_block_copy(pool: torch.Tensor, src_ids: torch.Tensor, dst_ids: torch.Tensor) -> None:
    """pool[:, :, dst_ids[i]] = pool[:, :, src_ids[i]] for every i (all K/V planes, all layers).

    Entries < 0 are skipped.  Source and destination pages must not overlap.
    """
    dev = require_cuda(pool, src_ids, dst_ids)
    _i32_contig("src_ids", src_ids)
    _i32_contig("dst_ids", dst_ids)
    if src_ids.numel() != dst_ids.numel():
        raise SlokvError("src_ids and dst_ids differ in length")
    planes, plane_stride, page_stride, page_bytes, cap = _pool_planes(pool)
    check(lib().slokv_kv_block_copy(
        pool.data_ptr(), plane_stride, page_stride, src_ids.data_ptr(), cap,
        pool.data_ptr(), plane_stride, page_stride, dst_ids.data_ptr(), cap,
        src_ids.numel(), planes, page_bytes, buffers.error_word(dev).data_ptr(),
        stream_ptr(dev)), "kv_block_copy")


def kv_block_gather(pool: torch.Tensor, ids: torch.Tensor, out: torch.Tensor | None = None
                    ) -> torch.Tensor:
    """Compact copy of pages `ids`: out[:, :, j] = pool[:, :, ids[j]] (swap-out / snapshot)."""
    dev = require_cuda(pool, ids)
    _i32_contig("ids", ids)
    planes, plane_stride, page_stride, page_bytes, cap = _pool_planes(pool)
    if out is None:
        shape = list(pool.shape)
        shape[2] = ids.numel()
        out = torch.empty(shape, dtype=pool.dtype, device=pool.device)
    o_planes, o_plane_stride, o_page_stride, o_page_bytes, o_cap = _pool_planes(out)
    if o_planes != planes or o_page_bytes != page_bytes or o_cap < ids.numel():
        raise SlokvError("gather destination geometry differs from the pool")
    check(lib().slokv_kv_block_copy(
        pool.data_ptr(), plane_stride, page_stride, ids.data_ptr(), cap,
        out.data_ptr(), o_plane_stride, o_page_stride, None, o_cap,
        ids.numel(), planes, page_bytes, buffers.error_word(dev).data_ptr(),
        stream_ptr(dev)), "kv_block_gather")
    return out


def kv_block_scatter(saved: torch.Tensor, pool: torch.Tensor, ids: torch.Tensor) -> None:
    """pool[:, :, ids[j]] = saved[:, :, j] (swap-in / restore_kv)."""
    dev = require_cuda(pool, ids, saved)
    _i32_contig("ids", ids)
    planes, plane_stride, page_stride, page_bytes, cap = _pool_planes(pool)
    s_planes, s_plane_stride, s_page_stride, s_page_bytes, s_cap = _pool_planes(saved)
    if s_planes != planes or s_page_bytes != page_bytes or s_cap < ids.numel():
        raise SlokvError("scatter source geometry differs from the pool")
    check(lib().slokv_kv_block_copy(
        saved.data_ptr(), s_plane_stride, s_page_stride, None, s_cap,
        pool.data_ptr(), plane_stride, page_stride, ids.data_ptr(), cap,
        ids.numel(), planes, page_bytes, buffers.error_word(dev).data_ptr(),
        stream_ptr(dev)), "kv_block_scatter")


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           softmax_scale=None, causal=True, block_table=None, out=None):
    """Causal varlen attention with the flash_attn_varlen_func calling convention.

    q: [Tq, Hq, D].  Without block_table, k/v are [Tk, Hkv, D] rows addressed by
    cu_seqlens_k (v may be a strided view of the fused QKV output); with
    block_table, k/v are the paged caches [num_blocks, block_size, Hkv, D] and
    row r's keys are gathered through block_table[r].  Query i of row r sees
    keys 0 .. k_len - q_len + i (bottom-right aligned).  Returns [Tq, Hq, D].
    """
    return _varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale,
                             causal, block_table, out, None)


def _varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal,
                      block_table, out, k_page_scale):
    """flash_attn_varlen_func's body; k_page_scale (fp32 [num_blocks, Hkv], paged
    only) multiplies the logits of each page's keys, for K pages that hold
    unscaled FP8 code values."""
    if not causal:
        raise SlokvError("only causal varlen attention is implemented (the engine's only use)")
    if q.dim() != 3:
        raise SlokvError("q must be [tokens, heads, head_dim]")
    Tq, Hq, D = q.shape
    dev = require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, block_table)
    _i32_contig("cu_seqlens_q", cu_seqlens_q)
    _i32_contig("cu_seqlens_k", cu_seqlens_k)
    if cu_seqlens_k.numel() != cu_seqlens_q.numel():
        raise SlokvError("cu_seqlens_q and cu_seqlens_k differ in length")
    if q.dtype != k.dtype or v.dtype != k.dtype:
        raise SlokvError("q, k and v dtypes differ")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise SlokvError("q, k and v need a contiguous last dimension")
    rows = cu_seqlens_q.numel() - 1
    scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
    if out is None:
        out = torch.empty(Tq, Hq, D, dtype=q.dtype, device=q.device)
    if block_table is not None:
        NB, bs, Hkv, Dk = k.shape
        if v.shape != k.shape or Dk != D:
            raise SlokvError("k_cache/v_cache shape mismatch with q")
        for name, c in (("k_cache", k), ("v_cache", v)):
            if c.stride(2) != D or c.stride(1) != Hkv * D:
                raise SlokvError(f"{name} blocks must be contiguous [block_size, Hkv, D]")
        if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
            raise SlokvError("block_table must be int32 with a contiguous last dimension")
        args = (k.data_ptr(), v.data_ptr(), 0, 0, 0, k.stride(0), v.stride(0),
                cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), rows, int(max_seqlen_q),
                block_table.data_ptr(), block_table.stride(0), block_table.shape[1], NB, bs)
    else:
        Tk, Hkv, Dk = k.shape
        if v.shape != k.shape or Dk != D or k.stride(1) != D or v.stride(1) != D:
            raise SlokvError("k/v must be [tokens, Hkv, D] with contiguous heads")
        args = (k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), Tk, 0, 0,
                cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), rows, int(max_seqlen_q),
                None, 0, 0, 0, 0)
    if Tq == 0 or rows == 0:
        return out
    err = buffers.error_word(dev)
    ws, ws_bytes = _prefill_workspace(dev, rows, int(max_seqlen_q))
    check(lib().slokv_paged_prefill(
        out.data_ptr(), out.stride(0), out.stride(1), q.data_ptr(), q.stride(0), q.stride(1), Tq,
        *args, Hq, Hkv, D, scale, _lib.dtype_code(q.dtype),
        None if k_page_scale is None else k_page_scale.data_ptr(), ws, ws_bytes, err.data_ptr(),
        stream_ptr(dev)),
        "paged_prefill")
    return out


def flash_attn_varlen_func_fp8(q, k_codes, v_codes, k_scale, v_scale, cu_seqlens_q,
                               cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale=None,
                               causal=True, block_table=None, out=None):
    """Prefix-cache varlen attention over an FP8 pool (block_table required),
    the dequantisation fused into the prefill kernel's tile loads.

    The kernel TMA-loads each 128-key tile of E4M3 codes straight from the pool
    pages and widens it in shared memory -- K as its unscaled code values
    (exact in f16) with the page's K scale applied to the logits, V as
    f16(decode(code) * V scale) -- so the tensor cores run f16 MMAs on them; a
    bf16 q is converted to f16 inside the kernel and the output is written in
    q's dtype.  Nothing is copied or allocated per call beyond `out`.  Needs
    an even number of query heads per KV head and max_seqlen_k <= 4330 pages.
    """
    if block_table is None:
        raise SlokvError("FP8 varlen attention reads the pool: block_table is required")
    if not causal:
        raise SlokvError("only causal varlen attention is implemented (the engine's only use)")
    NB, bs, Hkv, D = k_codes.shape
    if v_codes.shape != k_codes.shape or D != q.shape[-1]:
        raise SlokvError("FP8 pool shape mismatch with q")
    for name, c in (("k_codes", k_codes), ("v_codes", v_codes)):
        if not is_fp8_cache(c) or c.stride(3) != 1 or c.stride(2) != D or c.stride(1) != Hkv * D:
            raise SlokvError(f"{name} must be an FP8 pool with contiguous blocks")
    for name, sc in (("k_scale", k_scale), ("v_scale", v_scale)):
        if sc.dtype != torch.float32 or tuple(sc.shape) != (NB, Hkv) or not sc.is_contiguous():
            raise SlokvError(f"{name} must be contiguous fp32 [num_blocks, num_kv_heads]")
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise SlokvError("block_table must be int32 with a contiguous last dimension")
    if q.dim() != 3 or q.dtype not in (torch.bfloat16, torch.float16) or q.stride(-1) != 1:
        raise SlokvError("q must be bf16/f16 [tokens, heads, head_dim] with a contiguous last dim")
    dev = require_cuda(q, k_codes, v_codes, k_scale, v_scale, cu_seqlens_q, cu_seqlens_k,
                       block_table)
    _i32_contig("cu_seqlens_q", cu_seqlens_q)
    _i32_contig("cu_seqlens_k", cu_seqlens_k)
    if cu_seqlens_k.numel() != cu_seqlens_q.numel():
        raise SlokvError("cu_seqlens_q and cu_seqlens_k differ in length")
    Tq, Hq, _ = q.shape
    rows = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(Tq, Hq, D, dtype=q.dtype, device=q.device)
    elif out.dtype != q.dtype or out.shape != q.shape or out.stride(-1) != 1:
        raise SlokvError("out must match q's shape and dtype with a contiguous last dim")
    if Tq == 0 or rows <= 0:
        return out
    # the kernel keeps one K scale per page it can reach in shared memory: no
    # row reaches past ceil(max_seqlen_k / block_size) pages
    width = min(block_table.shape[1], max(1, (int(max_seqlen_k) + bs - 1) // bs))
    scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
    ws, ws_bytes = _prefill_workspace(dev, rows, int(max_seqlen_q))
    check(lib().slokv_paged_prefill_fp8(
        out.data_ptr(), out.stride(0), out.stride(1), q.data_ptr(), q.stride(0), q.stride(1), Tq,
        k_codes.data_ptr(), v_codes.data_ptr(), k_codes.stride(0), v_codes.stride(0),
        k_scale.data_ptr(), v_scale.data_ptr(), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(),
        rows, int(max_seqlen_q), block_table.data_ptr(), block_table.stride(0), width, NB, bs,
        Hq, Hkv, D, scale, _lib.dtype_code(q.dtype), ws, ws_bytes,
        buffers.error_word(dev).data_ptr(), stream_ptr(dev)), "paged_prefill_fp8")
    return out


# Smallest prefill work-order buffer (16K query tiles, e.g. 256 rows of 8K-token
# chunks), so graphs captured after a small warm-up rarely need a larger one.
_PREFILL_WS_MIN = 64 << 10


def _prefill_workspace(dev: torch.device, rows: int, max_seqlen_q: int):
    """(pointer, bytes) of the per-device prefill work-order buffer.  During graph
    capture a buffer too small for this geometry is not grown: the call then
    passes none and the tiles run in row-major order (same results)."""
    need = lib().slokv_paged_prefill_workspace_bytes(rows, max_seqlen_q)
    if need == 0:
        return None, 0
    if torch.cuda.is_current_stream_capturing() and not buffers.workspace_fits(dev, "prefill", need):
        return None, 0
    t = buffers.workspace(dev, "prefill", max(need, _PREFILL_WS_MIN))
    return t.data_ptr(), t.numel()
