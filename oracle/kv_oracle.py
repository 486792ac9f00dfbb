"""CPU restatement of the reference engine's KV-cache hot path (test infrastructure).

Every function cites the reference file:line whose behaviour it restates.  Tensor
arguments are CPU torch tensors; attention arithmetic is fp32 like the
reference's own oracle (benchmarks/v1_validation/reference.py).
"""
from __future__ import annotations

import bisect
import math

import numpy as np
import torch

# ---------------------------------------------------------------------------
# Paged append -- nanovllm/layers/attention.py:10-40 (store_kvcache_kernel):
# program i reads slot = slot_mapping[i]; slot == -1 returns; otherwise the D
# contiguous elements of key row i / value row i go to cache[slot*D : slot*D+D].
# ---------------------------------------------------------------------------


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    N, heads, head_dim = key.shape
    D = heads * head_dim
    kc = k_cache.view(-1, D)
    vc = v_cache.view(-1, D)
    slots = slot_mapping.tolist()
    for i, slot in enumerate(slots):
        if slot == -1:
            continue
        kc[slot] = key[i].reshape(D)
        vc[slot] = value[i].reshape(D)


# ---------------------------------------------------------------------------
# fp32 dense attention -- benchmarks/v1_validation/reference.py:7-23
# GQA by repeat_interleave, bottom-right aligned causal mask: query i of nq
# sees keys 0 .. nk-nq+i.
# ---------------------------------------------------------------------------


def dense_suffix_attention(q, k, v, scale=None):
    if q.ndim != 3 or k.ndim != 3 or v.shape != k.shape:
        raise ValueError("expected [tokens, heads, dim] Q/K/V")
    nq, heads, dim = q.shape
    nk, kv_heads, kd = k.shape
    if not 0 < nq <= nk or dim != kd or heads % kv_heads:
        raise ValueError("invalid causal suffix / GQA shape")
    q, k, v = (x.float() for x in (q, k, v))
    if not all(torch.isfinite(x).all().item() for x in (q, k, v)):
        raise ValueError("nonfinite Q/K/V")
    k = k.repeat_interleave(heads // kv_heads, dim=1)
    v = v.repeat_interleave(heads // kv_heads, dim=1)
    scores = torch.einsum("qhd,khd->hqk", q, k) * (dim ** -0.5 if scale is None else scale)
    qpos = torch.arange(nk - nq, nk)
    kpos = torch.arange(nk)
    scores = scores.masked_fill(kpos[None, :] > qpos[:, None], -math.inf)
    return torch.einsum("hqk,khd->qhd", scores.softmax(-1), v)


# ---------------------------------------------------------------------------
# Paged gather + the two flash-attn replacements --
# benchmarks/v1_validation/reference.py:60-82
# ---------------------------------------------------------------------------


def gather(cache, table, length):
    """Rows 0..length-1 of a sequence, through its block table (reference.py:60-62)."""
    pages = (length + cache.shape[1] - 1) // cache.shape[1]
    return cache[table[:pages].long()].flatten(0, 1)[:length]


def decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale):
    """flash_attn_with_kvcache replacement (reference.py:77-82); q is [B, 1, Hq, D].

    Rows with cache_seqlens <= 0 return zeros (the reference oracle rejects them;
    the kernels define them as zero output, like flash-attn's empty rows).
    """
    outs = []
    for i, n in enumerate(cache_seqlens.tolist()):
        if n <= 0:
            outs.append(torch.zeros(q.shape[1:], dtype=torch.float32))
            continue
        outs.append(dense_suffix_attention(q[i], gather(k_cache, block_table[i], n),
                                           gather(v_cache, block_table[i], n), softmax_scale))
    return torch.stack(outs)


def varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, softmax_scale, block_table=None):
    """flash_attn_varlen_func replacement (reference.py:64-75), causal only."""
    qs, ks = cu_seqlens_q.tolist(), cu_seqlens_k.tolist()
    outputs = []
    for i, (a, b) in enumerate(zip(qs, qs[1:])):
        length = ks[i + 1] - ks[i]
        pk = k[ks[i]:ks[i + 1]] if block_table is None else gather(k, block_table[i], length)
        pv = v[ks[i]:ks[i + 1]] if block_table is None else gather(v, block_table[i], length)
        outputs.append(dense_suffix_attention(q[a:b], pk, pv, softmax_scale))
    return torch.cat(outputs)


def forward_mixed(q, k, v, k_cache, v_cache, meta, slot_mapping, scale):
    """nanovllm/layers/mixed_attention.py:29-57 with the oracle attention bound in."""
    store_kvcache(k, v, k_cache, v_cache, slot_mapping)
    parts = []
    d = meta["num_decode"]
    if d:
        parts.append(decode(q[:d].unsqueeze(1), k_cache, v_cache, meta["decode_lens"],
                            meta["decode_tables"], scale).squeeze(1))
    if meta["num_prefill_tokens"]:
        hist = meta["prefill_has_history"]
        parts.append(varlen(q[d:], k_cache if hist else k[d:], v_cache if hist else v[d:],
                            meta["prefill_cu_q"], meta["prefill_cu_k"], scale,
                            meta["prefill_tables"] if hist else None))
    return parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)


# ---------------------------------------------------------------------------
# q/k RMSNorm + rotary embedding of one layer -- nanovllm/layers/layernorm.py
# rms_forward (fp32 statistics, rounded, times the weight) and
# nanovllm/layers/rotary_embedding.py (cos/sin table, rotate-half in fp32),
# as nanovllm/models/qwen3.py:76-85 chains them.  Eager torch on the CPU.
# ---------------------------------------------------------------------------


def rms_norm(x, weight, eps):
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(x.dtype) * weight


def rope_cos_sin(max_position, head_dim, base):
    """[max_position, head_dim] fp32: cos of the head_dim/2 frequencies, then sin
    (rotary_embedding.py RotaryEmbedding.__init__ with the unit axis squeezed)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def apply_rope(x, cos, sin):
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


def qk_norm_rope(qkv, num_q_heads, num_kv_heads, q_weight, k_weight, eps, positions, cos_sin):
    """(q, k, v) of one layer from the fused qkv rows [T, (Hq + 2 Hkv) * D]."""
    T = qkv.shape[0]
    D = cos_sin.shape[-1]
    q, k, v = qkv.split([num_q_heads * D, num_kv_heads * D, num_kv_heads * D], dim=-1)
    q = rms_norm(q.reshape(T, num_q_heads, D), q_weight, eps)
    k = rms_norm(k.reshape(T, num_kv_heads, D), k_weight, eps)
    cos, sin = cos_sin[positions.long()].chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v.reshape(T, num_kv_heads, D)


# ---------------------------------------------------------------------------
# Page copy -- diagnostics/online_token_replay/tensors.py:34-43 (restore_kv):
# pool[:, :, page].copy_(saved[:, :, j]) for every page, all planes.
# ---------------------------------------------------------------------------


def block_copy(pool, src_ids, dst_ids) -> None:
    for s, d in zip(list(src_ids), list(dst_ids)):
        if s < 0 or d < 0:
            continue
        pool[:, :, d].copy_(pool[:, :, s])


def block_gather(pool, ids):
    return torch.stack([pool[:, :, i] for i in list(ids)], dim=2)


def block_scatter(saved, pool, ids) -> None:
    for j, page in enumerate(list(ids)):
        if page < 0:
            continue
        pool[:, :, page].copy_(saved[:, :, j])


# ---------------------------------------------------------------------------
# E4M3FN codec -- benchmarks/v0/probe_quant_support.py:24-56 (scalar, exact)
# and :187-215 (vectorised bucketize-on-midpoints software path).
# ---------------------------------------------------------------------------


def decode_e4m3fn(code: int) -> float:
    sign = -1.0 if code & 0x80 else 1.0
    exponent = (code >> 3) & 0xF
    mantissa = code & 0x7
    if exponent == 15 and mantissa == 7:
        return math.nan
    if exponent == 0:
        return sign * mantissa * (2.0 ** -9)
    return sign * (1 + mantissa / 8) * (2.0 ** (exponent - 7))


POSITIVE_VALUES = [decode_e4m3fn(i) for i in range(127)]


def encode_e4m3fn(value: float) -> int:
    """Nearest of the 127 non-negative finite codes, ties to the even code,
    magnitude saturated at 448, sign from copysign; non-finite is an error."""
    if not math.isfinite(value):
        raise ValueError("non-finite input to the E4M3 encoder")
    sign = 0x80 if math.copysign(1.0, value) < 0 else 0
    magnitude = min(abs(value), 448.0)
    index = bisect.bisect_left(POSITIVE_VALUES, magnitude)
    candidates = {max(0, min(126, index)), max(0, min(126, index - 1))}
    code = min(candidates, key=lambda i: (abs(POSITIVE_VALUES[i] - magnitude), i & 1))
    return sign | code


_POS = np.array(POSITIVE_VALUES, dtype=np.float64)
_MID32 = ((_POS[:-1] + _POS[1:]) / 2).astype(np.float32)  # exact in fp32
DECODE_LUT = np.array([decode_e4m3fn(c) for c in range(256)], dtype=np.float32)


def encode_e4m3fn_array(x: np.ndarray) -> np.ndarray:
    """Vectorised encoder (software_fp8, probe_quant_support.py:201-215) on fp32 input.

    magnitude = min(|x|, 448); index = bucketize(magnitude, midpoints) (first
    midpoint >= magnitude); a magnitude exactly on a midpoint with an odd index
    moves up one code (ties to even); the sign bit comes from signbit(x).
    """
    x = np.asarray(x, dtype=np.float32)
    if not np.isfinite(x).all():
        raise ValueError("non-finite input to the E4M3 encoder")
    mag = np.minimum(np.abs(x), np.float32(448.0))
    idx = np.searchsorted(_MID32, mag, side="left").astype(np.int64)
    mid = _MID32[np.minimum(idx, 125)]
    ties_up = (idx < 126) & (mag == mid) & ((idx & 1) == 1)
    idx = idx + ties_up
    sign = np.signbit(x).astype(np.int64) << 7
    return (idx | sign).astype(np.uint8)


def decode_e4m3fn_array(codes: np.ndarray) -> np.ndarray:
    return DECODE_LUT[np.asarray(codes, dtype=np.uint8)]


# ---------------------------------------------------------------------------
# FP8-E4M3 KV cache contract (per-(block, kv-head) fp32 scale).
#
# The reference has the codec but no quantised KV path; the contract below is
# the one the kernels implement (it follows the scale definition of the
# reference manual, docs/project_manual.md:523-537, with the block granularity
# asked for by the north star):
#   * state per (block, head): scale s >= 0, fp32.  s == 0 means "no nonzero
#     value stored yet"; the divisor used for encoding is then 1 (the manual's
#     "amax = 0 -> scale = 1").
#   * an append call groups the new tokens of one block (they are adjacent in
#     slot_mapping with consecutive offsets, as the engine produces them).
#     a = max |fp32(x)| over those tokens and the head's D dims;
#     s_new = max(s_old, fp32(a / 448)), where s_old is the stored scale, or 0
#     when the group starts at offset 0 of the block: a block's first token is
#     always written at offset 0 and shared prefix blocks are full and
#     read-only (nanovllm/engine/block_manager.py:43-92 hands out blocks and
#     never writes a shared one), so a write at offset 0 means the page was
#     (re)assigned and whatever scale it holds belongs to its previous owner.
#   * if s_new > s_old > 0, every existing position p < (first new offset) of
#     that block/head is re-encoded: c' = encode(fp32(decode(c) * s_old) / s_new).
#   * new tokens: c = encode(fp32(x) / (s_new if s_new > 0 else 1)).
#   * dequantisation inside attention: decode(c) * s.
# All divisions/multiplications are IEEE fp32 round-to-nearest-even.
# ---------------------------------------------------------------------------


def _f32(x):
    return np.float32(x)


def fp8_append(key, value, k_codes, v_codes, k_scale, v_scale, slot_mapping) -> None:
    """Quantising append under the contract above.  key/value: [N, Hkv, D] (any
    float dtype); codes: uint8 [NB, bs, Hkv, D]; scales: fp32 [NB, Hkv]."""
    N, H, D = key.shape
    bs = k_codes.shape[1]
    slots = slot_mapping.tolist()
    i = 0
    while i < N:
        slot = slots[i]
        if slot < 0:
            i += 1
            continue
        blk, off = divmod(slot, bs)
        j = i + 1
        while j < N and slots[j] == slots[j - 1] + 1 and slots[j] // bs == blk:
            j += 1
        for x, codes, scales in ((key, k_codes, k_scale), (value, v_codes, v_scale)):
            run = x[i:j].float().numpy()                      # [n, H, D] fp32
            cb = codes[blk].numpy()                           # view [bs, H, D]
            sb = scales[blk].numpy()                          # view [H]
            for h in range(H):
                amax = np.float32(np.abs(run[:, h, :]).max())
                s_old = np.float32(0.0) if off == 0 else np.float32(sb[h])
                s_new = np.maximum(s_old, np.float32(amax / np.float32(448.0)))
                if s_new > s_old and s_old > 0 and off > 0:
                    old = decode_e4m3fn_array(cb[:off, h, :])
                    deq = (old * s_old).astype(np.float32)
                    cb[:off, h, :] = encode_e4m3fn_array((deq / s_new).astype(np.float32))
                div = s_new if s_new > 0 else np.float32(1.0)
                cb[off:off + (j - i), h, :] = encode_e4m3fn_array(
                    (run[:, h, :] / div).astype(np.float32))
                sb[h] = s_new
        i = j


def fp8_dequant(codes, scales):
    """decode(c) * s for a whole pool: [NB, bs, H, D] fp32."""
    deq = decode_e4m3fn_array(codes.numpy())
    return torch.from_numpy(deq * scales.numpy()[:, None, :, None].astype(np.float32))


def fp8_decode(q, k_codes, v_codes, k_scale, v_scale, cache_seqlens, block_table,
               softmax_scale):
    """Decode attention over the dequantised FP8 cache (fp32 oracle)."""
    return decode(q, fp8_dequant(k_codes, k_scale), fp8_dequant(v_codes, v_scale),
                  cache_seqlens, block_table, softmax_scale)
