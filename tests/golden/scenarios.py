"""Seeded KV-cache scenarios shared by the golden generator, the oracle tests and
the GPU parity tests.  All tensors are CPU torch tensors built from detgen, so
every consumer rebuilds bit-identical inputs.

The geometries mirror BASELINE config 1 and the reference's own attention tests
(tests/test_v1_attention_gpu.py:42-142, tests/test_v1_reference_gpu.py:10-66);
the values are synthetic (detgen), not the reference tests' torch.randn draws.
"""
from __future__ import annotations

import numpy as np
import torch

from .detgen import det_ints, det_normal, det_perm  # noqa: F401


def _t(arr, dtype):
    return torch.from_numpy(np.ascontiguousarray(arr)).to(dtype)


def _i32(x):
    return torch.tensor(x, dtype=torch.int32)


def cfg1_decode():
    """one Qwen3-4B attention layer, fp32, block 256, pool of 64
    blocks, batch 8 with context lengths uniform in [1, 2048] (seed 0), block
    tables a permutation of the pool, one appended token per sequence, then decode."""
    Hq, Hkv, D, bs, NB, B = 32, 8, 128, 256, 64, 8
    lens = det_ints(0, B, 1, 2048)
    tables = det_perm(0, NB).reshape(B, NB // B)
    slots = [int(tables[b, (L - 1) // bs]) * bs + (L - 1) % bs for b, L in enumerate(lens)]
    return dict(
        name="cfg1_decode", dtype=torch.float32, Hq=Hq, Hkv=Hkv, D=D, bs=bs, NB=NB,
        q=_t(det_normal(11, (B, Hq, D)), torch.float32),
        k=_t(det_normal(12, (B, Hkv, D)), torch.float32),
        v=_t(det_normal(13, (B, Hkv, D)), torch.float32),
        k_cache=_t(det_normal(14, (NB, bs, Hkv, D)), torch.float32),
        v_cache=_t(det_normal(15, (NB, bs, Hkv, D)), torch.float32),
        lens=_i32(lens.tolist()), tables=_i32(tables.tolist()), slots=_i32(slots),
        scale=D ** -0.5,
    )


def gqa_decode(dtype=torch.bfloat16):
    """GQA 8/2 decode over page tails and page boundaries, pages out of order,
    tables padded with -1 past each sequence's last page."""
    Hq, Hkv, D, bs, NB = 8, 2, 128, 256, 16
    lens = [1, 255, 256, 257, 700, 1024]
    B = len(lens)
    perm = det_perm(21, NB).tolist()
    W = 4
    tables, cursor = [], 0
    for L in lens:
        n = (L + bs - 1) // bs
        tables.append(perm[cursor:cursor + n] + [-1] * (W - n))
        cursor += n
    slots = [tables[b][(L - 1) // bs] * bs + (L - 1) % bs for b, L in enumerate(lens)]
    return dict(
        name="gqa_decode", dtype=dtype, Hq=Hq, Hkv=Hkv, D=D, bs=bs, NB=NB,
        q=_t(det_normal(22, (B, Hq, D)), dtype),
        k=_t(det_normal(23, (B, Hkv, D)), dtype),
        v=_t(det_normal(24, (B, Hkv, D)), dtype),
        k_cache=_t(det_normal(25, (NB, bs, Hkv, D)), dtype),
        v_cache=_t(det_normal(26, (NB, bs, Hkv, D)), dtype),
        lens=_i32(lens), tables=_i32(tables), slots=_i32(slots), scale=D ** -0.5,
    )


def _mixed_from_rows(name, seed, Hq, Hkv, NB, rows, poison, dtype=torch.bfloat16, D=128, bs=256):
    """rows: list of (history, count, table, phase) with decode rows first.
    Histories are written into the pool before the step (the pool is first filled
    with the `poison` pair so that stale bytes are visible)."""
    T = sum(r[1] for r in rows)
    k_cache = torch.full((NB, bs, Hkv, D), poison[0], dtype=dtype)
    v_cache = torch.full((NB, bs, Hkv, D), poison[1], dtype=dtype)
    q = _t(det_normal(seed, (T, Hq, D)), dtype)
    k = _t(det_normal(seed + 1, (T, Hkv, D)), dtype)
    v = _t(det_normal(seed + 2, (T, Hkv, D)), dtype)
    slots = []
    for i, (hist, count, table, _) in enumerate(rows):
        if hist:
            ok = _t(det_normal(seed + 10 + 2 * i, (hist, Hkv, D)), dtype)
            ov = _t(det_normal(seed + 11 + 2 * i, (hist, Hkv, D)), dtype)
            for pos in range(hist):
                k_cache[table[pos // bs], pos % bs] = ok[pos]
                v_cache[table[pos // bs], pos % bs] = ov[pos]
        slots.extend(table[p // bs] * bs + p % bs for p in range(hist, hist + count))
    decode_rows = [r for r in rows if r[3] == "decode"]
    prefill_rows = [r for r in rows if r[3] != "decode"]
    d = sum(r[1] for r in decode_rows)
    meta = dict(num_decode=d, num_prefill_tokens=T - d, decode_lens=None, decode_tables=None,
                prefill_cu_q=None, prefill_cu_k=None, prefill_tables=None, max_q=0, max_k=0,
                prefill_has_history=False)
    if decode_rows:
        W = max(len(r[2]) for r in decode_rows)
        meta["decode_lens"] = _i32([r[0] + r[1] for r in decode_rows])
        meta["decode_tables"] = _i32([list(r[2]) + [-1] * (W - len(r[2])) for r in decode_rows])
    if prefill_rows:
        cu_q, cu_k = [0], [0]
        for r in prefill_rows:
            cu_q.append(cu_q[-1] + r[1])
            cu_k.append(cu_k[-1] + r[0] + r[1])
        W = max(len(r[2]) for r in prefill_rows)
        meta.update(prefill_cu_q=_i32(cu_q), prefill_cu_k=_i32(cu_k),
                    prefill_tables=_i32([list(r[2]) + [-1] * (W - len(r[2]))
                                         for r in prefill_rows]),
                    max_q=max(r[1] for r in prefill_rows),
                    max_k=max(r[0] + r[1] for r in prefill_rows),
                    prefill_has_history=any(r[0] > 0 for r in prefill_rows))
    return dict(name=name, dtype=dtype, Hq=Hq, Hkv=Hkv, D=D, bs=bs, NB=NB, q=q, k=k, v=v,
                k_cache=k_cache, v_cache=v_cache, slots=_i32(slots), meta=meta, scale=D ** -0.5)


def mixed_page_reuse(round_id):
    """tests/test_v1_attention_gpu.py:42-81 geometry: decode with history 256 (+1),
    prefill with 255 cached tokens + a 3-token chunk, pages in reverse order;
    the second pass (round_id 1) changes the page mapping and re-poisons the pool."""
    tables = [[3, 1], [2, 0]] if round_id == 0 else [[0, 2], [1, 3]]
    rows = [(256, 1, tables[0], "decode"), (255, 3, tables[1], "prefill")]
    return _mixed_from_rows(f"mixed_page_reuse_{round_id}", 100 + 50 * round_id, 8, 2, 4, rows,
                            (99.0, -99.0))


def mixed_multi_prefill():
    """tests/test_v1_attention_gpu.py:106-142 geometry: rows of 1/255/257/513 new
    tokens over histories 256/0/256/513 on scattered physical pages."""
    lengths, histories = [1, 255, 257, 513], [256, 0, 256, 513]
    physical = iter([13, 2, 11, 4, 14, 0, 9, 1, 12, 7, 5])
    tables = [[next(physical) for _ in range((h + n + 255) // 256)]
              for h, n in zip(histories, lengths)]
    rows = [(histories[0], lengths[0], tables[0], "decode")]
    rows += [(h, n, t, "prefill") for h, n, t in zip(histories[1:], lengths[1:], tables[1:])]
    return _mixed_from_rows("mixed_multi_prefill", 300, 8, 2, 16, rows, (99.0, -99.0))


def mixed_qwen_geometry(round_id):
    """tests/test_v1_reference_gpu.py:10-45 geometry: real Qwen3-4B heads 32/8,
    decode 256+1, prefill 249+8 across a page boundary and a cold 17-token row."""
    tables = [[5, 1], [3, 0], [2]] if round_id == 0 else [[0, 4], [1, 5], [3]]
    rows = [(256, 1, tables[0], "decode"), (249, 8, tables[1], "prefill"),
            (0, 17, tables[2], "prefill")]
    return _mixed_from_rows(f"mixed_qwen_geometry_{round_id}", 500 + 50 * round_id, 32, 8, 6,
                            rows, (19.0, -23.0))


def cold_prefill():
    """tests/test_v1_attention_gpu.py:83-104: one cold 256-token prefill row, no
    history, stored to block 1; attention runs on the contiguous chunk."""
    rows = [(0, 256, [1], "prefill")]
    return _mixed_from_rows("cold_prefill", 700, 8, 2, 2, rows, (0.0, 0.0))


def qk_norm_rope_case():
    """q/k RMSNorm + rotary inputs in Qwen3 head geometry (8 q heads, 2 kv heads
    of 128, non-unit norm weights, positions spread over a 4096-entry table)."""
    T, Hq, Hkv, D = 37, 8, 2, 128
    qkv = torch.from_numpy(det_normal(960, (T, (Hq + 2 * Hkv) * D)) * 3.0).bfloat16()
    wq = torch.from_numpy(det_normal(961, (D,)) * 0.3 + 1.0).bfloat16()
    wk = torch.from_numpy(det_normal(962, (D,)) * 0.3 + 1.0).bfloat16()
    pos = torch.from_numpy(det_ints(963, T, 0, 4095).astype(np.int64))
    return dict(name="qk_norm_rope", qkv=qkv, Hq=Hq, Hkv=Hkv, D=D, wq=wq, wk=wk, pos=pos,
                eps=1e-6, base=1e6, max_position=4096)


def e4m3_probe_values():
    """fp32 values for the E4M3 encoder: every finite bf16 pattern, every
    midpoint between adjacent codes and its fp32 neighbours, and a detgen sweep
    of scaled normals (values of the form x / scale)."""
    bits = np.arange(1 << 16, dtype=np.uint32) << np.uint32(16)
    bf = bits.view(np.float32)
    bf = bf[np.isfinite(bf)]
    from oracle.kv_oracle import POSITIVE_VALUES  # noqa: E402 (test infrastructure)
    pos = np.array(POSITIVE_VALUES, dtype=np.float64)
    mids = ((pos[:-1] + pos[1:]) / 2).astype(np.float32)
    neigh = np.concatenate([np.nextafter(mids, np.float32(-np.inf)),
                            np.nextafter(mids, np.float32(np.inf)), mids, -mids])
    sweep = det_normal(900, (65536,)) * np.float32(120.0) / np.float32(0.37)
    return np.concatenate([bf, neigh, sweep]).astype(np.float32)
