"""GPU parity of the tcgen05 prefill / varlen attention and of the mixed
prefill/decode forward against the reference's fp32 attention (golden fixtures
produced by running the reference's forward_mixed) and the oracle.

Tolerance (bf16 attention): max |err| <= 2e-2, mean |err| <= 2e-3."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden import scenarios as S
from tests.golden.detgen import det_ints, det_normal, det_perm

pytestmark = pytest.mark.gpu

MAX_TOL, MEAN_TOL = 2e-2, 2e-3


def assert_attn_close(actual, expected, max_tol=MAX_TOL, mean_tol=MEAN_TOL):
    a = actual.float().cpu().reshape(expected.shape)
    assert torch.isfinite(a).all(), "non-finite attention output"
    err = (a - expected.float()).abs()
    assert err.max().item() <= max_tol, f"max abs err {err.max().item():.3e}"
    assert err.mean().item() <= mean_tol, f"mean abs err {err.mean().item():.3e}"


def _sha(t):
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def _meta_to(pkg, meta, device):
    m = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in meta.items()}
    return pkg.MixedAttentionContext(**m)


MIXED = [lambda: S.mixed_page_reuse(0), lambda: S.mixed_page_reuse(1), S.mixed_multi_prefill,
         lambda: S.mixed_qwen_geometry(0), lambda: S.mixed_qwen_geometry(1), S.cold_prefill]


@pytest.mark.parametrize("build", MIXED)
def test_forward_mixed_matches_reference_golden(pkg, golden, build):
    """The reference tests' mixed scenarios (tests/test_v1_attention_gpu.py:42-142,
    tests/test_v1_reference_gpu.py:10-66 geometries) through our forward_mixed:
    caches bit-exact with the reference's store, outputs within tolerance of the
    reference's own fp32 forward_mixed."""
    manifest, arrays = golden
    sc = build()
    ref = manifest["scenarios"][sc["name"]]
    kc, vc = sc["k_cache"].cuda(), sc["v_cache"].cuda()
    ctx = pkg.Context(slot_mapping=sc["slots"].cuda(), mixed=_meta_to(pkg, sc["meta"], "cuda"))
    out = pkg.forward_mixed(sc["q"].cuda(), sc["k"].cuda(), sc["v"].cuda(), kc, vc, ctx,
                            sc["scale"], pkg.store_kvcache)
    torch.cuda.synchronize()
    assert _sha(kc) == ref["k_cache_sha256"] and _sha(vc) == ref["v_cache_sha256"]
    assert list(out.shape) == ref["out_shape"]
    assert_attn_close(out[::ref["row_stride"]], torch.from_numpy(arrays[sc["name"] + "/out"]))
    assert pkg.read_device_errors() == 0


def _varlen_case(seed, q_lens, hist, Hq=32, Hkv=8, D=128, bs=256, dtype=torch.bfloat16):
    """Rows with `hist` cached tokens in the pool and q_lens new tokens (stored
    through the pool too, as the engine's prefix-cache prefill does)."""
    k_lens = [h + n for h, n in zip(hist, q_lens)]
    pages = [(k + bs - 1) // bs for k in k_lens]
    NB = sum(pages) + 2
    W = max(pages)
    perm = det_perm(seed, NB).tolist()
    tables, cur = [], 0
    for n in pages:
        tables.append(perm[cur:cur + n] + [-1] * (W - n))
        cur += n
    kc = torch.from_numpy(det_normal(seed + 1, (NB, bs, Hkv, D)) * 0.5).to(dtype)
    vc = torch.from_numpy(det_normal(seed + 2, (NB, bs, Hkv, D)) * 0.5).to(dtype)
    Tq = sum(q_lens)
    q = torch.from_numpy(det_normal(seed + 3, (Tq, Hq, D))).to(dtype)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32)
    return q, kc, vc, cu_q, cu_k, torch.tensor(tables, dtype=torch.int32), max(q_lens), max(k_lens)


@pytest.mark.parametrize("q_lens,hist,Hq,Hkv,seed", [
    ([2048, 2048, 2048], [0, 1024, 3072], 32, 8, 5000),   # config 3 prefill chunks
    ([1, 127, 128, 129, 300], [0, 5, 256, 1000, 40], 32, 8, 5001),
    ([513, 64], [513, 0], 8, 2, 5002),
    ([700], [4100], 16, 2, 5003),                          # group 8
    ([200, 33], [0, 777], 8, 8, 5004),                     # group 1
])
def test_paged_varlen_matches_oracle(pkg, q_lens, hist, Hq, Hkv, seed):
    q, kc, vc, cu_q, cu_k, tables, mq, mk = _varlen_case(seed, q_lens, hist, Hq, Hkv)
    out = pkg.flash_attn_varlen_func(q.cuda(), kc.cuda(), vc.cuda(), cu_seqlens_q=cu_q.cuda(),
                                     cu_seqlens_k=cu_k.cuda(), max_seqlen_q=mq, max_seqlen_k=mk,
                                     softmax_scale=128 ** -0.5, causal=True,
                                     block_table=tables.cuda())
    torch.cuda.synchronize()
    expect = O.varlen(q, kc, vc, cu_q, cu_k, 128 ** -0.5, tables)
    assert_attn_close(out, expect)
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("lens,seed", [([256], 5100), ([1, 2, 130, 1000], 5101),
                                       ([2048, 17], 5102)])
def test_contiguous_varlen_with_strided_v(pkg, lens, seed):
    """Cold prefill on the step's own k/v, v being a strided view of a fused QKV
    row (nanovllm/models/qwen3.py:77-81)."""
    Hq, Hkv, D = 32, 8, 128
    T = sum(lens)
    qkv = torch.from_numpy(det_normal(seed, (T, (Hq + 2 * Hkv) * D))).bfloat16()
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    q, k, v = q.reshape(T, Hq, D), k.reshape(T, Hkv, D), v.view(T, Hkv, D)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    qkv_d = qkv.cuda()
    qd, kd, vd = qkv_d.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    out = pkg.flash_attn_varlen_func(qd.reshape(T, Hq, D), kd.reshape(T, Hkv, D),
                                     vd.view(T, Hkv, D), cu_seqlens_q=cu.cuda(),
                                     cu_seqlens_k=cu.cuda(), max_seqlen_q=max(lens),
                                     max_seqlen_k=max(lens), softmax_scale=128 ** -0.5)
    expect = O.varlen(q, k, v, cu, cu, 128 ** -0.5, None)
    assert_attn_close(out, expect)


def test_fewer_keys_than_queries_gives_zero_rows(pkg):
    """Bottom-right alignment with q_len > k_len: the first q_len - k_len queries
    see no key and produce zeros; the rest match the oracle on their suffix."""
    Hq, Hkv, D = 8, 2, 128
    q = torch.from_numpy(det_normal(5200, (200, Hq, D))).bfloat16()
    k = torch.from_numpy(det_normal(5201, (150, Hkv, D))).bfloat16()
    v = torch.from_numpy(det_normal(5202, (150, Hkv, D))).bfloat16()
    cu_q = torch.tensor([0, 200], dtype=torch.int32)
    cu_k = torch.tensor([0, 150], dtype=torch.int32)
    out = pkg.flash_attn_varlen_func(q.cuda(), k.cuda(), v.cuda(), cu_q.cuda(), cu_k.cuda(),
                                     200, 150, softmax_scale=128 ** -0.5).float().cpu()
    assert out[:50].abs().sum() == 0
    expect = O.dense_suffix_attention(q[50:], k, v, 128 ** -0.5)
    assert_attn_close(out[50:], expect)


def test_config3_mixed_batch(pkg):
    """64 decode rows (context U[256, 4096]) + 3 prefill chunks
    of 2048 tokens over cached prefixes 0 / 1024 / 3072, in one forward_mixed."""
    Hq, Hkv, D, bs = 32, 8, 128, 256
    dec_lens = det_ints(1, 64, 256, 4096).tolist()
    hist = [0, 1024, 3072]
    rows = [(L - 1, 1) for L in dec_lens] + [(h, 2048) for h in hist]
    k_lens = [h + n for h, n in rows]
    pages = [(k + bs - 1) // bs for k in k_lens]
    NB = sum(pages) + 4
    perm = det_perm(7, NB).tolist()
    tables, cur = [], 0
    for n in pages:
        tables.append(perm[cur:cur + n])
        cur += n
    kc = torch.from_numpy(det_normal(8, (NB, bs, Hkv, D)) * 0.5).bfloat16()
    vc = torch.from_numpy(det_normal(9, (NB, bs, Hkv, D)) * 0.5).bfloat16()
    T = sum(n for _, n in rows)
    q = torch.from_numpy(det_normal(10, (T, Hq, D))).bfloat16()
    k = torch.from_numpy(det_normal(11, (T, Hkv, D)) * 0.5).bfloat16()
    v = torch.from_numpy(det_normal(12, (T, Hkv, D)) * 0.5).bfloat16()
    slots = [t[p // bs] * bs + p % bs for t, (h, n) in zip(tables, rows) for p in range(h, h + n)]
    W = max(pages)
    pad = lambda ts: torch.tensor([t + [-1] * (W - len(t)) for t in ts], dtype=torch.int32)
    cu_q = [0]
    cu_k = [0]
    for h, n in rows[64:]:
        cu_q.append(cu_q[-1] + n)
        cu_k.append(cu_k[-1] + h + n)
    meta = dict(num_decode=64, num_prefill_tokens=3 * 2048,
                decode_lens=torch.tensor(dec_lens, dtype=torch.int32), decode_tables=pad(tables[:64]),
                prefill_cu_q=torch.tensor(cu_q, dtype=torch.int32),
                prefill_cu_k=torch.tensor(cu_k, dtype=torch.int32), prefill_tables=pad(tables[64:]),
                max_q=2048, max_k=max(k_lens[64:]), prefill_has_history=True)
    sl = torch.tensor(slots, dtype=torch.int32)
    ek, ev = kc.clone(), vc.clone()
    expect = O.forward_mixed(q, k, v, ek, ev, meta, sl, 128 ** -0.5)
    kcd, vcd = kc.cuda(), vc.cuda()
    ctx = pkg.Context(slot_mapping=sl.cuda(), mixed=_meta_to(pkg, meta, "cuda"))
    out = pkg.forward_mixed(q.cuda(), k.cuda(), v.cuda(), kcd, vcd, ctx, 128 ** -0.5,
                            pkg.store_kvcache)
    torch.cuda.synchronize()
    assert torch.equal(kcd.cpu(), ek) and torch.equal(vcd.cpu(), ev)
    assert_attn_close(out, expect)
    assert pkg.read_device_errors() == 0


def test_attention_module_prefill_with_prefix_cache(pkg):
    """Attention.forward in a prefill context with block tables (prefix cache),
    as set by the reference's ModelRunner.prepare_prefill (model_runner.py:129-170)."""
    q, kc, vc, cu_q, cu_k, tables, mq, mk = _varlen_case(5300, [300, 50], [256, 0], 32, 8)
    Tq = q.shape[0]
    k = torch.from_numpy(det_normal(5301, (Tq, 8, 128)) * 0.5).bfloat16()
    v = torch.from_numpy(det_normal(5302, (Tq, 8, 128)) * 0.5).bfloat16()
    slots = []
    for r, (h, n) in enumerate([(256, 300), (0, 50)]):
        slots += [int(tables[r, p // 256]) * 256 + p % 256 for p in range(h, h + n)]
    sl = torch.tensor(slots, dtype=torch.int32)
    ek, ev = kc.clone(), vc.clone()
    O.store_kvcache(k, v, ek, ev, sl)
    expect = O.varlen(q, ek, ev, cu_q, cu_k, 128 ** -0.5, tables)
    attn = pkg.Attention(32, 128, 128 ** -0.5, 8)
    attn.k_cache, attn.v_cache = kc.cuda(), vc.cuda()
    pkg.set_context(True, cu_q.cuda(), cu_k.cuda(), mq, mk, sl.cuda(), None, tables.cuda())
    out = attn(q.cuda(), k.cuda(), v.cuda())
    pkg.reset_context()
    assert_attn_close(out, expect)


@pytest.mark.parametrize("q_lens,hist,seed", [
    ([2048, 2048, 2048], [0, 1024, 3072], 5400),
    ([1, 127, 128, 129, 300, 2000, 5], [0, 5, 256, 1000, 40, 9000, 3], 5401),
])
def test_longest_first_order_matches_row_major(pkg, q_lens, hist, seed):
    """The longest-first work order (workspace given) and the row-major order
    (no workspace) compute every query tile identically: outputs bit-equal."""
    from importlib import import_module
    _lib = import_module("slo-aware-llm-serving-engine_b200._lib")
    q, kc, vc, cu_q, cu_k, tables, mq, mk = _varlen_case(seed, q_lens, hist, 32, 8)
    q, kc, vc, cu_q, cu_k, tables = (t.cuda() for t in (q, kc, vc, cu_q, cu_k, tables))
    ordered = pkg.flash_attn_varlen_func(q, kc, vc, cu_q, cu_k, mq, mk,
                                         softmax_scale=128 ** -0.5, block_table=tables)
    plain = torch.full_like(ordered, float("nan"))
    rows = cu_q.numel() - 1
    assert _lib.lib().slokv_paged_prefill_workspace_bytes(rows, mq) >= rows * ((mq + 127) // 128) * 4
    err = _lib.buffers.error_word(q.device)
    _lib.check(_lib.lib().slokv_paged_prefill(
        plain.data_ptr(), plain.stride(0), plain.stride(1), q.data_ptr(), q.stride(0), q.stride(1),
        q.shape[0], kc.data_ptr(), vc.data_ptr(), 0, 0, 0, kc.stride(0), vc.stride(0),
        cu_q.data_ptr(), cu_k.data_ptr(), rows, mq, tables.data_ptr(), tables.stride(0),
        tables.shape[1], kc.shape[0], 256, 32, 8, 128, 128 ** -0.5, _lib.DTYPE_BF16, None, None, 0,
        err.data_ptr(), _lib.stream_ptr(q.device)), "paged_prefill")
    torch.cuda.synchronize()
    assert torch.equal(ordered, plain)
    assert pkg.read_device_errors() == 0
