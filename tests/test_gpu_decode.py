"""GPU parity: paged decode attention against the reference's fp32 torch
attention (golden fixtures) and the oracle restatement of it.

Tolerance (BF16 attention): max |err| <= 2e-2 and
mean |err| <= 2e-3 against the fp32 result on the same bf16 inputs."""
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


def make_decode_case(seed, B, Hq, Hkv, lens, NB=None, bs=256, D=128, dtype=torch.bfloat16,
                     poison=None):
    """Random paged layout: each sequence gets ceil(L/bs) distinct random blocks."""
    pages = [(L + bs - 1) // bs for L in lens]
    W = max(1, max(pages))
    NB = NB or max(sum(pages) + 3, 4)
    perm = det_perm(seed, NB).tolist()
    tables, cur = [], 0
    for n in pages:
        tables.append(perm[cur:cur + n] + [-1] * (W - n))
        cur += n
    kc = torch.from_numpy(det_normal(seed + 1, (NB, bs, Hkv, D)) * 0.5).to(dtype)
    vc = torch.from_numpy(det_normal(seed + 2, (NB, bs, Hkv, D)) * 0.5).to(dtype)
    if poison is not None:
        # stale bytes everywhere a sequence does not own a valid position
        valid = torch.zeros(NB, bs, dtype=torch.bool)
        for t, L in zip(tables, lens):
            for p in range(L):
                valid[t[p // bs], p % bs] = True
        kc[~valid] = poison
        vc[~valid] = poison
    q = torch.from_numpy(det_normal(seed + 3, (B, Hq, D))).to(dtype)
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32), torch.tensor(tables, dtype=torch.int32)


def run_decode(pkg, q, kc, vc, lens, tables, scale):
    out = pkg.flash_attn_with_kvcache(q.cuda().unsqueeze(1), kc.cuda(), vc.cuda(),
                                      cache_seqlens=lens.cuda(), block_table=tables.cuda(),
                                      softmax_scale=scale, causal=True)
    torch.cuda.synchronize()
    return out


def test_decode_matches_reference_golden(pkg, golden):
    """Store + decode of the GQA scenario against the reference's own fp32 decode."""
    manifest, arrays = golden
    sc = S.gqa_decode()
    kc, vc = sc["k_cache"].cuda(), sc["v_cache"].cuda()
    pkg.store_kvcache(sc["k"].cuda(), sc["v"].cuda(), kc, vc, sc["slots"].cuda())
    out = pkg.flash_attn_with_kvcache(sc["q"].cuda().unsqueeze(1), kc, vc,
                                      cache_seqlens=sc["lens"].cuda(),
                                      block_table=sc["tables"].cuda(),
                                      softmax_scale=sc["scale"], causal=True)
    assert out.shape == (6, 1, 8, 128) and out.dtype == torch.bfloat16
    assert_attn_close(out, torch.from_numpy(arrays["gqa_decode/out"]))
    assert pkg.read_device_errors() == 0


def test_decode_config1_geometry_bf16(pkg):
    """BASELINE config 1 (Qwen3-4B heads, pool 64 x 256, batch 8) run in bf16 on the
    GPU, checked against the fp32 oracle on the same bf16 values."""
    sc = S.cfg1_decode()
    bf = {k: sc[k].bfloat16() for k in ("q", "k", "v", "k_cache", "v_cache")}
    ek, ev = bf["k_cache"].clone(), bf["v_cache"].clone()
    O.store_kvcache(bf["k"], bf["v"], ek, ev, sc["slots"])
    expect = O.decode(bf["q"].unsqueeze(1), ek, ev, sc["lens"], sc["tables"], sc["scale"])
    kc, vc = bf["k_cache"].cuda(), bf["v_cache"].cuda()
    pkg.store_kvcache(bf["k"].cuda(), bf["v"].cuda(), kc, vc, sc["slots"].cuda())
    assert torch.equal(kc.cpu(), ek) and torch.equal(vc.cpu(), ev)
    out = run_decode(pkg, bf["q"], kc, vc, sc["lens"], sc["tables"], sc["scale"])
    assert_attn_close(out, expect)


@pytest.mark.parametrize("B,Hq,Hkv,lo,hi,seed", [
    (256, 32, 8, 512, 4096, 1000),   # config 2 shape (one layer)
    (3, 32, 8, 3000, 9000, 1001),    # few long sequences: many warp splits + merge
    (200, 32, 8, 1, 40, 1002),       # many tiny segments
    (17, 8, 8, 1, 700, 1003),        # GQA group 1
    (9, 16, 2, 1, 1500, 1004),       # group 8
    (5, 32, 2, 1, 900, 1005),        # group 16
    (64, 4, 1, 100, 3000, 1006),     # a TP=8 shard of Qwen3-4B (1 KV head)
])
def test_decode_random_layouts(pkg, B, Hq, Hkv, lo, hi, seed):
    lens = det_ints(seed, B, lo, hi).tolist()
    q, kc, vc, lens_t, tables = make_decode_case(seed, B, Hq, Hkv, lens)
    expect = O.decode(q.unsqueeze(1), kc, vc, lens_t, tables, 128 ** -0.5)
    out = run_decode(pkg, q, kc, vc, lens_t, tables, 128 ** -0.5)
    assert_attn_close(out, expect)
    assert pkg.read_device_errors() == 0


def test_decode_fp16(pkg):
    lens = det_ints(1010, 12, 1, 2000).tolist()
    q, kc, vc, lens_t, tables = make_decode_case(1010, 12, 32, 8, lens, dtype=torch.float16)
    expect = O.decode(q.unsqueeze(1), kc, vc, lens_t, tables, 0.088)
    out = run_decode(pkg, q, kc, vc, lens_t, tables, 0.088)
    assert out.dtype == torch.float16
    assert_attn_close(out, expect)


def test_zero_length_rows_and_nan_stale_pages(pkg):
    """Graph padding rows (context_lens = 0) give zeros; stale pool bytes (NaN)
    past each context never reach the output."""
    lens = [0, 1, 33, 0, 256, 257, 511]
    q, kc, vc, lens_t, tables = make_decode_case(1020, len(lens), 32, 8, lens,
                                                 poison=float("nan"))
    out = run_decode(pkg, q, kc, vc, lens_t, tables, 128 ** -0.5).float().cpu()
    assert torch.isfinite(out).all()
    assert out[0].abs().sum() == 0 and out[3].abs().sum() == 0
    expect = O.decode(q.unsqueeze(1), kc.nan_to_num(0.0), vc.nan_to_num(0.0), lens_t, tables,
                      128 ** -0.5)
    assert_attn_close(out, expect)


def test_stale_table_columns_are_not_read(pkg):
    """Entries past ceil(L / block_size) may be stale or garbage (graph replay
    overwrites only [:bs, :W]); they must not be dereferenced."""
    lens = [300, 40]
    q, kc, vc, lens_t, tables = make_decode_case(1030, 2, 32, 8, lens)
    wide = torch.full((2, 6), 10 ** 6, dtype=torch.int32)
    wide[:, :tables.shape[1]] = tables
    wide[0, 2:] = 10 ** 6
    wide[1, 1:] = -5
    out = run_decode(pkg, q, kc, vc, lens_t, wide, 128 ** -0.5)
    expect = O.decode(q.unsqueeze(1), kc, vc, lens_t, tables, 128 ** -0.5)
    assert_attn_close(out, expect)
    assert pkg.read_device_errors() == 0


def test_invalid_block_id_sets_error_without_fault(pkg):
    lens = [300]
    q, kc, vc, lens_t, tables = make_decode_case(1040, 1, 32, 8, lens)
    tables[0, 1] = 10 ** 6                        # inside ceil(L/256): will be read
    out = run_decode(pkg, q, kc, vc, lens_t, tables, 128 ** -0.5)
    assert torch.isfinite(out.float()).all()
    assert pkg.read_device_errors() & pkg._lib.DEVERR_BLOCK_RANGE


def test_decode_is_graph_capturable(pkg):
    """Capture once, replay with new lengths/tables/queries written into the same
    buffers, as the reference's decode graph replay does
    (nanovllm/engine/model_runner.py:196-212)."""
    B, Hq, Hkv = 16, 32, 8
    lens1 = det_ints(1050, B, 1, 1200).tolist()
    q, kc, vc, lens_t, tables = make_decode_case(1050, B, Hq, Hkv, lens1, NB=130)
    qd, kcd, vcd = q.cuda().unsqueeze(1), kc.cuda(), vc.cuda()
    ld, td = lens_t.cuda(), torch.full((B, 8), -1, dtype=torch.int32, device="cuda")
    td[:, :tables.shape[1]] = tables.cuda()
    out = pkg.flash_attn_with_kvcache(qd, kcd, vcd, cache_seqlens=ld, block_table=td,
                                      softmax_scale=128 ** -0.5)       # warm-up (workspace)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = pkg.flash_attn_with_kvcache(qd, kcd, vcd, cache_seqlens=ld, block_table=td,
                                          softmax_scale=128 ** -0.5)
    for step, seed in enumerate((1051, 1052)):
        lens2 = det_ints(seed, B, 0, 2000).tolist()
        perm = det_perm(seed, 130).tolist()
        t2 = torch.full((B, 8), -1, dtype=torch.int32)
        cur = 0
        for b, L in enumerate(lens2):
            n = (L + 255) // 256
            t2[b, :n] = torch.tensor(perm[cur:cur + n], dtype=torch.int32)
            cur += n
        q2 = torch.from_numpy(det_normal(seed, (B, Hq, 128))).bfloat16()
        qd.copy_(q2.cuda().unsqueeze(1))
        ld.copy_(torch.tensor(lens2, dtype=torch.int32).cuda())
        td.copy_(t2.cuda())
        g.replay()
        torch.cuda.synchronize()
        expect = O.decode(q2.unsqueeze(1), kc, vc, torch.tensor(lens2, dtype=torch.int32), t2,
                          128 ** -0.5)
        assert_attn_close(out, expect)
    del g


# fp32 pools (BASELINE config 1 is the reference's fp32 case): CUDA-core fp32
# arithmetic, so the bar is fp32 summation-order noise, not the bf16 one.
F32_MAX_TOL, F32_MEAN_TOL = 2e-5, 2e-6


def test_decode_config1_fp32_matches_reference_golden(pkg, golden):
    """BASELINE config 1 exactly as specified -- fp32 q/K/V, Qwen3-4B heads, pool
    64 x 256, batch 8, L ~ U[1, 2048] -- on the GPU: fp32 append bit-exact with
    the reference's Triton store (SHA-256 of its caches) and fp32 decode against
    the reference's own fp32 decode output."""
    import hashlib
    manifest, arrays = golden
    sc = S.cfg1_decode()
    assert sc["k_cache"].dtype == torch.float32
    kc, vc = sc["k_cache"].cuda(), sc["v_cache"].cuda()
    pkg.store_kvcache(sc["k"].cuda(), sc["v"].cuda(), kc, vc, sc["slots"].cuda())
    sha = lambda t: hashlib.sha256(t.cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    assert sha(kc) == manifest["scenarios"]["cfg1_decode"]["k_cache_sha256"]
    assert sha(vc) == manifest["scenarios"]["cfg1_decode"]["v_cache_sha256"]
    out = pkg.flash_attn_with_kvcache(sc["q"].cuda().unsqueeze(1), kc, vc,
                                      cache_seqlens=sc["lens"].cuda(),
                                      block_table=sc["tables"].cuda(),
                                      softmax_scale=sc["scale"], causal=True)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    assert_attn_close(out, torch.from_numpy(arrays["cfg1_decode/out"]), F32_MAX_TOL, F32_MEAN_TOL)
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("B,Hq,Hkv,lo,hi,seed", [
    (8, 32, 8, 1, 2048, 1100),      # config 1 distribution, other draws
    (5, 16, 2, 200, 3000, 1101),    # group 8, contexts over many chunks
    (7, 8, 8, 1, 300, 1102),        # group 1
])
def test_decode_fp32_random_layouts(pkg, B, Hq, Hkv, lo, hi, seed):
    lens = det_ints(seed, B, lo, hi).tolist()
    lens[0] = 0                       # a padded row: zeros
    q, kc, vc, lens_t, tables = make_decode_case(seed, B, Hq, Hkv, [max(L, 1) for L in lens],
                                                 dtype=torch.float32)
    lens_t[0] = 0
    expect = O.decode(q.unsqueeze(1), kc, vc, lens_t, tables, 128 ** -0.5)
    out = run_decode(pkg, q, kc, vc, lens_t, tables, 128 ** -0.5)
    assert_attn_close(out, expect, F32_MAX_TOL, F32_MEAN_TOL)
    assert out[0].abs().sum().item() == 0
    assert pkg.read_device_errors() == 0
