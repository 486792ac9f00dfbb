"""GPU parity: paged append and block-pool page copy are bit-exact against the
oracle (and, through the golden digests, against the reference's Triton store)."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden import scenarios as S
from tests.golden.detgen import det_ints, det_normal, det_perm

pytestmark = pytest.mark.gpu


def _sha(t):
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("build", [S.cfg1_decode, S.gqa_decode])
def test_append_matches_reference_digest(pkg, golden, build):
    manifest, _ = golden
    sc = build()
    kc, vc = sc["k_cache"].cuda(), sc["v_cache"].cuda()
    pkg.store_kvcache(sc["k"].cuda(), sc["v"].cuda(), kc, vc, sc["slots"].cuda())
    torch.cuda.synchronize()
    assert _sha(kc) == manifest["scenarios"][sc["name"]]["k_cache_sha256"]
    assert _sha(vc) == manifest["scenarios"][sc["name"]]["v_cache_sha256"]
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("n_tokens", [1, 7, 256, 8192])
def test_append_strided_value_view_and_padding(pkg, n_tokens):
    """v is a strided view of a fused qkv row, as Qwen3Attention produces it
    (nanovllm/models/qwen3.py:77-81); slot -1 rows (graph padding) are skipped."""
    Hq, Hkv, D, bs, NB = 32, 8, 128, 256, 48
    qkv = torch.from_numpy(det_normal(40 + n_tokens, (n_tokens, (Hq + 2 * Hkv) * D))).bfloat16()
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    k = k.view(-1, Hkv, D)
    v = v.view(-1, Hkv, D)
    perm = det_perm(41, NB * bs)[:n_tokens]
    slots = torch.from_numpy(perm.astype(np.int32))
    if n_tokens > 1:
        slots[::5] = -1
    kc = torch.from_numpy(det_normal(42, (NB, bs, Hkv, D))).bfloat16()
    vc = torch.from_numpy(det_normal(43, (NB, bs, Hkv, D))).bfloat16()
    ek, ev = kc.clone(), vc.clone()
    O.store_kvcache(k, v, ek, ev, slots)
    qkv_d = qkv.cuda()
    _, kd, vd = qkv_d.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    kcd, vcd = kc.cuda(), vc.cuda()
    pkg.store_kvcache(kd.view(-1, Hkv, D), vd.view(-1, Hkv, D), kcd, vcd, slots.cuda())
    assert torch.equal(kcd.cpu(), ek) and torch.equal(vcd.cpu(), ev)
    assert pkg.read_device_errors() == 0


def test_append_out_of_range_slot_sets_error_and_writes_nothing(pkg):
    k = torch.ones(3, 2, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([5, 512, -7], dtype=torch.int32, device="cuda")
    pkg.store_kvcache(k, k, kc, vc, slots)
    err = pkg.read_device_errors()
    assert err & pkg._lib.DEVERR_SLOT_RANGE
    assert kc.view(-1, 256)[5].float().sum().item() == 256.0
    assert kc.float().abs().sum().item() == 256.0


def _pool(NB=10, L=3, bs=256, Hkv=2, D=128, dtype=torch.bfloat16, seed=60):
    return torch.from_numpy(det_normal(seed, (2, L, NB, bs, Hkv, D))).to(dtype)


def test_block_copy_bit_exact(pkg):
    pool = _pool()
    src = torch.tensor([3, 7, 1, -1], dtype=torch.int32)
    dst = torch.tensor([0, 2, 9, 5], dtype=torch.int32)
    expect = pool.clone()
    O.block_copy(expect, src.tolist(), dst.tolist())
    dev = pool.cuda()
    pkg.kv_block_copy(dev, src.cuda(), dst.cuda())
    assert torch.equal(dev.cpu(), expect)


def test_block_gather_scatter_roundtrip(pkg, golden):
    pool = _pool(seed=61)
    ids = torch.tensor([8, 0, 4], dtype=torch.int32)
    dev = pool.cuda()
    saved = pkg.kv_block_gather(dev, ids.cuda())
    assert torch.equal(saved.cpu(), O.block_gather(pool, ids.tolist()))
    dev.fill_(-99)
    pkg.kv_block_scatter(saved, dev, ids.cuda())
    expect = torch.full_like(pool, -99)
    O.block_scatter(O.block_gather(pool, ids.tolist()), expect, ids.tolist())
    assert torch.equal(dev.cpu(), expect)


def test_block_scatter_matches_reference_restore(pkg, golden):
    """The reference's restore_kv outcome (golden) reproduced by the device scatter
    on a 16-byte-aligned page geometry (the golden pool's pages are 256 bytes)."""
    _, arrays = golden
    pool = torch.arange(2 * 3 * 6 * 4 * 2 * 8, dtype=torch.float32).reshape(2, 3, 6, 4, 2, 8)
    saved = torch.from_numpy(S.det_normal(950, (2, 3, 3, 4, 2, 8)))
    dev = pool.cuda()
    pkg.kv_block_scatter(saved.cuda(), dev, torch.tensor([4, 1, 5], dtype=torch.int32).cuda())
    np.testing.assert_array_equal(dev.cpu().numpy(), arrays["restore/pool"])


def test_block_copy_full_layer_pool_fp8_container(pkg):
    """A uint8 (FP8 code) pool copies bit-exactly too."""
    pool = torch.from_numpy(det_ints(62, 2 * 2 * 6 * 256 * 2 * 128, 0, 255).astype(np.uint8)
                            ).reshape(2, 2, 6, 256, 2, 128)
    src = torch.tensor([5, 4], dtype=torch.int32)
    dst = torch.tensor([1, 0], dtype=torch.int32)
    expect = pool.clone()
    O.block_copy(expect, src.tolist(), dst.tolist())
    dev = pool.cuda()
    pkg.kv_block_copy(dev, src.cuda(), dst.cuda())
    assert torch.equal(dev.cpu(), expect)


def test_kv_pool_bind_copy_and_scale_lifecycle(pkg):
    """KVPool binds layer views like allocate_kv_cache, copies whole blocks with
    their FP8 scales (copy-on-write), and zeroes scales of reassigned blocks."""
    pool = pkg.KVPool(num_layers=3, num_blocks=6, block_size=256, num_kv_heads=2, head_dim=128,
                      kv_dtype="fp8")
    attns = [pkg.Attention(8, 128, 128 ** -0.5, 2) for _ in range(3)]
    assert pool.bind(attns) == 3
    assert attns[2].k_cache.data_ptr() == pool.kv_cache[0, 2].data_ptr()
    assert attns[1].v_scale.data_ptr() == pool.v_scale[1].data_ptr()
    x = torch.from_numpy(det_normal(63, (300, 2, 128))).bfloat16().cuda()
    slots = torch.arange(300, dtype=torch.int32, device="cuda") + 256 * 2   # blocks 2, 3
    for a in attns:
        pkg.store_kvcache_fp8(x, x, a.k_cache, a.v_cache, a.k_scale, a.v_scale, slots)
    src = torch.tensor([2, 3], dtype=torch.int32, device="cuda")
    dst = torch.tensor([5, 0], dtype=torch.int32, device="cuda")
    pool.copy_blocks(src, dst)
    assert torch.equal(pool.kv_cache[:, :, 5], pool.kv_cache[:, :, 2])
    assert torch.equal(pool.kv_cache[:, :, 0], pool.kv_cache[:, :, 3])
    assert torch.equal(pool.k_scale[:, 5], pool.k_scale[:, 2]) and pool.k_scale[:, 5].gt(0).all()
    pool.reset_blocks(torch.tensor([5], device="cuda"))
    assert pool.k_scale[:, 5].abs().sum() == 0 and pool.v_scale[:, 5].abs().sum() == 0
    saved = pool.swap_out(torch.tensor([3], dtype=torch.int32, device="cuda"))
    pool.kv_cache[:, :, 3].zero_()
    pool.swap_in(saved, torch.tensor([3], dtype=torch.int32, device="cuda"))
    assert torch.equal(pool.kv_cache[:, :, 3], pool.kv_cache[:, :, 0])
