"""Host-side behaviour of the drop-in API that needs no GPU: the reference's own
assertions, loud failure on CPU tensors (no CPU fallback), Context plumbing."""
import pytest
import torch


def test_context_roundtrip(pkg):
    pkg.reset_context()
    assert pkg.get_context().is_prefill is False and pkg.get_context().slot_mapping is None
    sm = torch.tensor([1, 2], dtype=torch.int32)
    pkg.set_context(True, slot_mapping=sm, max_seqlen_q=3)
    ctx = pkg.get_context()
    assert ctx.is_prefill and ctx.slot_mapping is sm and ctx.max_seqlen_q == 3
    pkg.reset_context()
    assert pkg.get_context().max_seqlen_q == 0


def test_store_kvcache_reference_assertions(pkg):
    # nanovllm/layers/attention.py:36-39 assertions are kept verbatim
    k = torch.zeros(4, 2, 128)
    kc = torch.zeros(2, 256, 2, 128)
    with pytest.raises(AssertionError):
        pkg.store_kvcache(k.transpose(1, 2).contiguous().transpose(1, 2), k, kc, kc,
                          torch.zeros(4, dtype=torch.int32))
    with pytest.raises(AssertionError):
        pkg.store_kvcache(k, k, kc, kc, torch.zeros(3, dtype=torch.int32))


def test_cpu_tensors_fail_loudly(pkg):
    k = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(pkg.SlokvError, match="CUDA"):
        pkg.store_kvcache(k, k, kc, kc, torch.zeros(4, dtype=torch.int32))
    q = torch.zeros(4, 1, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(pkg.SlokvError, match="CUDA"):
        pkg.flash_attn_with_kvcache(q, kc, kc, torch.ones(4, dtype=torch.int32),
                                    torch.zeros(4, 1, dtype=torch.int32), 0.1)
    pool = torch.zeros(2, 1, 4, 256, 2, 128, dtype=torch.bfloat16)
    ids = torch.zeros(1, dtype=torch.int32)
    with pytest.raises(pkg.SlokvError, match="CUDA"):
        pkg.kv_block_copy(pool, ids, ids)


def test_decode_shape_checks(pkg):
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(pkg.SlokvError):
        pkg.flash_attn_with_kvcache(torch.zeros(4, 2, 8, 128, dtype=torch.bfloat16), kc, kc,
                                    torch.ones(4, dtype=torch.int32),
                                    torch.zeros(4, 1, dtype=torch.int32))


def test_attention_module_surface(pkg):
    attn = pkg.Attention(32, 128, 128 ** -0.5, 8)
    assert attn.num_heads == 32 and attn.num_kv_heads == 8 and attn.head_dim == 128
    assert attn.k_cache.numel() == 0 and attn.v_cache.numel() == 0
    meta = pkg.MixedAttentionContext(1, 0, None, None, None, None, None, 0, 0)
    assert meta.prefill_has_history is True


def test_mixed_requires_allocated_pool(pkg):
    # nanovllm/layers/mixed_attention.py:31-32
    ctx = pkg.Context(mixed=pkg.MixedAttentionContext(1, 0, None, None, None, None, None, 0, 0))
    empty = torch.tensor([])
    with pytest.raises(RuntimeError, match="allocated"):
        pkg.forward_mixed(torch.zeros(1, 8, 128), torch.zeros(1, 2, 128), torch.zeros(1, 2, 128),
                          empty, empty, ctx, 0.1, pkg.store_kvcache)


def test_bench_fp8_pool_fill_follows_the_config4_contract():
    """bench.fill_fp8_pool (the FP8 benches' pool contents): the blocks the
    batch reads hold E4M3 codes with per-(block, head) scale amax / 448 of
    N(0, 1) data with 1 % x20 outliers; untouched blocks stay zero."""
    import bench
    kv = torch.zeros(2, 1, 6, 256, 2, 128, dtype=torch.uint8)
    sc = torch.zeros(2, 1, 6, 2)
    g = torch.Generator().manual_seed(0)
    bench.fill_fp8_pool(kv, sc, [4, 1, 4], g, 1.0, True)
    assert (sc[:, :, [0, 2, 3, 5]] == 0).all() and (kv[:, :, [0, 2, 3, 5]] == 0).all()
    for blk in (1, 4):
        vals = kv[0, 0, blk].view(torch.float8_e4m3fn).float() * sc[0, 0, blk][None, :, None]
        amax = vals.abs().amax(dim=(0, 2))
        # the largest code of each head is the saturating 448 (scale = amax / 448)
        assert torch.allclose(amax, sc[0, 0, blk] * 448, rtol=0, atol=0)
        assert 1.5 < vals.std().item() < 3.5            # N(0,1) with 1 % x20: std ~ 2.2
