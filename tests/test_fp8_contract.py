"""CPU checks of the FP8-E4M3 KV contract as restated by the oracle (the
reference has the codec but no quantised KV path, so the contract's own
properties are what is pinned here; the codec itself is pinned to the
reference's encoder in test_oracle_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden.detgen import det_normal, det_outlier_mask


def _pool(NB=4, bs=256, H=2, D=128):
    return (torch.zeros(NB, bs, H, D, dtype=torch.uint8), torch.zeros(NB, bs, H, D, dtype=torch.uint8),
            torch.zeros(NB, H, dtype=torch.float32), torch.zeros(NB, H, dtype=torch.float32))


def kv_values(seed, shape, outlier_frac=0.01):
    x = det_normal(seed, shape)
    x = np.where(det_outlier_mask(seed + 1, shape, outlier_frac), x * np.float32(20.0), x)
    return torch.from_numpy(x.astype(np.float32)).bfloat16()


def test_scale_is_running_amax_over_448():
    kc, vc, ks, vs = _pool()
    x = kv_values(1, (300, 2, 128))
    slots = torch.arange(300, dtype=torch.int32)       # blocks 0 (256 tokens) and 1 (44)
    O.fp8_append(x, x, kc, vc, ks, vs, slots)
    xf = x.float().numpy()
    for blk, (a, b) in enumerate([(0, 256), (256, 300)]):
        for h in range(2):
            amax = np.float32(np.abs(xf[a:b, h]).max())
            assert ks[blk, h].item() == np.float32(amax / np.float32(448.0))


def test_roundtrip_error_is_within_half_a_code():
    kc, vc, ks, vs = _pool()
    x = kv_values(2, (256, 2, 128))
    O.fp8_append(x, x, kc, vc, ks, vs, torch.arange(256, dtype=torch.int32))
    deq = O.fp8_dequant(kc, ks)[0]
    err = (deq - x.float()).abs()
    # relative step of E4M3 is 2^-3 (half-step 2^-4) above the subnormal range
    bound = x.float().abs() * 2 ** -4 + ks[0].view(1, 2, 1) * 2 ** -9 + 1e-30
    assert bool((err <= bound * 1.0001).all())


def test_growing_amax_reencodes_earlier_tokens():
    kc, vc, ks, vs = _pool()
    small = torch.full((1, 2, 128), 0.5, dtype=torch.bfloat16)
    big = torch.full((1, 2, 128), 8.0, dtype=torch.bfloat16)
    O.fp8_append(small, small, kc, vc, ks, vs, torch.tensor([0], dtype=torch.int32))
    assert ks[0, 0].item() == np.float32(0.5) / np.float32(448)
    assert kc[0, 0, 0, 0].item() == O.encode_e4m3fn(448.0)
    O.fp8_append(big, big, kc, vc, ks, vs, torch.tensor([1], dtype=torch.int32))
    s_new = np.float32(8.0) / np.float32(448)
    assert ks[0, 0].item() == s_new
    # token 0 re-encoded: decode(126) * (0.5/448) / (8/448) = 28 -> code of 28
    assert kc[0, 0, 0, 0].item() == O.encode_e4m3fn(28.0)
    assert O.fp8_dequant(kc, ks)[0, 0, 0, 0].item() == pytest.approx(0.5, rel=1e-6)


def test_zero_block_keeps_zero_scale_and_padding_is_skipped():
    kc, vc, ks, vs = _pool()
    z = torch.zeros(2, 2, 128, dtype=torch.bfloat16)
    O.fp8_append(z, z, kc, vc, ks, vs, torch.tensor([-1, 5], dtype=torch.int32))
    assert ks.abs().sum() == 0 and kc.sum() == 0
    assert O.fp8_dequant(kc, ks).abs().sum() == 0


def test_separate_runs_per_block_and_skipped_slots():
    kc, vc, ks, vs = _pool()
    x = kv_values(3, (6, 2, 128))
    slots = torch.tensor([254, 255, 256, -1, 600, 601], dtype=torch.int32)
    O.fp8_append(x, x, kc, vc, ks, vs, slots)
    assert ks[0].gt(0).all() and ks[1].gt(0).all() and ks[2].gt(0).all() and ks[3].eq(0).all()
    # block 2 holds tokens 4, 5 at offsets 88, 89
    amax = np.abs(x[4:6].float().numpy()).max(axis=(0, 2))
    np.testing.assert_array_equal(ks[2].numpy(), (amax / np.float32(448)).astype(np.float32))


def test_write_at_offset_zero_ignores_a_stale_scale():
    """A page handed to a new sequence keeps its previous owner's scale in the
    pool (the block manager does not touch scales); the first write, which is
    always at offset 0, must not inherit it.  A later write at offset > 0 keeps
    the running amax of the new owner only."""
    kc, vc, ks, vs = _pool()
    big = kv_values(4, (256, 2, 128)).float() * 40                     # old owner: large amax
    O.fp8_append(big.bfloat16(), big.bfloat16(), kc, vc, ks, vs, torch.arange(256, dtype=torch.int32))
    stale = ks[0].clone()
    small = kv_values(5, (10, 2, 128))
    O.fp8_append(small, small, kc, vc, ks, vs, torch.arange(10, dtype=torch.int32))
    amax = np.abs(small.float().numpy()).max(axis=(0, 2))
    fresh = (amax / np.float32(448)).astype(np.float32)
    np.testing.assert_array_equal(ks[0].numpy(), fresh)
    assert (ks[0] < stale).all()
    # codes of the new tokens are encoded against the fresh scale
    expect = O.encode_e4m3fn_array((small.float().numpy() / fresh[None, :, None]).astype(np.float32))
    np.testing.assert_array_equal(kc[0, :10].numpy(), expect)
    # a decode token at offset 10 keeps the new owner's running scale
    more = kv_values(6, (1, 2, 128)) * 0.1
    O.fp8_append(more, more, kc, vc, ks, vs, torch.tensor([10], dtype=torch.int32))
    np.testing.assert_array_equal(ks[0].numpy(), fresh)
