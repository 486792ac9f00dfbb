"""Pin the CPU oracle to the reference: golden fixtures produced by running the
reference's own code (tests/golden/make_golden.py) and the reference tests'
known answers.  CPU only."""
import hashlib
import math

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden import scenarios as S


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("build", [S.cfg1_decode, S.gqa_decode])
def test_decode_scenarios_match_reference(build, golden):
    manifest, arrays = golden
    sc = build()
    ref = manifest["scenarios"][sc["name"]]
    kc, vc = sc["k_cache"].clone(), sc["v_cache"].clone()
    O.store_kvcache(sc["k"], sc["v"], kc, vc, sc["slots"])
    assert _sha(kc) == ref["k_cache_sha256"]
    assert _sha(vc) == ref["v_cache_sha256"]
    out = O.decode(sc["q"].unsqueeze(1), kc, vc, sc["lens"], sc["tables"], sc["scale"])
    np.testing.assert_allclose(out.numpy(), arrays[sc["name"] + "/out"], atol=2e-5, rtol=1e-5)


MIXED = [lambda: S.mixed_page_reuse(0), lambda: S.mixed_page_reuse(1), S.mixed_multi_prefill,
         lambda: S.mixed_qwen_geometry(0), lambda: S.mixed_qwen_geometry(1), S.cold_prefill]


@pytest.mark.parametrize("build", MIXED)
def test_mixed_scenarios_match_reference(build, golden):
    manifest, arrays = golden
    sc = build()
    ref = manifest["scenarios"][sc["name"]]
    kc, vc = sc["k_cache"].clone(), sc["v_cache"].clone()
    out = O.forward_mixed(sc["q"], sc["k"], sc["v"], kc, vc, sc["meta"], sc["slots"], sc["scale"])
    assert _sha(kc) == ref["k_cache_sha256"]
    assert _sha(vc) == ref["v_cache_sha256"]
    assert list(out.shape) == ref["out_shape"]
    np.testing.assert_allclose(out[::ref["row_stride"]].numpy(), arrays[sc["name"] + "/out"],
                               atol=2e-5, rtol=1e-5)


def test_e4m3_encoders_match_reference(golden):
    _, arrays = golden
    vals = S.e4m3_probe_values()
    ref = arrays["e4m3/codes"]
    assert ref.size == vals.size
    np.testing.assert_array_equal(O.encode_e4m3fn_array(vals), ref)
    # the scalar restatement on a deterministic subsample
    idx = np.arange(0, vals.size, 97)
    assert [O.encode_e4m3fn(float(vals[i])) for i in idx] == ref[idx].tolist()


def test_restore_matches_reference(golden):
    _, arrays = golden
    pool = torch.arange(2 * 3 * 6 * 4 * 2 * 8, dtype=torch.float32).reshape(2, 3, 6, 4, 2, 8)
    saved = torch.from_numpy(S.det_normal(950, (2, 3, 3, 4, 2, 8)))
    O.block_scatter(saved, pool, [4, 1, 5])
    np.testing.assert_array_equal(pool.numpy(), arrays["restore/pool"])


def test_qk_norm_rope_matches_reference(golden):
    """The oracle's RMSNorm + rotary embedding reproduces the reference's own
    RMSNorm / RotaryEmbedding modules bit for bit (both eager torch on the CPU)."""
    manifest, _ = golden
    nc = S.qk_norm_rope_case()
    cos_sin = O.rope_cos_sin(nc["max_position"], nc["D"], nc["base"])
    q, k, _ = O.qk_norm_rope(nc["qkv"], nc["Hq"], nc["Hkv"], nc["wq"], nc["wk"], nc["eps"],
                             nc["pos"], cos_sin)
    ref = manifest["scenarios"]["qk_norm_rope"]
    assert _sha(q) == ref["q_sha256"] and _sha(k) == ref["k_sha256"]


# ---- the reference tests' own known answers ---------------------------------

def test_e4m3_known_answers():
    # tests/test_v0_quant.py:8-28
    codes = [i for i in range(256) if (i & 127) != 127]
    assert len(codes) == 254
    assert all(O.encode_e4m3fn(O.decode_e4m3fn(c)) == c for c in codes)
    assert O.encode_e4m3fn(1.0625) == 56 and O.encode_e4m3fn(1.1875) == 58
    assert O.encode_e4m3fn(-0.0) == 128
    assert O.encode_e4m3fn(1e10) == 126 and O.encode_e4m3fn(-1e10) == 254
    assert O.decode_e4m3fn(126) == 448.0
    assert math.isnan(O.decode_e4m3fn(127))
    for v in (math.nan, math.inf, -math.inf):
        with pytest.raises(ValueError):
            O.encode_e4m3fn(v)
    arr = O.encode_e4m3fn_array(np.array([O.decode_e4m3fn(c) for c in codes], np.float32))
    assert arr.tolist() == codes
    with pytest.raises(ValueError):
        O.encode_e4m3fn_array(np.array([np.nan], np.float32))


def test_dense_mask_known_answer():
    # tests/test_v1_validation.py:39-47: bottom-right aligned causal + GQA
    q = torch.zeros(2, 4, 2)
    k = torch.zeros(4, 2, 2)
    v = torch.tensor([0., 3., 6., 90.])[:, None, None].expand(4, 2, 2)
    actual = O.dense_suffix_attention(q, k, v, scale=1.)
    expected = torch.tensor([3., 24.75])[:, None, None].expand(2, 4, 2)
    torch.testing.assert_close(actual, expected)
    with pytest.raises(ValueError):
        O.dense_suffix_attention(torch.zeros(3, 2, 2), torch.zeros(2, 1, 2), torch.zeros(2, 1, 2))
    with pytest.raises(ValueError):
        O.dense_suffix_attention(torch.full((1, 2, 2), float("nan")), torch.zeros(2, 1, 2),
                                 torch.zeros(2, 1, 2))


def test_gather_reordered_pages_and_tail():
    # tests/test_layer_replay_diagnostic.py:14-22 (page order and tail)
    cache = torch.arange(12.).reshape(3, 2, 1, 2)
    actual = O.gather(cache, torch.tensor([2, 0]), 3)
    torch.testing.assert_close(actual, torch.tensor([[[8., 9.]], [[10., 11.]], [[0., 1.]]]))


def test_restore_contract_example():
    # diagnostics/online_token_replay/tests/test_contract.py:43-60 page-copy semantics
    pool = torch.arange(6, dtype=torch.float32).reshape(1, 1, 3, 2, 1, 1).repeat(2, 1, 1, 1, 1, 1)
    saved = O.block_gather(pool, [0, 2])
    saved[:, :, 0] = torch.tensor([0., 0.]).reshape(2, 1, 1)  # sanitised tail as in the reference
    pool.fill_(-99)
    O.block_scatter(saved, pool, [0, 2])
    assert pool[0, 0, :, :, 0, 0].tolist() == [[0., 0.], [-99., -99.], [4., 5.]]


def test_store_skips_padding_slots():
    k = torch.arange(2 * 1 * 4, dtype=torch.float32).reshape(2, 1, 4)
    kc = torch.zeros(1, 4, 1, 4)
    vc = torch.zeros(1, 4, 1, 4)
    O.store_kvcache(k, -k, kc, vc, torch.tensor([-1, 2], dtype=torch.int32))
    assert kc.view(-1, 4)[2].tolist() == [4., 5., 6., 7.]
    assert kc.view(-1, 4)[[0, 1, 3]].abs().sum() == 0
