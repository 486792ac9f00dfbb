"""GPU parity of the fused q/k RMSNorm + rotary embedding + append
(qk_norm_rope_append) against the oracle's restatement of the reference's
RMSNorm and rotary embedding (nanovllm/layers/layernorm.py,
nanovllm/layers/rotary_embedding.py; pinned to the reference's own modules by
the golden fixture) and store_kvcache.

Bar: q and k equal to the oracle on at least 99 % of the elements.  The one
reordered step (the 128-term sum of squares, and rsqrtf against the CPU's
rsqrt) can move a normed value by one bf16 unit in the last place, which the
rotation carries into its outputs: every element within 2^-8 sqrt(x1^2 + x2^2)
(one unit of the rotated pair's inputs) + one unit of the output.  Cache rows
bit-equal to the returned k and to the raw v; rows of slot -1 tokens untouched."""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden.detgen import det_ints, det_normal, det_perm

pytestmark = pytest.mark.gpu


def _ulp_bf16(x):
    """One bf16 unit in the last place at |x| (x fp32)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(1e-30)))
    return torch.pow(2.0, e - 7)


@pytest.mark.parametrize("T,Hq,Hkv,seed", [(300, 32, 8, 7000), (1, 16, 4, 7001), (2048, 8, 2, 7002)])
def test_fused_norm_rope_append_matches_oracle(pkg, T, Hq, Hkv, seed):
    D, bs, NB, eps = 128, 256, 12, 1e-6
    qkv = torch.from_numpy(det_normal(seed, (T, (Hq + 2 * Hkv) * D)) * 3.0).bfloat16()
    wq = torch.from_numpy(det_normal(seed + 1, (D,)) * 0.3 + 1.0).bfloat16()
    wk = torch.from_numpy(det_normal(seed + 2, (D,)) * 0.3 + 1.0).bfloat16()
    pos = torch.from_numpy(det_ints(seed + 3, T, 0, 40959).astype(np.int64))
    cos_sin = O.rope_cos_sin(40960, D, 1e6)
    slots = torch.from_numpy(det_perm(seed + 4, NB * bs)[:T].astype(np.int32))
    slots[::7] = -1
    kc = torch.from_numpy(det_normal(seed + 5, (NB, bs, Hkv, D))).bfloat16()
    vc = torch.from_numpy(det_normal(seed + 6, (NB, bs, Hkv, D))).bfloat16()
    eq, ek, ev = O.qk_norm_rope(qkv, Hq, Hkv, wq, wk, eps, pos, cos_sin)
    kcd, vcd = kc.cuda(), vc.cuda()
    q, k = pkg.qk_norm_rope_append(qkv.cuda(), Hq, Hkv, wq.cuda(), wk.cuda(), eps, pos.cuda(),
                                   cos_sin.cuda(), slots.cuda(), kcd, vcd, k_out=True)
    torch.cuda.synchronize()
    assert pkg.read_device_errors() == 0
    qkv3 = qkv.view(T, Hq + 2 * Hkv, D)
    for got, want, normed in ((q.cpu().float(), eq.float(), O.rms_norm(qkv3[:, :Hq], wq, eps)),
                              (k.cpu().float(), ek.float(),
                               O.rms_norm(qkv3[:, Hq:Hq + Hkv], wk, eps))):
        x = normed.float()
        pair = torch.sqrt(x[..., :64] ** 2 + x[..., 64:] ** 2).repeat(1, 1, 2)
        diff = (got - want).abs()
        exact = (diff == 0).float().mean().item()
        bound = pair * 2.0 ** -8 + _ulp_bf16(want) + 1e-30
        print(f"exact {exact:.5f}, max diff / bound {(diff / bound).max().item():.3f}")
        assert (diff <= bound).all(), f"max diff {diff.max().item():.3e}"
        assert exact >= 0.99
    kcf, vcf = kcd.cpu().view(-1, Hkv, D), vcd.cpu().view(-1, Hkv, D)
    live = slots >= 0
    assert torch.equal(kcf[slots[live].long()], k.cpu()[live])
    assert torch.equal(vcf[slots[live].long()], ev[live])
    untouched = torch.ones(NB * bs, dtype=torch.bool)
    untouched[slots[live].long()] = False
    assert torch.equal(kcf[untouched], kc.view(-1, Hkv, D)[untouched])
    assert torch.equal(vcf[untouched], vc.view(-1, Hkv, D)[untouched])


def test_fused_norm_rope_position_outside_table_is_flagged(pkg):
    Hq, Hkv, D = 8, 2, 128
    qkv = torch.ones(2, (Hq + 2 * Hkv) * D, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    cos_sin = O.rope_cos_sin(16, D, 1e6).cuda()
    kc = torch.zeros(1, 256, Hkv, D, dtype=torch.bfloat16, device="cuda")
    pkg.qk_norm_rope_append(qkv, Hq, Hkv, w, w, 1e-6,
                            torch.tensor([3, 99], dtype=torch.int64, device="cuda"), cos_sin,
                            torch.tensor([0, 1], dtype=torch.int32, device="cuda"), kc,
                            kc.clone())
    assert pkg.read_device_errors() & pkg._lib.DEVERR_CONTEXT_LEN
