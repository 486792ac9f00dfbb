"""GPU test of the allocation-free decode entry point (slokv_paged_decode_noalloc).

That entry point exists for callers that cannot call cudaMalloc -- a host that
binds only the C ABI and has no device allocator, or an engine whose allocator
has already handed most of HBM to the KV pool -- so its split-K scratch is a
fixed device array inside the library instead of a caller-supplied workspace.
This test calls it through the C ABI twice in a row, on different inputs, and
checks each result against the workspace entry point (slokv_paged_decode,
reached through flash_attn_with_kvcache) and against the CPU oracle of the
reference's attention, with the decode tolerance used by every attention test:
max |err| <= 2e-2, mean |err| <= 2e-3.  The file sorts last so that a run
stopping at its first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as O
from tests.golden.detgen import det_ints, det_normal, det_perm

pytestmark = pytest.mark.gpu

MAX_TOL, MEAN_TOL = 2e-2, 2e-3


def _case(seed, B=48, Hq=32, Hkv=8, D=128, bs=256, lo=1, hi=3000):
    lens = det_ints(seed, B, lo, hi)
    pages = (lens + bs - 1) // bs
    NB = int(pages.sum()) + 4
    W = int(pages.max())
    perm = det_perm(seed + 1, NB)
    tables = np.full((B, W), -1, dtype=np.int32)
    cur = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[cur:cur + n]
        cur += n
    dev = "cuda"
    kc = torch.from_numpy(det_normal(seed + 2, (NB, bs, Hkv, D)) * 0.5).bfloat16().to(dev)
    vc = torch.from_numpy(det_normal(seed + 3, (NB, bs, Hkv, D)) * 0.5).bfloat16().to(dev)
    q = torch.from_numpy(det_normal(seed + 4, (B, 1, Hq, D))).bfloat16().to(dev)
    return (q, kc, vc, torch.from_numpy(lens.astype(np.int32)).to(dev),
            torch.from_numpy(tables).to(dev))


def _noalloc(lib, out, q, kc, vc, lens, tables, scale, err):
    B, _, Hq, D = q.shape
    NB, bs, Hkv, _ = kc.shape
    return lib.slokv_paged_decode_noalloc(
        out.data_ptr(), out.stride(0), out.stride(2), q.data_ptr(), q.stride(0), q.stride(2),
        kc.data_ptr(), vc.data_ptr(), kc.stride(0), vc.stride(0), NB, bs, Hq, Hkv, D,
        tables.data_ptr(), tables.stride(0), tables.shape[1], lens.data_ptr(), B, scale,
        0, err.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_decode_matches_workspace_entry_point(pkg):
    lib = pkg._lib.lib()
    assert lib.slokv_paged_decode_noalloc_scratch_bytes() == 6 << 20
    scale = 128 ** -0.5
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed in (4100, 4200):            # two calls in a row, different inputs
        q, kc, vc, lens, tables = _case(seed)
        expect = pkg.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens, block_table=tables,
                                             softmax_scale=scale)
        out = torch.full_like(q, float("nan"))
        status = _noalloc(lib, out, q, kc, vc, lens, tables, scale, err)
        assert status == 0, lib.slokv_status_string(status)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        diff = (out.float() - expect.float()).abs()
        assert diff.max().item() <= MAX_TOL and diff.mean().item() <= MEAN_TOL
        oracle = O.decode(q.cpu(), kc.cpu(), vc.cpu(), lens.cpu(), tables.cpu(), scale)
        odiff = (out.float().cpu() - oracle).abs()
        assert odiff.max().item() <= MAX_TOL and odiff.mean().item() <= MEAN_TOL, (
            f"vs oracle: max {odiff.max().item():.3e} mean {odiff.mean().item():.3e}")
        assert int(err.item()) == 0


def test_noalloc_rejects_geometry_beyond_scratch(pkg):
    lib = pkg._lib.lib()
    # 16 query heads per KV head: SMs x 3 warp slots x (2 x 16 x 132 x 4 + 16)
    # bytes of partials, beyond 6 MiB on a 148-SM part: rejected, nothing launched.
    need = lib.slokv_paged_decode_workspace_bytes(0, 32, 2, 128)
    if need <= lib.slokv_paged_decode_noalloc_scratch_bytes():
        pytest.skip("this device's SM count fits group 16 in the scratch")
    q, kc, vc, lens, tables = _case(4300, B=4, Hq=32, Hkv=2)
    out = torch.zeros_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = _noalloc(lib, out, q, kc, vc, lens, tables, 0.1, err)
    assert status == pkg._lib.ERR_SCRATCH_LIMIT
    assert b"fixed scratch" in lib.slokv_status_string(status)
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0


def test_noalloc_status_matches_workspace_entry_point(pkg):
    """Arguments the decode itself refuses get the decode's own status, not the
    scratch-limit one, and an empty batch is a no-op, whatever the geometry."""
    lib = pkg._lib.lib()
    q, kc, vc, lens, tables = _case(4400, B=4, Hq=32, Hkv=2)
    out = torch.zeros_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    B, _, Hq, D = q.shape
    NB, bs, Hkv, _ = kc.shape
    stream = torch.cuda.current_stream().cuda_stream

    def call(batch, hq, hkv):
        return lib.slokv_paged_decode_noalloc(
            out.data_ptr(), out.stride(0), out.stride(2), q.data_ptr(), q.stride(0),
            q.stride(2), kc.data_ptr(), vc.data_ptr(), kc.stride(0), vc.stride(0), NB, bs, hq,
            hkv, D, tables.data_ptr(), tables.stride(0), tables.shape[1], lens.data_ptr(), batch,
            0.1, 0, err.data_ptr(), stream)

    assert call(0, 32, 2) == pkg._lib.OK                 # empty batch: nothing to do
    assert call(B, 34, 2) == pkg._lib.ERR_UNSUPPORTED    # group 17: not built
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0 and int(err.item()) == 0
