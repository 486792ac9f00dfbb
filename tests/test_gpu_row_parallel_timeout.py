"""A rank that never arrives: the fused row-parallel all-reduce gives up.

Every wait of slokv_row_parallel_linear on a peer's flag is bounded (2 s).  On
one GPU this test builds the symmetric buffers of a 2- and a 4-rank group,
launches rank 0 alone (world = 2 or 4, rank_base = 0, local_ranks = 1) and never
launches the other ranks, so the flags rank 0 waits for are never set.  The call
must come back within a few seconds with SLOKV_DEVERR_TIMEOUT in the device
error word and leave the context usable: a plain decode-sized GEMM call right
after it (world 1) is checked against the fp32 product.  No GPU fault, trap or
hang is involved: the missing rank is simply never started."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

N = 2560


@pytest.mark.parametrize("world,T,K", [
    (2, 256, 512),      # single-CTA tiles
    (4, 256, 512),
    (2, 1024, 16384),   # CTA pairs (cta_group::2): the exchange waits of the pair kernel
])
def test_missing_rank_times_out_with_error_status(pkg, world, T, K):
    assert pkg.read_device_errors() == 0
    comm = pkg.RowParallelAllReduce.emulated(world, max_tokens=T, n_features=N, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(31 + world)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    out = torch.zeros(T, N, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    t0 = time.monotonic()
    comm._launch([x], [w], None, [out], 0)           # rank 0 of `world`, peers never start
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    errs = pkg.read_device_errors()
    comm.close()
    assert errs & pkg._lib.DEVERR_TIMEOUT, f"error word {errs:#x}"
    assert 1.5 <= elapsed <= 20.0, f"returned after {elapsed:.1f} s"
    # the context still works: the same GEMM with no exchange
    solo = pkg.RowParallelAllReduce.emulated(1, max_tokens=T, n_features=N, device="cuda")
    y = solo.emulate([x], [w])[0]
    torch.cuda.synchronize()
    exact = x.float() @ w.float().t()
    absum = x.float().abs() @ w.float().abs().t()
    assert ((y.float() - exact).abs() <= 2 ** -8 * (absum + exact.abs()) + 1e-6).all()
    assert pkg.read_device_errors() == 0
    solo.close()
