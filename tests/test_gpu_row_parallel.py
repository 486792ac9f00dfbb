"""Fused row-parallel linear + TP all-reduce (slokv_row_parallel_linear): the
reference's RowParallelLinear.forward (nanovllm/layers/linear.py:152-156,
y = all_reduce(F.linear(x_r, W_r))) on the tensor cores with the tile exchange
over peer memory.

On one GPU every rank of a 2/4/8-rank group runs inside one launch (emulated
ranks, one symmetric buffer per rank on this GPU), which exercises the whole
exchange: partial tiles pushed to their owner, owner reduce, broadcast of the
reduced tiles, per-call epochs.  Results are checked against the fp32 product
sum_r x_r W_r^T with the bound of the kernel's two roundings (each rank's
partial rounded to bf16, as the reference's F.linear output is, and the sum
rounded once), against cuBLAS per-rank partials summed the same way, and for
bit-equality across ranks.  tests/test_gpu_row_parallel_mp.py runs the same
check with one process per GPU."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

N = 2560  # Qwen3-4B hidden size: the o_proj / down_proj output width


def _case(seed, world, T, K, bias=False, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = [torch.randn(T, K, device="cuda", generator=g).to(dtype) for _ in range(world)]
    ws = [(torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype) for _ in range(world)]
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).to(dtype) if bias else None
    return xs, ws, b


def _check(ys, xs, ws, b):
    parts = [x.double() @ w.double().t() for x, w in zip(xs, ws)]
    exact = sum(parts) + (b.double() if b is not None else 0)
    # half an ulp of bf16 (2^-9 relative) per partial and for the final rounding,
    # doubled, plus the fp32 accumulation of each rank's K products (4 sqrt(K)
    # unit roundoffs of the sum of |products|: it dominates only where the
    # products cancel to near zero)
    absum = sum(x.double().abs() @ w.double().abs().t() for x, w in zip(xs, ws))
    K = xs[0].shape[1]
    bound = (2 ** -8 * (sum(p.abs() for p in parts) + exact.abs())
             + 4 * K ** 0.5 * 2 ** -24 * absum + 1e-6)
    for r, y in enumerate(ys):
        assert torch.isfinite(y.float()).all()
        assert torch.equal(y, ys[0]), f"rank {r} differs from rank 0"
    err = (ys[0].double() - exact).abs()
    assert (err <= bound).all(), f"max excess {(err - bound).max().item():.3e}"
    # the reference's arithmetic: cuBLAS bf16 partials, summed (fp32 here, rounded once)
    ref = sum(F.linear(x, w).float() for x, w in zip(xs, ws))
    if b is not None:
        ref = ref + b.float()
    d = (ys[0].float() - ref.to(ys[0].dtype).float()).abs()
    assert d.max().item() <= 2 ** -6 * max(1.0, ref.abs().max().item())
    assert (d == 0).float().mean().item() >= 0.95


@pytest.mark.parametrize("world,T,K,seed", [
    (1, 77, 512, 10),        # no exchange: the GEMM alone, ragged rows
    (2, 512, 2048, 11),      # o_proj at TP=2, decode batch 512
    (4, 700, 1216, 12),      # down_proj at TP=8 depth, 6 row tiles, ragged
    (8, 130, 512, 13),       # 8 ranks, 2 row tiles
    (2, 1, 1024, 14),        # a single row
    (4, 64, 8192, 15),       # long K: stream-K split with fp32 fix-ups, two-shot exchange
])
def test_row_parallel_emulated_matches_fp32(pkg, world, T, K, seed):
    xs, ws, _ = _case(seed, world, T, K)
    comm = pkg.RowParallelAllReduce.emulated(world, max_tokens=1024, n_features=N,
                                             device="cuda")
    try:
        ys = comm.emulate(xs, ws)
        torch.cuda.synchronize()
        assert pkg.read_device_errors() == 0
        _check(ys, xs, ws, None)
    finally:
        comm.close()


def test_row_parallel_f16(pkg):
    """16-bit float inputs (the f16 instantiation), two ranks."""
    xs, ws, b = _case(20, 2, 200, 1024, bias=True, dtype=torch.float16)
    comm = pkg.RowParallelAllReduce.emulated(2, max_tokens=256, n_features=N, device="cuda")
    try:
        ys = comm.emulate(xs, ws, biases=[b, b])
        torch.cuda.synchronize()
        assert pkg.read_device_errors() == 0
        _check(ys, xs, ws, b)
    finally:
        comm.close()


def test_row_parallel_bias_chunks_and_repeated_calls(pkg):
    """Bias added once; calls longer than max_tokens run in chunks; repeated
    calls on the same buffers (epochs advance, no reset) stay correct."""
    world = 4
    comm = pkg.RowParallelAllReduce.emulated(world, max_tokens=256, n_features=N, device="cuda")
    try:
        for it, T in enumerate((600, 3, 256, 129)):
            xs, ws, b = _case(100 + it, world, T, 512, bias=True)
            ys = comm.emulate(xs, ws, biases=[b] * world)
            torch.cuda.synchronize()
            assert pkg.read_device_errors() == 0
            _check(ys, xs, ws, b)
        assert int(comm.state[0].item()) == 3 + 1 + 1 + 1   # one epoch per launch (600 -> 3)
    finally:
        comm.close()


def test_row_parallel_graph_capture(pkg):
    """Captured in a CUDA graph (as the decode step is) and replayed with new
    inputs copied into the captured buffers."""
    world, T, K = 2, 384, 1024
    comm = pkg.RowParallelAllReduce.emulated(world, max_tokens=512, n_features=N, device="cuda")
    try:
        xs, ws, _ = _case(200, world, T, K)
        outs = [torch.empty(T, N, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        comm.emulate(xs, ws, outs=outs)          # eager warm-up
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            comm.emulate(xs, ws, outs=outs)
        for it in range(3):
            nx, nw, _ = _case(201 + it, world, T, K)
            for a, b in zip(xs + ws, nx + nw):
                a.copy_(b)
            graph.replay()
            torch.cuda.synchronize()
            assert pkg.read_device_errors() == 0
            _check(outs, xs, ws, None)
        del graph
    finally:
        comm.close()


def test_row_parallel_linear_module_single_rank(pkg):
    """RowParallelLinear without a process group is F.linear (TP = 1)."""
    m = pkg.RowParallelLinear(1024, N).cuda().bfloat16()
    torch.nn.init.normal_(m.weight, std=0.02)
    x = torch.randn(5, 1024, device="cuda").bfloat16()
    assert torch.equal(m(x), F.linear(x, m.weight))


def _plan(pkg, T, n, K, world, local):
    import ctypes
    plan = (ctypes.c_int32 * 5)()
    assert pkg._lib.lib().slokv_row_parallel_plan(T, n, K, world, local, plan) == 0
    return list(plan)


@pytest.mark.parametrize("world,T,n,K,seed", [
    (1, 1000, 2560, 8192, 40),    # 8 row tiles, ragged; 40 pair tiles over 74 pairs (split K)
    (1, 2048, 2560, 4096, 41),    # 80 pair tiles: stream-K over every pair
    (1, 300, 2560, 22528, 42),    # 3 row tiles: the second CTA of the last pair is padding
    (2, 1024, 640, 27648, 43),    # 5 column tiles: the last pair half is padding; one shot
    (4, 1024, 2560, 8192, 44),    # four emulated ranks of 18 pairs each, two-shot exchange
    (8, 1024, 2560, 8192, 45),    # eight emulated ranks of 9 pairs each
])
def test_row_parallel_pair_tiles(pkg, world, T, n, K, seed):
    """The 256 x 256 CTA-pair tiles (tcgen05.mma.cta_group::2), chosen for
    GEMMs of at least 2^34 multiply-adds, at shapes whose pair tiles are partly
    padding in rows or columns and whose K loops are split over pairs."""
    assert _plan(pkg, T, n, K, world, world)[0] == 2, "the pair kernel is not chosen"
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = [torch.randn(T, K, device="cuda", generator=g).bfloat16() for _ in range(world)]
    ws = [(torch.randn(n, K, device="cuda", generator=g) * 0.02).bfloat16()
          for _ in range(world)]
    comm = pkg.RowParallelAllReduce.emulated(world, max_tokens=2048, n_features=n, device="cuda")
    try:
        ys = comm.emulate(xs, ws)
        torch.cuda.synchronize()
        assert pkg.read_device_errors() == 0
        _check(ys, xs, ws, None)
    finally:
        comm.close()


def test_row_parallel_plan_query(pkg):
    """slokv_row_parallel_plan: decode-sized calls take the single-CTA kernel,
    large GEMMs the pairs; grids never exceed one CTA per SM or 160 per rank."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for T, K, world, local, kernel in ((512, 4096, 1, 1, 1), (512, 2048, 2, 1, 1),
                                       (2048, 4096, 1, 1, 2), (1024, 9728, 1, 1, 2),
                                       (1024, 8192, 4, 4, 2), (64, 4096, 8, 8, 1)):
        plan = _plan(pkg, T, 2560, K, world, local)
        assert plan[0] == kernel, (T, K, plan)
        assert 1 <= plan[2] <= plan[3] <= plan[1] <= min(160, sms // local)
        if kernel == 2:
            assert plan[1] % 2 == 0 and plan[2] % 2 == 0 and plan[3] % 2 == 0
            assert plan[1] * local <= 2 * plan[4]          # every pair co-resident
