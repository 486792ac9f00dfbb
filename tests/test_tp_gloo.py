"""Multi-rank host logic on CPU with the gloo backend (world size 2): the pool
capacity is the minimum over tensor-parallel ranks (as the reference's
MixedModelRunner.allocate_kv_cache does with an NCCL all-reduce), head shards
keep GQA groups rank-local, and every rank derives the same batch metadata."""
import hashlib
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import importlib
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
        per_block = pkg.block_bytes(36, 256, 8 // world, 128, "bf16")
        # ranks see different free memory; both must settle on the smaller count
        total = 180 * 2 ** 30
        used = (10 + 15 * rank) * 2 ** 30
        n = pkg.plan_num_blocks(total, used, 0, 0, per_block, 0.9)
        q_heads, kv_heads = pkg.tp_shard(32, 8, world, rank)
        import bench
        B, lens, pages, _ = bench.make_metadata(world)
        digest = hashlib.sha256(lens.numpy().tobytes()).hexdigest()
        queue.put((rank, n, list(q_heads), list(kv_heads), digest))
    finally:
        dist.destroy_process_group()


def test_two_rank_pool_sizing_sharding_and_metadata():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    counts = {r[1] for r in results}
    assert len(counts) == 1
    per_block = 2 * 36 * 256 * 4 * 128 * 2
    expect = int(180 * 2 ** 30 * 0.9 - 25 * 2 ** 30) // per_block   # the tighter rank
    assert counts == {expect}
    (_, _, q0, k0, d0), (_, _, q1, k1, d1) = results
    assert q0 == list(range(0, 16)) and q1 == list(range(16, 32))
    assert k0 == list(range(0, 4)) and k1 == list(range(4, 8))
    for qs, ks in ((q0, k0), (q1, k1)):
        assert all(h // 4 in ks for h in qs)          # GQA group of every query head is local
    assert d0 == d1


def test_block_bytes_counts_fp8_scales():
    import importlib
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    assert pkg.block_bytes(36, 256, 8, 128, "bf16") == 36 * 2 ** 20
    assert pkg.block_bytes(36, 256, 8, 128, "fp8") == 2 * 36 * (256 * 8 * 128 + 8 * 4)
    with pytest.raises(ValueError):
        pkg.tp_shard(32, 8, 3, 0)
    with pytest.raises(RuntimeError):
        pkg.plan_num_blocks(10, 10, 0, 0, 1)


def _rowpar_worker(rank, world, port, queue):
    import importlib
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
        full = torch.arange(2560 * 1024, dtype=torch.float32).view(2560, 1024)
        m = pkg.RowParallelLinear(1024, 2560)           # input dim sharded over the group
        m.weight.weight_loader(m.weight, full)
        shards = [torch.empty_like(m.weight.data) for _ in range(world)]
        dist.all_gather(shards, m.weight.data)
        reassembled = torch.equal(torch.cat(shards, dim=1), full)
        try:                                            # no CPU fallback for the fused op
            m(torch.zeros(3, 1024 // world))
            cpu_forward = "ran"
        except pkg.SlokvError:
            cpu_forward = "raised"
        # the buffer a rank would share over IPC for this group geometry
        nbytes = pkg.row_parallel_buffer_bytes(512, 2560, world)
        queue.put((rank, tuple(m.weight.shape), m.tp_size, reassembled, cpu_forward, nbytes))
    finally:
        dist.destroy_process_group()


def test_row_parallel_linear_two_ranks_shard_like_the_reference():
    """RowParallelLinear over a world-2 gloo group: each rank holds columns
    [r * K/2, (r + 1) * K/2) of the weight (nanovllm/layers/linear.py:141-149),
    the shards reassemble the full weight, both ranks size the same symmetric
    buffer, and a CPU forward at TP > 1 raises instead of falling back."""
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rowpar_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, shape, tp, reassembled, cpu_forward, nbytes in results:
        assert shape == (2560, 512) and tp == 2 and reassembled
        assert cpu_forward == "raised"
        assert nbytes == results[0][5] > 0


def _exchange_worker(rank, world, port, queue):
    import importlib
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lin = importlib.import_module("slo-aware-llm-serving-engine_b200.layers.linear")
        own = 0x1000 * (rank + 1)
        handle = bytes([rank]) * 64                     # stands in for a cudaIpcMemHandle_t
        opened = []

        def import_handle(h):                           # "maps" a peer: returns its tag
            opened.append(h[0])
            return 0xABC0000 + h[0]

        ptrs = lin.exchange_buffers(own, handle, import_handle)
        queue.put((rank, ptrs, opened))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_buffer_exchange_over_gloo(world):
    """The symmetric-buffer handshake of the fused row-parallel all-reduce: every
    rank gets rank r's buffer at index r (its own pointer at its own index, the
    peers' opened from their handles, each peer exactly once)."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ptrs, opened in results:
        assert ptrs == [0x1000 * (r + 1) if r == rank else 0xABC0000 + r for r in range(world)]
        assert sorted(opened) == [r for r in range(world) if r != rank]
