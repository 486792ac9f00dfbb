"""Tensor-parallel plumbing of the random-init Qwen3 harness on CPU (gloo):
head / MLP shards reassemble the TP=1 weights, and a two-rank forward (o_proj
and down_proj all-reduced, nanovllm/layers/linear.py:152-156) gives the same
hidden states and greedy tokens as one rank.  Attention here is a small dense
causal stand-in on CPU (the CUDA kernels are covered by the GPU tests)."""
import importlib
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TINY = dict(vocab_size=97, hidden_size=64, intermediate_size=96, num_layers=2, num_heads=4,
            num_kv_heads=2, head_dim=16, max_position=256)


def _harness():
    return importlib.import_module("slo-aware-llm-serving-engine_b200.qwen3_harness")


class _DenseCausal(torch.nn.Module):
    """Per-sequence causal GQA attention over the step's own k/v (prefill only)."""

    def __init__(self, scale, group):
        super().__init__()
        self.scale, self.group = scale, group
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q, k, v):
        ctx = importlib.import_module("slo-aware-llm-serving-engine_b200.utils.context").get_context()
        cu = ctx.cu_seqlens_q.tolist()
        outs = []
        for a, b in zip(cu, cu[1:]):
            kk = k[a:b].repeat_interleave(self.group, dim=1)
            vv = v[a:b].repeat_interleave(self.group, dim=1)
            s = torch.einsum("qhd,khd->hqk", q[a:b].float(), kk.float()) * self.scale
            n = b - a
            s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
            outs.append(torch.einsum("hqk,khd->qhd", s.softmax(-1), vv.float()).to(q.dtype))
        return torch.cat(outs)


def _forward(rank, world, group=None):
    h = _harness()
    ctxmod = importlib.import_module("slo-aware-llm-serving-engine_b200.utils.context")
    cfg = h.Qwen3Config(**TINY)
    m = h.Qwen3Model(cfg, rank, world, group, seed=3, device="cpu", dtype=torch.float32)
    for lw in m.layers:
        lw.attn = _DenseCausal(cfg.head_dim ** -0.5, cfg.num_heads // cfg.num_kv_heads)
    lens = [5, 11, 1]
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab_size, (sum(lens),), generator=g)
    pos = torch.cat([torch.arange(n) for n in lens])
    cu = torch.tensor([0, 5, 16, 17], dtype=torch.int32)
    ctxmod.set_context(True, cu, cu, 11, 11, None, None, None)
    hid = m.forward(ids, pos)
    ctxmod.reset_context()
    return hid, m.logits(hid).argmax(-1)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hid, tok = _forward(rank, world)
        queue.put((rank, hid, tok))
    finally:
        dist.destroy_process_group()


def test_shards_reassemble_the_full_weights():
    h = _harness()
    cfg = h.Qwen3Config(**TINY)
    full = h.Qwen3Model(cfg, 0, 1, seed=3, device="cpu", dtype=torch.float32)
    parts = [h.Qwen3Model(cfg, r, 2, seed=3, device="cpu", dtype=torch.float32) for r in range(2)]
    D, hq, hk = cfg.head_dim, cfg.num_heads // 2, cfg.num_kv_heads // 2
    for li, lf in enumerate(full.layers):
        p0, p1 = parts[0].layers[li], parts[1].layers[li]
        q = torch.cat([p0.wqkv[:hq * D], p1.wqkv[:hq * D]])
        k = torch.cat([p0.wqkv[hq * D:(hq + hk) * D], p1.wqkv[hq * D:(hq + hk) * D]])
        v = torch.cat([p0.wqkv[(hq + hk) * D:], p1.wqkv[(hq + hk) * D:]])
        assert torch.equal(torch.cat([q, k, v]), lf.wqkv)
        assert torch.equal(torch.cat([p0.wo, p1.wo], dim=1), lf.wo)
        il = cfg.intermediate_size // 2
        gate = torch.cat([p0.wgu[:il], p1.wgu[:il]])
        up = torch.cat([p0.wgu[il:], p1.wgu[il:]])
        assert torch.equal(torch.cat([gate, up]), lf.wgu)
        assert torch.equal(torch.cat([p0.wd, p1.wd], dim=1), lf.wd)
    assert torch.equal(parts[1].embed, full.embed)


def test_two_rank_forward_matches_one_rank():
    ref_hid, ref_tok = _forward(0, 1)
    world, ctx = 2, mp.get_context("spawn")
    queue, port = ctx.Queue(), _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((queue.get(timeout=240) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, hid, tok in results:
        assert torch.allclose(hid, ref_hid, atol=1e-5, rtol=1e-5)
        assert torch.equal(tok, ref_tok)
