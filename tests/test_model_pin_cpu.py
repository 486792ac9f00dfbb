"""The random-init Qwen3 harness computes what the reference's own
`Qwen3ForCausalLM` computes (nanovllm/models/qwen3.py:14-216), on the CPU.

tests/golden/make_model_golden.py ran the reference model (fp32, its fp32
diagnostic installed: fp32 RMSNorm, dense fp32 attention through its paged
pool) on weights drawn by `qwen3_harness.Qwen3Model(seed=7)` and stored its
greedy tokens and top-16 logits for a cold prefill of three prompts plus four
decode steps.  Here the harness runs the same weights and prompts with the
same attention arithmetic (the oracle's restatement of the reference's fp32
attention over a paged fp32 pool) and must reproduce them: same tokens, same
top-16 ids, logits within 1e-4 (fp32 summation order only).  With the layer
code pinned this way, the GPU greedy test (tests/test_gpu_model_reference.py)
compares attention implementations on the reference's model."""
import importlib
import json
import os

import numpy as np
import torch

from oracle import kv_oracle as O
from tests.golden import make_model_golden as G

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CTX = "slo-aware-llm-serving-engine_b200.utils.context"


class PagedOracleAttention(torch.nn.Module):
    """The reference Attention.forward on the CPU: store into an fp32 paged pool,
    then the fp32 oracle for prefill (the step's own rows) or decode (pages)."""

    def __init__(self, k_cache, v_cache, scale):
        super().__init__()
        self.k_cache, self.v_cache, self.scale = k_cache, v_cache, scale
        self.k_scale = self.v_scale = None

    def forward(self, q, k, v):
        ctx = importlib.import_module(CTX).get_context()
        O.store_kvcache(k, v, self.k_cache, self.v_cache, ctx.slot_mapping)
        if ctx.is_prefill:
            return O.varlen(q, k, v, ctx.cu_seqlens_q, ctx.cu_seqlens_k, self.scale)
        return O.decode(q.unsqueeze(1), self.k_cache, self.v_cache, ctx.context_lens,
                        ctx.block_tables, self.scale).squeeze(1)


def test_harness_reproduces_reference_qwen3_logits():
    with open(os.path.join(HERE, "model_pin.json")) as f:
        meta = json.load(f)
    gold = dict(np.load(os.path.join(HERE, "model_pin.npz")))
    h, cfg = G.harness_config()
    model = h.Qwen3Model(cfg, seed=meta["seed"], device="cpu", dtype=torch.float32)
    assert G.weight_digest(model) == meta["weights_sha256"], "weight generation changed"
    lens = list(meta["prompt_lens"])
    bs = G.BLOCK
    pages = [(n + meta["decode_steps"] + bs - 1) // bs for n in lens]
    nb = sum(pages)
    for lw in model.layers:   # every layer its own pool planes, pages in natural order
        kc = torch.zeros(nb, bs, cfg.num_kv_heads, cfg.head_dim)
        lw.attn = PagedOracleAttention(kc, torch.zeros_like(kc), cfg.head_dim ** -0.5)
    tables, cur = [], 0
    for p in pages:
        tables.append(list(range(cur, cur + p)) + [-1] * (max(pages) - p))
        cur += p
    tables_t = torch.tensor(tables, dtype=torch.int32)
    ctx = importlib.import_module(CTX)

    def slot(b, pos):
        return tables[b][pos // bs] * bs + pos % bs

    ps = G.prompts(cfg.vocab_size)
    with torch.no_grad():
        ids = torch.tensor([t for p in ps for t in p], dtype=torch.int64)
        pos = torch.cat([torch.arange(n) for n in lens])
        cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int32)
        slots = torch.tensor([slot(b, i) for b, n in enumerate(lens) for i in range(n)],
                             dtype=torch.int32)
        ctx.set_context(True, cu, cu, max(lens), max(lens), slots, None, None)
        hid = model.forward(ids, pos)
        ctx.reset_context()
        logits = model.logits(hid[cu[1:].long() - 1])
        for step in range(meta["decode_steps"] + 1):
            vals, top = logits.float().topk(meta["topk"], dim=-1)
            np.testing.assert_array_equal(top.numpy(), gold["top_ids"][step])
            np.testing.assert_allclose(vals.numpy(), gold["top_vals"][step], rtol=0, atol=1e-4)
            nxt = logits.argmax(dim=-1)
            np.testing.assert_array_equal(nxt.numpy(), gold["tokens"][:, step])
            if step == meta["decode_steps"]:
                break
            pos = torch.tensor(lens, dtype=torch.int64)
            slots = torch.tensor([slot(b, n) for b, n in enumerate(lens)], dtype=torch.int32)
            lens = [n + 1 for n in lens]
            ctx.set_context(False, slot_mapping=slots,
                            context_lens=torch.tensor(lens, dtype=torch.int32),
                            block_tables=tables_t)
            logits = model.logits(model.forward(nxt, pos))
            ctx.reset_context()
