"""Full-model greedy decode on a random-init Qwen3-4B (36 layers, hidden 2560,
N(0, 0.02) weights) through this package's Attention + Context (paged append,
tcgen05 prefill, paged decode, CUDA-graph decode step), checked against the
same model whose attention is the reference's fp32 torch attention
(benchmarks/v1_validation/reference.py:7-23, restated in oracle/kv_oracle.py)
over each sequence's own K/V history."""
import importlib

import pytest
import torch

from oracle import kv_oracle as O
from tests.golden.detgen import det_ints

pytestmark = pytest.mark.gpu

STEPS = 32


class OracleAttention(torch.nn.Module):
    """Reference attention: per-sequence K/V history, fp32 dense causal
    attention on the CPU, output rounded to bf16 as flash-attn returns it."""

    def __init__(self, scale):
        super().__init__()
        self.scale = scale
        self.k_cache = self.v_cache = torch.tensor([])
        self.k_scale = self.v_scale = None
        self.hist = []

    def forward(self, q, k, v):
        ctx = importlib.import_module("slo-aware-llm-serving-engine_b200.utils.context").get_context()
        outs = []
        if ctx.is_prefill:
            cu = ctx.cu_seqlens_q.tolist()
            for a, b in zip(cu, cu[1:]):
                kk, vv = k[a:b].clone(), v[a:b].clone()
                self.hist.append((kk, vv))
                outs.append(O.dense_suffix_attention(q[a:b].cpu(), kk.cpu(), vv.cpu(), self.scale))
            return torch.cat(outs).to(q.dtype).to(q.device)
        for i in range(q.shape[0]):
            kk = torch.cat([self.hist[i][0], k[i:i + 1]])
            vv = torch.cat([self.hist[i][1], v[i:i + 1]])
            self.hist[i] = (kk, vv)
            outs.append(O.dense_suffix_attention(q[i:i + 1].cpu(), kk.cpu(), vv.cpu(), self.scale))
        return torch.cat(outs).to(q.dtype).to(q.device)


def _reference_run(model, lens, prompts):
    """Free-running greedy decode with the oracle attention; returns the tokens
    [B, STEPS] and the top-2 logit gap of every step [B, STEPS]."""
    h = importlib.import_module("slo-aware-llm-serving-engine_b200.qwen3_harness")
    ours = [lw.attn for lw in model.layers]
    for lw in model.layers:
        lw.attn = OracleAttention(model.cfg.head_dim ** -0.5)
    gaps = []

    def logits(hid):
        lg = h.Qwen3Model.logits(model, hid)
        top = lg.float().topk(2, dim=-1).values
        gaps.append((top[:, 0] - top[:, 1]).cpu())
        return lg

    model.logits = logits
    runner = h.GreedyRunner(model, lens, STEPS, seed=1)
    cur = runner.prefill(prompts, chunk_tokens=4096)
    toks = [cur]
    for _ in range(STEPS - 1):
        cur = runner.decode(cur, use_graph=False)
        toks.append(cur)
    del model.logits
    for lw, a in zip(model.layers, ours):
        lw.attn = a
    return torch.stack(toks, dim=1).cpu(), torch.stack(gaps, dim=1)


def test_random_init_qwen3_4b_greedy_decode_agrees_with_reference_attention(pkg):
    """Teacher-forced: at every step both paths see the reference's token
    history, so one disagreement does not derail the rest.  On a random-init
    model the 36 layers amplify the bf16 rounding of attention (~0.15 % per
    layer) into logit changes of up to ~0.2 (logit std ~1) and the bf16 logits
    tie outright in a few percent of steps, so free-running tokens cannot match
    a non-bit-identical attention everywhere; the bar is that every
    disagreement sits at a reference top-2 gap inside that perturbation and
    that the paths agree on the large majority of steps."""
    h = importlib.import_module("slo-aware-llm-serving-engine_b200.qwen3_harness")
    cfg = h.Qwen3Config()
    model = h.Qwen3Model(cfg, seed=11, device="cuda")
    lens = [37, 300, 129, 517, 256, 1, 700, 64]
    ids = det_ints(4242, sum(lens), 0, cfg.vocab_size - 1).tolist()
    prompts, cur = [], 0
    for n in lens:
        prompts.append(ids[cur:cur + n])
        cur += n
    ref, gaps = _reference_run(model, lens, prompts)
    runner = h.GreedyRunner(model, lens, STEPS, seed=1)
    ours = [runner.prefill(prompts, chunk_tokens=4096).cpu()]
    for t in range(STEPS - 1):
        ours.append(runner.decode(ref[:, t].cuda(), use_graph=True).cpu())
    ours = torch.stack(ours, dim=1)
    assert pkg.read_device_errors() == 0
    agree = ours == ref
    rate = agree.float().mean().item()
    worst = gaps[~agree].max().item() if (~agree).any() else 0.0
    print(f"teacher-forced greedy agreement {rate:.4f} over {agree.numel()} steps; "
          f"largest reference top-2 gap at a disagreement {worst:.4f}")
    assert rate >= 0.75, f"agreement {rate:.4f}"
    assert worst <= 0.25, f"a disagreement at reference top-2 gap {worst:.4f}"
