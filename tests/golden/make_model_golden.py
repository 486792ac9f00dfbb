"""Pin the random-init Qwen3 harness to the REFERENCE's own model, on the CPU.

Run where the reference checkout is available:

    python tests/golden/make_model_golden.py --reference /path/to/SLO-Aware-LLM-Serving-Engine

What runs: the reference's `Qwen3ForCausalLM` (nanovllm/models/qwen3.py:14-216)
at the Qwen3-4B layer geometry (hidden 2560, 32 / 8 heads, head_dim 128,
intermediate 9728, vocab 151936, q/k RMSNorm, RoPE theta 1e6, tied LM head)
with MODEL_LAYERS decoder layers, in fp32 with its fp32 diagnostic installed
exactly as `install_fp32_diagnostic` (benchmarks/v1_validation/reference.py:
34-96) installs it: fp32 RMSNorm, dense fp32 attention in place of flash-attn,
its Triton `store_kvcache` writing a paged pool (TRITON_INTERPRET=1).  Its
weights are the ones `qwen3_harness.Qwen3Model(seed=MODEL_SEED, device="cpu",
dtype=float32)` draws, loaded into the reference modules; the harness is only
the weight source here.  The script prefills PROMPT_LENS prompts through
nanovllm's Context (cold prefill, slots into the paged pool), then decodes
DECODE_STEPS greedy tokens (paged decode through block tables), and stores the
greedy tokens plus the top-16 logits (values and ids) of every step in
tests/golden/model_pin.npz.  tests/test_model_pin_cpu.py runs the harness on
the same weights and checks it against them.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys
import types

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.golden.detgen import det_ints  # noqa: E402

MODEL_LAYERS = 2
MODEL_SEED = 7
PROMPT_LENS = [37, 5, 64]
DECODE_STEPS = 4
TOPK = 16
BLOCK = 256


def harness_config():
    h = importlib.import_module("slo-aware-llm-serving-engine_b200.qwen3_harness")
    return h, h.Qwen3Config(num_layers=MODEL_LAYERS)


def prompts(vocab):
    ids = det_ints(6160, sum(PROMPT_LENS), 0, vocab - 1).tolist()
    out, cur = [], 0
    for n in PROMPT_LENS:
        out.append(ids[cur:cur + n])
        cur += n
    return out


def weight_digest(model) -> str:
    """SHA-256 over the harness weights (embedding and every layer's matrices)."""
    d = hashlib.sha256()
    for t in [model.embed] + [w for lw in model.layers for w in (lw.wqkv, lw.wo, lw.wgu, lw.wd)]:
        d.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return d.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference project (read only)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch.distributed as dist
    from transformers import Qwen3Config as HFConfig
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=os.environ.get("MASTER_PORT", "29533"))
    dist.init_process_group("gloo", rank=0, world_size=1)
    from benchmarks.v1_validation.reference import install_fp32_diagnostic
    from nanovllm.models.qwen3 import Qwen3ForCausalLM
    from nanovllm.utils.context import reset_context, set_context

    h, cfg = harness_config()
    src = h.Qwen3Model(cfg, seed=MODEL_SEED, device="cpu", dtype=torch.float32)
    hf = HFConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                  intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_layers,
                  num_attention_heads=cfg.num_heads, num_key_value_heads=cfg.num_kv_heads,
                  head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                  max_position_embeddings=cfg.max_position, tie_word_embeddings=True,
                  attention_bias=False, hidden_act="silu")
    torch.set_default_dtype(torch.float32)
    model = Qwen3ForCausalLM(hf)
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(src.embed)
        for layer, lw in zip(model.model.layers, src.layers):
            layer.self_attn.qkv_proj.weight.copy_(lw.wqkv)
            layer.self_attn.o_proj.weight.copy_(lw.wo)
            layer.mlp.gate_up_proj.weight.copy_(lw.wgu)
            layer.mlp.down_proj.weight.copy_(lw.wd)
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    rope = model.model.layers[0].self_attn.rotary_emb.cos_sin_cache.squeeze(1)
    assert torch.equal(rope[:, :cfg.head_dim // 2], src.cos[:rope.shape[0]]), "RoPE tables differ"

    pages = [(n + DECODE_STEPS + BLOCK - 1) // BLOCK for n in PROMPT_LENS]
    nb = sum(pages)
    kv = torch.zeros(2, cfg.num_layers, nb, BLOCK, cfg.num_kv_heads, cfg.head_dim)
    engine = types.SimpleNamespace(
        config=types.SimpleNamespace(tensor_parallel_size=1, enforce_eager=True),
        model_runner=types.SimpleNamespace(model=model, kv_cache=kv))
    install_fp32_diagnostic(engine)
    # block tables: the reverse of the natural order, so pages are not contiguous
    order = list(range(nb))[::-1]
    tables, cur = [], 0
    for p in pages:
        tables.append(order[cur:cur + p] + [-1] * (max(pages) - p))
        cur += p
    tables_t = torch.tensor(tables, dtype=torch.int32)

    def slot(b, pos):
        return tables[b][pos // BLOCK] * BLOCK + pos % BLOCK

    ps = prompts(cfg.vocab_size)
    tokens, top_vals, top_ids = [], [], []
    with torch.no_grad():
        ids = torch.tensor([t for p in ps for t in p], dtype=torch.int64)
        pos = torch.cat([torch.arange(n) for n in PROMPT_LENS])
        cu = torch.tensor(np.cumsum([0] + PROMPT_LENS), dtype=torch.int32)
        slots = torch.tensor([slot(b, i) for b, n in enumerate(PROMPT_LENS) for i in range(n)],
                             dtype=torch.int32)
        set_context(True, cu, cu, max(PROMPT_LENS), max(PROMPT_LENS), slots, None, None)
        logits = model.compute_logits(model(ids, pos))
        reset_context()
        lens = list(PROMPT_LENS)
        for step in range(DECODE_STEPS + 1):
            v, i = logits.float().topk(TOPK, dim=-1)
            top_vals.append(v.numpy())
            top_ids.append(i.numpy())
            nxt = logits.argmax(dim=-1)
            tokens.append(nxt.numpy())
            if step == DECODE_STEPS:
                break
            pos = torch.tensor(lens, dtype=torch.int64)
            slots = torch.tensor([slot(b, n) for b, n in enumerate(lens)], dtype=torch.int32)
            lens = [n + 1 for n in lens]
            set_context(False, slot_mapping=slots, context_lens=torch.tensor(lens, dtype=torch.int32),
                        block_tables=tables_t)
            logits = model.compute_logits(model(nxt, pos))
            reset_context()
    out = {"tokens": np.stack(tokens, axis=1), "top_vals": np.stack(top_vals),
           "top_ids": np.stack(top_ids)}
    np.savez_compressed(os.path.join(HERE, "model_pin.npz"), **out)
    meta = {"generator": "tests/golden/make_model_golden.py", "layers": MODEL_LAYERS,
            "seed": MODEL_SEED, "prompt_lens": PROMPT_LENS, "decode_steps": DECODE_STEPS,
            "topk": TOPK, "weights_sha256": weight_digest(src), "torch": torch.__version__}
    with open(os.path.join(HERE, "model_pin.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    gaps = out["top_vals"][..., 0] - out["top_vals"][..., 1]
    print("tokens", out["tokens"].tolist(), "min top-2 gap", float(gaps.min()))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
