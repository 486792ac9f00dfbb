"""Generate the golden fixtures by running the REFERENCE engine's own code on CPU.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/SLO-Aware-LLM-Serving-Engine

What runs (all reference code, unmodified, imported from its checkout):
  * store_kvcache + its Triton kernel (nanovllm/layers/attention.py:10-40),
    executed by the Triton CPU interpreter (TRITON_INTERPRET=1);
  * the fp32 attention oracle that replaces flash-attn's two entry points
    (benchmarks/v1_validation/reference.py:34-96, installed exactly as the
    reference's FP32 diagnostic installs it);
  * forward_mixed (nanovllm/layers/mixed_attention.py:29-57);
  * encode_e4m3fn (benchmarks/v0/probe_quant_support.py:39-56);
  * restore_kv (diagnostics/online_token_replay/tensors.py:34-43);
  * RMSNorm (nanovllm/layers/layernorm.py) and RotaryEmbedding
    (nanovllm/layers/rotary_embedding.py) as qwen3.py:82-85 apply them to q/k,
    eager (TORCHDYNAMO_DISABLE=1 turns their torch.compile into a no-op).
Inputs come from tests/golden/scenarios.py (deterministic), so only outputs and
digests are stored, in tests/golden/golden.npz + golden.json.
"""
from __future__ import annotations

import argparse
import hashlib
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

from tests.golden import scenarios as S  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def install_reference_oracle():
    """Bind the reference's fp32 attention oracle into its attention modules, the
    way install_fp32_diagnostic does for a live engine (a stub engine with no
    layers satisfies its preconditions)."""
    from benchmarks.v1_validation.reference import install_fp32_diagnostic

    class _Stub(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList()

    engine = types.SimpleNamespace(
        config=types.SimpleNamespace(tensor_parallel_size=1, enforce_eager=True),
        model_runner=types.SimpleNamespace(model=_Stub(), kv_cache=torch.zeros(2, 0)))
    install_fp32_diagnostic(engine)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (read only)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    install_reference_oracle()
    import nanovllm.layers.attention as ref_attn
    from nanovllm.layers.mixed_attention import MixedAttentionContext, forward_mixed
    from benchmarks.v0.probe_quant_support import encode_e4m3fn
    from diagnostics.online_token_replay.tensors import restore_kv

    arrays, manifest = {}, {"generator": "tests/golden/make_golden.py", "scenarios": {}}

    # --- decode scenarios: store (Triton, interpreted) then the fp32 decode oracle
    for sc in (S.cfg1_decode(), S.gqa_decode()):
        kc, vc = sc["k_cache"].clone(), sc["v_cache"].clone()
        ref_attn.store_kvcache(sc["k"], sc["v"], kc, vc, sc["slots"])
        out = ref_attn.flash_attn_with_kvcache(
            sc["q"].unsqueeze(1), kc, vc, cache_seqlens=sc["lens"], block_table=sc["tables"],
            softmax_scale=sc["scale"], causal=True)
        arrays[sc["name"] + "/out"] = out.float().numpy()
        manifest["scenarios"][sc["name"]] = {
            "k_cache_sha256": sha(kc), "v_cache_sha256": sha(vc),
            "out_shape": list(out.shape), "row_stride": 1}
        print(sc["name"], tuple(out.shape))

    # --- mixed / prefill scenarios through the reference forward_mixed
    for sc in (S.mixed_page_reuse(0), S.mixed_page_reuse(1), S.mixed_multi_prefill(),
               S.mixed_qwen_geometry(0), S.mixed_qwen_geometry(1), S.cold_prefill()):
        kc, vc = sc["k_cache"].clone(), sc["v_cache"].clone()
        meta = MixedAttentionContext(**sc["meta"])
        ctx = types.SimpleNamespace(mixed=meta, slot_mapping=sc["slots"])
        out = forward_mixed(sc["q"], sc["k"], sc["v"], kc, vc, ctx, sc["scale"],
                            ref_attn.store_kvcache)
        stride = 8 if out.shape[0] > 64 else 1  # keep the fixture small
        arrays[sc["name"] + "/out"] = out[::stride].float().numpy()
        manifest["scenarios"][sc["name"]] = {
            "k_cache_sha256": sha(kc), "v_cache_sha256": sha(vc),
            "out_shape": list(out.shape), "row_stride": stride}
        print(sc["name"], tuple(out.shape))

    # --- E4M3 encoder on the probe values
    vals = S.e4m3_probe_values()
    codes = np.array([encode_e4m3fn(float(x)) for x in vals.tolist()], dtype=np.uint8)
    arrays["e4m3/codes"] = codes
    manifest["scenarios"]["e4m3"] = {"count": int(codes.size),
                                     "values_sha256": hashlib.sha256(vals.tobytes()).hexdigest()}
    print("e4m3", codes.size)

    # --- restore_kv page copy on a small pool
    pool = torch.arange(2 * 3 * 6 * 4 * 2 * 8, dtype=torch.float32).reshape(2, 3, 6, 4, 2, 8)
    saved = torch.from_numpy(S.det_normal(950, (2, 3, 3, 4, 2, 8)))
    image = {"block_ids": [4, 1, 5], "kv": saved, "pool_shape": list(pool.shape)}
    restore_kv(pool, image)
    arrays["restore/pool"] = pool.numpy()
    manifest["scenarios"]["restore"] = {"block_ids": [4, 1, 5]}

    # --- q/k RMSNorm + rotary embedding of one layer (qwen3.py:82-85)
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.rotary_embedding import RotaryEmbedding
    nc = S.qk_norm_rope_case()
    T, Hq, Hkv, D = nc["qkv"].shape[0], nc["Hq"], nc["Hkv"], nc["D"]
    q, k, _ = nc["qkv"].split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    q_norm, k_norm = RMSNorm(D, eps=nc["eps"]), RMSNorm(D, eps=nc["eps"])
    q_norm.weight.data = nc["wq"].clone()
    k_norm.weight.data = nc["wk"].clone()
    rope = RotaryEmbedding(D, D, nc["max_position"], nc["base"])
    with torch.no_grad():
        qn = q_norm(q.reshape(T, Hq, D))
        kn = k_norm(k.reshape(T, Hkv, D))
        qr, kr = rope(nc["pos"], qn, kn)
    arrays["qk_norm_rope/q"] = qr.float().numpy()
    arrays["qk_norm_rope/k"] = kr.float().numpy()
    manifest["scenarios"]["qk_norm_rope"] = {"q_sha256": sha(qr), "k_sha256": sha(kr)}
    print("qk_norm_rope", tuple(qr.shape), tuple(kr.shape))

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "golden.npz"))


if __name__ == "__main__":
    main()
