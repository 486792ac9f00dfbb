#!/usr/bin/env python
"""Decode-step benchmark of the B200 KV-cache hot path.

One step = for each of the 36 Qwen3-4B layers: append one new K/V token per
sequence into the paged pool (kv_append) and run GQA-4 paged decode attention
over the whole context (paged_decode).  Batch 256 per GPU, context lengths
uniform in [512, 4096], block size 256, block pool sized to ~70% of HBM with a
random block assignment, K/V ~ 0.5*N(0,1), Q ~ N(0,1) (synthetic data).

N > 1 (torchrun): tensor parallelism over KV heads with weak scaling -- every
rank holds Hkv/N KV heads (and 4x as many query heads) for a global batch of
256*N sequences, so each rank streams the same bytes as one GPU at N=1; there is
no collective inside the hot path (attention is head-local).  The timed region
is bracketed by barrier + synchronize and the max over ranks is reported.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/sec and paged-attn HBM GB/s (% of 8 TB/s), Qwen3-4B, 1/2/4/8 B200"
LAYERS, HQ, HKV, D, BS = 36, 32, 8, 128, 256
BATCH_PER_GPU = 256
CTX_LO, CTX_HI = 512, 4096
POOL_FRAC = 0.70
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        props = torch.cuda.get_device_properties(device)
        bus = getattr(props, "pci_bus_id", None)
        dom = getattr(props, "pci_domain_id", None)
        dev = getattr(props, "pci_device_id", None)
        self.sel = (f"{dom:08X}:{bus:02X}:{dev:02X}.0" if None not in (bus, dom, dev)
                    else str(device.index or 0))

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.sel, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.samples = []
        if self.proc is None:
            return False
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)
        return False

    def summary(self):
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[4:8])
                          if v.lower() == "active"})
        under = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(under) if under else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------

def make_metadata(n_gpus, seed=2, batch_per_gpu=BATCH_PER_GPU, lo=CTX_LO, hi=CTX_HI):
    """Global batch metadata, identical on every rank (same generator)."""
    gen = torch.Generator().manual_seed(seed)
    B = batch_per_gpu * n_gpus
    lens = torch.randint(lo, hi + 1, (B,), generator=gen, dtype=torch.int64)
    pages = (lens + BS - 1) // BS
    return B, lens.to(torch.int32), pages, gen


def build_gpu_workload(args, rank, n, device):
    hkv, hq = HKV // n, HQ // n
    fp8 = args.kv == "fp8"
    B, lens, pages, gen = make_metadata(n, batch_per_gpu=args.batch, lo=args.ctx_lo,
                                        hi=args.ctx_hi)
    W = int(pages.max())
    need = int(pages.sum())
    block_bytes = 2 * args.layers * (BS * hkv * D * (1 if fp8 else 2) + (hkv * 4 if fp8 else 0))
    free, total = torch.cuda.mem_get_info(device)
    if args.pool_blocks:
        NB = args.pool_blocks
    else:
        NB = int(POOL_FRAC * total) // block_bytes
        NB = min(NB, int((free - (6 << 30)) // block_bytes))
    if NB < need:
        raise SystemExit(f"pool of {NB} blocks cannot hold the {need} blocks of the batch")
    perm = torch.randperm(NB, generator=gen)[:need].to(torch.int32)
    tables = torch.full((B, W), -1, dtype=torch.int32)
    cur = 0
    for b in range(B):
        p = int(pages[b])
        tables[b, :p] = perm[cur:cur + p]
        cur += p
    last = (lens - 1).to(torch.int64)
    slots = (tables[torch.arange(B), last // BS].to(torch.int64) * BS + last % BS).to(torch.int32)

    log(f"[rank {rank}] pool {NB} blocks x {block_bytes / 2**20:.1f} MiB = "
        f"{NB * block_bytes / 2**30:.1f} GiB ({NB * block_bytes / total:.0%} of HBM), "
        f"batch {B}, Hkv {hkv}, layers {args.layers}")
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    scales = None
    if fp8:
        # N(0, 1) bf16 with 1 % x20 outliers, quantised per
        # (block, kv head) with scale amax / 448, in the blocks the batch reads
        kv = torch.zeros(2, args.layers, NB, BS, hkv, D, dtype=torch.uint8, device=device)
        scales = torch.zeros((2, args.layers, NB, hkv), dtype=torch.float32, device=device)
        fill_fp8_pool(kv, scales, perm.tolist(), g, 1.0, True)
    else:
        kv = torch.empty(2, args.layers, NB, BS, hkv, D, dtype=torch.bfloat16, device=device)
        for i in range(2):
            for l in range(args.layers):
                kv[i, l].normal_(0.0, 0.5, generator=g)
    q = torch.randn(args.layers, B, hq, D, device=device, generator=g).to(torch.bfloat16)
    std = 1.0 if fp8 else 0.5        # config 4: N(0, 1) (+ outliers); config 2: 0.5 N(0, 1)
    knew = torch.randn(args.layers, B, hkv, D, device=device, generator=g) * std
    vnew = torch.randn(args.layers, B, hkv, D, device=device, generator=g) * std
    if fp8:  # 1% outliers x20
        knew = torch.where(torch.rand(knew.shape, device=device, generator=g) < 0.01, knew * 20, knew)
        vnew = torch.where(torch.rand(vnew.shape, device=device, generator=g) < 0.01, vnew * 20, vnew)
    knew, vnew = knew.bfloat16(), vnew.bfloat16()
    out = torch.empty(args.layers, B, hq, D, dtype=torch.bfloat16, device=device)
    return dict(B=B, hq=hq, hkv=hkv, NB=NB, W=W, lens_cpu=lens, tables_cpu=tables,
                slots_cpu=slots, lens=lens.to(device), tables=tables.to(device),
                slots=slots.to(device), kv=kv, q=q, knew=knew, vnew=vnew, out=out,
                block_bytes=block_bytes, fp8=fp8, scales=scales)


def fill_fp8_pool(kv, scales, blocks, gen, std, outliers):
    """FP8 pool contents as BASELINE config 4 specifies them: per layer plane,
    bf16 values N(0, std^2) (1 % of elements x20 when `outliers`) for the blocks
    the batch reads, stored as E4M3 codes with per-(block, kv-head) scale
    amax / 448 (round to nearest, saturating; unused blocks keep zeros)."""
    ids = torch.as_tensor(sorted(set(int(b) for b in blocks)), dtype=torch.long,
                          device=kv.device)
    n, hkv = ids.numel(), kv.shape[-2]
    for i in range(kv.shape[0]):
        for l in range(kv.shape[1]):
            for c in range(0, n, 1024):                      # bounded temporaries
                sel = ids[c:c + 1024]
                x = torch.randn((sel.numel(),) + tuple(kv.shape[3:]), device=kv.device,
                                generator=gen) * std
                if outliers:
                    x = torch.where(torch.rand(x.shape, device=kv.device, generator=gen) < 0.01,
                                    x * 20, x)
                x = x.bfloat16().float()
                s = x.abs().amax(dim=(1, 3)) / 448.0                 # [blocks, hkv]
                q = (x / s.clamp_min(1e-30)[:, None, :, None]).clamp(-448, 448)
                kv[i, l, sel] = q.to(torch.float8_e4m3fn).view(torch.uint8)
                scales[i, l, sel] = s
                del x, q


def decode_config(args, n):
    """The `config` of the decode workload (configs 2 / 4) at N GPUs, computed
    from the seeded metadata alone, so both arms of the bench print the same
    dict whatever device they run on."""
    fp8 = args.kv == "fp8"
    B, lens, pages, _ = make_metadata(n, batch_per_gpu=args.batch, lo=args.ctx_lo,
                                      hi=args.ctx_hi)
    hkv = HKV // n
    kv_bytes = int(lens.to(torch.int64).sum()) * hkv * D * (1 if fp8 else 2) * 2
    return {
        "workload": ("BASELINE config 4: FP8-E4M3 KV decode step, 36 layers of "
                     "quantising append + fused-dequant GQA-4 paged decode"
                     if fp8 else
                     "BASELINE config 2: pure decode step, 36 layers of kv_append + "
                     "GQA-4 paged decode, Qwen3-4B KV geometry"),
        "batch_per_gpu": args.batch, "global_batch": B, "layers": args.layers,
        "kv_heads_per_gpu": hkv, "q_heads_per_gpu": HQ // n, "head_dim": D,
        "block_size": BS, "context": f"U[{args.ctx_lo},{args.ctx_hi}]",
        "kv_cache": "fp8_e4m3" if fp8 else "bf16",
        "parallelism": f"tp{n} over KV heads (weak: global batch {args.batch}*N)",
        "l2": "inputs larger than L2: ~%.2f GB of K/V read per layer" % (kv_bytes / 1e9)}


def decode_bytes(wl):
    """Algorithmic HBM bytes of one paged_decode launch (one layer)."""
    ctx = int(wl["lens_cpu"].to(torch.int64).sum())
    pages = int(((wl["lens_cpu"].to(torch.int64) + BS - 1) // BS).sum())
    kv = ctx * wl["hkv"] * D * (1 if wl["fp8"] else 2) * 2
    scales = pages * wl["hkv"] * 4 * 2 if wl["fp8"] else 0
    qo = wl["B"] * wl["hq"] * D * 2 * 2
    meta = wl["B"] * 4 + pages * 4
    return kv + scales + qo + meta


def append_bytes(wl):
    """Algorithmic HBM bytes of one kv_append launch: read new K and V, write them
    (bf16) or their codes and scales (FP8)."""
    if wl["fp8"]:
        return wl["B"] * wl["hkv"] * D * (2 + 1) * 2 + wl["B"] * wl["hkv"] * 4 * 2 * 2 + wl["B"] * 4
    return wl["B"] * wl["hkv"] * D * 2 * 2 * 2 + wl["B"] * 4


def flash_attn_decode(wl, L, reps):
    """The reference's own GPU decode dependency on this box: flash-attn's
    flash_attn_with_kvcache (nanovllm/layers/attention.py:76-78) over the same
    pool, tables, lengths and queries, timed with CUDA events over reps x L
    launches (eager, as the reference calls it outside its graph).  Returns its
    per-layer time, GB/s of the same algorithmic bytes and the largest
    difference from our output of the same layers, or why it did not run."""
    try:
        import flash_attn
        from flash_attn import flash_attn_with_kvcache
    except Exception as e:  # noqa: BLE001 - report any import failure
        return {"unavailable": f"import flash_attn: {type(e).__name__}: {e}"[:300]}
    kc, vc = wl["kv"][0], wl["kv"][1]
    tables = wl["tables"].clamp(min=0)      # padding -> a valid id: reads stay in bounds
    def layer(l):
        return flash_attn_with_kvcache(wl["q"][l].unsqueeze(1), kc[l], vc[l],
                                       cache_seqlens=wl["lens"], block_table=tables,
                                       softmax_scale=D ** -0.5, causal=True)
    try:
        diff = 0.0
        for l in range(min(L, 4)):
            o = layer(l).squeeze(1)
            diff = max(diff, (o.float() - wl["out"][l].float()).abs().max().item())
        torch.cuda.synchronize()
        for l in range(L):
            layer(l)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            for l in range(L):
                layer(l)
        e.record()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 - a missing sm_100 kernel image lands here
        return {"unavailable": f"flash_attn {flash_attn.__version__}: {type(e).__name__}: {e}"[:300]}
    ms = s.elapsed_time(e) / (reps * L)
    return {"version": flash_attn.__version__, "ms_per_layer": round(ms, 5),
            "gbs": round(decode_bytes(wl) / (ms * 1e-3) / 1e9, 1),
            "max_abs_diff_vs_ours": diff}


# ----------------------------------------------------------------------------
# our implementation
# ----------------------------------------------------------------------------

def run_ours(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = args.gpus
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if n > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    pkg._lib.lib()

    wl = build_gpu_workload(args, rank, n, device)
    L, B = args.layers, wl["B"]
    scale = D ** -0.5
    kv = wl["kv"]

    sc = wl["scales"]

    def decode_layer(l):
        if wl["fp8"]:
            pkg.flash_attn_with_kvcache_fp8(wl["q"][l].unsqueeze(1), kv[0, l], kv[1, l],
                                            sc[0, l], sc[1, l], cache_seqlens=wl["lens"],
                                            block_table=wl["tables"], softmax_scale=scale,
                                            out=wl["out"][l].unsqueeze(1))
        else:
            pkg.flash_attn_with_kvcache(wl["q"][l].unsqueeze(1), kv[0, l], kv[1, l],
                                        cache_seqlens=wl["lens"], block_table=wl["tables"],
                                        softmax_scale=scale, out=wl["out"][l].unsqueeze(1))

    def step():
        for l in range(L):
            if wl["fp8"]:
                pkg.store_kvcache_fp8(wl["knew"][l], wl["vnew"][l], kv[0, l], kv[1, l],
                                      sc[0, l], sc[1, l], wl["slots"])
            else:
                pkg.store_kvcache(wl["knew"][l], wl["vnew"][l], kv[0, l], kv[1, l], wl["slots"])
            decode_layer(l)

    def decode_only():
        for l in range(L):
            decode_layer(l)

    def barrier():
        if dist is not None:
            dist.barrier()

    step()                                   # eager pass: allocates the workspace
    torch.cuda.synchronize()
    if pkg.read_device_errors():
        raise SystemExit("device error word set during warm-up")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    dgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dgraph):
        decode_only()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    # ---- timed region: K decode steps ----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(device)
    with clocks:
        barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(end) / args.steps

    # ---- kernel timing for the roofline: decode launches alone ----
    reps = max(2, args.steps // 2)
    dgraph.replay()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(reps):
        dgraph.replay()
    e2.record()
    torch.cuda.synchronize()
    dec_ms = s2.elapsed_time(e2) / (reps * L)
    errs = pkg.read_device_errors()

    # ---- end to end through the public API with host buffers ----
    e2e = run_e2e(args, pkg, wl, device, barrier) if not args.no_e2e else None

    t = torch.tensor([ms, dec_ms, e2e["ms"] if e2e else 0.0, e2e["eager_ms"] if e2e else 0.0],
                     device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, dec_ms, e2e_ms, e2e_eager_ms = t.tolist()

    line = None
    if rank == 0:
        peak, peak_kind = measured_hbm_peak()
        dbytes = decode_bytes(wl)
        abytes = append_bytes(wl)
        step_bytes = L * (dbytes + abytes)
        achieved = dbytes / (dec_ms * 1e-3) / 1e9
        step_gbs = step_bytes / (ms * 1e-3) / 1e9
        tok_s = B / (ms * 1e-3)
        traffic = None
        name = "paged_decode_fp8_traffic.json" if wl["fp8"] else "paged_decode_traffic.json"
        try:
            with open(os.path.join(ROOT, "profiles", name)) as f:
                tr = json.load(f)
            # the captures were taken on the one-GPU configurations 2 and 4 only
            if n == 1 and args.batch == (128 if wl["fp8"] else BATCH_PER_GPU):
                traffic = tr.get("dram_bytes_per_launch")
        except Exception:
            pass
        line = {
            "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8_e4m3 KV, f16 MMA, bf16 q/out" if wl["fp8"] else "bf16",
            "data": ("synthetic: K/V ~ N(0,1) with 1% x20 outliers, quantised per (block, kv head) "
                     "with scale amax/448" if wl["fp8"] else "synthetic: K/V ~ 0.5*N(0,1)")
                    + f", Q ~ N(0,1), context ~ U[{args.ctx_lo},"
                    f"{args.ctx_hi}], random block assignment (seeded)",
            "config": decode_config(args, n),
            "setup": {"pool_blocks": wl["NB"],
                      "pool_gib": round(wl["NB"] * wl["block_bytes"] / 2 ** 30, 1),
                      "graph": "one CUDA graph per step (append + decode for every layer)"},
            "hbm": {"step_gbs": round(step_gbs, 1),
                    "frac_of_8tbs": round(step_gbs / NOMINAL_HBM_GBS, 4),
                    "frac_of_measured": round(step_gbs / peak, 4),
                    "step_bytes": step_bytes},
            "roofline": {"kernel": "paged_decode (main + merge launch, one layer)",
                         "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind, "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                         "algorithmic_bytes": dbytes, "launch_ms": round(dec_ms, 5),
                         "traffic": traffic,
                         "traffic_source": (f"profiles/{name}: dram__bytes_read.sum + "
                                            "dram__bytes_write.sum per launch from a recorded ncu "
                                            "capture of this kernel on this configuration (not "
                                            "measured in this run)") if traffic else None},
            "gpu_launches": args.steps * L * 3,
            "clocks": clocks.summary(),
            "device_errors": errs,
        }
        if e2e:
            line["e2e"] = {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                           "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                           "ms_per_step": round(e2e_ms, 3),
                           "eager_ms_per_step": round(e2e_eager_ms, 3),
                           "path": "Attention.forward + Context per layer (store_kvcache + "
                                   "flash_attn_with_kvcache) for all layers, with each layer's "
                                   "H2D of q/k/v from pinned host buffers and D2H of its "
                                   "output on forked streams, captured as one CUDA graph per "
                                   "step as the reference replays its decode step; "
                                   "eager_ms_per_step: the same step with every layer called "
                                   "from Python"}
        if n == 1 and not args.no_cpu_baseline and not wl["fp8"]:
            line["cpu_baseline"] = cpu_baseline(args, sample_seconds=args.cpu_seconds)
        if args.against_flash_attn and n == 1 and not wl["fp8"]:
            fa = flash_attn_decode(wl, L, reps)
            if "ms_per_layer" in fa:
                fa["ours_ms_per_layer"] = round(dec_ms, 5)
                fa["speedup"] = round(fa["ms_per_layer"] / dec_ms, 3)
            line["library_decode"] = {"flash_attn_with_kvcache": fa}
    del graph, dgraph
    if not args.no_model_step and not wl["fp8"]:
        # The decode path itself has no exchange step (attention is head-local), so
        # the line also carries the full-model step at TP = N (config 5), whose
        # o_proj / down_proj all-reduce is the one collective around the path:
        # fused row-parallel kernel vs cuBLAS + NCCL, both timed on the device.
        kv = sc = None                       # drop the decode pool (closures hold these cells)
        wl.clear()
        torch.cuda.empty_cache()
        mb = 512 if n > 1 else 256          # batch 512 bf16 does not fit one B200
        msteps = max(2, min(args.steps, 10))
        r = measure_model_step(args, rank, n, device, dist, mb, msteps, 3)
        if rank == 0:
            sub = {"metric": MODEL_METRIC, "value": round(mb / (r["ms"] * 1e-3), 1),
                   "unit": "tok/s", "ms_per_step": round(r["ms"], 3), "steps": msteps,
                   "warmup": 3, "parallelism": f"tp{n}", "global_batch": mb,
                   "context": f"U[{CTX_LO},{CTX_HI}] after prefill",
                   "prefill_seconds": round(r["prefill_s"], 2),
                   "all_reduce": ("fused row-parallel kernel (GEMM + tile exchange over NVLink "
                                  "peer memory)" if n > 1 else "none (TP = 1)"),
                   "gpu_launches": r["gpu_launches"], "device_errors": r["errors"],
                   "clocks": r["clocks"]}
            if r["nccl_ms"] is not None:
                sub["cublas_nccl_ms_per_step"] = round(r["nccl_ms"], 3)
                sub["cublas_nccl_value"] = round(mb / (r["nccl_ms"] * 1e-3), 1)
            line["model_step"] = sub
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, pkg, wl, device, barrier):
    """The same decode step driven through the public Attention/Context API from
    pinned host buffers: per step the metadata and every layer's q/k/v go
    host->device and every layer's attention output comes back device->host.

    As the reference engine runs its decode step (nanovllm/engine/
    model_runner.py:196-257: one CUDA graph replay per step), the step is
    captured as one graph: the metadata and each layer's q/k/v copied from
    pinned host memory on a forked stream, each layer's Attention.forward
    (under one Context) waiting for its inputs, each layer's output copied back
    on another forked stream, so the copies overlap the neighbouring layers.
    The same step is also timed eagerly (every layer's Attention.forward called
    from Python, copies per layer pipelined on the side streams): `eager_ms`
    reports it; it depends on the host's dispatch speed (14.0 ms on one box,
    17.9 on another against 13.6 for the graph)."""
    L, B = args.layers, wl["B"]
    attn = []
    for l in range(L):
        a = pkg.Attention(wl["hq"], D, D ** -0.5, wl["hkv"])
        a.k_cache, a.v_cache = wl["kv"][0, l], wl["kv"][1, l]
        if wl["fp8"]:
            a.k_scale, a.v_scale = wl["scales"][0, l], wl["scales"][1, l]
        attn.append(a)
    h_q = wl["q"].cpu().pin_memory()
    h_k = wl["knew"].cpu().pin_memory()
    h_v = wl["vnew"].cpu().pin_memory()
    h_out = torch.empty(wl["out"].shape, dtype=torch.bfloat16).pin_memory()
    h_slots = wl["slots_cpu"].pin_memory()
    h_lens = wl["lens_cpu"].pin_memory()
    h_tables = wl["tables_cpu"].pin_memory()
    h2d = (h_slots.numel() + h_lens.numel() + h_tables.numel()) * 4 + L * (
        h_q[0].numel() + h_k[0].numel() + h_v[0].numel()) * 2
    d2h = L * h_out[0].numel() * 2

    main = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # device input buffers: two sets alternating across the eager steps
    sets = [dict(q=torch.empty_like(wl["q"]), k=torch.empty_like(wl["knew"]),
                 v=torch.empty_like(wl["vnew"]), slots=torch.empty_like(wl["slots"]),
                 lens=torch.empty_like(wl["lens"]), tables=torch.empty_like(wl["tables"]),
                 free=torch.cuda.Event(), meta=torch.cuda.Event(),
                 inp=[torch.cuda.Event() for _ in range(L)]) for _ in range(2)]
    for st in sets:
        st["free"].record(main)
    done = [torch.cuda.Event() for _ in range(L)]

    def eager_step(i):
        st = sets[i & 1]
        with torch.cuda.stream(s_in):
            s_in.wait_event(st["free"])          # the previous user of this set finished
            st["slots"].copy_(h_slots, non_blocking=True)
            st["lens"].copy_(h_lens, non_blocking=True)
            st["tables"].copy_(h_tables, non_blocking=True)
            st["meta"].record(s_in)
            for l in range(L):
                st["q"][l].copy_(h_q[l], non_blocking=True)
                st["k"][l].copy_(h_k[l], non_blocking=True)
                st["v"][l].copy_(h_v[l], non_blocking=True)
                st["inp"][l].record(s_in)
        main.wait_event(st["meta"])
        pkg.set_context(False, slot_mapping=st["slots"], context_lens=st["lens"],
                        block_tables=st["tables"])
        for l in range(L):
            main.wait_event(st["inp"][l])
            o = attn[l](st["q"][l], st["k"][l], st["v"][l])
            done[l].record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[l])
                h_out[l].copy_(o.view(B, wl["hq"], D), non_blocking=True)
                o.record_stream(s_out)
        st["free"].record(main)
        pkg.reset_context()

    def timed(step_fn, warm):
        for i in range(max(1, warm)):
            step_fn(i)
        torch.cuda.synchronize()
        steps = max(2, args.steps)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        s.record(main)
        for i in range(steps):
            step_fn(i)
        main.wait_stream(s_out)                  # the last outputs are on the host
        e.record(main)
        torch.cuda.synchronize()
        barrier()
        return s.elapsed_time(e) / steps

    eager_ms = timed(eager_step, args.warmup)     # (also sizes the workspaces for capture)

    # the whole step in one graph: per-layer H2D on a forked stream, the layers
    # waiting on their inputs, per-layer D2H on another forked stream, so the
    # copies overlap the neighbouring layers within the step
    st = sets[0]
    keep = []

    def captured_step():
        cap = torch.cuda.current_stream(device)
        fork = torch.cuda.Event()
        fork.record(cap)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        with torch.cuda.stream(s_in):
            st["slots"].copy_(h_slots, non_blocking=True)
            st["lens"].copy_(h_lens, non_blocking=True)
            st["tables"].copy_(h_tables, non_blocking=True)
            st["meta"].record(s_in)
            for l in range(L):
                st["q"][l].copy_(h_q[l], non_blocking=True)
                st["k"][l].copy_(h_k[l], non_blocking=True)
                st["v"][l].copy_(h_v[l], non_blocking=True)
                st["inp"][l].record(s_in)
        cap.wait_event(st["meta"])
        pkg.set_context(False, slot_mapping=st["slots"], context_lens=st["lens"],
                        block_tables=st["tables"])
        for l in range(L):
            cap.wait_event(st["inp"][l])
            o = attn[l](st["q"][l], st["k"][l], st["v"][l])
            keep.append(o)                       # no reuse of o's block inside the capture
            done[l].record(cap)
            s_out.wait_event(done[l])
            with torch.cuda.stream(s_out):
                h_out[l].copy_(o.view(B, wl["hq"], D), non_blocking=True)
        pkg.reset_context()
        cap.wait_stream(s_in)
        cap.wait_stream(s_out)

    whole = torch.cuda.CUDAGraph()
    with torch.cuda.graph(whole):
        captured_step()
    whole_ms = timed(lambda i: whole.replay(), args.warmup)
    del whole, keep
    return {"ms": whole_ms, "eager_ms": eager_ms, "h2d": h2d, "d2h": d2h}


# ----------------------------------------------------------------------------
# CPU baseline: the oracle (restatement of the reference's torch path)
# ----------------------------------------------------------------------------

def _cpu_sample(batch=BATCH_PER_GPU, seed=2):
    from oracle import kv_oracle as O  # test infrastructure: the timed CPU baseline only
    B, lens, pages, gen = make_metadata(1, seed=seed, batch_per_gpu=batch)
    need = int(pages.sum())
    W = int(pages.max())
    tables = torch.full((B, W), -1, dtype=torch.int32)
    perm = torch.randperm(need, generator=gen).to(torch.int32)
    cur = 0
    for b in range(B):
        p = int(pages[b])
        tables[b, :p] = perm[cur:cur + p]
        cur += p
    kc = (torch.randn(need, BS, HKV, D, generator=gen) * 0.5).bfloat16()
    vc = (torch.randn(need, BS, HKV, D, generator=gen) * 0.5).bfloat16()
    q = torch.randn(B, HQ, D, generator=gen).bfloat16()
    k = (torch.randn(B, HKV, D, generator=gen) * 0.5).bfloat16()
    v = (torch.randn(B, HKV, D, generator=gen) * 0.5).bfloat16()
    last = (lens - 1).to(torch.int64)
    slots = (tables[torch.arange(B), last // BS].to(torch.int64) * BS + last % BS).to(torch.int32)

    def layer():
        O.store_kvcache(k, v, kc, vc, slots)
        O.decode(q.unsqueeze(1), kc, vc, lens, tables, D ** -0.5)
    return B, layer


def cpu_baseline(args, sample_seconds=10.0):
    torch.set_num_threads(os.cpu_count() or 1)
    B, layer = _cpu_sample(batch=args.cpu_batch)
    layer()                                      # warm-up
    times = []
    t_end = time.perf_counter() + sample_seconds
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        layer()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(B / (LAYERS * t), 3), "unit": "tok/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} x one layer (append + decode) of a {B}-sequence batch with "
                      f"context U[{CTX_LO},{CTX_HI}], fp32 oracle arithmetic on bf16 K/V; "
                      f"tok/s = batch / (36 x median layer time {t * 1e3:.1f} ms)"}


# ----------------------------------------------------------------------------
# config 3: mixed prefill / decode step (reported separately, not the headline)
# ----------------------------------------------------------------------------

MIXED_DECODE, MIXED_CHUNK, MIXED_PREFIX = 64, 2048, (0, 1024, 3072)


def measured_tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def run_mixed(args):
    """36 layers of forward_mixed over 64 decode rows + 3 prefill chunks (with
    --kv fp8: forward_mixed_fp8 over an FP8-E4M3 pool -- quantising append, FP8
    decode, and the prefill rows attended through their pages copied to f16)."""
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    L = args.layers
    gen = torch.Generator().manual_seed(1)
    dec_lens = torch.randint(256, 4097, (MIXED_DECODE,), generator=gen)
    rows = [(int(n) - 1, 1) for n in dec_lens] + [(h, MIXED_CHUNK) for h in MIXED_PREFIX]
    pages = [(h + n + BS - 1) // BS for h, n in rows]
    W = max(pages)
    fp8 = args.kv == "fp8"
    block_bytes = 2 * L * (BS * HKV * D + HKV * 4) if fp8 else 2 * L * BS * HKV * D * 2
    free, total = torch.cuda.mem_get_info(device)
    NB = args.pool_blocks or min(int(POOL_FRAC * total) // block_bytes,
                                 int((free - (8 << 30)) // block_bytes))
    perm = torch.randperm(NB, generator=gen)[:sum(pages)].tolist()
    tables, cur = [], 0
    for n in pages:
        tables.append(perm[cur:cur + n] + [-1] * (W - n))
        cur += n
    slots = [t[pos // BS] * BS + pos % BS for t, (h, n) in zip(tables, rows)
             for pos in range(h, h + n)]
    T = len(slots)
    g = torch.Generator(device=device).manual_seed(77)
    sc = None
    if fp8:  # the bf16 pool's values (0.5 N(0, 1)) quantised per (block, head), amax / 448
        kv = torch.zeros(2, L, NB, BS, HKV, D, dtype=torch.uint8, device=device)
        sc = torch.zeros((2, L, NB, HKV), dtype=torch.float32, device=device)
        fill_fp8_pool(kv, sc, perm, g, 0.5, False)
    else:
        kv = torch.empty(2, L, NB, BS, HKV, D, dtype=torch.bfloat16, device=device)
        for i in range(2):
            for l in range(L):
                kv[i, l].normal_(0.0, 0.5, generator=g)
    q = torch.randn(L, T, HQ, D, device=device, generator=g).bfloat16()
    k = (torch.randn(L, T, HKV, D, device=device, generator=g) * 0.5).bfloat16()
    v = (torch.randn(L, T, HKV, D, device=device, generator=g) * 0.5).bfloat16()
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=device)
    cu_q, cu_k = [0], [0]
    for h, n in rows[MIXED_DECODE:]:
        cu_q.append(cu_q[-1] + n)
        cu_k.append(cu_k[-1] + h + n)
    meta = pkg.MixedAttentionContext(
        MIXED_DECODE, T - MIXED_DECODE, i32(dec_lens.tolist()), i32(tables[:MIXED_DECODE]),
        i32(cu_q), i32(cu_k), i32(tables[MIXED_DECODE:]), MIXED_CHUNK,
        max(h + n for h, n in rows[MIXED_DECODE:]), True)
    ctx = pkg.Context(slot_mapping=i32(slots), mixed=meta)
    scale = D ** -0.5

    def step():
        for l in range(L):
            if fp8:
                pkg.forward_mixed_fp8(q[l], k[l], v[l], kv[0, l], kv[1, l], sc[0, l], sc[1, l],
                                      ctx, scale)
            else:
                pkg.forward_mixed(q[l], k[l], v[l], kv[0, l], kv[1, l], ctx, scale,
                                  pkg.store_kvcache)

    def prefill_only():
        for l in range(L):
            if fp8:
                pkg.flash_attn_varlen_func_fp8(q[l, MIXED_DECODE:], kv[0, l], kv[1, l], sc[0, l],
                                               sc[1, l], meta.prefill_cu_q, meta.prefill_cu_k,
                                               meta.max_q, meta.max_k, softmax_scale=scale,
                                               block_table=meta.prefill_tables)
            else:
                pkg.flash_attn_varlen_func(q[l, MIXED_DECODE:], kv[0, l], kv[1, l],
                                           meta.prefill_cu_q, meta.prefill_cu_k, meta.max_q,
                                           meta.max_k, softmax_scale=scale,
                                           block_table=meta.prefill_tables)

    step()
    prefill_only()                  # eager: sizes the per-device buffers before capture
    torch.cuda.synchronize()
    graph, pgraph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    with torch.cuda.graph(pgraph):
        prefill_only()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    clocks = Clocks(device)
    with clocks:
        ev[0].record()
        for _ in range(args.steps):
            graph.replay()
        ev[1].record()
        torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    pgraph.replay()
    ev[2].record()
    for _ in range(args.steps):
        pgraph.replay()
    ev[3].record()
    torch.cuda.synchronize()
    pre_ms = ev[2].elapsed_time(ev[3]) / (args.steps * L)
    pairs = sum(n * h + n * (n + 1) // 2 for h, n in rows[MIXED_DECODE:])
    flops = 4 * HQ * D * pairs
    peak, kind = measured_tensor_peak()
    achieved = flops / (pre_ms * 1e-3) / 1e12
    traffic = None
    try:
        if not fp8:
            with open(os.path.join(ROOT, "profiles", "paged_prefill_traffic.json")) as f:
                traffic = json.load(f).get("dram_bytes_per_launch")
    except Exception:
        pass
    line = {
        "metric": "mixed prefill/decode step tokens/s (config 3) and prefill tensor TFLOP/s",
        "value": round(T / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("fp8_e4m3 KV (prefill: S as E4M3 MMAs on the K codes, PV in f16 on V "
                  "widened in shared memory; decode: f16 MMAs on codes widened in registers), "
                  "bf16 q/out") if fp8 else "bf16",
        "data": "synthetic (seed 1)",
        "config": {"workload": "BASELINE config 3: 64 decode rows (context U[256,4096]) + 3 "
                               "prefill chunks of 2048 over cached prefixes 0/1024/3072, 36 layers "
                               "of forward_mixed (store + paged decode + paged varlen)"
                               + (" over an FP8-E4M3 pool (forward_mixed_fp8)" if fp8 else ""),
                   "tokens_per_step": T, "layers": L, "pool_blocks": NB},
        "roofline": {"kernel": ("paged_prefill_fp8 (tcgen05, one layer, reading the FP8 "
                                "code pages)") if fp8 else "paged_prefill (tcgen05, one layer)",
                     "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind_str(kind),
                     "algorithmic_flops": flops, "launch_ms": round(pre_ms, 4),
                     "traffic": traffic},
        # per layer: append (FP8: amax, encode, scale commit), decode + merge, prefill
        # work order + prefill
        "gpu_launches": args.steps * L * (7 if fp8 else 5),
        "clocks": clocks.summary(),
        "device_errors": pkg.read_device_errors(),
    }
    print(json.dumps(line), flush=True)
    del graph, pgraph


def run_copy(args):
    """Block-pool copy (copy-on-write / swap of whole block ids): `--batch` random
    source blocks copied to distinct free blocks across all 72 K/V planes of the
    36-layer bf16 pool, one launch per step."""
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    L = args.layers
    block_bytes = 2 * L * BS * HKV * D * 2
    free, total = torch.cuda.mem_get_info(device)
    NB = args.pool_blocks or int((free - (8 << 30)) // block_bytes)
    kv = torch.empty(2, L, NB, BS, HKV, D, dtype=torch.bfloat16, device=device)
    kv.view(torch.int16).random_(-30000, 30000)
    gen = torch.Generator().manual_seed(5)
    perm = torch.randperm(NB, generator=gen)
    n = args.batch
    src = perm[:n].to(torch.int32).to(device)
    dst = perm[n:2 * n].to(torch.int32).to(device)

    def step():
        pkg.kv_block_copy(kv, src, dst)

    step()
    torch.cuda.synchronize()
    bits = kv.view(torch.int16)  # random bit patterns include NaNs: compare bits
    for i in (0, n // 2, n - 1):
        assert torch.equal(bits[:, :, int(dst[i])], bits[:, :, int(src[i])]), "copy mismatch"
    for _ in range(args.warmup):
        step()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    clocks = Clocks(device)
    with clocks:
        ev[0].record()
        for _ in range(args.steps):
            step()
        ev[1].record()
        torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    moved = n * block_bytes * 2
    peak, kind = measured_hbm_peak()
    gbs = moved / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "block-pool copy GB/s (read + write), 36-layer bf16 pool", "value": round(gbs, 1),
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (bit copy)", "data": "synthetic",
        "config": {"workload": f"copy {n} block ids x {L} layers x K/V (CoW / swap)",
                   "pool_blocks": NB, "bytes_per_step": moved},
        "roofline": {"kernel": "kv_block_copy", "bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "peak_kind": kind, "algorithmic_bytes": moved, "launch_ms": round(ms, 4),
                     "traffic": None},
        "gpu_launches": args.steps, "clocks": clocks.summary()}), flush=True)


ROWPAR_METRIC = "row-parallel linear + TP all-reduce, us per call (o_proj, down_proj of Qwen3-4B)"


def run_rowpar(args):
    """The o_proj / down_proj step of config 5 alone at TP = --gpus: x [T, K/t] @
    W_r^T [2560, K/t] then the sum over ranks, T = --batch rows (the decode
    batch), as the fused row-parallel kernel and as the reference's cuBLAS
    F.linear + NCCL all-reduce (each also alone).  Every variant is captured as
    a CUDA graph of `reps` back-to-back calls and timed with CUDA events over
    --steps replays; max over ranks.  Roofline of the fused call: the slower of
    its tensor-core time (FLOPs / measured bf16 peak) and its NVLink time
    (2 (t-1)/t of y per rank over the measured 770 GB/s peer-copy rate)."""
    import torch.nn.functional as F
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    T, N, reps = args.batch, 2560, 8
    comm = pkg.RowParallelAllReduce(T, N, device)
    g = torch.Generator(device=device).manual_seed(77 + rank)
    peak, peak_kind = measured_tensor_peak()
    results = {}
    for name, K in (("o_proj", 4096 // world), ("down_proj", 9728 // world)):
        x = torch.randn(T, K, device=device, generator=g).bfloat16()
        w = (torch.randn(N, K, device=device, generator=g) * 0.02).bfloat16()
        y = torch.empty(T, N, dtype=torch.bfloat16, device=device)
        yr = torch.empty(T, N, dtype=torch.bfloat16, device=device)

        def fused():
            comm(x, w, out=y)

        def gemm():
            torch.matmul(x, w.t(), out=yr)

        def allreduce():
            if dist is not None:
                dist.all_reduce(yr)

        def reference():
            gemm()
            allreduce()

        times = {}
        for vname, fn in (("fused", fused), ("cublas_gemm", gemm), ("nccl_all_reduce", allreduce),
                          ("cublas_plus_nccl", reference)):
            if vname == "nccl_all_reduce" and dist is None:
                continue
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    fn()
            for _ in range(args.warmup):
                graph.replay()
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.steps):
                graph.replay()
            e.record()
            torch.cuda.synchronize()
            us = s.elapsed_time(e) * 1e3 / (args.steps * reps)
            t = torch.tensor([us], device=device)
            if dist is not None:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times[vname] = round(t.item(), 2)
            del graph
        # correctness of the fused call against the reference arithmetic
        fused()
        reference()
        torch.cuda.synchronize()
        diff = (y.float() - yr.float()).abs().max().item()
        flops = 2.0 * T * N * K
        link_bytes = 2.0 * (world - 1) / world * T * N * 2
        target_us = max(flops / (peak * 1e12), link_bytes / 770e9) * 1e6
        results[name] = dict(K_per_rank=K, us=times, max_abs_diff_vs_reference=diff,
                             roofline={"target_us": round(target_us, 2),
                                       "frac": round(target_us / times["fused"], 4),
                                       "tensor_tflops": round(flops / (times["fused"] * 1e-6) / 1e12, 1),
                                       "peak_tflops": peak, "peak_kind": peak_kind,
                                       "nvlink_bytes_per_rank": int(link_bytes)})
    errs = pkg.read_device_errors()
    if rank == 0:
        per_layer = sum(r["us"]["fused"] for r in results.values())
        ref_layer = sum(r["us"]["cublas_plus_nccl"] for r in results.values())
        print(json.dumps({
            "metric": ROWPAR_METRIC, "value": round(per_layer, 2), "unit": "us/layer",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic N(0,1) activations, N(0, 0.02) weights",
            "config": {"workload": "o_proj + down_proj of one Qwen3-4B layer with their TP "
                                   "all-reduce (RowParallelLinear.forward)", "rows": T,
                       "out_features": N, "parallelism": f"tp{world}",
                       "graph": f"{reps} calls per CUDA graph"},
            "reference_us_per_layer": round(ref_layer, 2),
            "shapes": results, "gpu_launches": args.steps * reps * 2, "device_errors": errs,
        }), flush=True)
    comm.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


MODEL_METRIC = "full-model greedy decode tokens/s, random-init Qwen3-4B (config 5), TP = n_gpus"


def measure_model_step(args, rank, world, device, dist, batch, steps, warmup, kv="bf16",
                       unfused_qk=False, nccl_all_reduce=False, ctx_lo=CTX_LO, ctx_hi=CTX_HI):
    """Config 5 at TP = world: build the random-init Qwen3-4B shard of this rank,
    prefill `batch` prompts of random ids (context U[ctx_lo, ctx_hi]) through the
    tcgen05 varlen kernel, then time `steps` graph-captured greedy decode steps
    (o_proj / down_proj + TP all-reduce as the fused row-parallel kernel, or
    cuBLAS + NCCL); at TP > 1 the same step re-captured with cuBLAS + NCCL is
    timed right after.  Device-timed, max over ranks.  Returns a dict (the same
    on every rank)."""
    h = importlib.import_module("slo-aware-llm-serving-engine_b200.qwen3_harness")
    pkg = importlib.import_module("slo-aware-llm-serving-engine_b200")
    cfg = h.Qwen3Config()
    B = batch
    gen = torch.Generator().manual_seed(5)
    lens = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=gen).tolist()
    ids = torch.randint(0, cfg.vocab_size, (sum(lens),), generator=gen).tolist()
    prompts, cur = [], 0
    for n in lens:
        prompts.append(ids[cur:cur + n])
        cur += n
    model = h.Qwen3Model(cfg, rank, world, None, seed=0, device=device,
                         fused_qk_norm_rope=not unfused_qk, fused_all_reduce=not nccl_all_reduce)
    compare = world > 1 and not nccl_all_reduce
    runner = h.GreedyRunner(model, lens, (warmup + steps) * (2 if compare else 1) + 2,
                            seed=1, kv_dtype=kv)
    t0 = time.time()
    tok = runner.prefill(prompts, chunk_tokens=32768)
    torch.cuda.synchronize()
    prefill_s = time.time() - t0
    for _ in range(warmup):
        tok = runner.decode(tok)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(device)
    with clocks:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(steps):
            tok = runner.decode(tok)
        end.record()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    ms = start.elapsed_time(end) / steps
    errs = pkg.read_device_errors()
    nccl_ms = 0.0
    if compare:   # the same step with cuBLAS + NCCL for o_proj / down_proj
        fused_comm, model.rowpar = model.rowpar, None
        runner.graph = None
        for _ in range(warmup):
            tok = runner.decode(tok)
        dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(steps):
            tok = runner.decode(tok)
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
        nccl_ms = start.elapsed_time(end) / steps
        model.rowpar = fused_comm
    t = torch.tensor([ms, nccl_ms, prefill_s], device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, nccl_ms, prefill_s = t.tolist()
    # per-rank HBM bytes of one step: the KV read by attention (mean context
    # over the timed steps) + the append + this rank's weights
    ctx = sum(lens) + B * (warmup + steps // 2 + 1)
    kv_bytes = 2 * cfg.num_layers * ctx * model.hkv * cfg.head_dim * (1 if kv == "fp8" else 2)
    w_bytes = sum(t.numel() * 2 for lw in model.layers
                  for t in (lw.wqkv, lw.wo, lw.wgu, lw.wd)) + model.embed.numel() * 2
    fused = world > 1 and not nccl_all_reduce
    res = dict(ms=ms, nccl_ms=nccl_ms if compare else None, prefill_s=prefill_s, B=B,
               kv_bytes=kv_bytes, w_bytes=w_bytes, clocks=clocks.summary(), errors=errs,
               fused_all_reduce=fused,
               # per layer: the append (fused with q/k norm + RoPE, or alone), the
               # decode's main + merge launches, and two fused row-parallel launches
               gpu_launches=steps * cfg.num_layers * (3 + (2 if fused else 0)))
    runner.release()
    model.close()
    del runner, model
    torch.cuda.empty_cache()
    return res


def run_model(args):
    """random-init Qwen3-4B (36 layers, N(0, 0.02) weights)
    decode step at TP = --gpus (measure_model_step), one JSON line."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    r = measure_model_step(args, rank, world, device, dist, args.batch, args.steps, args.warmup,
                           kv=args.kv, unfused_qk=args.unfused_qk,
                           nccl_all_reduce=args.nccl_all_reduce, ctx_lo=args.ctx_lo,
                           ctx_hi=args.ctx_hi)
    if rank == 0:
        B, ms = r["B"], r["ms"]
        peak, peak_kind = measured_hbm_peak()
        achieved = (r["kv_bytes"] + r["w_bytes"]) / (ms * 1e-3) / 1e9
        line = {
            "metric": MODEL_METRIC, "value": round(B / (ms * 1e-3), 1), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: random-init weights "
            "N(0, 0.02), random prompt ids (seed 5)",
            "config": {"workload": "BASELINE config 5: random-init Qwen3-4B greedy decode step "
                                   f"(36 layers), batch {B}, context U[{args.ctx_lo}, "
                                   f"{args.ctx_hi}] after prefill, KV {args.kv}, q/k norm + "
                                   f"RoPE {'torch ops' if args.unfused_qk else 'fused with the append'}"
                                   + (", o_proj/down_proj + all-reduce "
                                      + ("cuBLAS + NCCL" if args.nccl_all_reduce or world == 1
                                         else "fused row-parallel kernel")),
                       "parallelism": f"tp{world}", "global_batch": B,
                       "prefill_seconds": round(r["prefill_s"], 2)},
            "roofline": {"kernel": "whole decode step per rank (KV read + weights)",
                         "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind,
                         "algorithmic_bytes": r["kv_bytes"] + r["w_bytes"], "traffic": None},
            "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"],
            "device_errors": r["errors"],
        }
        if r["nccl_ms"] is not None:
            line["all_reduce_compare"] = {
                "fused_ms_per_step": round(ms, 3), "nccl_ms_per_step": round(r["nccl_ms"], 3),
                "note": "same step re-captured with cuBLAS o_proj/down_proj + NCCL all-reduce, "
                        "timed right after (contexts longer by warmup + steps tokens)"}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def peak_kind_str(kind):
    return f"{kind} bf16 dense (burst)"


def run_reference(args):
    """--impl reference: the reference's torch path for the hot path, as restated
    by the oracle, on the host cores (the reference has no CPU kernel of its own
    to build).  Rank 0 only; other ranks exit without work.

    One timed step is a bounded sample of the decode step: ONE layer (append +
    decode) of the 256-sequence batch, so `ms_per_step` is that layer's measured
    time and `layers_timed_per_step` says so; `value` scales it to the whole
    36-layer step (batch / (36 x layer time)).  Under weak scaling the N-GPU job
    is N such batches, so the CPU rate is the same at every N."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    B, layer = _cpu_sample(batch=args.cpu_batch)
    for _ in range(args.warmup):
        layer()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer()
    t = (time.perf_counter() - t0) / args.steps
    value = B / (LAYERS * t)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2), "layers_timed_per_step": 1,
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded), as the GPU arm",
        "config": decode_config(args, args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s",
                         "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"each step: one layer (append + decode) of a {B}-sequence "
                                   f"batch, context U[{CTX_LO},{CTX_HI}], fp32 oracle "
                                   f"arithmetic; value = batch / (36 x mean layer time)"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0,
                "note": "CPU implementation: inputs and outputs stay in host memory, "
                        "so there are no host-device copies to time"},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "mixed", "copy", "model", "rowpar"],
                    default="decode",
                    help="decode: config 2/4 (the headline); mixed: config 3 prefill + decode; "
                         "model: config 5 full random-init model at TP = --gpus; "
                         "rowpar: the fused row-parallel linear + all-reduce alone")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16",
                    help="cache format: bf16 (config 2, the headline) or fp8 (config 4)")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU")
    ap.add_argument("--ctx-lo", type=int, default=None)
    ap.add_argument("--ctx-hi", type=int, default=None)
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers per step (36 for the bench; fewer only for profiling)")
    ap.add_argument("--pool-blocks", type=int, default=0,
                    help="pool size in blocks (default: ~70%% of HBM); profiling only")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--unfused-qk", action="store_true",
                    help="model workload: q/k norm + RoPE as torch ops and the plain append")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model-step", action="store_true",
                    help="decode workload: skip the config-5 model-step sub-record")
    ap.add_argument("--nccl-all-reduce", action="store_true",
                    help="model workload: cuBLAS o_proj/down_proj + NCCL all-reduce instead of "
                         "the fused row-parallel kernel")
    ap.add_argument("--against-flash-attn", action="store_true",
                    help="also time the reference's flash-attn decode on the same pool (N=1, bf16)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--cpu-batch", type=int, default=BATCH_PER_GPU)
    args = ap.parse_args()
    fp8_defaults = args.kv == "fp8"
    if args.workload == "model":
        # config 5: batch 512, context U[512, 4096]; at TP = 1 a bf16 cache of
        # that batch (~174 GB) does not fit one B200, so TP = 1 bf16 runs 256
        if args.batch is None:
            args.batch = 512 if (args.gpus > 1 or fp8_defaults) else 256
        args.ctx_lo = args.ctx_lo or CTX_LO
        args.ctx_hi = args.ctx_hi or CTX_HI
    if args.workload == "rowpar" and args.batch is None:
        args.batch = 512
    if args.batch is None:
        args.batch = 128 if fp8_defaults else BATCH_PER_GPU
    if args.ctx_lo is None:
        args.ctx_lo = 1024 if fp8_defaults else CTX_LO
    if args.ctx_hi is None:
        args.ctx_hi = 8192 if fp8_defaults else CTX_HI
    if args.warmup < 3 and args.impl == "ours":
        log("note: warm-up raised to 3 steps")
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "mixed":
        run_mixed(args)
    elif args.workload == "copy":
        run_copy(args)
    elif args.workload == "model":
        run_model(args)
    elif args.workload == "rowpar":
        run_rowpar(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
