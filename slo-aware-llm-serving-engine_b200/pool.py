"""KV block pool: sizing, allocation, binding and block lifecycle, bf16 or FP8.

Mirrors the reference engine's pool handling (nanovllm/engine/model_runner.py:103-121,
nanovllm/engine/mixed_model_runner.py:17-47): the pool is one tensor
kv_cache[2, num_layers, num_blocks, block_size, Hkv_local, head_dim], sized from
free device memory as
    int(total * gpu_memory_utilization - used - peak + current) // block_bytes,
optionally capped, and reduced to the minimum over tensor-parallel ranks so every
rank schedules the same block ids.  Layer l's attention module is bound to
kv_cache[0, l] / kv_cache[1, l].

FP8-E4M3 pools keep uint8 codes in the same layout plus fp32 scales
k_scale/v_scale [num_layers, num_blocks, Hkv_local]; block_bytes counts the
scales.  A reused page never inherits an old amax without any call from the
block manager: the quantising append ignores a block's stored scale when its
write starts at offset 0, where every newly assigned block is first written
(reset_blocks remains as an eager helper for tools that want clean scales).
"""
from __future__ import annotations

import torch

from . import kvcache


def tp_shard(num_heads: int, num_kv_heads: int, tp_size: int, rank: int):
    """Query / KV head ranges of one tensor-parallel rank (heads split evenly, as
    nanovllm/models/qwen3.py:29-35 divides them); GQA groups never straddle ranks."""
    if num_heads % tp_size or num_kv_heads % tp_size:
        raise ValueError("head counts must divide by the tensor-parallel size")
    if not 0 <= rank < tp_size:
        raise ValueError("rank out of range")
    hq, hk = num_heads // tp_size, num_kv_heads // tp_size
    return range(rank * hq, (rank + 1) * hq), range(rank * hk, (rank + 1) * hk)


def block_bytes(num_layers: int, block_size: int, num_kv_heads: int, head_dim: int,
                kv_dtype: str = "bf16") -> int:
    """Bytes one block id occupies over all layers, K and V (plus FP8 scales)."""
    if kv_dtype == "fp8":
        return 2 * num_layers * (block_size * num_kv_heads * head_dim + num_kv_heads * 4)
    if kv_dtype in ("bf16", "f16"):
        return 2 * num_layers * block_size * num_kv_heads * head_dim * 2
    raise ValueError(f"unknown kv dtype {kv_dtype}")


def plan_num_blocks(total: int, used: int, peak: int, current: int, per_block: int,
                    gpu_memory_utilization: float = 0.9, cap: int | None = None,
                    group=None) -> int:
    """Block count of the reference's formula, capped, minimum over `group`."""
    count = int(total * gpu_memory_utilization - used - peak + current) // per_block
    if cap is not None:
        count = min(count, cap)
    import torch.distributed as dist
    if group is not None or (dist.is_available() and dist.is_initialized()):
        if dist.get_world_size(group) > 1:
            backend = dist.get_backend(group)
            dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
            t = torch.tensor([count], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
            count = int(t.item())
    if count <= 0:
        raise RuntimeError("no KV blocks available on at least one TP rank")
    return count


class KVPool:
    """The paged KV pool of one rank."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                 head_dim: int, kv_dtype: str = "bf16", device="cuda"):
        self.num_layers, self.num_blocks, self.block_size = num_layers, num_blocks, block_size
        self.num_kv_heads, self.head_dim, self.kv_dtype = num_kv_heads, head_dim, kv_dtype
        shape = (2, num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        if kv_dtype == "fp8":
            self.kv_cache = torch.zeros(shape, dtype=torch.uint8, device=device)
            self.k_scale = torch.zeros(num_layers, num_blocks, num_kv_heads, dtype=torch.float32,
                                       device=device)
            self.v_scale = torch.zeros_like(self.k_scale)
        else:
            dt = torch.bfloat16 if kv_dtype == "bf16" else torch.float16
            self.kv_cache = torch.empty(shape, dtype=dt, device=device)
            self.k_scale = self.v_scale = None

    @classmethod
    def from_free_memory(cls, num_layers, block_size, num_kv_heads, head_dim, kv_dtype="bf16",
                         gpu_memory_utilization=0.9, cap=None, group=None, device=None):
        """Size the pool like allocate_kv_cache does (min over TP ranks)."""
        device = device or torch.device("cuda", torch.cuda.current_device())
        free, total = torch.cuda.mem_get_info(device)
        stats = torch.cuda.memory_stats(device)
        per_block = block_bytes(num_layers, block_size, num_kv_heads, head_dim, kv_dtype)
        n = plan_num_blocks(total, total - free, stats["allocated_bytes.all.peak"],
                            stats["allocated_bytes.all.current"], per_block,
                            gpu_memory_utilization, cap, group)
        return cls(num_layers, n, block_size, num_kv_heads, head_dim, kv_dtype, device)

    def bind(self, modules) -> int:
        """Bind every module with k_cache/v_cache attributes, in order, to its layer."""
        layer = 0
        for m in modules:
            if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
                m.k_cache = self.kv_cache[0, layer]
                m.v_cache = self.kv_cache[1, layer]
                if self.k_scale is not None:
                    m.k_scale, m.v_scale = self.k_scale[layer], self.v_scale[layer]
                layer += 1
        if layer != self.num_layers:
            raise RuntimeError(f"bound {layer} attention layers, pool has {self.num_layers}")
        return layer

    def reset_blocks(self, block_ids: torch.Tensor) -> None:
        """Zero the FP8 scales of `block_ids` (no-op for bf16).  Optional: the
        append already treats a block whose write starts at offset 0 as fresh,
        so the engine's block manager never has to call this."""
        if self.k_scale is not None and block_ids.numel():
            idx = block_ids.to(device=self.k_scale.device, dtype=torch.long)
            self.k_scale[:, idx] = 0
            self.v_scale[:, idx] = 0

    def copy_blocks(self, src_ids: torch.Tensor, dst_ids: torch.Tensor) -> None:
        """Copy whole blocks (all layers, K and V, and FP8 scales): copy-on-write
        of a shared tail block, or a move for defragmentation."""
        kvcache.kv_block_copy(self.kv_cache, src_ids, dst_ids)
        if self.k_scale is not None:
            s = src_ids.long()
            d = dst_ids.long()
            keep = (s >= 0) & (d >= 0)
            self.k_scale[:, d[keep]] = self.k_scale[:, s[keep]]
            self.v_scale[:, d[keep]] = self.v_scale[:, s[keep]]

    def swap_out(self, block_ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Gather blocks into a compact device buffer [2, L, n, ...] (one launch) for
        swap-based preemption; the caller may then copy it to pinned host memory."""
        return kvcache.kv_block_gather(self.kv_cache, block_ids, out)

    def swap_in(self, saved: torch.Tensor, block_ids: torch.Tensor) -> None:
        kvcache.kv_block_scatter(saved, self.kv_cache, block_ids)
