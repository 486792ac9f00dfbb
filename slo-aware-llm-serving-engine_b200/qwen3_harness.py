"""Random-init Qwen3 decoder and a greedy runner around the KV-cache path.

This is the caller used to measure and check the path end to end (the
full-model decode configuration): the layer structure of
nanovllm/models/qwen3.py:14-215 -- qkv projection, per-head q/k RMSNorm,
rotary embedding, attention through this package's `Attention` + `Context`,
o_proj, add-RMSNorm, SiLU-gated MLP, tied embedding / LM head -- and the
per-step metadata the reference's ModelRunner builds
(nanovllm/engine/model_runner.py:123-212: slot_mapping, context_lens,
block_tables, cu_seqlens).  The dense math is plain torch (cuBLAS GEMMs) and is
not part of the path.

Tensor parallelism splits query / KV heads and the MLP columns over the
process group and all-reduces the o_proj and down_proj outputs
(nanovllm/layers/linear.py:152-156) -- by default with the fused row-parallel
kernel (GEMM + tile exchange over NVLink in one launch), else cuBLAS + NCCL;
the embedding / LM head is replicated on
every rank, so every rank computes the same logits and the same greedy token.
Weights are N(0, init_std) drawn per full tensor from a seeded generator and
then sliced, so the global model is identical for every TP size.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .kvcache import qk_norm_rope_append
from .layers.attention import Attention
from .layers.linear import RowParallelAllReduce
from .pool import KVPool, tp_shard
from .utils.context import get_context, reset_context, set_context


@dataclass(frozen=True)
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 2560
    intermediate_size: int = 9728
    num_layers: int = 36
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position: int = 40960
    init_std: float = 0.02


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMS over the last dim, rounded to x's dtype, times w
    (nanovllm/layers/layernorm.py rms_forward)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return xf.to(x.dtype) * w


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """(norm(x + residual), x + residual) with the sum formed in fp32 and the new
    residual rounded to x's dtype (nanovllm/layers/layernorm.py add_rms_forward)."""
    s = x.float() + residual.float()
    new_res = s.to(x.dtype)
    s = s * torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    return s.to(x.dtype) * w, new_res


class _Layer:
    __slots__ = ("wqkv", "wo", "wgu", "wd", "ln1", "ln2", "qn", "kn", "attn")


class Qwen3Model:
    """One tensor-parallel rank of a random-init Qwen3 decoder."""

    def __init__(self, cfg: Qwen3Config, tp_rank: int = 0, tp_size: int = 1, group=None,
                 seed: int = 0, device="cuda", dtype=torch.bfloat16,
                 fused_qk_norm_rope: bool = True, fused_all_reduce: bool = True,
                 row_parallel_max_tokens: int = 4096):
        self.cfg, self.tp_rank, self.tp_size, self.group = cfg, tp_rank, tp_size, group
        # q/k RMSNorm + RoPE + append in one kernel (qk_norm_rope_append) for
        # layers whose attention is this package's module on a bf16/f16 pool
        self.fused_qk_norm_rope = fused_qk_norm_rope
        self.device, self.dtype = torch.device(device), dtype
        qh, kh = tp_shard(cfg.num_heads, cfg.num_kv_heads, tp_size, tp_rank)
        if cfg.intermediate_size % tp_size:
            raise ValueError("intermediate size must divide by the tensor-parallel size")
        self.hq, self.hkv = len(qh), len(kh)
        D, H, inter = cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
        il = inter // tp_size
        qr = slice(qh.start * D, qh.stop * D)
        kr = slice(kh.start * D, kh.stop * D)
        ir = slice(tp_rank * il, (tp_rank + 1) * il)
        ones = lambda n: torch.ones(n, dtype=dtype, device=self.device)
        self.embed = self._normal((cfg.vocab_size, H), seed, 0)
        self.norm = ones(H)
        self.layers = []
        for i in range(cfg.num_layers):
            base = 16 * (i + 1)
            wq = self._normal((cfg.num_heads * D, H), seed, base + 0)[qr]
            wk = self._normal((cfg.num_kv_heads * D, H), seed, base + 1)[kr]
            wv = self._normal((cfg.num_kv_heads * D, H), seed, base + 2)[kr]
            lw = _Layer()
            lw.wqkv = torch.cat([wq, wk, wv]).contiguous()
            lw.wo = self._normal((H, cfg.num_heads * D), seed, base + 3)[:, qr].contiguous()
            gate = self._normal((inter, H), seed, base + 4)[ir]
            up = self._normal((inter, H), seed, base + 5)[ir]
            lw.wgu = torch.cat([gate, up]).contiguous()
            lw.wd = self._normal((H, inter), seed, base + 6)[:, ir].contiguous()
            lw.ln1, lw.ln2, lw.qn, lw.kn = ones(H), ones(H), ones(D), ones(D)
            lw.attn = Attention(self.hq, D, D ** -0.5, self.hkv)
            self.layers.append(lw)
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        freqs = torch.outer(torch.arange(cfg.max_position, dtype=torch.float32), inv_freq)
        self.cos = freqs.cos().to(self.device)
        self.sin = freqs.sin().to(self.device)
        self.cos_sin = torch.cat((self.cos, self.sin), dim=-1).contiguous()
        # o_proj / down_proj + TP all-reduce as one kernel per rank
        # (slokv_row_parallel_linear); collective construction over `group`.
        # (CPU instances exist only for the weight-sharding checks.)
        self.rowpar = None
        if tp_size > 1 and fused_all_reduce and self.device.type == "cuda":
            self.rowpar = RowParallelAllReduce(row_parallel_max_tokens, H, self.device, group)

    def close(self):
        """Release the fused all-reduce buffers (collective over the TP group)."""
        if self.rowpar is not None:
            self.rowpar.close()
            self.rowpar = None

    def _normal(self, shape, seed: int, idx: int) -> torch.Tensor:
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1_000_003 + idx)
        t = torch.randn(shape, generator=g, device=self.device, dtype=torch.float32)
        return t.mul_(self.cfg.init_std).to(self.dtype)

    def attention_modules(self):
        return [lw.attn for lw in self.layers]

    def _rope(self, positions, x):
        """Rotate-half rotary embedding in fp32 (nanovllm/layers/rotary_embedding.py)."""
        cos = self.cos[positions].unsqueeze(1)
        sin = self.sin[positions].unsqueeze(1)
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)

    def _row_parallel(self, x, w):
        """RowParallelLinear.forward (nanovllm/layers/linear.py:152-156)."""
        if self.rowpar is not None:
            return self.rowpar(x, w)
        y = F.linear(x, w)
        if self.tp_size > 1:
            torch.distributed.all_reduce(y, group=self.group)
        return y

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """Final normed hidden states [T, hidden]; the Context must be set."""
        cfg = self.cfg
        eps, D = cfg.rms_norm_eps, cfg.head_dim
        qs, kvs = self.hq * D, self.hkv * D
        h = F.embedding(input_ids, self.embed)
        res = None
        for lw in self.layers:
            if res is None:
                x, res = rms_norm(h, lw.ln1, eps), h
            else:
                x, res = add_rms_norm(h, res, lw.ln1, eps)
            qkv = F.linear(x, lw.wqkv)
            if (self.fused_qk_norm_rope and type(lw.attn) is Attention
                    and lw.attn.k_scale is None and lw.attn.k_cache.numel()):
                ctx = get_context()
                cold = ctx.is_prefill and ctx.block_tables is None   # attends on its own rows
                out = qk_norm_rope_append(qkv, self.hq, self.hkv, lw.qn, lw.kn, eps, positions,
                                          self.cos_sin, ctx.slot_mapping, lw.attn.k_cache,
                                          lw.attn.v_cache, k_out=cold)
                q, k = out if cold else (out, None)
                v = qkv[:, qs + kvs:].view(-1, self.hkv, D)
                o = lw.attn.attend(q, k, v)
            else:
                q, k, v = qkv.split([qs, kvs, kvs], dim=-1)
                q = rms_norm(q.view(-1, self.hq, D), lw.qn, eps)
                k = rms_norm(k.view(-1, self.hkv, D), lw.kn, eps)
                v = v.view(-1, self.hkv, D)                # strided view, as the reference
                q, k = self._rope(positions, q), self._rope(positions, k)
                o = lw.attn(q, k, v)
            h = self._row_parallel(o.flatten(1, -1), lw.wo)
            x, res = add_rms_norm(h, res, lw.ln2, eps)
            gate, up = F.linear(x, lw.wgu).chunk(2, dim=-1)
            h = self._row_parallel(F.silu(gate) * up, lw.wd)
        h, _ = add_rms_norm(h, res, self.norm, eps)
        return h

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return F.linear(h, self.embed)


class GreedyRunner:
    """Prefill a batch of prompts into a paged pool, then decode greedily.

    Each sequence owns the blocks it will need for prompt + `max_new` tokens,
    drawn from a seeded permutation of the pool (so pages are scattered, as in
    a long-running engine).  Prefill runs in chunks of whole sequences
    (cold prompts: varlen on the step's own k/v, as `prepare_prefill` sets it
    up without a prefix cache); decode builds slot_mapping / context_lens /
    block_tables like `prepare_decode` and can be captured in a CUDA graph.
    """

    def __init__(self, model: Qwen3Model, prompt_lens, max_new: int, block_size: int = 256,
                 seed: int = 0, spare_blocks: int = 0, kv_dtype: str = "bf16"):
        self.model, self.bs = model, block_size
        self.lens = [int(n) for n in prompt_lens]
        self.B = len(self.lens)
        dev = model.device
        need = [(n + max_new + block_size - 1) // block_size for n in self.lens]
        nb = sum(need) + spare_blocks
        self.pool = KVPool(model.cfg.num_layers, nb, block_size, model.hkv, model.cfg.head_dim,
                           kv_dtype=kv_dtype, device=dev)
        self.pool.bind(model.attention_modules())
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(nb, generator=g).tolist()
        self.W = max(need)
        tables, cur = [], 0
        for n in need:
            tables.append(perm[cur:cur + n] + [-1] * (self.W - n))
            cur += n
        self.tables = torch.tensor(tables, dtype=torch.int32, device=dev)
        self.graph = None

    def _slots(self, b: int, start: int, stop: int) -> list[int]:
        row = self.tables[b].tolist()
        return [row[p // self.bs] * self.bs + p % self.bs for p in range(start, stop)]

    @torch.inference_mode()
    def prefill(self, prompts, chunk_tokens: int = 16384) -> torch.Tensor:
        """Run every prompt; returns the first greedy token of each sequence [B]."""
        dev = self.model.device
        out = torch.empty(self.B, dtype=torch.int64, device=dev)
        b = 0
        while b < self.B:
            e, tot = b, 0
            while e < self.B and (e == b or tot + self.lens[e] <= chunk_tokens):
                tot += self.lens[e]
                e += 1
            ids = torch.tensor([t for i in range(b, e) for t in prompts[i]], dtype=torch.int64,
                               device=dev)
            pos = torch.tensor([p for i in range(b, e) for p in range(self.lens[i])],
                               dtype=torch.int64, device=dev)
            cu = [0]
            for i in range(b, e):
                cu.append(cu[-1] + self.lens[i])
            cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
            slots = torch.tensor([s for i in range(b, e) for s in self._slots(i, 0, self.lens[i])],
                                 dtype=torch.int32, device=dev)
            mx = max(self.lens[b:e])
            set_context(True, cu_t, cu_t, mx, mx, slots, None, None)
            h = self.model.forward(ids, pos)
            reset_context()
            out[b:e] = self.model.logits(h[cu_t[1:].long() - 1]).argmax(dim=-1)
            b = e
        self.pos = torch.tensor(self.lens, dtype=torch.int64, device=dev)
        return out

    def _decode_body(self, ids, pos, ctx_lens, slots):
        """One decode forward over static buffers (graph-capturable)."""
        blk = torch.gather(self.tables, 1, (pos // self.bs).unsqueeze(1)).squeeze(1)
        slots.copy_(blk * self.bs + (pos % self.bs).to(torch.int32))
        ctx_lens.copy_((pos + 1).to(torch.int32))
        set_context(False, None, None, 0, 0, slots, ctx_lens, self.tables)
        h = self.model.forward(ids, pos)
        reset_context()
        return self.model.logits(h).argmax(dim=-1)

    @torch.inference_mode()
    def decode(self, tokens: torch.Tensor, use_graph: bool = True) -> torch.Tensor:
        """Append `tokens` (the last token of every sequence) and return the next
        greedy token of each [B]."""
        dev = self.model.device
        if self.graph is None and use_graph:
            self._ids = torch.zeros(self.B, dtype=torch.int64, device=dev)
            self._pos = torch.zeros(self.B, dtype=torch.int64, device=dev)
            self._lens = torch.zeros(self.B, dtype=torch.int32, device=dev)
            self._slots_buf = torch.zeros(self.B, dtype=torch.int32, device=dev)
            self._ids.copy_(tokens)
            self._pos.copy_(self.pos)
            self._decode_body(self._ids, self._pos, self._lens, self._slots_buf)  # warm-up
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._next = self._decode_body(self._ids, self._pos, self._lens, self._slots_buf)
        if use_graph:
            self._ids.copy_(tokens)
            self._pos.copy_(self.pos)
            self.graph.replay()
            nxt = self._next.clone()
        else:
            lens = torch.empty(self.B, dtype=torch.int32, device=dev)
            slots = torch.empty(self.B, dtype=torch.int32, device=dev)
            nxt = self._decode_body(tokens, self.pos, lens, slots)
        self.pos += 1
        return nxt

    def release(self):
        """Drop the captured graph (it holds NCCL calls under TP)."""
        self.graph = None
