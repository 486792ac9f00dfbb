"""Row-parallel linear layer with its tensor-parallel all-reduce fused into one
kernel (`slokv_row_parallel_linear`).

The reference's `RowParallelLinear` (nanovllm/layers/linear.py:130-156) shards
the input dimension over the TP ranks, runs `F.linear` on each rank (bias on
rank 0 only) and then `dist.all_reduce(y)`.  Here one launch per rank does the
GEMM on the tensor cores and exchanges 128 x 128 output tiles with the other
ranks through their symmetric buffers over NVLink peer memory, so the
collective overlaps the GEMM and no NCCL call is made.

`RowParallelAllReduce` owns the exchange state of one TP group: a zeroed
symmetric buffer per rank (allocated by the library, shared with CUDA IPC
handles exchanged over the process group) and a per-process call counter.  It
can also run every rank of a group inside one process on one GPU ("emulated"
ranks, one launch for all of them), which is how the exchange is tested
without several GPUs.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F
from torch import nn

from .. import _lib
from .._lib import SlokvError, buffers, check, lib, require_cuda, stream_ptr

__all__ = ["RowParallelAllReduce", "RowParallelLinear", "exchange_buffers",
           "row_parallel_buffer_bytes"]

_TILE_N = 128
_TILE_K = 64


def row_parallel_buffer_bytes(max_tokens: int, n_features: int, world: int) -> int:
    """Bytes of one rank's symmetric buffer (0 for an unsupported geometry)."""
    return int(lib().slokv_row_parallel_buffer_bytes(int(max_tokens), int(n_features), int(world)))


def exchange_buffers(own_ptr: int, own_handle: bytes, import_handle, group=None) -> list[int]:
    """All-gather every rank's IPC handle over `group` and map the peers'
    buffers: returns the pointer of rank r's buffer as seen by this process at
    index r (this rank's own `own_ptr` at its own index), then waits on a
    barrier so no rank writes into a peer before every rank has mapped.
    `import_handle(handle_bytes) -> int` opens one peer handle."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    handles = [None] * world
    dist.all_gather_object(handles, bytes(own_handle), group=group)
    ptrs = [own_ptr if r == rank else import_handle(h) for r, h in enumerate(handles)]
    dist.barrier(group=group)
    return ptrs


def _ptr_array(values):
    arr = (ctypes.c_void_p * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


class RowParallelAllReduce:
    """Exchange state of one TP group for the fused row-parallel linear.

    RowParallelAllReduce(max_tokens, n_features, device, group=None)
        one rank per process: every rank of `group` (default: the default
        process group) constructs it collectively; buffers are exchanged with
        all_gather_object.
    RowParallelAllReduce.emulated(world, max_tokens, n_features, device)
        every rank in this process, on one GPU; call `emulate(xs, ws)`.

    Calls with more than `max_tokens` rows run in max_tokens-row chunks.  Every
    rank must make the same sequence of calls with the same row counts.
    """

    def __init__(self, max_tokens: int, n_features: int, device, group=None, *,
                 _emulate_world: int | None = None):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise SlokvError("the fused row-parallel linear runs on CUDA devices only")
        if n_features % _TILE_N:
            raise SlokvError(f"n_features must be a multiple of {_TILE_N}")
        self.max_tokens = int(max_tokens)
        self.n_features = int(n_features)
        self.group = group
        self._own, self._peers = [], []
        if _emulate_world is not None:
            self.world, self.rank, self.local_ranks = int(_emulate_world), 0, int(_emulate_world)
        else:
            import torch.distributed as dist
            if dist.is_available() and dist.is_initialized():
                self.world = dist.get_world_size(group)
                self.rank = dist.get_rank(group)
            else:                      # no process group: one rank, the GEMM alone
                self.world, self.rank = 1, 0
            self.local_ranks = 1
        if self.world not in (1, 2, 4, 8):
            raise SlokvError(f"the fused row-parallel linear supports TP sizes 1, 2, 4 and 8, "
                             f"not {self.world}")
        self.buffer_bytes = row_parallel_buffer_bytes(self.max_tokens, self.n_features, self.world)
        if self.buffer_bytes == 0:
            raise SlokvError("unsupported row-parallel geometry")
        with torch.cuda.device(self.device):
            self.state = torch.zeros(2, dtype=torch.int32, device=self.device)
            self._err = buffers.error_word(self.device)
            if self.world == 1 or _emulate_world is not None:
                self.rank_buffers = [self._alloc() for _ in range(self.world)]
            else:
                own = self._alloc()
                self.rank_buffers = self._exchange(own)
        self._buf_arr = _ptr_array(self.rank_buffers)

    @classmethod
    def emulated(cls, world: int, max_tokens: int, n_features: int, device):
        return cls(max_tokens, n_features, device, _emulate_world=world)

    # ---- buffers ------------------------------------------------------------
    def _alloc(self) -> int:
        p = ctypes.c_void_p()
        check(lib().slokv_device_alloc(self.buffer_bytes, ctypes.byref(p)), "device_alloc")
        self._own.append(p.value)
        return p.value

    def _exchange(self, own: int) -> list[int]:
        hsize = lib().slokv_ipc_handle_size()
        h = ctypes.create_string_buffer(hsize)
        check(lib().slokv_ipc_export(own, h), "ipc_export")

        def import_handle(hb: bytes) -> int:
            p = ctypes.c_void_p()
            check(lib().slokv_ipc_import(ctypes.create_string_buffer(hb, hsize), ctypes.byref(p)),
                  "ipc_import")
            self._peers.append(p.value)
            return p.value

        return exchange_buffers(own, h.raw, import_handle, self.group)

    def close(self):
        """Release the peer mappings and this process's buffers.  Collective:
        call it on every rank after the last fused call has finished."""
        if not self._own and not self._peers:
            return
        torch.cuda.synchronize(self.device)
        if self.local_ranks == 1 and self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        for p in self._peers:
            lib().slokv_ipc_close(p)
        for p in self._own:
            lib().slokv_device_free(p)
        self._own, self._peers = [], []

    # ---- calls --------------------------------------------------------------
    def _check(self, x, w, bias, out):
        if x.dim() != 2 or w.dim() != 2 or w.shape[0] != self.n_features or x.shape[1] != w.shape[1]:
            raise SlokvError(f"x [T, K] and w [{self.n_features}, K] expected, got "
                             f"{tuple(x.shape)} and {tuple(w.shape)}")
        if x.dtype not in (torch.bfloat16, torch.float16) or w.dtype != x.dtype:
            raise SlokvError("x and w must share a 16-bit dtype")
        if x.shape[1] % _TILE_K:
            raise SlokvError(f"the input features per rank must be a multiple of {_TILE_K}")
        if x.stride(1) != 1 or w.stride(1) != 1:
            raise SlokvError("x and w need a contiguous last dimension")
        if bias is not None and (bias.dtype != x.dtype or bias.shape != (self.n_features,)
                                 or not bias.is_contiguous()):
            raise SlokvError("bias must be a contiguous [n_features] tensor of x's dtype")
        if out is None:
            out = torch.empty(x.shape[0], self.n_features, dtype=x.dtype, device=x.device)
        elif out.shape != (x.shape[0], self.n_features) or out.dtype != x.dtype or out.stride(1) != 1:
            raise SlokvError("out must be [T, n_features] of x's dtype with contiguous rows")
        return out

    def _launch(self, xs, ws, biases, outs, rank_base):
        T, K = xs[0].shape
        n = len(xs)
        check(lib().slokv_row_parallel_linear(
            _ptr_array([x.data_ptr() for x in xs]), xs[0].stride(0),
            _ptr_array([w.data_ptr() for w in ws]), ws[0].stride(0),
            None if biases is None else _ptr_array([b.data_ptr() for b in biases]),
            _ptr_array([o.data_ptr() for o in outs]), outs[0].stride(0),
            T, self.n_features, K, self._buf_arr, self.world, rank_base, n, self.max_tokens,
            self.state.data_ptr(), _lib.dtype_code(xs[0].dtype), self._err.data_ptr(),
            stream_ptr(self.device)), "row_parallel_linear")

    def _chunks(self, T):
        for s in range(0, T, self.max_tokens):
            yield s, min(T, s + self.max_tokens)

    def __call__(self, x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """all_reduce(F.linear(x, w[, bias on one rank])) over the group, fused."""
        if self.local_ranks != 1:
            raise SlokvError("an emulated group is driven through emulate()")
        require_cuda(x, w, bias, out)
        out = self._check(x, w, bias, out)
        for s, e in self._chunks(x.shape[0]):
            self._launch([x[s:e]], [w], None if bias is None else [bias], [out[s:e]], self.rank)
        return out

    def emulate(self, xs, ws, biases=None, outs=None):
        """Every rank of an emulated group in one launch: xs[r], ws[r] are rank
        r's input and weight shard; returns the list of per-rank outputs (all
        equal)."""
        if self.local_ranks != self.world or len(xs) != self.world or len(ws) != self.world:
            raise SlokvError("emulate() takes one input and one weight per rank")
        require_cuda(*xs, *ws)
        outs = list(outs) if outs is not None else [None] * self.world
        for r in range(self.world):
            outs[r] = self._check(xs[r], ws[r], None if biases is None else biases[r], outs[r])
            if xs[r].shape != xs[0].shape or xs[r].stride(0) != xs[0].stride(0) or \
                    ws[r].stride(0) != ws[0].stride(0) or outs[r].stride(0) != outs[0].stride(0):
                raise SlokvError("emulated ranks need equal shapes and strides")
        for s, e in self._chunks(xs[0].shape[0]):
            self._launch([x[s:e] for x in xs], ws, biases, [o[s:e] for o in outs], 0)
        return outs


class RowParallelLinear(nn.Module):
    """Drop-in for the reference's RowParallelLinear (nanovllm/layers/linear.py:
    130-156): same constructor, weight shard [output_size, input_size / tp],
    weight_loader and forward contract; the all-reduce runs inside the fused
    kernel.  `comm` (a RowParallelAllReduce over the default process group) is
    shared by every layer of one output width; it is created on first use with
    `max_tokens` rows per launch."""

    _comms: dict = {}

    def __init__(self, input_size: int, output_size: int, bias: bool = False,
                 max_tokens: int = 8192):
        super().__init__()
        import torch.distributed as dist
        self.tp_rank = dist.get_rank() if dist.is_initialized() else 0
        self.tp_size = dist.get_world_size() if dist.is_initialized() else 1
        if input_size % self.tp_size:
            raise SlokvError(f"{input_size} is not divisible by the TP size {self.tp_size}")
        self.input_size = input_size // self.tp_size
        self.output_size = output_size
        self.max_tokens = max_tokens
        self.weight = nn.Parameter(torch.empty(output_size, self.input_size))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        data = param.data
        if data.ndim == 1:
            data.copy_(loaded_weight)
            return
        shard = data.size(1)
        data.copy_(loaded_weight.narrow(1, self.tp_rank * shard, shard))

    def comm(self) -> RowParallelAllReduce:
        key = (self.weight.device, self.output_size, self.max_tokens)
        c = RowParallelLinear._comms.get(key)
        if c is None:
            c = RowParallelAllReduce(self.max_tokens, self.output_size, self.weight.device)
            RowParallelLinear._comms[key] = c
        return c

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return F.linear(x, self.weight, self.bias)
        lead = x.shape[:-1]
        y = self.comm()(x.reshape(-1, x.shape[-1]), self.weight, self.bias)
        return y.view(*lead, self.output_size)
