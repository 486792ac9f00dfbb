"""ctypes binding of the C ABI declared in include/slokv.h.

The library is loaded from this package directory only (it is built in-tree by
build.py).  There is no fallback: if it is missing, or if a tensor handed to an
entry point is not on a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libslokv.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# status codes / device error bits (mirrors include/slokv.h)
OK = 0
ERR_INVALID_ARG = -1
ERR_ALIGNMENT = -2
ERR_UNSUPPORTED = -3
ERR_CUDA = -4
ERR_WORKSPACE = -5
ERR_SCRATCH_LIMIT = -6

DEVERR_SLOT_RANGE = 0x1
DEVERR_BLOCK_RANGE = 0x2
DEVERR_CONTEXT_LEN = 0x4
DEVERR_TIMEOUT = 0x8
DEVERR_NONFINITE = 0x10

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2
DTYPE_FP8_E4M3 = 3

_c_i32, _c_i64, _c_f32, _c_sz, _c_vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                         ctypes.c_size_t, ctypes.c_void_p)

# name -> (restype, argtypes)
SIGNATURES = {
    "slokv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "slokv_abi_version": (ctypes.c_int, []),
    "slokv_kv_append": (ctypes.c_int, [
        _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i32, _c_i32, _c_i32, _c_i64,
        _c_vp, _c_vp]),
    "slokv_paged_decode_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32, _c_i32]),
    "slokv_paged_decode": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64,            # out, strides
        _c_vp, _c_i64, _c_i64,            # q, strides
        _c_vp, _c_vp, _c_i64, _c_i64,     # k_cache, v_cache, block strides
        _c_i32, _c_i32,                   # num_blocks, block_size
        _c_i32, _c_i32, _c_i32,           # Hq, Hkv, D
        _c_vp, _c_i64, _c_i32,            # block_tables, stride, width
        _c_vp, _c_i32,                    # context_lens, batch
        _c_f32, _c_i32,                   # scale, dtype
        _c_vp, _c_sz, _c_vp, _c_vp]),     # workspace, bytes, dev_error, stream
    "slokv_paged_prefill": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64,                    # out, token / head strides
        _c_vp, _c_i64, _c_i64, _c_i64,            # q, strides, rows
        _c_vp, _c_vp, _c_i64, _c_i64, _c_i64,     # k, v, row strides, kv rows
        _c_i64, _c_i64,                           # block strides
        _c_vp, _c_vp, _c_i32, _c_i32,             # cu_q, cu_k, rows, max_seqlen_q
        _c_vp, _c_i64, _c_i32, _c_i32, _c_i32,    # tables, stride, width, num_blocks, bs
        _c_i32, _c_i32, _c_i32, _c_f32, _c_i32,   # Hq, Hkv, D, scale, dtype
        _c_vp,                                    # k_page_scale (FP8 pools) or None
        _c_vp, _c_sz, _c_vp, _c_vp]),             # workspace, bytes, dev_error, stream
    "slokv_paged_prefill_workspace_bytes": (_c_sz, [_c_i32, _c_i32]),
    "slokv_paged_prefill_fp8": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64,                    # out, token / head strides
        _c_vp, _c_i64, _c_i64, _c_i64,            # q, strides, rows
        _c_vp, _c_vp, _c_i64, _c_i64,             # k / v codes, block strides (bytes)
        _c_vp, _c_vp,                             # k / v scales
        _c_vp, _c_vp, _c_i32, _c_i32,             # cu_q, cu_k, rows, max_seqlen_q
        _c_vp, _c_i64, _c_i32, _c_i32, _c_i32,    # tables, stride, width, num_blocks, bs
        _c_i32, _c_i32, _c_i32, _c_f32, _c_i32,   # Hq, Hkv, D, scale, q dtype
        _c_vp, _c_sz, _c_vp, _c_vp]),             # workspace, bytes, dev_error, stream
    "slokv_fp8_pages_dequant": (ctypes.c_int, [
        _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp,   # codes, block strides, scales
        _c_i32, _c_i32, _c_i32, _c_i32,               # num_blocks, block_size, Hkv, D
        _c_vp, _c_i64, _c_i32, _c_vp, _c_i32, _c_i32,  # tables, stride, width, cu_k, rows, pages
        _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),          # dst_k, dst_v, dst_k_scale, err, stream
    "slokv_qk_norm_rope_append": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,  # qkv, row stride, T, Hq, Hkv, D
        _c_vp, _c_vp, _c_f32,                         # q_weight, k_weight, eps
        _c_vp, _c_vp, _c_i32,                         # positions, cos_sin, max_position
        _c_vp, _c_vp, _c_vp, _c_i64,                  # slot_mapping, k_cache, v_cache, slots
        _c_vp, _c_i64, _c_vp, _c_i64,                 # q_out, stride, k_out, stride
        _c_i32, _c_vp, _c_vp]),                       # dtype, dev_error, stream
    "slokv_kv_append_fp8_runs_workspace_bytes": (_c_sz, [_c_i32, _c_i32]),
    "slokv_kv_append_fp8_runs": (ctypes.c_int, [
        _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i32, _c_i32,
        _c_i32, _c_i32, _c_i32, _c_i32,           # as slokv_kv_append_fp8, then
        _c_vp, _c_sz, _c_vp, _c_vp]),             # workspace, bytes, dev_error, stream
    "slokv_kv_append_fp8": (ctypes.c_int, [
        _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i32, _c_i32,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp]),
    "slokv_paged_decode_fp8_workspace_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32, _c_i32]),
    "slokv_paged_decode_fp8": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64,
        _c_vp, _c_vp,                     # k_scale, v_scale
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp, _c_i32,
        _c_f32, _c_i32, _c_vp, _c_sz, _c_vp, _c_vp]),
    "slokv_fp8_e4m3_encode": (ctypes.c_int, [_c_vp, _c_vp, _c_i64, _c_vp, _c_vp]),
    "slokv_fp8_e4m3_decode": (ctypes.c_int, [_c_vp, _c_vp, _c_i64, _c_vp]),
    "slokv_paged_decode_noalloc": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp, _c_i32,
        _c_f32, _c_i32, _c_vp, _c_vp]),   # as slokv_paged_decode, without the workspace
    "slokv_paged_decode_noalloc_scratch_bytes": (_c_sz, []),
    "slokv_row_parallel_buffer_bytes": (_c_sz, [_c_i32, _c_i32, _c_i32]),
    "slokv_row_parallel_plan": (ctypes.c_int, [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp]),
    "slokv_row_parallel_linear": (ctypes.c_int, [
        _c_vp, _c_i64, _c_vp, _c_i64,             # x[], row stride, w[], row stride
        _c_vp, _c_vp, _c_i64,                     # bias[] (or None), y[], row stride
        _c_i32, _c_i32, _c_i32,                   # tokens, n_features, k_features
        _c_vp, _c_i32, _c_i32, _c_i32, _c_i32,    # rank_buffers[], world, rank_base, local, max_tokens
        _c_vp, _c_i32, _c_vp, _c_vp]),            # state, dtype, dev_error, stream
    "slokv_device_alloc": (ctypes.c_int, [_c_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "slokv_device_free": (ctypes.c_int, [_c_vp]),
    "slokv_ipc_handle_size": (ctypes.c_int, []),
    "slokv_ipc_export": (ctypes.c_int, [_c_vp, _c_vp]),
    "slokv_ipc_import": (ctypes.c_int, [_c_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "slokv_ipc_close": (ctypes.c_int, [_c_vp]),
    "slokv_kv_block_copy": (ctypes.c_int, [
        _c_vp, _c_i64, _c_i64, _c_vp, _c_i32,     # src, strides, ids, capacity
        _c_vp, _c_i64, _c_i64, _c_vp, _c_i32,     # dst, strides, ids, capacity
        _c_i32, _c_i32, _c_i64, _c_vp, _c_vp]),   # pages, planes, page bytes, dev_error, stream
}

_lock = threading.Lock()
_lib = None


class SlokvError(RuntimeError):
    """A C-ABI entry point rejected its arguments or a CUDA launch failed."""


def lib() -> ctypes.CDLL:
    """Load libslokv.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise SlokvError(
                    f"{LIB_NAME} is not built: run `python -c 'import __graft_entry__ as g; g.build()'` "
                    "or the package's build.py (there is no CPU fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != OK:
        msg = lib().slokv_status_string(status).decode()
        raise SlokvError(f"{what}: {msg} (status {status})")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise SlokvError("the KV-cache kernels run on CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise SlokvError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float16:
        return DTYPE_F16
    if dt == torch.float32:
        return DTYPE_F32
    if dt == torch.uint8 or dt == getattr(torch, "float8_e4m3fn", None):
        return DTYPE_FP8_E4M3
    raise SlokvError(f"unsupported dtype {dt}")


class _PerDevice:
    """Per-device fixed-address buffers: the device error word and workspaces.

    They are allocated once (outside graph capture) and reused by every call, so
    captured graphs keep pointing at live memory.
    """

    def __init__(self):
        self._err = {}
        self._ws = {}

    def error_word(self, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        t = self._err.get(idx)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            self._err[idx] = t
        return t

    def workspace(self, device: torch.device, key: str, nbytes: int,
                  zero: bool = False) -> torch.Tensor:
        """Buffer `key` of at least nbytes; `zero`: allocated zero-filled (for
        buffers the kernels leave zero after every call)."""
        idx = device.index if device.index is not None else torch.cuda.current_device()
        t = self._ws.get((idx, key))
        if t is None or t.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise SlokvError(
                    f"workspace '{key}' must be allocated before CUDA graph capture; call the op "
                    "once eagerly (warm-up) with the largest geometry first")
            t = (torch.zeros if zero else torch.empty)(max(nbytes, 256), dtype=torch.uint8,
                                                       device=torch.device("cuda", idx))
            self._ws[(idx, key)] = t
        return t

    def workspace_fits(self, device: torch.device, key: str, nbytes: int) -> bool:
        """Whether workspace `key` of `device` already holds nbytes (no allocation)."""
        idx = device.index if device.index is not None else torch.cuda.current_device()
        t = self._ws.get((idx, key))
        return t is not None and t.numel() >= nbytes


buffers = _PerDevice()


def read_device_errors(device: torch.device | None = None, reset: bool = True) -> int:
    """Return (and by default clear) the device error bits of `device`.

    This synchronises the device's current stream; call it outside graph capture.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    word = buffers.error_word(device)
    val = int(word.item()) & 0xFFFFFFFF
    if reset and val:
        word.zero_()
    return val
