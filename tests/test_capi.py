"""C-ABI library: it loads, exports every symbol include/*.h declares, and its
host-side argument checks reject bad calls before any launch.  CPU only: no call
here reaches a kernel or the CUDA runtime."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(slokv_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("slokv_kv_append", "slokv_paged_decode", "slokv_kv_block_copy",
                     "slokv_paged_decode_workspace_bytes"):
        assert required in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(pkg._lib.SIGNATURES) >= set(declared_symbols())


def test_status_strings(pkg):
    lib = pkg._lib.lib()
    assert lib.slokv_status_string(0) == b"ok"
    assert b"unsupported" in lib.slokv_status_string(-3)
    assert lib.slokv_abi_version() >= 1


def test_append_argument_checks(pkg):
    lib = pkg._lib.lib()
    # zero tokens is a no-op; negative sizes and bad element widths are rejected
    assert lib.slokv_kv_append(None, 0, None, 0, None, None, None, 0, 1024, 2, 64, None, None) == 0
    assert lib.slokv_kv_append(None, 0, None, 0, None, None, None, -1, 1024, 2, 64, None, None) == -1
    assert lib.slokv_kv_append(None, 0, None, 0, None, None, None, 4, 1024, 3, 64, None, None) == -3
    assert lib.slokv_kv_append(None, 0, None, 0, None, None, None, 4, 1024, 2, 64, None, None) == -1


def _decode(lib, **kw):
    args = dict(out=None, osb=0, osh=0, q=None, qsb=0, qsh=0, kc=None, vc=None, kbs=0, vbs=0,
                nb=64, bs=256, hq=32, hkv=8, d=128, bt=None, bts=0, w=16, lens=None, batch=4,
                scale=0.1, dtype=0, ws=None, wsb=0, err=None, stream=None)
    args.update(kw)
    return lib.slokv_paged_decode(*args.values())


def test_decode_argument_checks(pkg):
    lib = pkg._lib.lib()
    assert _decode(lib, batch=0) == 0                   # empty batch: nothing to do
    assert _decode(lib, batch=-1) == -1
    assert _decode(lib, d=64) == -3                     # head_dim 128 only
    assert _decode(lib, dtype=2) == -1                  # fp32 path: null pointers rejected
    assert _decode(lib, dtype=3) == -3                  # FP8 codes need slokv_paged_decode_fp8
    assert _decode(lib, hq=30) == -1                    # Hq % Hkv
    assert _decode(lib, hq=8 * 17) == -3                # group > 16
    assert _decode(lib, bs=48) == -3                    # block size multiple of 32
    assert _decode(lib) == -1                           # null pointers


def test_block_copy_argument_checks(pkg):
    lib = pkg._lib.lib()
    def call(src=None, sps=0, dst=None, dps=0, n=0, cap=8, pb=1024):
        return lib.slokv_kv_block_copy(src, 0, sps, None, cap, dst, 0, dps, None, cap, n, 4, pb,
                                       None, None)
    assert call(n=0) == 0
    assert call(n=-1) == -1
    assert call(n=2) == -1
    assert call(n=2, cap=-1) == -1
    p = ctypes.c_void_p(16)
    assert call(src=p, sps=8, dst=p, dps=16, n=2) == -2


def test_row_parallel_argument_checks(pkg):
    lib = pkg._lib.lib()
    def call(tokens=4, n=2560, k=1024, world=2, base=0, local=1, max_tokens=512, dtype=0,
             x=None, w=None, y=None, bufs=None, state=None):
        return lib.slokv_row_parallel_linear(x, k, w, k, None, y, n, tokens, n, k, bufs, world,
                                             base, local, max_tokens, state, dtype, None, None)
    assert call(tokens=0) == 0                       # nothing to do
    assert call(tokens=-1) == -1
    assert call(tokens=600) == -1                    # more rows than the buffers hold
    assert call(world=9) == -1 and call(world=0) == -1
    assert call(base=1, local=2) == -1               # ranks beyond the group
    assert call(n=2500) == -3 and call(k=1000) == -3  # 128-wide output / 64-deep K tiles
    assert call(dtype=2) == -3                       # 16-bit inputs only
    assert call(world=3) == -3                       # TP sizes 1, 2, 4, 8
    assert call() == -1                              # null pointers


def test_row_parallel_buffer_layout(pkg):
    lib = pkg._lib.lib()
    # stream-K fix-up slots (160 CTAs x 128 rows x 256 fp32 columns, the width of
    # a CTA-pair tile) + flags, then for world > 1 partial slots
    # [world][ceil(tiles / world)] (two ranks: [2][tiles]) + result slots [tiles]
    # of 32 KB tiles + their flags
    fix = 160 * 128 * 256 * 4 + 160 * 4
    for T, n, world in ((1, 2560, 2), (512, 2560, 4), (8192, 2560, 8), (130, 1024, 1)):
        tiles = -(-T // 128) * (n // 128)
        got = lib.slokv_row_parallel_buffer_bytes(T, n, world)
        owned = tiles if world == 2 else -(-tiles // world)   # two ranks: one shot
        data = fix + ((world * owned + tiles) * 32768 if world > 1 else 0)
        flags = 4 * (world * owned + 4 * tiles) if world > 1 else 0
        assert data < got <= data + flags + 5 * 4096
        assert got % 4096 == 0
    assert lib.slokv_row_parallel_buffer_bytes(128, 2500, 2) == 0
    assert lib.slokv_row_parallel_buffer_bytes(0, 2560, 2) == 0
    assert lib.slokv_row_parallel_buffer_bytes(128, 2560, 9) == 0


def test_fp8_runs_append_and_page_widen_argument_checks(pkg):
    lib = pkg._lib.lib()
    ws_bytes = lib.slokv_kv_append_fp8_runs_workspace_bytes(100, 8)
    assert ws_bytes == 100 * 8 * 2 * 4
    assert lib.slokv_kv_append_fp8_runs_workspace_bytes(0, 8) == 0

    def runs(n=4, hd=128, ws=None, wsb=0, ptr=None):
        return lib.slokv_kv_append_fp8_runs(ptr, 1024, ptr, 1024, ptr, ptr, ptr, ptr, ptr, n, 8,
                                            hd, 256, 100, 0, ws, wsb, None, None)
    assert runs(n=0) == 0                              # nothing to do
    assert runs(n=-1) == -1
    assert runs(hd=64) == -3                           # head_dim 128 only
    assert runs() == -1                                # null pointers
    assert runs(ptr=16, ws=None) == -5                 # workspace missing
    assert runs(ptr=16, ws=256, wsb=ws_bytes - 4) == -5  # workspace too small

    def widen(rows=2, width=3, hd=128, ptr=None):
        return lib.slokv_fp8_pages_dequant(ptr, ptr, 0, 0, ptr, ptr, 100, 256, 8, hd, ptr, 4, 4,
                                           ptr, rows, width, ptr, ptr, ptr, None, None)
    assert widen(rows=0) == 0 and widen(width=0) == 0
    assert widen(rows=-1) == -1
    assert widen(hd=64) == -3
    assert widen() == -1                               # null pointers


def test_fused_fp8_prefill_argument_checks(pkg):
    lib = pkg._lib.lib()

    def call(rows=2, maxq=128, hq=32, hkv=8, hd=128, bs=256, qdt=0, ptr=None, align=16, kbs=1 << 20):
        return lib.slokv_paged_prefill_fp8(
            ptr, 32 * 128, 128, ptr, 32 * 128, 128, 256, ptr, ptr, kbs, kbs, ptr, ptr, ptr, ptr,
            rows, maxq, ptr, 16, 16, 100, bs, hq, hkv, hd, 0.1, qdt, None, 0, None, None)
    assert call(rows=0) == 0 and call(maxq=0) == 0     # nothing to do
    assert call(rows=-1) == -1
    assert call(hd=64) == -3                           # head_dim 128 only
    assert call(qdt=2) == -3                           # q/out are bf16 or f16
    assert call(hq=24, hkv=8) == -3                    # odd GQA group: two heads per CTA
    assert call(hq=30, hkv=8) == -1                    # heads not divisible
    assert call() == -1                                # null pointers
    assert call(ptr=16, bs=200) == -3                  # block size not a multiple of 128
    assert call(ptr=24) == -2                          # misaligned base
    assert call(ptr=16, kbs=1000) == -2                # block stride not a 16-byte multiple
