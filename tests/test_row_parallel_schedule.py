"""The stream-K work split of the fused row-parallel kernel, restated on the CPU
and checked exhaustively over decode- and prefill-sized shapes.

Restates `make_sched` / `Sched::get` / the predecessor scan of
slo-aware-llm-serving-engine_b200/csrc/row_parallel.cu (CTA c owns chunk units
[c*U/G, (c+1)*U/G) of U = tiles * k_chunks, cut into per-tile segments; a first
segment that continues a tile begun by earlier CTAs is processed last).  The
invariants the kernel relies on:
  * every (tile, K chunk) is computed by exactly one CTA;
  * every tile has exactly one finishing segment (the one holding its last
    chunk), and the CTAs whose fix-up sums it adds -- the scan down from c - 1
    to the CTA holding the tile's first chunk -- are exactly the CTAs with a
    contributing (unfinished) segment of that tile;
  * a CTA has at most one contributing segment, and processes it before its
    own finishing segment, so the fix-up waits form no cycle.
"""
import pytest


def unit_begin(c, G, U):
    return c * U // G


def sched(c, G, U, k):
    if c >= G:                                   # CTAs past the GEMM count: no work
        return []
    beg, end = unit_begin(c, G, U), unit_begin(c + 1, G, U)
    if end <= beg:
        return []
    t0 = beg // k
    n = (end - 1) // k - t0 + 1
    defer = n > 1 and beg > t0 * k
    out = []
    for i in range(n):
        j = (i + 1) % n if defer else i
        kc0 = beg - t0 * k if j == 0 else 0
        kc1 = end - (t0 + n - 1) * k if j == n - 1 else k
        out.append((t0 + j, kc0, kc1))
    return out


def predecessors(c, tile, G, U, k):
    fp = c - 1
    while unit_begin(fp, G, U) > tile * k:
        fp -= 1
    return list(range(fp, c))


@pytest.mark.parametrize("tiles", [1, 5, 20, 40, 80, 160, 1280])
@pytest.mark.parametrize("k", [8, 16, 19, 32, 38, 76, 152])
def test_stream_k_schedule_invariants(tiles, k):
    U = tiles * k
    for per_rank in (18, 37, 74, 148):
        G = min(per_rank, -(-U // 4))            # at least 4 K chunks per CTA
        cover, finish, contrib = {}, {}, {}
        for c in range(G + 2):                   # (two idle CTAs beyond G)
            segs = sched(c, G, U, k)
            assert c < G or not segs
            for t, a, b in segs:
                assert 0 <= a < b <= k
                for kc in range(a, b):
                    assert (t, kc) not in cover
                    cover[(t, kc)] = c
                if b == k:
                    assert t not in finish
                    finish[t] = (c, a)
                else:
                    contrib.setdefault(t, []).append(c)
            assert sum(1 for s in segs if s[2] < k) <= 1
        assert len(cover) == U
        assert set(finish) == set(range(tiles))
        for t, (c, a) in finish.items():
            preds = predecessors(c, t, G, U, k) if a > 0 else []
            assert preds == sorted(contrib.get(t, []))
            if a > 0:
                assert sched(c, G, U, k)[-1][0] == t          # finishing segment last
            for pc in preds:
                segs = sched(pc, G, U, k)
                ci = next(i for i, s in enumerate(segs) if s[2] < k)
                fi = [i for i, s in enumerate(segs) if s[2] == k and s[1] > 0]
                assert not fi or ci < fi[0]                   # publishes before it waits
