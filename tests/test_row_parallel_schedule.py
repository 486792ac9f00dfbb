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


# ---- the CTA-pair kernel (256 x 256 pair tiles, cta_group::2) ----------------

BM = BN = 128
FIX_FLOATS = BM * 2 * BN          # one CTA's fp32 fix-up slot (128 rows x 256 columns)
MAX_CTAS = 160
MIN_CHUNKS = 4
PAIR_MIN_MACS = 1 << 34


def pair_grid(m_tiles, n_tiles, k, per_rank):
    """The host's choice for the pair kernel (plan_grid in row_parallel.cu):
    gemm_pairs for `per_rank` CTAs (already even): stream-K over every pair,
    at least MIN_CHUNKS K chunks each."""
    pair_tiles = ((m_tiles + 1) // 2) * ((n_tiles + 1) // 2)
    return min(-(-(pair_tiles * k) // MIN_CHUNKS), per_rank // 2)


def test_pair_kernel_size_rule():
    """Pairs from 2^34 multiply-adds per call (T x N x K) with two row and two
    column tiles."""
    def pair(T, N, K):
        return -(-T // BM) >= 2 and N // BN >= 2 and T * N * K >= PAIR_MIN_MACS
    assert not pair(512, 2560, 4096) and not pair(512, 2560, 9728)    # decode batches
    assert not pair(1024, 2560, 4096) and pair(1024, 2560, 9728)
    assert pair(2048, 2560, 4096) and not pair(2048, 2560, 1024)
    assert not pair(128, 2560, 1 << 20)                                # one row tile


@pytest.mark.parametrize("tokens", [129, 256, 300, 512, 1024])
@pytest.mark.parametrize("n_tiles", [2, 3, 20])
@pytest.mark.parametrize("k", [8, 32, 64, 152, 352])
def test_pair_schedule_produces_every_output_tile_once(tokens, n_tiles, k):
    """Every 128 x 128 output tile (m < m_tiles, nt < n_tiles) is written by
    exactly one (pair, CTA position, half) of a finishing segment; padding
    halves (m or nt past the end) are never pushed; fix-up reads and writes of
    CTA position r stay inside slot 2 c + r of the contributing pair c."""
    m_tiles = -(-tokens // BM)
    pm_tiles, pn_tiles = (m_tiles + 1) // 2, (n_tiles + 1) // 2
    for sms, local_ranks in ((148, 1), (148, 4), (140, 8)):
        per_rank = min(sms // local_ranks, MAX_CTAS) & ~1
        G = pair_grid(m_tiles, n_tiles, k, per_rank)
        assert 2 * G <= per_rank and G >= 1
        U = pm_tiles * pn_tiles * k
        written = {}
        for pair in range(per_rank // 2):
            for t, a, b in sched(pair, G, U, k):
                if b < k:
                    continue                            # contributing segment: fix-up only
                preds = predecessors(pair, t, G, U, k) if a > 0 else []
                for r in (0, 1):
                    for c in preds:
                        slot = 2 * c + r
                        assert 0 <= slot < per_rank
                    pm, pn = divmod(t, pn_tiles)
                    m = 2 * pm + r
                    if m >= m_tiles:
                        continue
                    for h in (0, 1):
                        nt = 2 * pn + h
                        if nt >= n_tiles:
                            continue
                        assert (m, nt) not in written
                        written[(m, nt)] = (pair, r, h)
        assert set(written) == {(m, nt) for m in range(m_tiles) for nt in range(n_tiles)}
    # the largest fix-up float a thread touches: float4 group 8 q + c = 63 of row
    # 127 (groups of 128 rows, 4 floats each)
    assert ((7 * 8 + 7) * BM + 127) * 4 + 3 < FIX_FLOATS
