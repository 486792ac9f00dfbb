// Paged GQA decode attention for sm_100a.
//
// Replaces flash_attn_with_kvcache as called by the reference engine
// (nanovllm/layers/attention.py:75-78 and nanovllm/layers/mixed_attention.py:117-121):
// one query token per sequence, K/V gathered from the paged pool through
// block_tables, cache_seqlens already counting the token appended this step.
//
// Design (B200-first, HBM-bound):
//  * Persistent grid: one CTA per SM, 4 autonomous warps per CTA.  The work is
//    the list of 32-token tiles of every (sequence, kv-head) segment, ordered
//    (b, kv_head, tile).  Warp slot s of S processes the contiguous range
//    [s*T/S, (s+1)*T/S) of the T tiles, so every warp streams the same number of
//    bytes whatever the mix of context lengths (balanced split-K, a.k.a.
//    flash-decoding with stream-K partitioning).
//  * Each warp owns a 3-stage ring of 16 KB stages in shared memory.  Lane 0
//    issues TMA tensor loads (4-D map over [block, token, kv_head, dim], 128-byte
//    swizzle, evict-first L2 policy) of the K and V tile two stages ahead and
//    the warp waits on the stage's mbarrier (bounded by a time limit).
//  * QK^T and PV run on the warp-level tensor-core MMA (m16n8k16, fp32
//    accumulate): the G query heads that share a KV head are the M rows, so the
//    K/V tile is read from shared memory once for all of them.  The online
//    softmax is kept in registers per row and reduced with quad shuffles.
//  * A segment that lies inside one warp's range is finalised in place; a
//    segment that straddles warp ranges leaves (m, l, acc) partials in the
//    workspace, which a small merge kernel combines.  At most two partials per
//    warp exist, so the workspace does not depend on batch or context length.
#include "common.cuh"
#include "fp8_e4m3.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

namespace slokv {
namespace decode {

constexpr int kD = 128;                         // head_dim
constexpr int kTile = 32;                       // tokens per pipeline stage
constexpr int kHalfBytes = kTile * 128;         // 32 rows x 64 dims x 2 B
constexpr int kStageBytes = 4 * kHalfBytes;     // K lo/hi + V lo/hi halves
constexpr int kRingBytes = 192 * 1024;          // K/V stages of all warps of a CTA
constexpr int kRowFloats = kD + 4;              // partial row: m, l, pad, pad, acc[kD]
constexpr int kAccOff = 4;                      // acc starts 16-byte aligned
constexpr int kMaxBatch = 8192;

struct Params {
  void *out;
  int64_t out_sb, out_sh;
  const void *q;
  int64_t q_sb, q_sh;
  const int32_t *block_tables;
  int64_t bt_stride;
  int32_t max_blocks;
  const int32_t *context_lens;
  int32_t batch;
  int32_t num_blocks, block_size, hkv, group;
  float scale_log2;
  const float *k_scale;  // FP8 cache only: [num_blocks, hkv] fp32
  const float *v_scale;
  float *partials;  // [nslots][2][group][kRowFloats]
  int4 *jobs;       // [nslots]: merge job of the warp slot (x = -1: none)
  uint32_t *err;
  int32_t nslots;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Number of tiles of sequence b (its segment length per kv head).
__device__ __forceinline__ int32_t seq_tiles(const Params &p, int b, uint32_t *err_bits) {
  int32_t len = __ldg(p.context_lens + b);
  if (len <= 0) return 0;
  const int32_t cap = p.max_blocks * p.block_size;
  if (len > cap) {
    *err_bits |= SLOKV_DEVERR_CONTEXT_LEN;
    len = cap;
  }
  return (len + kTile - 1) / kTile;
}

__device__ __forceinline__ int32_t seq_len_clamped(const Params &p, int b) {
  int32_t len = __ldg(p.context_lens + b);
  const int32_t cap = p.max_blocks * p.block_size;
  return len > cap ? cap : len;
}

// Exclusive prefix over sequences of (tiles_b * hkv) into prefix[0..batch].
// Called by all threads of the CTA.
__device__ void build_prefix(const Params &p, int32_t *prefix, uint32_t *err_bits) {
  __shared__ int32_t warp_sums[32];
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int per = (p.batch + nthr - 1) / nthr;
  const int lo = min(tid * per, p.batch), hi = min(lo + per, p.batch);
  int32_t local = 0;
  for (int b = lo; b < hi; ++b) local += seq_tiles(p, b, err_bits) * p.hkv;
  // inclusive scan of `local` across the CTA
  const int lane = tid & 31, warp = tid >> 5;
  int32_t v = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int32_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = nthr >> 5;
    int32_t w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < nw) warp_sums[lane] = w;
  }
  __syncthreads();
  int32_t run = v - local + (warp > 0 ? warp_sums[warp - 1] : 0);
  for (int b = lo; b < hi; ++b) {
    prefix[b] = run;
    uint32_t dummy = 0;
    run += seq_tiles(p, b, &dummy) * p.hkv;
  }
  if (tid == nthr - 1) prefix[p.batch] = run;
  __syncthreads();
}

struct TileRef {
  int32_t b, h, j, nt, seg_start;
};

// Locate global tile t: largest b with prefix[b] <= t.
__device__ __forceinline__ TileRef locate(const Params &p, const int32_t *prefix, int64_t t) {
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  TileRef r;
  r.b = lo;
  r.nt = (prefix[lo + 1] - prefix[lo]) / p.hkv;
  const int32_t rel = static_cast<int32_t>(t - prefix[lo]);
  r.h = rel / r.nt;
  r.j = rel - r.h * r.nt;
  r.seg_start = prefix[lo] + r.h * r.nt;
  return r;
}

__device__ __forceinline__ int64_t range_start(int64_t s, int64_t total, int64_t nslots) {
  return (s * total) / nslots;
}

// Slot that owns global tile t (max s with range_start(s) <= t).
__device__ __forceinline__ int64_t owner_slot(int64_t t, int64_t total, int64_t nslots) {
  int64_t s = (t * nslots) / total;
  if (s >= nslots) s = nslots - 1;
  while (s + 1 < nslots && range_start(s + 1, total, nslots) <= t) ++s;
  while (s > 0 && range_start(s, total, nslots) > t) --s;
  return s;
}

// The next tile a warp's producer lane issues, advanced tile by tile in the
// work-list order (segment (b, h) after segment, tiles in order) so the issue
// path needs no search; the page's block id is read once per page.
struct IssueCursor {
  int32_t b, h, j, nt, page, blk;
};

__device__ __forceinline__ void cursor_init(IssueCursor &c, const Params &p,
                                            const int32_t *prefix, int64_t t) {
  const TileRef r = locate(p, prefix, t);
  c.b = r.b;
  c.h = r.h;
  c.j = r.j;
  c.nt = r.nt;
  c.page = -1;
  c.blk = 0;
}

// Step to the following tile; call only when one exists (it then lies in a
// later non-empty sequence at worst, so b stays below batch).
__device__ __forceinline__ void cursor_next(IssueCursor &c, const Params &p,
                                            const int32_t *prefix) {
  if (++c.j < c.nt) return;
  c.j = 0;
  c.page = -1;
  if (++c.h < p.hkv) return;
  c.h = 0;
  do {
    ++c.b;
    c.nt = (prefix[c.b + 1] - prefix[c.b]) / p.hkv;
  } while (c.nt == 0 && c.b + 1 < p.batch);
}

// Issue the TMA loads of the cursor's tile into `stage` of this warp's ring.
template <bool kFp8>
__device__ __forceinline__ void issue_cursor_tile(const Params &p, IssueCursor &c,
                                                  const CUtensorMap *kmap,
                                                  const CUtensorMap *vmap, uint32_t ring,
                                                  uint32_t bars, int stage, uint64_t policy) {
  const int tiles_per_block = p.block_size / kTile;
  const int page = c.j / tiles_per_block;
  if (page != c.page) {
    c.page = page;
    c.blk = __ldg(p.block_tables + static_cast<int64_t>(c.b) * p.bt_stride + page);
    if (c.blk < 0 || c.blk >= p.num_blocks) record_error(p.err, SLOKV_DEVERR_BLOCK_RANGE);
  }
  const int off = (c.j - page * tiles_per_block) * kTile;
  // Out-of-range block ids load as zeros (TMA bounds fill); never a fault.
  const uint32_t bar = bars + stage * 8;
  fence_proxy_async_smem();
  if constexpr (kFp8) {
    const uint32_t dst = ring + stage * (2 * kTile * 128);
    mbar_arrive_expect_tx(bar, 2 * kTile * 128);
    tma_load_4d(dst, kmap, bar, 0, c.h, off, c.blk, policy);
    tma_load_4d(dst + kTile * 128, vmap, bar, 0, c.h, off, c.blk, policy);
  } else {
    const uint32_t dst = ring + stage * kStageBytes;
    mbar_arrive_expect_tx(bar, kStageBytes);
    tma_load_4d(dst + 0 * kHalfBytes, kmap, bar, 0, c.h, off, c.blk, policy);
    tma_load_4d(dst + 1 * kHalfBytes, kmap, bar, 64, c.h, off, c.blk, policy);
    tma_load_4d(dst + 2 * kHalfBytes, vmap, bar, 0, c.h, off, c.blk, policy);
    tma_load_4d(dst + 3 * kHalfBytes, vmap, bar, 64, c.h, off, c.blk, policy);
  }
}

// Shared-memory ring geometry of the two cache formats.  Both use 192 KiB of
// ring: bf16/f16 tiles are 16 KiB (K and V, two 64-dim halves each), FP8 tiles
// are 8 KiB, so the FP8 variant runs twice as many warps per SM.
template <bool kFp8>
struct Ring {
  // bf16: 3 warps x 4 stages measured 1.6 % faster than 4 x 3 (deeper ring per
  // warp); FP8 is issue-bound and needs its 8 warps (6 x 4 measured 29 % slower).
  static constexpr int kWarpsPerCta = kFp8 ? 8 : 3;
  static constexpr int kStages = kFp8 ? 3 : 4;                       // ring depth per warp
  static constexpr int kStage = kFp8 ? 2 * kTile * 128 : kStageBytes;
  static constexpr int kVOff = kFp8 ? kTile * 128 : 2 * kHalfBytes;  // V offset in a stage
  static constexpr int kBytes = kWarpsPerCta * kStages * kStage;
};
static_assert(Ring<true>::kBytes == kRingBytes && Ring<false>::kBytes == kRingBytes, "ring");

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// Both byte pairs of a 32-bit word of E4M3 codes -> two f16x2 (low byte of a
// pair -> low half).
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t word(const uint4 &w, int i) {
  return i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w;
}

// Output dims of accumulator elements (n-tile n, quad c): bf16/f16 n-tile n
// holds dims [8n, 8n+8), so the pair (c0, c1) is dims 8n+2c, 8n+2c+1.  FP8:
// the V fragments of n-tile n take dim 16*g + n for B column g, so c0 / c1 are
// dims 32c + n and 32c + 16 + n.
template <bool kFp8>
__device__ __forceinline__ int out_dim0(int n, int c) {
  return kFp8 ? 32 * c + n : 8 * n + 2 * c;
}
template <bool kFp8>
__device__ __forceinline__ int out_dim1(int n, int c) {
  return kFp8 ? 32 * c + 16 + n : 8 * n + 2 * c + 1;
}

template <typename T, bool kFp8>
__global__ void __launch_bounds__(Ring<kFp8>::kWarpsPerCta * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p) {
  using R = Ring<kFp8>;
  using MQ = Mma<typename std::conditional<kFp8, __half, T>::type>;  // MMA input type
  using MO = Mma<T>;                                                  // output type
  constexpr int kW = R::kWarpsPerCta;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t *base_ptr = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t bars_all = base + kRingBytes;
  int32_t *prefix = reinterpret_cast<int32_t *>(base_ptr + kRingBytes + kW * R::kStages * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  if (lane == 0) {
    for (int i = 0; i < R::kStages; ++i) mbar_init(bars_all + (warp * R::kStages + i) * 8, 1);
    fence_barrier_init();
  }
  uint32_t err_bits = 0;
  build_prefix(p, prefix, &err_bits);  // contains __syncthreads
  if (err_bits && threadIdx.x == 0) record_error(p.err, err_bits);

  const int64_t total = prefix[p.batch];
  const int G = p.group;

  // Sequences with no context (graph padding rows) produce zeros; nothing else
  // touches their output rows.
  for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
    if (prefix[b + 1] != prefix[b]) continue;
    T *ob = static_cast<T *>(p.out) + static_cast<int64_t>(b) * p.out_sb;
    const int pairs = kD / 2;
    for (int i = threadIdx.x; i < p.hkv * G * pairs; i += blockDim.x) {
      const int row = i / pairs, pr = i - row * pairs;
      *reinterpret_cast<uint32_t *>(ob + row * p.out_sh + 2 * pr) = 0u;
    }
  }

  const int64_t s = static_cast<int64_t>(blockIdx.x) * kW + warp;
  const int64_t a = range_start(s, total, p.nslots);
  const int64_t e = range_start(s + 1, total, p.nslots);
  // The merge job of this warp slot: the segment whose last piece this warp
  // holds while earlier pieces sit in other slots.  Rewritten on every call.
  int4 job = make_int4(-1, 0, 0, 0);
  if (a >= e) {
    if (lane == 0) p.jobs[s] = job;
    return;
  }

  const uint32_t ring = base + warp * R::kStages * R::kStage;
  const uint32_t bars = bars_all + warp * R::kStages * 8;
  const uint64_t policy = l2_evict_first_policy();
  const int tiles_per_block = p.block_size / kTile;

  IssueCursor cur;                        // lane 0: next tile to issue (a + issued)
  int64_t issued = 0;
  if (lane == 0) {
    cursor_init(cur, p, prefix, a);
    for (; issued < R::kStages && a + issued < e; ++issued) {
      issue_cursor_tile<kFp8>(p, cur, &kmap, &vmap, ring, bars, static_cast<int>(issued), policy);
      if (a + issued + 1 < e) cursor_next(cur, p, prefix);
    }
  }
  __syncwarp();

  int64_t t = a;
  while (t < e) {
    const TileRef r = locate(p, prefix, t);
    const int64_t seg_end = static_cast<int64_t>(r.seg_start) + r.nt;
    const int64_t piece_end = seg_end < e ? seg_end : e;
    const int32_t len = seq_len_clamped(p, r.b);

    // Q fragments (A operand) for the G heads of kv head r.h; rows >= G are 0.
    uint32_t qa[8][4];
    {
      const T *qb = static_cast<const T *>(p.q) + static_cast<int64_t>(r.b) * p.q_sb +
                    static_cast<int64_t>(r.h * G) * p.q_sh;
      const bool r0 = g < G, r1 = g + 8 < G;
      if constexpr (!kFp8) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int d0 = ks * 16 + 2 * c;
          qa[ks][0] = r0 ? *reinterpret_cast<const uint32_t *>(qb + g * p.q_sh + d0) : 0u;
          qa[ks][1] = r1 ? *reinterpret_cast<const uint32_t *>(qb + (g + 8) * p.q_sh + d0) : 0u;
          qa[ks][2] = r0 ? *reinterpret_cast<const uint32_t *>(qb + g * p.q_sh + d0 + 8) : 0u;
          qa[ks][3] = r1 ? *reinterpret_cast<const uint32_t *>(qb + (g + 8) * p.q_sh + d0 + 8) : 0u;
        }
      } else {
        // f16 fragments in the dim order of the FP8 K fragments: k-step
        // 4*gi + tq takes dims 64*gi + 16*c + 4*tq + {0,1} (k = 2c, 2c+1) and
        // + {2,3} (k = 2c+8, 2c+9).
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int d0 = 64 * (ks >> 2) + 16 * c + 4 * (ks & 3);
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (r0) {
            w[0] = *reinterpret_cast<const uint32_t *>(qb + g * p.q_sh + d0);
            w[1] = *reinterpret_cast<const uint32_t *>(qb + g * p.q_sh + d0 + 2);
          }
          if (r1) {
            w[2] = *reinterpret_cast<const uint32_t *>(qb + (g + 8) * p.q_sh + d0);
            w[3] = *reinterpret_cast<const uint32_t *>(qb + (g + 8) * p.q_sh + d0 + 2);
          }
          const float2 f0 = MO::unpack(w[0]), f1 = MO::unpack(w[1]);
          const float2 f2 = MO::unpack(w[2]), f3 = MO::unpack(w[3]);
          qa[ks][0] = MQ::pack(f0.x, f0.y);
          qa[ks][2] = MQ::pack(f1.x, f1.y);
          qa[ks][1] = MQ::pack(f2.x, f2.y);
          qa[ks][3] = MQ::pack(f3.x, f3.y);
        }
      }
    }
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float vs_cur = 1.f;  // FP8: o is kept in units of this page's V scale
    float ks_tile = 1.f, vs_tile = 1.f;
    int scale_page = -1;

    for (int64_t tt = t; tt < piece_end; ++tt) {
      const int64_t idx = tt - a;
      const int stage = static_cast<int>(idx % R::kStages);
      const uint32_t parity = static_cast<uint32_t>((idx / R::kStages) & 1);
      const int j = static_cast<int>(tt - r.seg_start);
      if constexpr (kFp8) {
        const int page = j / tiles_per_block;
        if (page != scale_page) {          // scales change per page (8 tiles)
          scale_page = page;
          const int32_t blk =
              __ldg(p.block_tables + static_cast<int64_t>(r.b) * p.bt_stride + page);
          if (blk >= 0 && blk < p.num_blocks) {
            const int64_t si = static_cast<int64_t>(blk) * p.hkv + r.h;
            ks_tile = __ldg(p.k_scale + si);
            vs_tile = __ldg(p.v_scale + si);
          } else {
            ks_tile = 0.f;
            vs_tile = 0.f;
          }
          if (!(vs_tile > 0.f)) vs_tile = 1.f;  // an all-zero page: any unit works
        }
      }
      if (!mbar_wait(bars + stage * 8, parity)) {
        if (lane == 0) record_error(p.err, SLOKV_DEVERR_TIMEOUT);
        return;
      }
      const int valid = min(kTile, len - j * kTile);
      const uint32_t kb = ring + stage * R::kStage;
      const uint32_t vb = kb + R::kVOff;
      if (valid < kTile) {
        // Rows past the context hold stale pool bytes (possibly NaN); zero the
        // V rows so that P = 0 really contributes nothing.
        uint8_t *vrow = base_ptr + (vb - base);
        if constexpr (!kFp8) {
          for (int i = lane; i < (kTile - valid) * 16; i += 32) {
            const int row = valid + (i >> 4), part = i & 15;
            const int half = part >> 3, chunk = part & 7;
            *reinterpret_cast<int4 *>(vrow + half * kHalfBytes + row * 128 + chunk * 16) =
                make_int4(0, 0, 0, 0);
          }
        } else {
          for (int i = lane; i < (kTile - valid) * 8; i += 32) {
            const int row = valid + (i >> 3), chunk = i & 7;
            *reinterpret_cast<int4 *>(vrow + row * 128 + chunk * 16) = make_int4(0, 0, 0, 0);
          }
        }
        __syncwarp();
      }

      // ---- S = Q K^T  (16 rows x 32 tokens) ----
      float sc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      if constexpr (!kFp8) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const int row = nt * 8 + (lane & 7);
            const int chunk = kk * 4 + (lane >> 3);
            const uint32_t addr = kb + (chunk >> 3) * kHalfBytes + swz128(row, chunk & 7);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(b0, b1, b2, b3, addr);
            MQ::run(sc[nt], qa[2 * kk], b0, b1);
            MQ::run(sc[nt], qa[2 * kk + 1], b2, b3);
          }
        }
      } else {
        // Lane (g, c) reads 16-byte chunks c (dims 16c..) and c + 4 (dims
        // 64 + 16c..) of token row 8*nt + g: word t of a chunk feeds k-step
        // 4*gi + t (see the Q fragment order above).
        uint4 w0[4], w1[4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          w0[nt] = lds128(kb + swz128(nt * 8 + g, c));
          w1[nt] = lds128(kb + swz128(nt * 8 + g, c + 4));
        }
        // Two accumulator sets (dims 0-63 and 64-127), summed after: eight
        // dependent MMA chains of four instead of four of eight.
        float sc2[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) sc2[nt][0] = sc2[nt][1] = sc2[nt][2] = sc2[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            uint32_t b0, b1, b2, b3;
            e4m3x4_to_f16x2x2(word(w0[nt], ks), b0, b1);
            e4m3x4_to_f16x2x2(word(w1[nt], ks), b2, b3);
            MQ::run(sc[nt], qa[ks], b0, b1);
            MQ::run(sc2[nt], qa[ks + 4], b2, b3);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) sc[nt][e2] += sc2[nt][e2];
      }

      // ---- online softmax (log2 domain) ----
      const float sl = kFp8 ? ks_tile * p.scale_log2 : p.scale_log2;
      float mx0 = -INFINITY, mx1 = -INFINITY;
      // Unmasked fast path for full tiles: measured faster for the FP8 tile,
      // slower for the bf16 one (longer loop body), so bf16 always masks.
      if (kFp8 && valid == kTile) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            sc[nt][e2] *= sl;
            sc[nt][2 + e2] *= sl;
            mx0 = fmaxf(mx0, sc[nt][e2]);
            mx1 = fmaxf(mx1, sc[nt][2 + e2]);
          }
        }
      } else {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int tok = nt * 8 + 2 * c + e2;
            const bool ok = tok < valid;
            sc[nt][e2] = ok ? sc[nt][e2] * sl : -INFINITY;
            sc[nt][2 + e2] = ok ? sc[nt][2 + e2] * sl : -INFINITY;
            mx0 = fmaxf(mx0, sc[nt][e2]);
            mx1 = fmaxf(mx1, sc[nt][2 + e2]);
          }
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
      const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = fast_exp2(m0 - mu0), al1 = fast_exp2(m1 - mu1);
      m0 = mn0;
      m1 = mn1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        sc[nt][0] = fast_exp2(sc[nt][0] - mu0);
        sc[nt][1] = fast_exp2(sc[nt][1] - mu0);
        sc[nt][2] = fast_exp2(sc[nt][2] - mu1);
        sc[nt][3] = fast_exp2(sc[nt][3] - mu1);
        rs0 += sc[nt][0] + sc[nt][1];
        rs1 += sc[nt][2] + sc[nt][3];
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      float oa0 = al0, oa1 = al1;
      if constexpr (kFp8) {
        // Re-express o in units of this tile's V scale (1 when it is unchanged).
        const float ratio = tt == t ? 1.f : vs_cur / vs_tile;
        oa0 *= ratio;
        oa1 *= ratio;
        vs_cur = vs_tile;
      }
      // FP8: rescale the accumulators only when some row's running max or the V
      // unit moved (it settles after a few tiles).  The vote costs the bf16
      // tile more than the multiplies it saves (measured), so bf16 always does them.
      if (!kFp8 || (tt != t && __any_sync(0xffffffffu, oa0 != 1.f || oa1 != 1.f))) {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][0] *= oa0;
          o[n][1] *= oa0;
          o[n][2] *= oa1;
          o[n][3] *= oa1;
        }
      }
      uint32_t pa[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        pa[i][0] = MQ::pack(sc[2 * i][0], sc[2 * i][1]);
        pa[i][1] = MQ::pack(sc[2 * i][2], sc[2 * i][3]);
        pa[i][2] = MQ::pack(sc[2 * i + 1][0], sc[2 * i + 1][1]);
        pa[i][3] = MQ::pack(sc[2 * i + 1][2], sc[2 * i + 1][3]);
      }

      // ---- O += P V ----
      if constexpr (!kFp8) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
          for (int np = 0; np < 8; ++np) {
            const int row = i * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int chunk = np * 2 + (lane >> 4);
            const uint32_t addr = vb + (chunk >> 3) * kHalfBytes + swz128(row, chunk & 7);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(b0, b1, b2, b3, addr);
            MQ::run(o[2 * np], pa[i], b0, b1);
            MQ::run(o[2 * np + 1], pa[i], b2, b3);
          }
        }
      } else {
        // B fragment of n-tile n for lane (g, c): V[tokens 2c, 2c+1 | 2c+8,
        // 2c+9][dim 16g + n].  The lane loads chunk g (dims 16g..16g+15) of those
        // four token rows -- rows with different swizzle phases, so the loads
        // are conflict-free -- and prmt pairs the two tokens' codes of a dim
        // before one cvt makes the f16x2 register.
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r0 = 16 * i + 2 * c;
          const uint4 a0 = lds128(vb + swz128(r0, g)), a1 = lds128(vb + swz128(r0 + 1, g));
          const uint4 a8 = lds128(vb + swz128(r0 + 8, g)), a9 = lds128(vb + swz128(r0 + 9, g));
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t lo01 = prmt(word(a0, wi), word(a1, wi), 0x5140u);  // dims 4wi, 4wi+1
            const uint32_t hi01 = prmt(word(a0, wi), word(a1, wi), 0x7362u);  // dims 4wi+2, +3
            const uint32_t lo89 = prmt(word(a8, wi), word(a9, wi), 0x5140u);
            const uint32_t hi89 = prmt(word(a8, wi), word(a9, wi), 0x7362u);
            uint32_t b[4][2];
            e4m3x4_to_f16x2x2(lo01, b[0][0], b[1][0]);
            e4m3x4_to_f16x2x2(hi01, b[2][0], b[3][0]);
            e4m3x4_to_f16x2x2(lo89, b[0][1], b[1][1]);
            e4m3x4_to_f16x2x2(hi89, b[2][1], b[3][1]);
#pragma unroll
            for (int e = 0; e < 4; ++e) MQ::run(o[4 * wi + e], pa[i], b[e][0], b[e][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0 && tt + R::kStages < e) {
        issue_cursor_tile<kFp8>(p, cur, &kmap, &vmap, ring, bars, stage, policy);
        if (tt + R::kStages + 1 < e) cursor_next(cur, p, prefix);
      }
    }

    // ---- finish the piece ----
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const bool whole = (t == r.seg_start) && (piece_end == seg_end);
    if (whole) {
      const float inv0 = l0 > 0.f ? vs_cur / l0 : 0.f;
      const float inv1 = l1 > 0.f ? vs_cur / l1 : 0.f;
      T *ob = static_cast<T *>(p.out) + static_cast<int64_t>(r.b) * p.out_sb +
              static_cast<int64_t>(r.h * G) * p.out_sh;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        if constexpr (!kFp8) {
          const int d = out_dim0<false>(n, c);
          if (g < G)
            *reinterpret_cast<uint32_t *>(ob + g * p.out_sh + d) =
                MO::pack(o[n][0] * inv0, o[n][1] * inv0);
          if (g + 8 < G)
            *reinterpret_cast<uint32_t *>(ob + (g + 8) * p.out_sh + d) =
                MO::pack(o[n][2] * inv1, o[n][3] * inv1);
        } else {
          const int d0 = out_dim0<true>(n, c), d1 = out_dim1<true>(n, c);
          const uint32_t v0 = MO::pack(o[n][0] * inv0, o[n][1] * inv0);
          const uint32_t v1 = MO::pack(o[n][2] * inv1, o[n][3] * inv1);
          if (g < G) {
            reinterpret_cast<uint16_t *>(ob + g * p.out_sh + d0)[0] = static_cast<uint16_t>(v0);
            reinterpret_cast<uint16_t *>(ob + g * p.out_sh + d1)[0] = static_cast<uint16_t>(v0 >> 16);
          }
          if (g + 8 < G) {
            reinterpret_cast<uint16_t *>(ob + (g + 8) * p.out_sh + d0)[0] = static_cast<uint16_t>(v1);
            reinterpret_cast<uint16_t *>(ob + (g + 8) * p.out_sh + d1)[0] = static_cast<uint16_t>(v1 >> 16);
          }
        }
      }
    } else {
      const int slot_idx = (t == a && t > r.seg_start) ? 0 : 1;
      if (slot_idx == 0 && piece_end == seg_end)
        job = make_int4(r.b, r.h, static_cast<int>(owner_slot(r.seg_start, total, p.nslots)),
                        static_cast<int>(total));
      float *pb = p.partials + ((s * 2 + slot_idx) * G) * static_cast<int64_t>(kRowFloats);
      const float mu0 = m0 == -INFINITY ? 0.f : m0;
      const float mu1 = m1 == -INFINITY ? 0.f : m1;
      if (g < G) {
        float *row = pb + g * kRowFloats;
        if (c == 0) {
          row[0] = mu0;
          row[1] = l0;
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          row[kAccOff + out_dim0<kFp8>(n, c)] = o[n][0] * vs_cur;
          row[kAccOff + out_dim1<kFp8>(n, c)] = o[n][1] * vs_cur;
        }
      }
      if (g + 8 < G) {
        float *row = pb + (g + 8) * kRowFloats;
        if (c == 0) {
          row[0] = mu1;
          row[1] = l1;
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          row[kAccOff + out_dim0<kFp8>(n, c)] = o[n][2] * vs_cur;
          row[kAccOff + out_dim1<kFp8>(n, c)] = o[n][3] * vs_cur;
        }
      }
    }
    t = piece_end;
  }
  if (lane == 0) p.jobs[s] = job;
}

// Combine the partials of every segment that straddles warp ranges.  One CTA
// per warp slot of the main kernel; the slot's job names the segment whose
// last piece it holds (pieces: slot s_lo's tail partial, then the head partial
// of every non-empty slot up to this one).  Warp w merges query-head rows w,
// w + 4, ... in one pass with a running max, so each piece costs one round of
// independent loads; lane l owns dims [4l, 4l+4).
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_merge_kernel(const Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t s = blockIdx.x;
  if (s >= p.nslots) return;
  const int4 job = p.jobs[s];
  if (job.x < 0) return;
  const int G = p.group;
  const int64_t total = job.w, s_lo = job.z;
  for (int row = warp; row < G; row += 4) {
    float m = -INFINITY, l = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t t = s_lo; t <= s; ++t) {
      if (t > s_lo && range_start(t + 1, total, p.nslots) == range_start(t, total, p.nslots))
        continue;
      const float *pr = p.partials + ((t * 2 + (t == s_lo ? 1 : 0)) * G + row) *
                                         static_cast<int64_t>(kRowFloats);
      const float mt = pr[0], lt = pr[1];
      const float4 v = *reinterpret_cast<const float4 *>(pr + kAccOff + lane * 4);
      const float mn = fmaxf(m, mt);
      const float a = m == -INFINITY ? 0.f : fast_exp2(m - mn);
      const float b = mt == -INFINITY ? 0.f : fast_exp2(mt - mn);
      l = l * a + lt * b;
      acc[0] = acc[0] * a + v.x * b;
      acc[1] = acc[1] * a + v.y * b;
      acc[2] = acc[2] * a + v.z * b;
      acc[3] = acc[3] * a + v.w * b;
      m = mn;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T *ob = static_cast<T *>(p.out) + static_cast<int64_t>(job.x) * p.out_sb +
            static_cast<int64_t>(job.y * G + row) * p.out_sh + lane * 4;
    *reinterpret_cast<uint2 *>(ob) = make_uint2(Mma<T>::pack(acc[0] * inv, acc[1] * inv),
                                                Mma<T>::pack(acc[2] * inv, acc[3] * inv));
  }
}

// ---- host side -------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int device_sms(int dev) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return -1;
  return n;
}

bool encode_cache_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int elem_bytes,
                      int64_t block_stride, int num_blocks, int block_size, int hkv) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(hkv),
                        static_cast<cuuint64_t>(block_size), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD) * elem_bytes,
                           static_cast<cuuint64_t>(kD) * hkv * elem_bytes,
                           static_cast<cuuint64_t>(block_stride) * elem_bytes};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / elem_bytes), 1, kTile, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // Promote L2 fills only up to the size of one head's row (256 B bf16, 128 B
  // FP8): a wider fill would drag in a neighbouring head's row that another
  // warp streams much later (it is evicted first), doubling DRAM reads.
  CUresult r = fn(map, dt, 4, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  elem_bytes == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                  : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

size_t partial_bytes_for(int sms, int group, int warps = Ring<false>::kWarpsPerCta) {
  return static_cast<size_t>(sms) * warps * 2 * group * kRowFloats * sizeof(float);
}

// Workspace of the decode (default: the bf16/f16 warp slots per SM).
size_t workspace_bytes_for(int sms, int group, int warps = Ring<false>::kWarpsPerCta) {
  return partial_bytes_for(sms, group, warps) + static_cast<size_t>(sms) * warps * sizeof(int4);
}

template <typename T, bool kFp8>
int launch(const Params &p0, const CUtensorMap &km, const CUtensorMap &vm, int sms,
           cudaStream_t stream) {
  constexpr int kW = Ring<kFp8>::kWarpsPerCta;
  const size_t smem = 1024 + kRingBytes + kW * Ring<kFp8>::kStages * 8 +
                      static_cast<size_t>(p0.batch + 1) * sizeof(int32_t);
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(paged_decode_kernel<T, kFp8>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              1024 + kRingBytes + kW * Ring<kFp8>::kStages * 8 +
                                  (kMaxBatch + 1) * sizeof(int32_t)) == cudaSuccess;
  });
  if (!ok) return SLOKV_ERR_CUDA;
  paged_decode_kernel<T, kFp8><<<sms, kW * 32, smem, stream>>>(km, vm, p0);
  if (cudaGetLastError() != cudaSuccess) return SLOKV_ERR_CUDA;
  paged_decode_merge_kernel<T><<<p0.nslots, 128, 0, stream>>>(p0);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

// ---- fp32 pool: the reference's fp32 configuration --------------------------
//
// q, cache and out in fp32 (the reference engine's fp32 diagnostic runs its
// whole model, pool included, in fp32).  CUDA-core arithmetic, one CTA per
// (sequence, KV head) and its G query heads: every K/V row is read once for
// the group.  Keys go in chunks of 256: thread t scores key t of the chunk for
// all G heads (its 128-float K row against the group's q in shared memory),
// each head's chunk max and exponentials update an online softmax, and thread
// d accumulates output dim d over the chunk's V rows (coalesced 512-byte row
// reads).  A parity path: HBM traffic is the rows' K and V once; no TMA, no
// workspace.
namespace f32dec {
constexpr int kThreads = 128;
constexpr int kChunk = 256;
}  // namespace f32dec

template <int G>
__global__ void __launch_bounds__(f32dec::kThreads)
    paged_decode_f32_kernel(float *__restrict__ out, int64_t out_sb, int64_t out_sh,
                            const float *__restrict__ q, int64_t q_sb, int64_t q_sh,
                            const float *__restrict__ k_cache, const float *__restrict__ v_cache,
                            int64_t k_bs, int64_t v_bs, int32_t num_blocks, int32_t block_size,
                            int32_t hkv, const int32_t *__restrict__ tables, int64_t bt_stride,
                            int32_t max_blocks, const int32_t *__restrict__ lens, float scale,
                            uint32_t *err) {
  using f32dec::kChunk;
  using f32dec::kThreads;
  __shared__ float sq[G][kD];
  __shared__ float ss[G][kChunk];
  __shared__ float red[2][G][kThreads / 32];
  const int b = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  int L = __ldg(lens + b);
  if (L > static_cast<int64_t>(max_blocks) * block_size) {
    if (tid == 0) record_error(err, SLOKV_DEVERR_CONTEXT_LEN);
    L = max_blocks * block_size;
  }
  float *orow = out + static_cast<int64_t>(b) * out_sb + static_cast<int64_t>(hk) * G * out_sh;
  if (L <= 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) orow[g * out_sh + tid] = 0.f;
    return;
  }
  const float *qrow = q + static_cast<int64_t>(b) * q_sb + static_cast<int64_t>(hk) * G * q_sh;
#pragma unroll
  for (int g = 0; g < G; ++g) sq[g][tid] = __ldg(qrow + g * q_sh + tid);
  const int32_t *trow = tables + static_cast<int64_t>(b) * bt_stride;
  const int64_t row_elems = static_cast<int64_t>(hkv) * kD;
  float acc[G], m_run[G], l_run[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    acc[g] = 0.f;
    m_run[g] = -INFINITY;
    l_run[g] = 0.f;
  }
  // (block id or -1 outside the pool, offset in the block) of a key
  auto block_of = [&](int key) {
    const int page = key / block_size;
    const int32_t blk = __ldg(trow + page);
    return make_int2(blk >= 0 && blk < num_blocks ? blk : -1, key - page * block_size);
  };
  for (int c0 = 0; c0 < L; c0 += kChunk) {
    const int n = min(kChunk, L - c0);
    __syncthreads();                      // q loaded; the previous chunk's P consumed
    for (int t = tid; t < n; t += kThreads) {
      const int2 bo = block_of(c0 + t);
      const int blk = bo.x, off = bo.y;
      float dot[G];
#pragma unroll
      for (int g = 0; g < G; ++g) dot[g] = 0.f;
      if (blk >= 0) {
        const float4 *kr = reinterpret_cast<const float4 *>(
            k_cache + static_cast<int64_t>(blk) * k_bs + off * row_elems + hk * kD);
#pragma unroll 4
        for (int d4 = 0; d4 < kD / 4; ++d4) {
          const float4 kv = __ldg(kr + d4);
#pragma unroll
          for (int g = 0; g < G; ++g)
            dot[g] += sq[g][4 * d4] * kv.x + sq[g][4 * d4 + 1] * kv.y + sq[g][4 * d4 + 2] * kv.z +
                      sq[g][4 * d4 + 3] * kv.w;
        }
      } else {                            // a block id outside the pool reads as zeros
        record_error(err, SLOKV_DEVERR_BLOCK_RANGE);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) ss[g][t] = dot[g] * scale;
    }
    __syncthreads();
    // chunk max of every head
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = -INFINITY;
      for (int t = tid; t < n; t += kThreads) mx = fmaxf(mx, ss[g][t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) red[0][g][warp] = mx;
    }
    __syncthreads();
    float alpha[G], m_new[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = red[0][g][0];
#pragma unroll
      for (int w = 1; w < kThreads / 32; ++w) mx = fmaxf(mx, red[0][g][w]);
      m_new[g] = fmaxf(m_run[g], mx);
      alpha[g] = expf(m_run[g] - m_new[g]);           // 0 on the first chunk
      m_run[g] = m_new[g];
    }
    // P = exp(s - m), its chunk sum, then O += P V (thread tid = output dim)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sum = 0.f;
      for (int t = tid; t < n; t += kThreads) {
        const float pv = expf(ss[g][t] - m_new[g]);
        ss[g][t] = pv;
        sum += pv;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) red[1][g][warp] = sum;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) sum += red[1][g][w];
      l_run[g] = l_run[g] * alpha[g] + sum;
      acc[g] *= alpha[g];
    }
    for (int t = 0; t < n; ++t) {
      const int2 bo = block_of(c0 + t);
      const int blk = bo.x, off = bo.y;
      const float v = blk >= 0 ? __ldg(v_cache + static_cast<int64_t>(blk) * v_bs +
                                       off * row_elems + hk * kD + tid)
                               : 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] += ss[g][t] * v;
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) orow[g * out_sh + tid] = acc[g] / l_run[g];
}

int run_decode_f32(void *out, int64_t out_stride_b, int64_t out_stride_h, const void *q,
                   int64_t q_stride_b, int64_t q_stride_h, const void *k_cache,
                   const void *v_cache, int64_t k_block_stride, int64_t v_block_stride,
                   int32_t num_blocks, int32_t block_size, int32_t num_kv_heads, int32_t group,
                   const int32_t *block_tables, int64_t block_table_stride,
                   int32_t max_blocks_per_seq, const int32_t *context_lens, int32_t batch,
                   float softmax_scale, uint32_t *dev_error, cudaStream_t st) {
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens || max_blocks_per_seq <= 0)
    return SLOKV_ERR_INVALID_ARG;
  // float4 K rows: 16-byte cache bases and block strides
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u)
    return SLOKV_ERR_ALIGNMENT;
  if ((k_block_stride | v_block_stride) & 3) return SLOKV_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 3u)
    return SLOKV_ERR_ALIGNMENT;
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(num_kv_heads));
  auto go = [&](auto kernel) {
    kernel<<<grid, f32dec::kThreads, 0, st>>>(
        static_cast<float *>(out), out_stride_b, out_stride_h, static_cast<const float *>(q),
        q_stride_b, q_stride_h, static_cast<const float *>(k_cache),
        static_cast<const float *>(v_cache), k_block_stride, v_block_stride, num_blocks,
        block_size, num_kv_heads, block_tables, block_table_stride, max_blocks_per_seq,
        context_lens, softmax_scale, dev_error);
    return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
  };
  switch (group) {
    case 1: return go(paged_decode_f32_kernel<1>);
    case 2: return go(paged_decode_f32_kernel<2>);
    case 4: return go(paged_decode_f32_kernel<4>);
    case 8: return go(paged_decode_f32_kernel<8>);
    case 16: return go(paged_decode_f32_kernel<16>);
    default: return SLOKV_ERR_UNSUPPORTED;
  }
}

// Shared argument checks and launch of both cache formats.
int run_decode(bool fp8, void *out, int64_t out_stride_b, int64_t out_stride_h, const void *q,
               int64_t q_stride_b, int64_t q_stride_h, const void *k_cache, const void *v_cache,
               int64_t k_block_stride, int64_t v_block_stride, const float *k_scale,
               const float *v_scale, int32_t num_blocks, int32_t block_size,
               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
               const int32_t *block_tables, int64_t block_table_stride,
               int32_t max_blocks_per_seq, const int32_t *context_lens, int32_t batch,
               float softmax_scale, int32_t dtype, void *workspace, size_t workspace_bytes,
               uint32_t *dev_error, void *stream) {
  if (batch < 0 || num_blocks <= 0 || block_size <= 0 || num_kv_heads <= 0 || num_q_heads <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (batch == 0) return SLOKV_OK;
  if (batch > kMaxBatch) return SLOKV_ERR_UNSUPPORTED;
  if (head_dim != kD) return SLOKV_ERR_UNSUPPORTED;
  const bool f32 = !fp8 && dtype == SLOKV_DTYPE_F32;
  if (dtype != SLOKV_DTYPE_BF16 && dtype != SLOKV_DTYPE_F16 && !f32) return SLOKV_ERR_UNSUPPORTED;
  if (num_q_heads % num_kv_heads) return SLOKV_ERR_INVALID_ARG;
  const int group = num_q_heads / num_kv_heads;
  if (group > 16) return SLOKV_ERR_UNSUPPORTED;
  if (f32)
    return run_decode_f32(out, out_stride_b, out_stride_h, q, q_stride_b, q_stride_h, k_cache,
                          v_cache, k_block_stride, v_block_stride, num_blocks, block_size,
                          num_kv_heads, group, block_tables, block_table_stride,
                          max_blocks_per_seq, context_lens, batch, softmax_scale, dev_error,
                          static_cast<cudaStream_t>(stream));
  if (block_size % kTile) return SLOKV_ERR_UNSUPPORTED;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens || max_blocks_per_seq <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (fp8 && (!k_scale || !v_scale)) return SLOKV_ERR_INVALID_ARG;
  const int cache_bytes = fp8 ? 1 : 2;
  // 16-byte rule of TMA for base and strides; 4-byte pairs for q/out.
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u)
    return SLOKV_ERR_ALIGNMENT;
  if (((k_block_stride * cache_bytes) | (v_block_stride * cache_bytes)) & 15)
    return SLOKV_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 3u)
    return SLOKV_ERR_ALIGNMENT;
  if ((q_stride_b | q_stride_h | out_stride_b | out_stride_h) & 1) return SLOKV_ERR_ALIGNMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SLOKV_ERR_CUDA;
  const int sms = device_sms(dev);
  if (sms <= 0) return SLOKV_ERR_CUDA;
  const int warps = fp8 ? Ring<true>::kWarpsPerCta : Ring<false>::kWarpsPerCta;
  const size_t need = workspace_bytes_for(sms, group, warps);
  if (!workspace || workspace_bytes < need) return SLOKV_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15u) return SLOKV_ERR_ALIGNMENT;

  const CUtensorMapDataType dt =
      fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
          : (dtype == SLOKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUtensorMap km, vm;
  if (!encode_cache_map(&km, k_cache, dt, cache_bytes, k_block_stride, num_blocks, block_size,
                        num_kv_heads) ||
      !encode_cache_map(&vm, v_cache, dt, cache_bytes, v_block_stride, num_blocks, block_size,
                        num_kv_heads))
    return SLOKV_ERR_CUDA;

  Params p;
  p.out = out;
  p.out_sb = out_stride_b;
  p.out_sh = out_stride_h;
  p.q = q;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.context_lens = context_lens;
  p.batch = batch;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.hkv = num_kv_heads;
  p.group = group;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.partials = static_cast<float *>(workspace);
  p.jobs = reinterpret_cast<int4 *>(static_cast<char *>(workspace) +
                                    partial_bytes_for(sms, group, warps));
  p.err = dev_error;
  p.nslots = sms * warps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp8)
    return dtype == SLOKV_DTYPE_BF16 ? launch<__nv_bfloat16, true>(p, km, vm, sms, st)
                                     : launch<__half, true>(p, km, vm, sms, st);
  return dtype == SLOKV_DTYPE_BF16 ? launch<__nv_bfloat16, false>(p, km, vm, sms, st)
                                   : launch<__half, false>(p, km, vm, sms, st);
}

size_t query_workspace(int32_t device, int32_t num_q_heads, int32_t num_kv_heads,
                       int32_t head_dim, int warps) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return 0;
  if (head_dim != kD) return 0;
  int dev = device;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return 0;
  const int sms = device_sms(dev);
  if (sms <= 0) return 0;
  return workspace_bytes_for(sms, num_q_heads / num_kv_heads, warps);
}

}  // namespace decode
}  // namespace slokv

extern "C" size_t slokv_paged_decode_workspace_bytes(int32_t device, int32_t num_q_heads,
                                                     int32_t num_kv_heads, int32_t head_dim) {
  using namespace slokv::decode;
  return query_workspace(device, num_q_heads, num_kv_heads, head_dim,
                         Ring<false>::kWarpsPerCta);
}

extern "C" size_t slokv_paged_decode_fp8_workspace_bytes(int32_t device, int32_t num_q_heads,
                                                         int32_t num_kv_heads, int32_t head_dim) {
  using namespace slokv::decode;
  return query_workspace(device, num_q_heads, num_kv_heads, head_dim, Ring<true>::kWarpsPerCta);
}

extern "C" int slokv_paged_decode(void *out, int64_t out_stride_b, int64_t out_stride_h,
                                  const void *q, int64_t q_stride_b, int64_t q_stride_h,
                                  const void *k_cache, const void *v_cache,
                                  int64_t k_block_stride, int64_t v_block_stride,
                                  int32_t num_blocks, int32_t block_size, int32_t num_q_heads,
                                  int32_t num_kv_heads, int32_t head_dim,
                                  const int32_t *block_tables, int64_t block_table_stride,
                                  int32_t max_blocks_per_seq, const int32_t *context_lens,
                                  int32_t batch, float softmax_scale, int32_t dtype,
                                  void *workspace, size_t workspace_bytes, uint32_t *dev_error,
                                  void *stream) {
  return slokv::decode::run_decode(
      false, out, out_stride_b, out_stride_h, q, q_stride_b, q_stride_h, k_cache, v_cache,
      k_block_stride, v_block_stride, nullptr, nullptr, num_blocks, block_size, num_q_heads,
      num_kv_heads, head_dim, block_tables, block_table_stride, max_blocks_per_seq,
      context_lens, batch, softmax_scale, dtype, workspace, workspace_bytes, dev_error, stream);
}

extern "C" int slokv_paged_decode_fp8(void *out, int64_t out_stride_b, int64_t out_stride_h,
                                      const void *q, int64_t q_stride_b, int64_t q_stride_h,
                                      const void *k_codes, const void *v_codes,
                                      int64_t k_block_stride, int64_t v_block_stride,
                                      const float *k_scale, const float *v_scale,
                                      int32_t num_blocks, int32_t block_size,
                                      int32_t num_q_heads, int32_t num_kv_heads,
                                      int32_t head_dim, const int32_t *block_tables,
                                      int64_t block_table_stride, int32_t max_blocks_per_seq,
                                      const int32_t *context_lens, int32_t batch,
                                      float softmax_scale, int32_t q_dtype, void *workspace,
                                      size_t workspace_bytes, uint32_t *dev_error, void *stream) {
  return slokv::decode::run_decode(
      true, out, out_stride_b, out_stride_h, q, q_stride_b, q_stride_h, k_codes, v_codes,
      k_block_stride, v_block_stride, k_scale, v_scale, num_blocks, block_size, num_q_heads,
      num_kv_heads, head_dim, block_tables, block_table_stride, max_blocks_per_seq,
      context_lens, batch, softmax_scale, q_dtype, workspace, workspace_bytes, dev_error, stream);
}

// ---- allocation-free decode entry point -------------------------------------
//
// For callers that cannot call cudaMalloc: a host runtime bound to this library
// through its C ABI alone (no device allocator of its own), or an engine whose
// caching allocator has already handed ~90% of HBM to the KV pool, so a fresh
// cudaMalloc would fail or would have to synchronise the device mid-step.  The
// split-K scratch then lives in this file-scope device array instead of a
// caller-supplied workspace.  Every GPU that loads the library holds the array
// until the process exits.
namespace slokv {
namespace decode {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(6) << 20;  // 6 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `dev` (which must be the current
// device).  In host code the array's name is only a host-side stand-in, so the
// address is looked up with cudaGetSymbolAddress once per device and cached.
int noalloc_scratch(int dev, void **out) {
  if (dev < 0 || dev >= kMaxDevices) return SLOKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return SLOKV_ERR_CUDA;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return SLOKV_OK;
}

}  // namespace
}  // namespace decode
}  // namespace slokv

extern "C" size_t slokv_paged_decode_noalloc_scratch_bytes(void) {
  return slokv::decode::kNoAllocScratchBytes;
}

extern "C" int slokv_paged_decode_noalloc(void *out, int64_t out_stride_b, int64_t out_stride_h,
                                          const void *q, int64_t q_stride_b, int64_t q_stride_h,
                                          const void *k_cache, const void *v_cache,
                                          int64_t k_block_stride, int64_t v_block_stride,
                                          int32_t num_blocks, int32_t block_size,
                                          int32_t num_q_heads, int32_t num_kv_heads,
                                          int32_t head_dim, const int32_t *block_tables,
                                          int64_t block_table_stride, int32_t max_blocks_per_seq,
                                          const int32_t *context_lens, int32_t batch,
                                          float softmax_scale, int32_t dtype,
                                          uint32_t *dev_error, void *stream) {
  using namespace slokv;
  using namespace slokv::decode;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SLOKV_ERR_CUDA;
  // The scratch holds the per-warp split-K partials: SMs x 3 warp slots x
  // (2 x group x 132 x 4 + 16) bytes, so on a 148-SM B200 up to 13 query heads
  // per KV head fit in 6 MiB.  For a geometry that does not fit, the workspace
  // entry point is asked with no workspace at all: it runs every argument
  // check, launches nothing, and answers SLOKV_ERR_WORKSPACE only when the
  // arguments are otherwise valid -- so both entry points return the same
  // status for the same arguments, and only a call that would have run gets
  // SLOKV_ERR_SCRATCH_LIMIT.
  if (num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0 &&
      head_dim == kD) {
    const int sms = device_sms(dev);
    if (sms <= 0) return SLOKV_ERR_CUDA;
    if (workspace_bytes_for(sms, num_q_heads / num_kv_heads) > kNoAllocScratchBytes) {
      const int st = slokv_paged_decode(
          out, out_stride_b, out_stride_h, q, q_stride_b, q_stride_h, k_cache, v_cache,
          k_block_stride, v_block_stride, num_blocks, block_size, num_q_heads, num_kv_heads,
          head_dim, block_tables, block_table_stride, max_blocks_per_seq, context_lens, batch,
          softmax_scale, dtype, nullptr, 0, dev_error, stream);
      return st == SLOKV_ERR_WORKSPACE ? SLOKV_ERR_SCRATCH_LIMIT : st;
    }
  }
  void *scratch = nullptr;
  const int rc = noalloc_scratch(dev, &scratch);
  if (rc != SLOKV_OK) return rc;
  return slokv_paged_decode(out, out_stride_b, out_stride_h, q, q_stride_b, q_stride_h, k_cache,
                            v_cache, k_block_stride, v_block_stride, num_blocks, block_size,
                            num_q_heads, num_kv_heads, head_dim, block_tables,
                            block_table_stride, max_blocks_per_seq, context_lens, batch,
                            softmax_scale, dtype, scratch, kNoAllocScratchBytes, dev_error,
                            stream);
}
