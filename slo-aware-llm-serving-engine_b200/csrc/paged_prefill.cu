// Causal varlen (prefill / prefix-cache / mixed-batch prefill) attention on the
// sm_100a tensor cores.
//
// Replaces flash_attn_varlen_func as the reference engine calls it
// (nanovllm/layers/attention.py:69-74, nanovllm/layers/mixed_attention.py:123-133):
// rows r with q_len = cu_q[r+1]-cu_q[r] queries and k_len = cu_k[r+1]-cu_k[r]
// keys; query i sees keys 0 .. k_len-q_len+i (bottom-right aligned causal
// mask); keys come from the paged pool through block_tables (prefix cache) or
// from contiguous k/v rows (cold prefill).  GQA: query head h uses kv head
// h / (Hq/Hkv).
//
// Two kernels.  GQA groups of even size (the engine's geometries) run the
// warp-specialised two-head kernel further down (two query heads share one
// K/V stream; tensor-core issue, TMA and two softmax warpgroups in separate
// warps, P kept in TMEM).  Odd groups run the single-head kernel described here.
//
// Single-head design (one CTA = 128 queries of one head of one row, 4 warps):
//  * TMA loads Q once and K/V tiles of 128 keys (two 64-dim halves each,
//    128-byte swizzle = the canonical K-major UMMA layout) into double-buffered
//    K and V rings; every CTA loads its own tiles.
//  * One thread issues tcgen05.mma (kind::f16, M=128, fp32 accumulate in TMEM):
//    S_j = Q K_j^T into one of two TMEM S buffers -- S_{j+1} is issued before the
//    softmax of S_j, so the tensor core works while the CUDA cores do exp --
//    and O += P_j V_j with V as an MN-major operand (two N=64 halves).
//  * Softmax: thread t owns query row t (TMEM lane t): it loads its 128 scores
//    with tcgen05.ld, so max/sum need no shuffles; P is written as bf16/f16
//    into a swizzled shared-memory tile (the A operand of the PV MMA).  O stays
//    in TMEM and is rescaled there (tcgen05.ld/st) only when a warp's row max
//    moved.
//  * V rows past k_len in the last tile are zeroed before PV so stale pool bytes
//    (possibly NaN) never reach O; masked scores are -inf, not multiplied.
#include "common.cuh"
#include "fp8_e4m3.cuh"
#include "tcgen05.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

namespace slokv {
namespace prefill {

constexpr int kD = 128;
constexpr int kBM = 128;                  // queries per CTA
constexpr int kBN = 128;                  // keys per tile
constexpr int kHalf = 128 * 128;          // 128 rows x 128 bytes (one 64-dim half)
constexpr int kTile = 2 * kHalf;          // 32 KiB: 128 x 128 16-bit elements
constexpr int kOffQ = 0;
constexpr int kOffK = kTile;              // two stages
constexpr int kOffV = 3 * kTile;          // two stages
constexpr int kOffP = 5 * kTile;
constexpr int kTiles = 6 * kTile;         // 192 KiB
// barriers after the tiles: Q, K[2], V[2], S[2], PV
constexpr int kBarQ = 0, kBarK = 1, kBarV = 3, kBarS = 5, kBarPV = 7, kNumBars = 8;
constexpr int kSmemBytes = 1024 + kTiles + kNumBars * 8 + 16;
constexpr uint32_t kTmemCols = 512;       // S0 | S1 | O (128 columns each)
constexpr uint32_t kColS = 0, kColO = 256;

struct Params {
  void *out;
  int64_t out_st, out_sh;                 // out[token][head][dim]
  const int32_t *cu_q, *cu_k;
  const int32_t *block_tables;            // null: contiguous k/v
  int64_t bt_stride;
  int32_t max_blocks;
  int32_t num_blocks, block_size;
  int32_t hq, hkv, group;
  float scale_log2;
  uint32_t *err;
  // Two-head kernel work order: linear block b runs query tile order[b / (hq/2)]
  // (row * m_tiles + m, longest first; -1 = no tile); null: row-major order.
  const int32_t *order;
  int32_t m_tiles;                        // ceil(max_seqlen_q / 128)
  // Optional per-(page, kv head) factor of S (two-head kernel only): K holds
  // unscaled FP8 codes and the logits of a key tile in page `pid` are
  // S * k_page_scale[pid * hkv + kv head].  Null: 1.
  const float *k_page_scale;
  // FP8 kernel only: the pool's V scales; V codes of page `pid` widen to
  // f16(decode(code) * v_page_scale[pid * hkv + kv head]).
  const float *v_page_scale;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input max (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed pairs of fp32 for the sm_100 f32x2 arithmetic (each lane rounds as
// the scalar instruction does).
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f32x2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t two(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <>
struct Pack<__half> {
  __device__ __forceinline__ static uint32_t two(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

// Coordinates of key tile j (keys 128j .. 128j+127 of row r) for the K/V maps.
struct KvCoord {
  int32_t c2, c3;
  bool ok;
};

__device__ __forceinline__ KvCoord kv_coord(const Params &p, int r, int k0, int j) {
  KvCoord c;
  const int key = j * kBN;
  if (p.block_tables == nullptr) {
    c.c2 = k0 + key;
    c.c3 = 0;
    c.ok = true;
  } else {
    const int page = key / p.block_size;
    c.c2 = key - page * p.block_size;
    // A page past the table width or an id outside the pool loads as zeros
    // (TMA bounds fill) and is flagged; the table row is never over-read.
    c.c3 = page < p.max_blocks
               ? __ldg(p.block_tables + static_cast<int64_t>(r) * p.bt_stride + page) : -1;
    c.ok = c.c3 >= 0 && c.c3 < p.num_blocks;
  }
  return c;
}

template <typename T>
__global__ void __launch_bounds__(128, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const Params p) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = tc::idesc_f16(kBf16, false, 128, 128);
  constexpr uint32_t kIdescPV = tc::idesc_f16(kBf16, true, 128, 64);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int r = blockIdx.z, h = blockIdx.y;
  const int m = gridDim.x - 1 - blockIdx.x;  // longest (last) query tiles first
  const int q0 = __ldg(p.cu_q + r), q_len = __ldg(p.cu_q + r + 1) - q0;
  const int k0 = __ldg(p.cu_k + r), k_len = __ldg(p.cu_k + r + 1) - k0;
  if (m * kBM >= q_len) return;
  const int hk = h / p.group;
  const int qk_off = k_len - q_len;
  const int last_q = min((m + 1) * kBM, q_len) - 1;
  const int need = min(k_len, qk_off + last_q + 1);   // keys any query of the tile sees
  const int nk = need > 0 ? (need + kBN - 1) / kBN : 0;
  // query row of this thread and the last key it may see (inclusive)
  const int qi = m * kBM + tid;
  const bool row_ok = qi < q_len;
  const int kmax = row_ok ? min(qk_off + qi, k_len - 1) : -1;
  T *orow = static_cast<T *>(p.out) + static_cast<int64_t>(q0 + qi) * p.out_st +
            static_cast<int64_t>(h) * p.out_sh;

  if (nk == 0) {  // no query of the tile sees any key: zero output
    if (row_ok)
      for (int d = 0; d < kD; d += 8)
        *reinterpret_cast<uint4 *>(orow + d) = make_uint4(0, 0, 0, 0);
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *base_ptr = smem_raw + (base - raw);
  const uint32_t bars = base + kTiles;
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(base_ptr + kTiles + kNumBars * 8);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  if (tid == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int i = 0; i < kNumBars; ++i) mbar_init(bars + i * 8, 1);
    fence_barrier_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(const_cast<uint32_t *>(tmem_slot)), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint64_t policy = l2_evict_first_policy();

  auto bar = [&](int i) { return bars + i * 8; };
  auto issue_k = [&](int j) {
    const KvCoord c = kv_coord(p, r, k0, j);
    if (!c.ok) record_error(p.err, SLOKV_DEVERR_BLOCK_RANGE);
    const uint32_t dst = base + kOffK + (j & 1) * kTile;
    mbar_arrive_expect_tx(bar(kBarK + (j & 1)), kTile);
    tma_load_4d(dst, &kmap, bar(kBarK + (j & 1)), 0, hk, c.c2, c.c3, policy);
    tma_load_4d(dst + kHalf, &kmap, bar(kBarK + (j & 1)), 64, hk, c.c2, c.c3, policy);
  };
  auto issue_v = [&](int j) {
    const KvCoord c = kv_coord(p, r, k0, j);
    const uint32_t dst = base + kOffV + (j & 1) * kTile;
    mbar_arrive_expect_tx(bar(kBarV + (j & 1)), kTile);
    tma_load_4d(dst, &vmap, bar(kBarV + (j & 1)), 0, hk, c.c2, c.c3, policy);
    tma_load_4d(dst + kHalf, &vmap, bar(kBarV + (j & 1)), 64, hk, c.c2, c.c3, policy);
  };
  auto wait_or_abort = [&](int i, uint32_t parity) {
    if (!mbar_wait(bar(i), parity)) {
      record_error(p.err, SLOKV_DEVERR_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
    return true;
  };
  // S_j = Q K_j^T -> TMEM S buffer j&1 (issued by thread 0)
  auto issue_s = [&](int j) {
    if (*abort_flag || !wait_or_abort(kBarK + (j & 1), (j >> 1) & 1)) return;
    tc::fence_after_sync();
    const uint32_t qa = base + kOffQ, kb = base + kOffK + (j & 1) * kTile;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
      tc::mma_f16_ss(tmem + kColS + (j & 1) * 128, tc::smem_desc_sw128(qa + off, 16, 1024),
                     tc::smem_desc_sw128(kb + off, 16, 1024), kIdescS, kk > 0);
    }
    tc::commit(bar(kBarS + (j & 1)));
  };

  if (tid == 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar(kBarQ), kTile);
    tma_load_4d(base + kOffQ, &qmap, bar(kBarQ), 0, h, q0 + m * kBM, 0, policy);
    tma_load_4d(base + kOffQ + kHalf, &qmap, bar(kBarQ), 64, h, q0 + m * kBM, 0, policy);
    issue_k(0);
    issue_v(0);
    if (nk > 1) {
      issue_k(1);
      issue_v(1);
    }
    if (wait_or_abort(kBarQ, 0)) issue_s(0);
  }

  float m_run = -INFINITY, l_run = 0.f;
  uint32_t sreg[32];
  for (int j = 0; j < nk; ++j) {
    __syncthreads();               // every exit decision is taken here, by all threads
    if (*abort_flag) break;
    if (tid == 0 && j + 1 < nk) issue_s(j + 1);
    wait_or_abort(kBarS + (j & 1), (j >> 1) & 1);   // S_j in TMEM
    tc::fence_after_sync();
    if (tid == 0 && j + 2 < nk && !*abort_flag) issue_k(j + 2);  // S_j freed K stage j&1

    // ---- pass 1: running max of row qi over keys 128j .. 128j+127 ----
    const int key0 = j * kBN;
    const bool full = key0 + kBN - 1 <= kmax;
    const uint32_t s_addr = tmem + lane_base + kColS + (j & 1) * 128;
    float mx = -INFINITY;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      tc::ld32(s_addr + cb * 32, sreg);
      tc::wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int key = key0 + cb * 32 + c;
        if (full || key <= kmax) mx = fmaxf(mx, __uint_as_float(sreg[c]) * p.scale_log2);
      }
    }
    const float m_new = fmaxf(m_run, mx);
    const float mu = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = fast_exp2(m_run - mu);
    m_run = m_new;

    // PV_{j-1} must be done before P, O and V stage (j-1)&1 are reused.
    if (j > 0) {
      wait_or_abort(kBarPV, (j - 1) & 1);
      tc::fence_after_sync();
      if (tid == 0 && j + 1 < nk && !*abort_flag) issue_v(j + 1);
    }

    // ---- pass 2: P = exp2(s - m) -> shared memory (K-major, 128-byte swizzle) ----
    float rs = 0.f;
    uint8_t *prow = base_ptr + kOffP + tid * 128;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      tc::ld32(s_addr + cb * 32, sreg);
      tc::wait_ld();
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const int key = key0 + cb * 32 + c;
        const float a = (full || key <= kmax)
                            ? fast_exp2(__uint_as_float(sreg[c]) * p.scale_log2 - mu) : 0.f;
        const float b = (full || key + 1 <= kmax)
                            ? fast_exp2(__uint_as_float(sreg[c + 1]) * p.scale_log2 - mu) : 0.f;
        rs += a + b;
        pk[c >> 1] = Pack<T>::two(a, b);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int chunk = cb * 4 + i;  // 8 keys per 16-byte chunk
        *reinterpret_cast<uint4 *>(prow + (chunk >> 3) * kHalf + (((chunk & 7) ^ (tid & 7)) << 4)) =
            make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
    l_run = l_run * alpha + rs;

    // rescale O when the running max moved for any row of this warp
    if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
      const uint32_t o_addr = tmem + lane_base + kColO;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        tc::ld32(o_addr + cb * 32, sreg);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) sreg[c] = __float_as_uint(__uint_as_float(sreg[c]) * alpha);
        tc::st32(o_addr + cb * 32, sreg);
      }
      tc::wait_st();
    }
    // zero V rows past the sequence end in the last tile
    if (key0 + kBN > k_len && wait_or_abort(kBarV + (j & 1), (j >> 1) & 1)) {
      const int valid = k_len - key0;
      uint8_t *vt = base_ptr + kOffV + (j & 1) * kTile;
      for (int i = tid; i < (kBN - valid) * 16; i += 128) {
        const int row = valid + (i >> 4), part = i & 15;
        *reinterpret_cast<uint4 *>(vt + (part >> 3) * kHalf + row * 128 + (part & 7) * 16) =
            make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0 && !*abort_flag) {
      tc::fence_after_sync();
      if (wait_or_abort(kBarV + (j & 1), (j >> 1) & 1)) {
        const uint32_t pa = base + kOffP, vb = base + kOffV + (j & 1) * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t adesc =
              tc::smem_desc_sw128(pa + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
#pragma unroll
          for (int nh = 0; nh < 2; ++nh)
            tc::mma_f16_ss(tmem + kColO + nh * 64, adesc,
                           tc::smem_desc_sw128(vb + nh * kHalf + kk * 16 * 128, 1024, 1024),
                           kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc::commit(bar(kBarPV));
      }
    }
  }

  // ---- epilogue: O / l -> out ----
  __syncthreads();
  const bool ok = !*abort_flag && wait_or_abort(kBarPV, (nk - 1) & 1);
  tc::fence_after_sync();
  if (__all_sync(0xffffffffu, ok)) {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    const uint32_t o_addr = tmem + lane_base + kColO;
#pragma unroll
    for (int cblk = 0; cblk < 4; ++cblk) {
      tc::ld32(o_addr + cblk * 32, sreg);
      tc::wait_ld();
      if (row_ok) {
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 w;
          w.x = Pack<T>::two(__uint_as_float(sreg[c]) * inv, __uint_as_float(sreg[c + 1]) * inv);
          w.y = Pack<T>::two(__uint_as_float(sreg[c + 2]) * inv, __uint_as_float(sreg[c + 3]) * inv);
          w.z = Pack<T>::two(__uint_as_float(sreg[c + 4]) * inv, __uint_as_float(sreg[c + 5]) * inv);
          w.w = Pack<T>::two(__uint_as_float(sreg[c + 6]) * inv, __uint_as_float(sreg[c + 7]) * inv);
          *reinterpret_cast<uint4 *>(orow + cblk * 32 + c) = w;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ---- longest-first work order ------------------------------------------------
//
// A query tile's cost is its number of key tiles, which grows along the causal
// diagonal and with the row's cached prefix.  Blocks are dispatched in linear
// order, so listing the tiles longest first (list scheduling by decreasing
// cost) keeps the long tiles out of the last wave.  One block counting-sorts
// the rows x m_tiles tiles by cost (costs above kSchedBuckets - 1 share the top
// bucket); ties come out in any order.
constexpr int kSchedBuckets = 2048;
constexpr int kSchedThreads = 1024;

__device__ __forceinline__ int tile_cost(const int32_t *cu_q, const int32_t *cu_k, int idx,
                                         int m_tiles) {
  const int r = idx / m_tiles, m = idx - r * m_tiles;
  const int q_len = __ldg(cu_q + r + 1) - __ldg(cu_q + r);
  if (m * kBM >= q_len) return -1;
  const int k_len = __ldg(cu_k + r + 1) - __ldg(cu_k + r);
  const int need = min(k_len, k_len - q_len + min((m + 1) * kBM, q_len));
  const int nk = need > 0 ? (need + kBN - 1) / kBN : 0;
  return min(nk, kSchedBuckets - 1);
}

__global__ void __launch_bounds__(kSchedThreads)
    prefill_schedule_kernel(const int32_t *cu_q, const int32_t *cu_k, int rows, int m_tiles,
                            int32_t *order) {
  __shared__ int start[kSchedBuckets];
  __shared__ int warp_tot[kSchedThreads / 32];
  __shared__ int total;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int n = rows * m_tiles;
  for (int i = tid; i < kSchedBuckets; i += kSchedThreads) start[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kSchedThreads) {
    const int c = tile_cost(cu_q, cu_k, i, m_tiles);
    if (c >= 0) atomicAdd(&start[c], 1);
  }
  __syncthreads();
  // exclusive scan of the counts from the highest cost down: thread t owns
  // costs hi = top - 2t and hi - 1
  static_assert(kSchedBuckets == 2 * kSchedThreads, "two buckets per thread");
  const int hi = kSchedBuckets - 1 - 2 * tid;
  const int c_hi = start[hi], c_lo = start[hi - 1];
  int incl = c_hi + c_lo;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;                       // inclusive over warps
    if (lane == 31) total = t;
  }
  __syncthreads();
  const int excl = incl - (c_hi + c_lo) + (w > 0 ? warp_tot[w - 1] : 0);
  start[hi] = excl;
  start[hi - 1] = excl + c_hi;
  __syncthreads();
  for (int i = tid; i < n; i += kSchedThreads) {
    const int c = tile_cost(cu_q, cu_k, i, m_tiles);
    if (c >= 0) order[atomicAdd(&start[c], 1)] = i;
  }
  for (int i = total + tid; i < n; i += kSchedThreads) order[i] = -1;
}

// ---- warp-specialised two-head variant ---------------------------------------
//
// One CTA = 128 queries of two query heads that share a KV head (GQA group of
// even size), so one K/V stream feeds both.  Warps 0-3 / 4-7: softmax warpgroups
// of head 0 / head 1 (thread = query row = TMEM lane).  Warp 8: tensor-core issue
// (lane 0).  Warp 9: TMA producer (lane 0).  Warps 10-11 only complete the
// issue warpgroup, whose registers setmaxnreg moves to the softmax warpgroups:
// a softmax thread holds its whole 128-key S row after one TMEM load, so each
// tile costs one TMEM round trip, one row max and one exponentiation pass.
// While one warpgroup runs the softmax of tile j, the tensor core runs the
// other head's PV and next S.
//
// TMEM (512 columns): S_0 | S_1 | O_0 | O_1, 128 columns each.  P_h (bf16/f16)
// is written over the first 64 columns of S_h and read as the TMEM A operand of
// PV_h; S_h of the next tile is issued after PV_h, so the in-order tensor core
// reads P_h before overwriting it.
// Shared memory: Q_0 | Q_1 | K stage 0 | K stage 1 | V stage 0 | V stage 1.
namespace ws {
constexpr int kOffQ = 0;
constexpr int kOffK = 2 * kTile;
constexpr int kOffV = 4 * kTile;
constexpr int kTilesBytes = 6 * kTile;
enum Bar { kQ = 0, kK = 1, kV = 3, kFreeK = 5, kFreeV = 7, kS = 9, kP = 11, kPV = 13, kNum = 15 };
constexpr int kSmem = 1024 + kTilesBytes + kNum * 8 + 16;
// FP8 pools: the row's per-page K scales (one float per page of the row, for
// the CTA's KV head) follow, so the tile loop reads them from shared memory.
constexpr int kOffScale = kTilesBytes + kNum * 8 + 16;
constexpr int kSmemMax = 232448;   // per-block opt-in limit of sm_100
constexpr int kThreads = 384;
// Register split (setmaxnreg): the block launches with 168 registers a thread
// (384 threads x 168 = 64512); warps 8-11 drop to kRegsIssue and the two softmax
// warpgroups rise to kRegsSoftmax: 2*128*kRegsSoftmax + 128*kRegsIssue = 64512.
constexpr int kRegsLaunch = 168, kRegsIssue = 56, kRegsSoftmax = 224;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsIssue <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");

constexpr uint32_t kColS = 0, kColO = 256;
}  // namespace ws

// kPageScale: the K pages hold unscaled FP8 code values and every tile's logits
// take the page's K scale (FP8 pools).  A separate instantiation, so the plain
// bf16/f16 kernel keeps its register allocation (the scale bookkeeping costs
// the softmax warps a few spilled registers).
template <typename T, bool kPageScale>
__global__ void __launch_bounds__(ws::kThreads, 1)
    paged_prefill_ws_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const Params p) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = tc::idesc_f16(kBf16, false, 128, 128);
  constexpr uint32_t kIdescPV = tc::idesc_f16(kBf16, true, 128, 128);

  const int tid = threadIdx.x, lane = tid & 31;
  // warp index made visibly warp-uniform for the compiler (role dispatch, setmaxnreg)
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);
  // 1-D grid: head pair fastest, then query tiles (longest first when ordered)
  const int pairs = p.hq >> 1;
  const int rank = blockIdx.x / pairs;
  const int h0 = 2 * (blockIdx.x - rank * pairs);   // query heads h0, h0 + 1
  int r, m;
  if (p.order != nullptr) {
    const int item = __ldg(p.order + rank);
    if (item < 0) return;
    r = item / p.m_tiles;
    m = item - r * p.m_tiles;
  } else {
    r = rank / p.m_tiles;
    m = p.m_tiles - 1 - (rank - r * p.m_tiles);
  }
  const int q0 = __ldg(p.cu_q + r), q_len = __ldg(p.cu_q + r + 1) - q0;
  const int k0 = __ldg(p.cu_k + r), k_len = __ldg(p.cu_k + r + 1) - k0;
  if (m * kBM >= q_len) return;
  const int hk = h0 / p.group;
  const int qk_off = k_len - q_len;
  const int last_q = min((m + 1) * kBM, q_len) - 1;
  const int need = min(k_len, qk_off + last_q + 1);
  const int nk = need > 0 ? (need + kBN - 1) / kBN : 0;
  if (nk == 0) {
    if (tid < 256) {
      const int qi = m * kBM + (tid & 127);
      if (qi < q_len) {
        T *orow = static_cast<T *>(p.out) + static_cast<int64_t>(q0 + qi) * p.out_st +
                  static_cast<int64_t>(h0 + (tid >> 7)) * p.out_sh;
        for (int d = 0; d < kD; d += 8) *reinterpret_cast<uint4 *>(orow + d) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *base_ptr = smem_raw + (base - raw);
  const uint32_t bars = base + ws::kTilesBytes;
  volatile uint32_t *tmem_slot =
      reinterpret_cast<volatile uint32_t *>(base_ptr + ws::kTilesBytes + ws::kNum * 8);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  auto bar = [&](int i) { return bars + i * 8; };
  float *s_ks = reinterpret_cast<float *>(base_ptr + ws::kOffScale);
  if constexpr (kPageScale) {  // the row's page scales, read after the barrier below
    // (the table holds max_blocks entries: pages past the block table, i.e.
    // contexts longer than the table, are neither written nor read)
    const int npg = min((need + p.block_size - 1) / p.block_size, p.max_blocks);
    for (int pg = tid; pg < npg; pg += ws::kThreads) {
      const int32_t pid = __ldg(p.block_tables + static_cast<int64_t>(r) * p.bt_stride + pg);
      s_ks[pg] = pid >= 0 && pid < p.num_blocks
                     ? __ldg(p.k_page_scale + static_cast<int64_t>(pid) * p.hkv + hk)
                     : 0.f;
    }
  }

  if (tid == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int i = 0; i < ws::kNum; ++i)
      mbar_init(bar(i), (i == ws::kP || i == ws::kP + 1) ? 128u : 1u);
    fence_barrier_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(const_cast<uint32_t *>(tmem_slot)), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](int i, uint32_t parity) {
    if (*abort_flag) return false;
    if (!mbar_wait(bar(i), parity)) {
      record_error(p.err, SLOKV_DEVERR_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
    return true;
  };

  if (warp >= 8) {
    // Warps 8-11 (one warpgroup) give registers to the softmax warpgroups.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(ws::kRegsIssue));
    if (warp == 9) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        const uint64_t policy = l2_evict_first_policy();
        mbar_arrive_expect_tx(bar(ws::kQ), 2 * kTile);
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t dst = base + ws::kOffQ + hh * kTile;
          tma_load_4d(dst, &qmap, bar(ws::kQ), 0, h0 + hh, q0 + m * kBM, 0, policy);
          tma_load_4d(dst + kHalf, &qmap, bar(ws::kQ), 64, h0 + hh, q0 + m * kBM, 0, policy);
        }
        for (int j = 0; j < nk; ++j) {
          const int st = j & 1;
          // K stage st frees once both S MMAs of tile j-2 finish, V stage st once
          // both PV MMAs of tile j-2 finish (later): K loads run ahead.
          if (j >= 2 && !wait(ws::kFreeK + st, ((j - 2) >> 1) & 1)) break;
          const KvCoord c = kv_coord(p, r, k0, j);
          if (!c.ok) record_error(p.err, SLOKV_DEVERR_BLOCK_RANGE);
          const uint32_t kd = base + ws::kOffK + st * kTile, vd = base + ws::kOffV + st * kTile;
          mbar_arrive_expect_tx(bar(ws::kK + st), kTile);
          tma_load_4d(kd, &kmap, bar(ws::kK + st), 0, hk, c.c2, c.c3, policy);
          tma_load_4d(kd + kHalf, &kmap, bar(ws::kK + st), 64, hk, c.c2, c.c3, policy);
          if (j >= 2 && !wait(ws::kFreeV + st, ((j - 2) >> 1) & 1)) break;
          mbar_arrive_expect_tx(bar(ws::kV + st), kTile);
          tma_load_4d(vd, &vmap, bar(ws::kV + st), 0, hk, c.c2, c.c3, policy);
          tma_load_4d(vd + kHalf, &vmap, bar(ws::kV + st), 64, hk, c.c2, c.c3, policy);
        }
      }
    } else if (warp == 8) {
      // ---------------- tensor-core issue (lane 0 issues, the warp helps zero V) ----
      auto issue_s = [&](int hh, int j) {
        const uint32_t qa = base + ws::kOffQ + hh * kTile;
        const uint32_t kb = base + ws::kOffK + (j & 1) * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          tc::mma_f16_ss(tmem + ws::kColS + hh * 128, tc::smem_desc_sw128(qa + off, 16, 1024),
                         tc::smem_desc_sw128(kb + off, 16, 1024), kIdescS, kk > 0);
        }
        tc::commit(bar(ws::kS + hh));
      };
      bool ok = wait(ws::kQ, 0) && wait(ws::kK, 0);
      if (ok && lane == 0) {
        tc::fence_after_sync();
        issue_s(0, 0);
        issue_s(1, 0);
        tc::commit(bar(ws::kFreeK));                      // K stage 0 free after S(0)
      }
      __syncwarp();
      for (int j = 0; j < nk && ok; ++j) {
        const int st = j & 1;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          ok = wait(ws::kP + hh, j & 1);                  // P_h(j) in TMEM, O_h rescaled
          if (ok && hh == 0) {
            ok = wait(ws::kV + st, (j >> 1) & 1);
            const int key0 = j * kBN;
            if (ok && key0 + kBN > k_len) {               // zero V rows past the sequence end
              const int valid = k_len - key0;
              uint8_t *vt = base_ptr + ws::kOffV + st * kTile;
              for (int i = lane; i < (kBN - valid) * 16; i += 32) {
                const int row = valid + (i >> 4), part = i & 15;
                *reinterpret_cast<uint4 *>(vt + (part >> 3) * kHalf + row * 128 + (part & 7) * 16) =
                    make_uint4(0, 0, 0, 0);
              }
              fence_proxy_async_smem();
            }
            __syncwarp();
          }
          if (ok && lane == 0) {
            tc::fence_after_sync();
            const uint32_t vb = base + ws::kOffV + st * kTile;
            const uint32_t pa = tmem + ws::kColS + hh * 128;
            // N = 128 in one instruction: V is MN-major with the two 64-dim
            // halves (128-byte swizzle atoms along N) kHalf bytes apart (LBO);
            // 8-key row groups are 1024 bytes apart (SBO).
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              tc::mma_f16_ts(tmem + ws::kColO + hh * 128, pa + kk * 8,
                             tc::smem_desc_sw128(vb + kk * 16 * 128, kHalf, 1024), kIdescPV,
                             (j > 0 || kk > 0) ? 1u : 0u);
            tc::commit(bar(ws::kPV + hh));
          }
          if (ok && j + 1 < nk) {
            if (hh == 0) ok = wait(ws::kK + ((j + 1) & 1), ((j + 1) >> 1) & 1);
            if (ok && lane == 0) issue_s(hh, j + 1);
          }
          __syncwarp();
        }
        if (ok && lane == 0) {
          tc::commit(bar(ws::kFreeV + st));                   // after PV(j) of both heads
          if (j + 1 < nk) tc::commit(bar(ws::kFreeK + ((j + 1) & 1)));   // after S(j+1)
        }
        __syncwarp();
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(ws::kRegsSoftmax));
    // ---------------- softmax warpgroup hh (rows = TMEM lanes) ----------------
    const int hh = warp >> 2;
    const int row = tid & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qi = m * kBM + row;
    const bool row_ok = qi < q_len;
    const int kmax = row_ok ? min(qk_off + qi, k_len - 1) : -1;
    const uint32_t s_addr = tmem + lane_base + ws::kColS + hh * 128;
    const uint32_t o_addr = tmem + lane_base + ws::kColO + hh * 128;
    // Lazy rescaling: the row keeps a stale max m_run while a tile's P row sum
    // against it stays <= kSumLimit, so every P <= 2^8 (exact in the bf16/f16
    // range) and O in TMEM is rescaled only when that bound would break.
    constexpr float kSumLimit = 256.f;
    // Padding rows (no query) start from a finite max; all their keys are
    // masked, so P = 0 and l = 0.
    float m_run = row_ok ? -INFINITY : 0.f, l_run = 0.f;
    uint32_t s[4][32];                            // S row of the tile, keys 32*i + c
    bool ok = true;
    // P = 2^(S * sl - mu) of the S row in registers (sl: scale_log2 times the
    // tile's K page scale), packed (keys 2w, 2w+1 in column w) over the first 64
    // columns of S; returns the row sum.  The scale-and-shift and the sum run
    // two keys per f32x2 instruction.
    auto exp_store = [&](float mu, float sl) {
      const uint64_t sl2 = f32x2(sl, sl), nmu2 = f32x2(-mu, -mu);
      uint64_t rs2[4] = {0ull, 0ull, 0ull, 0ull};  // {0.f, 0.f}
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t pk[32];
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          const int i = 2 * hb + (w >> 4), c = (w & 15) * 2;
          const float2 x = f32x2_split(ffma2(
              f32x2(__uint_as_float(s[i][c]), __uint_as_float(s[i][c + 1])), sl2, nmu2));
          const float a = fast_exp2(x.x);
          const float b = fast_exp2(x.y);
          rs2[w & 3] = fadd2(rs2[w & 3], f32x2(a, b));
          pk[w] = Pack<T>::two(a, b);
        }
        tc::st32(s_addr + 32 * hb, pk);
      }
      const float2 r01 = f32x2_split(fadd2(rs2[0], rs2[1]));
      const float2 r23 = f32x2_split(fadd2(rs2[2], rs2[3]));
      return (r01.x + r01.y) + (r23.x + r23.y);
    };
    for (int j = 0; j < nk && ok; ++j) {
      // S_h(j) complete implies PV_h(j-1) complete (both issued in order by one
      // thread; a commit covers every earlier MMA): O_h and the P columns are free.
      ok = wait(ws::kS + hh, j & 1);
      tc::fence_after_sync();
      const int key0 = j * kBN;
      const bool full = key0 + kBN - 1 <= kmax;   // no key of the tile is masked
      // K page scale of the tile (FP8 pools); a zero scale, a page of zero
      // codes, must keep masked -inf keys at -inf
      const int kpage = key0 / p.block_size;
      const float sl =
          kPageScale ? p.scale_log2 * fmaxf(kpage < p.max_blocks ? s_ks[kpage] : 0.f, 1e-30f)
                     : p.scale_log2;
#pragma unroll
      for (int i = 0; i < 4; ++i) tc::ld32(s_addr + 32 * i, s[i]);
      tc::wait_ld();
      if (!full) {                                // masked keys -> -inf (exp2 -> 0)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (key0 + 32 * i + c > kmax) s[i][c] = 0xff800000u;
      }
      // P against the running max without a row max first.  A warp with a row
      // sum above kSumLimit (or on a row's first tile) takes the row max,
      // rescales and recomputes P from the S row still in registers.
      const bool fresh = __any_sync(0xffffffffu, m_run == -INFINITY);
      float alpha = 1.f, rs = 0.f;
      bool redo = fresh;
      if (!fresh) {
        rs = exp_store(m_run, sl);
        redo = __any_sync(0xffffffffu, !(rs <= kSumLimit));
      }
      if (redo) {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 32; ++c) mx = fmaxf(mx, __uint_as_float(s[i][c]));
        mx *= sl;
        if (mx > m_run) {                          // first tile: m_run = -inf, alpha = 0
          alpha = fast_exp2(m_run - mx);
          m_run = mx;
        }
        if (!fresh) tc::wait_st();                 // first P stores land before rewrite
        rs = exp_store(m_run == -INFINITY ? 0.f : m_run, sl);
      }
      l_run = l_run * alpha + rs;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int i = 0; i < 4; ++i) tc::ld32(o_addr + 32 * i, s[i]);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int c = 0; c < 32; ++c) s[i][c] = __float_as_uint(__uint_as_float(s[i][c]) * alpha);
          tc::st32(o_addr + 32 * i, s[i]);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(bar(ws::kP + hh));
    }
    // epilogue: O_h / l -> out
    ok = ok && wait(ws::kPV + hh, (nk - 1) & 1);
    tc::fence_after_sync();
    if (__all_sync(0xffffffffu, ok)) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T *orow = static_cast<T *>(p.out) + static_cast<int64_t>(q0 + qi) * p.out_st +
                static_cast<int64_t>(h0 + hh) * p.out_sh;
#pragma unroll
      for (int i = 0; i < 4; ++i) tc::ld32(o_addr + 32 * i, s[i]);
      tc::wait_ld();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 w;
            w.x = Pack<T>::two(__uint_as_float(s[i][c]) * inv, __uint_as_float(s[i][c + 1]) * inv);
            w.y = Pack<T>::two(__uint_as_float(s[i][c + 2]) * inv, __uint_as_float(s[i][c + 3]) * inv);
            w.z = Pack<T>::two(__uint_as_float(s[i][c + 4]) * inv, __uint_as_float(s[i][c + 5]) * inv);
            w.w = Pack<T>::two(__uint_as_float(s[i][c + 6]) * inv, __uint_as_float(s[i][c + 7]) * inv);
            *reinterpret_cast<uint4 *>(orow + 32 * i + c) = w;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}


// ---- FP8-E4M3 pool: the two-head kernel reading the code pages directly -----
//
// Replaces the page copy of the FP8 prefix-cache path.  K and V pages of E4M3
// codes are TMA-loaded as they lie in the pool (16 KB per 128-key tile, one
// head) into two-slot K and V code rings; tiles two ahead are prefetched into
// L2.
//  * S = Q K^T runs on the codes themselves (tcgen05 kind::f8f6f4, fp32
//    accumulate): each softmax thread splits its query row, scaled by a power of
//    two 2^e so its largest element lies in [128, 256), into two E4M3 rows,
//    hi = e4m3(q 2^e) and lo = e4m3(q 2^e - hi), written over the row's q in
//    shared memory.  A bf16 (8-bit) or f16 element is then exactly hi + lo
//    whenever it is at least 2^-10 of the row's largest (below that the split
//    drops bits under 2^-17 of the row max), so S = (hi K^T + lo K^T) 2^-e: two
//    MMAs of K = 32 per 32 dims, the tensor time of one f16 MMA, and no K
//    conversion.
//  * V is widened to its unscaled code values (exact in f16) by six converter
//    warps, rows past the keys zeroed (stale pool bytes may hold NaN codes).
//  * Scales in the softmax, per 128-key tile (a tile never spans two pages):
//    logits S * k_scale * 2^-e; P multiplied by r = v_scale / v_ref (v_ref the
//    largest V scale among the row's pages) through the exponent,
//    P = 2^(s - m + log2 r) (r <= 1, so P stays <= 2^8 in f16), the row sum
//    taking P / r and the output O * v_ref / l.  PV runs in f16 (kind::f16).
//  * CTA: 16 warps -- 0-7 softmax (two heads), 8 MMA issue, 9 TMA, 10-15
//    converters -- with a setmaxnreg split of 208 / 48 on a 128-register launch.
//  * The output is written in q's dtype.
namespace f8 {
constexpr int kCodeTile = kBN * kD;                  // 16 KB of codes per 128-key tile
constexpr int kOffQ = 0;                             // per head: hi rows | lo rows
constexpr int kOffKc = 2 * kTile;                    // K codes, two slots
constexpr int kOffVc = kOffKc + 2 * kCodeTile;       // V codes, two slots
constexpr int kOffV = kOffVc + 2 * kCodeTile;        // two f16 V stages
constexpr int kTilesBytes = kOffV + 2 * kTile;       // 192 KB
enum Bar {
  kQ = 0, kQ8 = 1, kKc = 2, kVc = 4, kFreeK = 6, kVcFree = 8, kV16 = 10, kFreeV = 12,
  kS = 14, kP = 16, kPV = 18, kNum = 20
};
// after the barriers: TMEM slot, abort flag, v_ref; then (k scale, v scale)
// of every page of the table row
constexpr int kOffScale = kTilesBytes + kNum * 8 + 16;
constexpr int kSmemFixed = 1024 + kOffScale;        // + 8 bytes per page of the table row
// Warps 0-7 softmax, 8 MMA issue, 9 TMA, 10 .. 10 + kConvWarps - 1 widen V.
// Register split (setmaxnreg): launch kRegsLaunch a thread; the softmax
// warpgroups rise to kRegsSoftmax, every other warp drops to kRegsIssue.
constexpr int kConvWarps = 6;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kThreads = (10 + kConvWarps) * 32;
constexpr int kRegsLaunch = 128, kRegsIssue = 48, kRegsSoftmax = 208;
static_assert(2 * 128 * kRegsSoftmax + (kThreads - 256) * kRegsIssue <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");
static_assert(kThreads * kRegsLaunch <= 65536, "launch allocation exceeds the register file");
}  // namespace f8

// Widen one 128-key tile of E4M3 codes (128-byte rows, 128-byte swizzle) into
// the f16 operand layout (two 64-dim halves of 128-byte rows, 128-byte
// swizzle), rows >= valid written as zeros.  Thread ct of the kConvThreads
// converters takes 16-code chunks g = ct, ct + kConvThreads, ...: chunk
// (g >> 3) & 7 of row (g & 7) + 8 (g >> 6), so the 8 lanes of a shared-memory
// phase touch one chunk of 8 consecutive rows, whose swizzled positions are
// all distinct for the load and for both stores (no bank conflict).
__device__ __forceinline__ void widen_tile(const uint8_t *codes, uint8_t *dst, int ct, int valid) {
#pragma unroll 4
  for (int g = ct; g < kBN * 8; g += f8::kConvThreads) {
    const int row = (g & 7) | ((g >> 6) << 3), c = (g >> 3) & 7;
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    if (row < valid) {
      const uint4 w = *reinterpret_cast<const uint4 *>(codes + swz128(row, c));
      lo.x = e4m3x2_to_f16x2(w.x & 0xffffu);
      lo.y = e4m3x2_to_f16x2(w.x >> 16);
      lo.z = e4m3x2_to_f16x2(w.y & 0xffffu);
      lo.w = e4m3x2_to_f16x2(w.y >> 16);
      hi.x = e4m3x2_to_f16x2(w.z & 0xffffu);
      hi.y = e4m3x2_to_f16x2(w.z >> 16);
      hi.z = e4m3x2_to_f16x2(w.w & 0xffffu);
      hi.w = e4m3x2_to_f16x2(w.w >> 16);
    }
    uint8_t *half = dst + (c >> 2) * kHalf;
    *reinterpret_cast<uint4 *>(half + swz128(row, 2 * (c & 3))) = lo;
    *reinterpret_cast<uint4 *>(half + swz128(row, 2 * (c & 3) + 1)) = hi;
  }
}

template <typename Tq>
__device__ __forceinline__ float2 to_float2(uint32_t u);
template <>
__device__ __forceinline__ float2 to_float2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
}
template <>
__device__ __forceinline__ float2 to_float2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&u));
}

// Two E4M3 codes (low byte first) of two fp32 values, round to nearest even,
// saturated to the finite range.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float a, float b) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

template <typename Tq>
__global__ void __launch_bounds__(f8::kThreads, 1)
    paged_prefill_fp8_kernel(const __grid_constant__ CUtensorMap qmap,
                             const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const Params p) {
  constexpr uint32_t kIdescS = tc::idesc_f16(false, false, 128, 128);   // E4M3 x E4M3 (format 0)
  constexpr uint32_t kIdescPV = tc::idesc_f16(false, true, 128, 128);   // f16, V MN-major

  const int tid = threadIdx.x, lane = tid & 31;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);
  const int pairs = p.hq >> 1;
  const int rank = blockIdx.x / pairs;
  const int h0 = 2 * (blockIdx.x - rank * pairs);
  int r, m;
  if (p.order != nullptr) {
    const int item = __ldg(p.order + rank);
    if (item < 0) return;
    r = item / p.m_tiles;
    m = item - r * p.m_tiles;
  } else {
    r = rank / p.m_tiles;
    m = p.m_tiles - 1 - (rank - r * p.m_tiles);
  }
  const int q0 = __ldg(p.cu_q + r), q_len = __ldg(p.cu_q + r + 1) - q0;
  const int k0 = __ldg(p.cu_k + r), k_len = __ldg(p.cu_k + r + 1) - k0;
  if (m * kBM >= q_len) return;
  const int hk = h0 / p.group;
  const int qk_off = k_len - q_len;
  const int last_q = min((m + 1) * kBM, q_len) - 1;
  const int need = min(k_len, qk_off + last_q + 1);
  const int nk = need > 0 ? (need + kBN - 1) / kBN : 0;
  if (nk == 0) {
    if (tid < 256) {
      const int qi = m * kBM + (tid & 127);
      if (qi < q_len) {
        Tq *orow = static_cast<Tq *>(p.out) + static_cast<int64_t>(q0 + qi) * p.out_st +
                   static_cast<int64_t>(h0 + (tid >> 7)) * p.out_sh;
        for (int d = 0; d < kD; d += 8) *reinterpret_cast<uint4 *>(orow + d) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *base_ptr = smem_raw + (base - raw);
  const uint32_t bars = base + f8::kTilesBytes;
  volatile uint32_t *tmem_slot =
      reinterpret_cast<volatile uint32_t *>(base_ptr + f8::kTilesBytes + f8::kNum * 8);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  uint32_t *v_ref_bits = const_cast<uint32_t *>(tmem_slot + 2);
  auto bar = [&](int i) { return bars + i * 8; };
  float2 *s_kv = reinterpret_cast<float2 *>(base_ptr + f8::kOffScale);
  // the row's (K scale, V scale) per page for this KV head (pages the tiles
  // reach, <= table width); v_ref = the largest V scale (0 when all are 0)
  const int npg = min((need + p.block_size - 1) / p.block_size, p.max_blocks);
  if (tid == 0) *v_ref_bits = 0u;
  __syncthreads();
  for (int pg = tid; pg < npg; pg += f8::kThreads) {
    const int32_t pid = __ldg(p.block_tables + static_cast<int64_t>(r) * p.bt_stride + pg);
    float2 kv = make_float2(0.f, 0.f);
    if (pid >= 0 && pid < p.num_blocks) {
      const int64_t si = static_cast<int64_t>(pid) * p.hkv + hk;
      kv = make_float2(__ldg(p.k_page_scale + si), __ldg(p.v_page_scale + si));
    }
    s_kv[pg] = kv;
    if (kv.y > 0.f) atomicMax(v_ref_bits, __float_as_uint(kv.y));   // non-negative floats
  }

  if (tid == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int i = 0; i < f8::kNum; ++i) {
      uint32_t count = 1;
      if (i == f8::kQ8) count = 256;
      if (i == f8::kVcFree || i == f8::kVcFree + 1 || i == f8::kV16 || i == f8::kV16 + 1)
        count = f8::kConvThreads;
      if (i == f8::kP || i == f8::kP + 1) count = 128;
      mbar_init(bar(i), count);
    }
    fence_barrier_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(const_cast<uint32_t *>(tmem_slot)), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](int i, uint32_t parity) {
    if (*abort_flag) return false;
    if (!mbar_wait(bar(i), parity)) {
      record_error(p.err, SLOKV_DEVERR_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
    return true;
  };

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(f8::kRegsIssue));
    if (warp == 9) {
      // ---------------- TMA producer: q once, then the code tiles ----------------
      if (lane == 0) {
        const uint64_t policy = l2_evict_first_policy();
        mbar_arrive_expect_tx(bar(f8::kQ), 2 * kTile);
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t dst = base + f8::kOffQ + hh * kTile;
          tma_load_4d(dst, &qmap, bar(f8::kQ), 0, h0 + hh, q0 + m * kBM, 0, policy);
          tma_load_4d(dst + kHalf, &qmap, bar(f8::kQ), 64, h0 + hh, q0 + m * kBM, 0, policy);
        }
        auto prefetch = [&](int jj) {
          if (jj >= nk) return;
          const KvCoord c = kv_coord(p, r, k0, jj);
          tma_prefetch_4d(&kmap, 0, hk, c.c2, c.c3);
          tma_prefetch_4d(&vmap, 0, hk, c.c2, c.c3);
        };
        prefetch(1);
        for (int j = 0; j < nk; ++j) {
          const int st = j & 1;
          const KvCoord c = kv_coord(p, r, k0, j);
          if (!c.ok) record_error(p.err, SLOKV_DEVERR_BLOCK_RANGE);
          prefetch(j + 2);
          // K slot st frees once both heads' S(j-2) are done, V slot st once
          // the converters have widened tile j-2
          if (j >= 2 && !wait(f8::kFreeK + st, ((j - 2) >> 1) & 1)) break;
          mbar_arrive_expect_tx(bar(f8::kKc + st), f8::kCodeTile);
          tma_load_4d(base + f8::kOffKc + st * f8::kCodeTile, &kmap, bar(f8::kKc + st), 0, hk,
                      c.c2, c.c3, policy);
          if (j >= 2 && !wait(f8::kVcFree + st, ((j - 2) >> 1) & 1)) break;
          mbar_arrive_expect_tx(bar(f8::kVc + st), f8::kCodeTile);
          tma_load_4d(base + f8::kOffVc + st * f8::kCodeTile, &vmap, bar(f8::kVc + st), 0, hk,
                      c.c2, c.c3, policy);
        }
      }
    } else if (warp >= 10) {
      // ---------------- converters: V codes -> f16 code values ----------------
      const int ct = tid - 10 * 32;
      for (int j = 0; j < nk; ++j) {
        const int st = j & 1;
        if (!wait(f8::kVc + st, (j >> 1) & 1)) break;
        if (j >= 2 && !wait(f8::kFreeV + st, ((j - 2) >> 1) & 1)) break;
        widen_tile(base_ptr + f8::kOffVc + st * f8::kCodeTile, base_ptr + f8::kOffV + st * kTile,
                   ct, k_len - j * kBN);
        fence_proxy_async_smem();
        mbar_arrive(bar(f8::kVcFree + st));
        mbar_arrive(bar(f8::kV16 + st));
      }
    } else {
      // ---------------- tensor-core issue (lane 0) ----------------
      // S_hh(j) = Q_hi K^T + Q_lo K^T over the code tile in K slot j & 1
      auto issue_s = [&](int hh, int j) {
        const uint32_t qa = base + f8::kOffQ + hh * kTile;
        const uint32_t kb = base + f8::kOffKc + (j & 1) * f8::kCodeTile;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_f8_ss(tmem + ws::kColS + hh * 128,
                          tc::smem_desc_sw128(qa + t * kHalf + kk * 32, 16, 1024),
                          tc::smem_desc_sw128(kb + kk * 32, 16, 1024), kIdescS, t | kk);
        tc::commit(bar(f8::kS + hh));
      };
      bool ok = wait(f8::kQ8, 0) && wait(f8::kKc, 0);
      if (ok && lane == 0) {
        tc::fence_after_sync();
        issue_s(0, 0);
        issue_s(1, 0);
        tc::commit(bar(f8::kFreeK));                    // K slot 0 free after both S(0)
      }
      __syncwarp();
      for (int j = 0; j < nk && ok; ++j) {
        const int st = j & 1;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          ok = wait(f8::kP + hh, j & 1);
          if (ok && hh == 0) ok = wait(f8::kV16 + st, (j >> 1) & 1);
          if (ok && lane == 0) {
            tc::fence_after_sync();
            const uint32_t vb = base + f8::kOffV + st * kTile;
            const uint32_t pa = tmem + ws::kColS + hh * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              tc::mma_f16_ts(tmem + ws::kColO + hh * 128, pa + kk * 8,
                             tc::smem_desc_sw128(vb + kk * 16 * 128, kHalf, 1024), kIdescPV,
                             (j > 0 || kk > 0) ? 1u : 0u);
            tc::commit(bar(f8::kPV + hh));
          }
          if (ok && j + 1 < nk) {
            if (hh == 0) ok = wait(f8::kKc + ((j + 1) & 1), ((j + 1) >> 1) & 1);
            if (ok && lane == 0) {
              tc::fence_after_sync();
              issue_s(hh, j + 1);
            }
          }
          __syncwarp();
        }
        if (ok && lane == 0) {
          tc::commit(bar(f8::kFreeV + st));
          if (j + 1 < nk) tc::commit(bar(f8::kFreeK + ((j + 1) & 1)));   // both heads' S(j+1)
        }
        __syncwarp();
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(f8::kRegsSoftmax));
    const int hh = warp >> 2;
    const int row = tid & 127;
    // Split this thread's query row (head hh, row `row`) into E4M3 hi / lo rows
    // scaled by 2^qe, written over the row's q (hi into the first 64-dim half's
    // 128 bytes of the row, lo into the second's).
    float qe = 0.f;
    if (wait(f8::kQ, 0)) {
      uint8_t *qrow = base_ptr + f8::kOffQ + hh * kTile;
      uint32_t w[64];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = *reinterpret_cast<const uint4 *>(qrow + (c >> 3) * kHalf + swz128(row, c & 7));
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float2 f = to_float2<Tq>(w[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      // 2^qe puts the row's largest element in [128, 256) (exponent clamped so
      // a row of denormals cannot overflow the scale)
      const int e = amax > 0.f
                        ? max(static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127, -100)
                        : 7;
      qe = static_cast<float>(7 - e);
      const float sc = exp2f(qe);
#pragma unroll
      for (int c = 0; c < 8; ++c) {        // 16-dim chunks c (hi) -> row chunk c, half 0 / 1
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a = to_float2<Tq>(w[8 * c + 2 * i]);
          const float2 b = to_float2<Tq>(w[8 * c + 2 * i + 1]);
          const float x0 = a.x * sc, x1 = a.y * sc, x2 = b.x * sc, x3 = b.y * sc;
          const uint32_t h01 = f32x2_to_e4m3x2(x0, x1), h23 = f32x2_to_e4m3x2(x2, x3);
          const uint32_t d01u = e4m3x2_to_f16x2(h01), d23u = e4m3x2_to_f16x2(h23);
          const float2 d01 = __half22float2(*reinterpret_cast<const __half2 *>(&d01u));
          const float2 d23 = __half22float2(*reinterpret_cast<const __half2 *>(&d23u));
          const uint32_t l01 = f32x2_to_e4m3x2(x0 - d01.x, x1 - d01.y);
          const uint32_t l23 = f32x2_to_e4m3x2(x2 - d23.x, x3 - d23.y);
          hi[i] = h01 | (h23 << 16);
          lo[i] = l01 | (l23 << 16);
        }
        *reinterpret_cast<uint4 *>(qrow + swz128(row, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(qrow + kHalf + swz128(row, c)) =
            make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async_smem();
    }
    mbar_arrive(bar(f8::kQ8));
    const float v_ref = __uint_as_float(*v_ref_bits);
    const float q_unscale = exp2f(-qe);
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qi = m * kBM + row;
    const bool row_ok = qi < q_len;
    const int kmax = row_ok ? min(qk_off + qi, k_len - 1) : -1;
    const uint32_t s_addr = tmem + lane_base + ws::kColS + hh * 128;
    const uint32_t o_addr = tmem + lane_base + ws::kColO + hh * 128;
    constexpr float kSumLimit = 256.f;
    float m_run = row_ok ? -INFINITY : 0.f, l_run = 0.f;
    uint32_t s[4][32];
    bool ok = true;
    // P' = 2^(S * sl - mu + lv) of the S row in registers, packed f16 over the
    // first 64 columns of S; returns the row sum of P'.
    auto exp_store = [&](float mu, float sl, float lv) {
      const uint64_t sl2 = f32x2(sl, sl), nmu2 = f32x2(lv - mu, lv - mu);
      uint64_t rs2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t pk[32];
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          const int i = 2 * hb + (w >> 4), c = (w & 15) * 2;
          const float2 x = f32x2_split(ffma2(
              f32x2(__uint_as_float(s[i][c]), __uint_as_float(s[i][c + 1])), sl2, nmu2));
          const float a = fast_exp2(x.x);
          const float b = fast_exp2(x.y);
          rs2[w & 3] = fadd2(rs2[w & 3], f32x2(a, b));
          pk[w] = Pack<__half>::two(a, b);
        }
        tc::st32(s_addr + 32 * hb, pk);
      }
      const float2 r01 = f32x2_split(fadd2(rs2[0], rs2[1]));
      const float2 r23 = f32x2_split(fadd2(rs2[2], rs2[3]));
      return (r01.x + r01.y) + (r23.x + r23.y);
    };
    for (int j = 0; j < nk && ok; ++j) {
      ok = wait(f8::kS + hh, j & 1);
      tc::fence_after_sync();
      const int key0 = j * kBN;
      const bool full = key0 + kBN - 1 <= kmax;
      const int kpage = key0 / p.block_size;
      const float2 kv = kpage < p.max_blocks ? s_kv[kpage] : make_float2(0.f, 0.f);
      // a zero K scale (a page of zero codes) must keep masked -inf keys at -inf
      const float sl = p.scale_log2 * q_unscale * fmaxf(kv.x, 1e-30f);
      // V scale relative to v_ref (<= 1); a zero-scale page has zero codes,
      // so any factor works there and 1 keeps its P in the row sum exact
      const float rv = kv.y > 0.f ? __fdividef(kv.y, v_ref) : 1.f;
      const float irv = kv.y > 0.f ? __fdividef(v_ref, kv.y) : 1.f;
      const float lv = __log2f(rv);
#pragma unroll
      for (int i = 0; i < 4; ++i) tc::ld32(s_addr + 32 * i, s[i]);
      tc::wait_ld();
      if (!full) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (key0 + 32 * i + c > kmax) s[i][c] = 0xff800000u;
      }
      const bool fresh = __any_sync(0xffffffffu, m_run == -INFINITY);
      float alpha = 1.f, rs = 0.f;
      bool redo = fresh;
      if (!fresh) {
        rs = exp_store(m_run, sl, lv) * irv;
        redo = __any_sync(0xffffffffu, !(rs <= kSumLimit));
      }
      if (redo) {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 32; ++c) mx = fmaxf(mx, __uint_as_float(s[i][c]));
        mx *= sl;
        if (mx > m_run) {
          alpha = fast_exp2(m_run - mx);
          m_run = mx;
        }
        if (!fresh) tc::wait_st();
        rs = exp_store(m_run == -INFINITY ? 0.f : m_run, sl, lv) * irv;
      }
      l_run = l_run * alpha + rs;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int i = 0; i < 4; ++i) tc::ld32(o_addr + 32 * i, s[i]);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int c = 0; c < 32; ++c) s[i][c] = __float_as_uint(__uint_as_float(s[i][c]) * alpha);
          tc::st32(o_addr + 32 * i, s[i]);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(bar(f8::kP + hh));
    }
    ok = ok && wait(f8::kPV + hh, (nk - 1) & 1);
    tc::fence_after_sync();
    if (__all_sync(0xffffffffu, ok)) {
      // O is in units of v_ref: out = O * v_ref / l
      const float inv = l_run > 0.f ? v_ref / l_run : 0.f;
      Tq *orow = static_cast<Tq *>(p.out) + static_cast<int64_t>(q0 + qi) * p.out_st +
                 static_cast<int64_t>(h0 + hh) * p.out_sh;
#pragma unroll
      for (int i = 0; i < 4; ++i) tc::ld32(o_addr + 32 * i, s[i]);
      tc::wait_ld();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 w;
            w.x = Pack<Tq>::two(__uint_as_float(s[i][c]) * inv, __uint_as_float(s[i][c + 1]) * inv);
            w.y = Pack<Tq>::two(__uint_as_float(s[i][c + 2]) * inv, __uint_as_float(s[i][c + 3]) * inv);
            w.z = Pack<Tq>::two(__uint_as_float(s[i][c + 4]) * inv, __uint_as_float(s[i][c + 5]) * inv);
            w.w = Pack<Tq>::two(__uint_as_float(s[i][c + 6]) * inv, __uint_as_float(s[i][c + 7]) * inv);
            *reinterpret_cast<uint4 *>(orow + 32 * i + c) = w;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
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

// 4-D map {dim 128, head, row, page} with a {64, 1, 128, 1} box, 128-byte swizzle.
bool encode_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, uint64_t heads,
                uint64_t head_stride, uint64_t rows, uint64_t row_stride, uint64_t pages,
                uint64_t page_stride) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {kD, heads, rows, pages};
  cuuint64_t strides[3] = {head_stride * 2, row_stride * 2, page_stride * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, dt, 4, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map of an E4M3 code pool {dim 128, head, row, page} (bytes) with a
// {128, 1, 128, 1} box: one 128-key tile of one head, 128-byte rows, 128-byte
// swizzle.
bool encode_code_map(CUtensorMap *map, const void *base, uint64_t heads, uint64_t rows,
                     uint64_t pages, uint64_t page_stride_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {kD, heads, rows, pages};
  cuuint64_t strides[3] = {kD, heads * kD, page_stride_bytes};
  cuuint32_t box[4] = {kD, 1, kBN, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename Tq>
int launch_fp8(const Params &p, const CUtensorMap &qm, const CUtensorMap &km,
               const CUtensorMap &vm, int rows, cudaStream_t stream) {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    cudaFuncAttributes fa;
    // the register split hands out exactly the launch allocation (see f8::kRegsLaunch)
    ok = cudaFuncSetAttribute(paged_prefill_fp8_kernel<Tq>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, ws::kSmemMax) ==
             cudaSuccess &&
         cudaFuncGetAttributes(&fa, paged_prefill_fp8_kernel<Tq>) == cudaSuccess &&
         fa.numRegs == f8::kRegsLaunch;
  });
  if (!ok) return SLOKV_ERR_UNSUPPORTED;
  const int64_t smem = f8::kSmemFixed + 8 * static_cast<int64_t>(p.max_blocks);
  if (smem > ws::kSmemMax) return SLOKV_ERR_UNSUPPORTED;
  if (p.order != nullptr)
    prefill_schedule_kernel<<<1, kSchedThreads, 0, stream>>>(p.cu_q, p.cu_k, rows, p.m_tiles,
                                                               const_cast<int32_t *>(p.order));
  const int64_t blocks = static_cast<int64_t>(rows) * p.m_tiles * (p.hq / 2);
  if (blocks > 0x7fffffff) return SLOKV_ERR_UNSUPPORTED;
  paged_prefill_fp8_kernel<Tq><<<static_cast<unsigned>(blocks), f8::kThreads,
                                 static_cast<unsigned>(smem), stream>>>(qm, km, vm, p);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

template <typename T>
int launch(const Params &p, const CUtensorMap &qm, const CUtensorMap &km, const CUtensorMap &vm,
           int rows, int max_q, cudaStream_t stream) {
  static std::once_flag once;
  static bool ok = false, ws_ok = false, ws_scaled_ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(paged_prefill_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes) == cudaSuccess &&
         cudaFuncSetAttribute(paged_prefill_ws_kernel<T, false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, ws::kSmem) == cudaSuccess &&
         cudaFuncSetAttribute(paged_prefill_ws_kernel<T, true>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, ws::kSmemMax) ==
             cudaSuccess;
    // The register split in the two-head kernel hands out exactly the launch
    // allocation; with any other per-thread count setmaxnreg.inc could not be
    // satisfied, so that kernel is used only when the build matches.
    cudaFuncAttributes fa;
    ws_ok = ok && cudaFuncGetAttributes(&fa, paged_prefill_ws_kernel<T, false>) == cudaSuccess &&
            fa.numRegs == ws::kRegsLaunch;
    ws_scaled_ok = ok &&
                   cudaFuncGetAttributes(&fa, paged_prefill_ws_kernel<T, true>) == cudaSuccess &&
                   fa.numRegs == ws::kRegsLaunch;
  });
  if (!ok) return SLOKV_ERR_CUDA;
  const bool scaled = p.k_page_scale != nullptr;
  if (scaled && !(p.group % 2 == 0 && ws_scaled_ok)) return SLOKV_ERR_UNSUPPORTED;
  const int64_t smem_scaled = ws::kSmem + 4 * static_cast<int64_t>(p.max_blocks);
  if (scaled && smem_scaled > ws::kSmemMax) return SLOKV_ERR_UNSUPPORTED;
  if (p.group % 2 == 0 && (scaled || ws_ok)) {  // two query heads of one KV head per CTA
    if (p.order != nullptr) {
      prefill_schedule_kernel<<<1, kSchedThreads, 0, stream>>>(
          p.cu_q, p.cu_k, rows, p.m_tiles, const_cast<int32_t *>(p.order));
    }
    const int64_t blocks = static_cast<int64_t>(rows) * p.m_tiles * (p.hq / 2);
    if (blocks > 0x7fffffff) return SLOKV_ERR_UNSUPPORTED;
    if (scaled)
      paged_prefill_ws_kernel<T, true><<<static_cast<unsigned>(blocks), ws::kThreads,
                                         static_cast<unsigned>(smem_scaled), stream>>>(qm, km, vm,
                                                                                        p);
    else
      paged_prefill_ws_kernel<T, false><<<static_cast<unsigned>(blocks), ws::kThreads, ws::kSmem,
                                          stream>>>(qm, km, vm, p);
  } else {
    dim3 grid((max_q + kBM - 1) / kBM, p.hq, rows);
    paged_prefill_kernel<T><<<grid, 128, kSmemBytes, stream>>>(qm, km, vm, p);
  }
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

}  // namespace prefill
}  // namespace slokv

extern "C" size_t slokv_paged_prefill_workspace_bytes(int32_t num_rows, int32_t max_seqlen_q) {
  if (num_rows <= 0 || max_seqlen_q <= 0) return 0;
  const size_t items = static_cast<size_t>(num_rows) *
                       static_cast<size_t>((max_seqlen_q + slokv::prefill::kBM - 1) /
                                           slokv::prefill::kBM);
  return (items * sizeof(int32_t) + 255) & ~static_cast<size_t>(255);
}

extern "C" int slokv_paged_prefill(void *out, int64_t out_stride_t, int64_t out_stride_h,
                                   const void *q, int64_t q_stride_t, int64_t q_stride_h,
                                   int64_t q_rows, const void *k, const void *v,
                                   int64_t kv_stride_t, int64_t v_stride_t, int64_t kv_rows,
                                   int64_t k_block_stride, int64_t v_block_stride,
                                   const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                                   int32_t num_rows, int32_t max_seqlen_q,
                                   const int32_t *block_tables, int64_t block_table_stride,
                                   int32_t max_blocks_per_seq, int32_t num_blocks,
                                   int32_t block_size, int32_t num_q_heads, int32_t num_kv_heads,
                                   int32_t head_dim, float softmax_scale, int32_t dtype,
                                   const float *k_page_scale, void *workspace,
                                   size_t workspace_bytes, uint32_t *dev_error, void *stream) {
  using namespace slokv;
  using namespace slokv::prefill;
  if (num_rows < 0 || max_seqlen_q < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (num_rows == 0 || max_seqlen_q == 0) return SLOKV_OK;
  if (head_dim != kD) return SLOKV_ERR_UNSUPPORTED;
  if (dtype != SLOKV_DTYPE_BF16 && dtype != SLOKV_DTYPE_F16) return SLOKV_ERR_UNSUPPORTED;
  if (num_q_heads % num_kv_heads) return SLOKV_ERR_INVALID_ARG;
  if (!out || !q || !k || !v || !cu_seqlens_q || !cu_seqlens_k || q_rows <= 0)
    return SLOKV_ERR_INVALID_ARG;
  const bool paged = block_tables != nullptr;
  if (paged && (block_size <= 0 || block_size % kBN || num_blocks <= 0 || max_blocks_per_seq <= 0))
    return paged && block_size % kBN ? SLOKV_ERR_UNSUPPORTED : SLOKV_ERR_INVALID_ARG;
  if (!paged && kv_rows <= 0) return SLOKV_ERR_INVALID_ARG;
  // TMA: 16-byte aligned bases and strides; 16-byte output stores.
  const uint64_t bits = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  if (bits & 15u) return SLOKV_ERR_ALIGNMENT;
  if (((q_stride_t | q_stride_h | out_stride_t | out_stride_h) * 2) & 15) return SLOKV_ERR_ALIGNMENT;
  if (paged ? (((k_block_stride | v_block_stride) * 2) & 15) : (((kv_stride_t | v_stride_t) * 2) & 15))
    return SLOKV_ERR_ALIGNMENT;

  const CUtensorMapDataType dt =
      dtype == SLOKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap qm, km, vm;
  const uint64_t hkv = static_cast<uint64_t>(num_kv_heads);
  bool ok = encode_map(&qm, q, dt, num_q_heads, q_stride_h, q_rows, q_stride_t, 1,
                       q_rows * q_stride_t);
  if (paged) {
    ok = ok && encode_map(&km, k, dt, hkv, kD, block_size, hkv * kD, num_blocks, k_block_stride) &&
         encode_map(&vm, v, dt, hkv, kD, block_size, hkv * kD, num_blocks, v_block_stride);
  } else {
    ok = ok && encode_map(&km, k, dt, hkv, kD, kv_rows, kv_stride_t, 1, kv_rows * kv_stride_t) &&
         encode_map(&vm, v, dt, hkv, kD, kv_rows, v_stride_t, 1, kv_rows * v_stride_t);
  }
  if (!ok) return SLOKV_ERR_CUDA;

  Params p;
  p.out = out;
  p.out_st = out_stride_t;
  p.out_sh = out_stride_h;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  p.m_tiles = (max_seqlen_q + kBM - 1) / kBM;
  p.k_page_scale = k_page_scale;
  p.v_page_scale = nullptr;
  // page scales are applied by the two-head kernel only (even GQA groups, paged)
  if (k_page_scale != nullptr && (p.group % 2 != 0 || !paged)) return SLOKV_ERR_UNSUPPORTED;
  // The work order needs rows x m_tiles int32 (slokv_paged_prefill_workspace_bytes);
  // without it the tiles run in row-major order.
  p.order = workspace != nullptr &&
                    workspace_bytes >= slokv_paged_prefill_workspace_bytes(num_rows, max_seqlen_q) &&
                    (reinterpret_cast<uintptr_t>(workspace) & 3u) == 0
                ? static_cast<const int32_t *>(workspace)
                : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == SLOKV_DTYPE_BF16
             ? launch<__nv_bfloat16>(p, qm, km, vm, num_rows, max_seqlen_q, st)
             : launch<__half>(p, qm, km, vm, num_rows, max_seqlen_q, st);
}

extern "C" int slokv_paged_prefill_fp8(void *out, int64_t out_stride_t, int64_t out_stride_h,
                                       const void *q, int64_t q_stride_t, int64_t q_stride_h,
                                       int64_t q_rows, const void *k_codes, const void *v_codes,
                                       int64_t k_block_stride, int64_t v_block_stride,
                                       const float *k_scale, const float *v_scale,
                                       const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                                       int32_t num_rows, int32_t max_seqlen_q,
                                       const int32_t *block_tables, int64_t block_table_stride,
                                       int32_t max_blocks_per_seq, int32_t num_blocks,
                                       int32_t block_size, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_dim,
                                       float softmax_scale, int32_t q_dtype, void *workspace,
                                       size_t workspace_bytes, uint32_t *dev_error, void *stream) {
  using namespace slokv;
  using namespace slokv::prefill;
  if (num_rows < 0 || max_seqlen_q < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (num_rows == 0 || max_seqlen_q == 0) return SLOKV_OK;
  if (head_dim != kD) return SLOKV_ERR_UNSUPPORTED;
  if (q_dtype != SLOKV_DTYPE_BF16 && q_dtype != SLOKV_DTYPE_F16) return SLOKV_ERR_UNSUPPORTED;
  if (num_q_heads % num_kv_heads) return SLOKV_ERR_INVALID_ARG;
  if ((num_q_heads / num_kv_heads) % 2) return SLOKV_ERR_UNSUPPORTED;   // two heads per CTA
  if (!out || !q || !k_codes || !v_codes || !k_scale || !v_scale || !cu_seqlens_q ||
      !cu_seqlens_k || !block_tables || q_rows <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (block_size <= 0 || block_size % kBN) return SLOKV_ERR_UNSUPPORTED;
  const uint64_t bits = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                        reinterpret_cast<uintptr_t>(k_codes) | reinterpret_cast<uintptr_t>(v_codes);
  if (bits & 15u) return SLOKV_ERR_ALIGNMENT;
  if (((q_stride_t | q_stride_h | out_stride_t | out_stride_h) * 2) & 15) return SLOKV_ERR_ALIGNMENT;
  if ((k_block_stride | v_block_stride) & 15) return SLOKV_ERR_ALIGNMENT;   // bytes (codes)

  const CUtensorMapDataType dt = q_dtype == SLOKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap qm, km, vm;
  const uint64_t hkv = static_cast<uint64_t>(num_kv_heads);
  if (!encode_map(&qm, q, dt, num_q_heads, q_stride_h, q_rows, q_stride_t, 1,
                  q_rows * q_stride_t) ||
      !encode_code_map(&km, k_codes, hkv, block_size, num_blocks, k_block_stride) ||
      !encode_code_map(&vm, v_codes, hkv, block_size, num_blocks, v_block_stride))
    return SLOKV_ERR_CUDA;
  Params p;
  p.out = out;
  p.out_st = out_stride_t;
  p.out_sh = out_stride_h;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  p.m_tiles = (max_seqlen_q + kBM - 1) / kBM;
  p.k_page_scale = k_scale;
  p.v_page_scale = v_scale;
  p.order = workspace != nullptr &&
                    workspace_bytes >= slokv_paged_prefill_workspace_bytes(num_rows, max_seqlen_q) &&
                    (reinterpret_cast<uintptr_t>(workspace) & 3u) == 0
                ? static_cast<const int32_t *>(workspace)
                : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return q_dtype == SLOKV_DTYPE_BF16 ? launch_fp8<__nv_bfloat16>(p, qm, km, vm, num_rows, st)
                                     : launch_fp8<__half>(p, qm, km, vm, num_rows, st);
}
