// Row-parallel linear layer fused with its tensor-parallel all-reduce: the
// o_proj / down_proj step of every decoder layer
// (nanovllm/layers/linear.py:152-156: y = F.linear(x, W_rank) then
// dist.all_reduce(y) over the TP group), as ONE persistent kernel per rank.
//
// Phase 1 (GEMM).  The rank's partial Y_r = X_r W_r^T is computed in 128 x 128
// output tiles on the 5th-generation tensor cores, stream-K: the K loops of all
// tiles (tiles x K/64 chunk units) are split evenly over up to one CTA per SM,
// so a decode-sized problem (a few dozen tiles) still fills all 148 SMs.  A TMA
// warp streams 128 x 64 slices of X and W (128-byte swizzle) through a 4-stage
// shared-memory ring, one elected thread issues tcgen05.mma (kind::f16, M = N =
// 128, K = 16) into one of two TMEM accumulators, and four epilogue warps read
// the finished accumulator.  A CTA whose range ends inside a tile writes that
// segment's fp32 sum to its fix-up slot (this GPU's memory) and flags it; the
// CTA that reaches the tile's last chunk adds its predecessors' fix-up sums in
// CTA order (it processes that segment last, so no wait can cycle).  The
// finished tile's epilogue then reads
// the whole tile's fp32 sum, rounds it to 16 bits once (the reference's
// per-rank F.linear output is rounded the same way) and stages it in shared
// memory; one thread then
// pushes the staged 32 KB tile with a single plain bulk copy (cp.async.bulk,
// shared to global) into the symmetric buffer of the tile's owner rank (tile % world)
// over NVLink peer memory.  The MMA of the next tile overlaps the epilogue of
// this one.  When its last tile is out, the CTA waits for its copies, issues
// ONE system-scope fence and sets the owners' flags with relaxed stores (a
// system-scope fence costs microseconds here, so it is paid once per CTA and
// phase, not per tile).
//
// Phase 2 (owner reduce), in 32-row quarter tiles spread over all CTAs.  For
// each quarter it owns, a rank waits for the partial flags of every source
// rank, loads the world partial slices at once (world x 3 16-byte loads in
// flight per thread), sums them in fp32 in rank order (plus the bias, once),
// rounds once, writes its own Y rows, stages the quarter and bulk-copies the
// 8 KB into every peer's result slot; the CTA's flags follow one fence, as in
// phase 1.
//
// Phase 3.  Every rank copies the reduced quarters it does not own from its own
// result slots (written by their owners) into Y.
//
// Two shots (reduce-scatter then all-gather) move 2 (world - 1) / world of Y
// over NVLink per rank, the ring all-reduce volume, but with one hop each and
// with the first shot overlapping the GEMM tile by tile.  Every rank ends with
// bit-identical Y.  All loads are from this GPU's own memory (X, W, its
// symmetric buffer); only stores cross NVLink.  Every TMA load is a plain
// single-CTA load of local memory.
//
// Large GEMMs (>= 2^34 multiply-adds per call) run phase 1 on CTA pairs
// instead (row_parallel_pair_kernel: clusters of two CTAs, 256 x 256 tiles,
// tcgen05.mma.cta_group::2), which halves the operand bytes per output; the
// tiles they produce are 128 x 128 halves, so phases 2 and 3 are shared.
//
// The world size is a template parameter (1, 2, 4 or 8: the TP sizes of the
// 8-KV-head model), so the per-source loops unroll into independent loads.
//
// Flags carry a per-call epoch (a device counter advanced by the last CTA of
// each call), so nothing is reset between calls and the call is CUDA-graph
// capturable.  Every wait is bounded (kWaitLimitNs); a wait that gives up sets
// SLOKV_DEVERR_TIMEOUT and the CTA skips its remaining work.  The grid never
// exceeds one CTA per SM and is launched cooperatively, so every CTA is
// resident and the phase-2/3 waits (which only depend on other CTAs' phase 1/2
// work) always end.  One launch may also run several ranks as virtual ranks
// over buffers of this GPU (tests run the whole exchange on one GPU this way).
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

#include <cudaTypedefs.h>

namespace slokv {
namespace rp {

constexpr int kBM = 128, kBN = 128, kBK = 64;
constexpr int kStages = 4;
constexpr uint32_t kSlice = kBM * kBK * 2;         // 16 KB: 128 rows x 64 elements
constexpr uint32_t kStageBytes = 2 * kSlice;       // X slice + W slice
constexpr uint32_t kTileBytes = kBM * kBN * 2;     // 32 KB output tile
constexpr int kChunks = kTileBytes / 16;           // 16-byte chunks per tile
constexpr int kQuarters = 4;                       // exchange unit: 32 rows of a tile
constexpr int kQRows = kBM / kQuarters;
constexpr uint32_t kQBytes = kTileBytes / kQuarters;
constexpr int kQChunks = kChunks / kQuarters;      // 512
constexpr int kThreads = 192;                      // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int kEpiThreads = 128;
constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 160;                      // >= SMs per GPU (fix-up slots)
constexpr int kMinChunks = 4;                      // K chunks per CTA at least
constexpr int64_t kPairMinMacs = int64_t(1) << 34;  // GEMM size from which CTA pairs run
constexpr uint32_t kFixBytes = kBM * 2 * kBN * 4;  // fp32 fix-up slot of one CTA (pair width)
constexpr uint32_t kTmemCols = 256;                // two 128-column accumulators
constexpr uint32_t kOffStaging = kStages * kStageBytes;
constexpr uint32_t kOffBars = kOffStaging + kTileBytes;
constexpr int kNumBars = 2 * kStages + 4;          // full, empty, acc_full[2], acc_empty[2]
constexpr uint32_t kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;

// CTA-pair variant (tcgen05.mma.cta_group::2): a pair of CTAs on two SMs
// computes a 256 x 256 output tile, CTA r of the pair holding rows 128 r ..
// 128 r + 127 of it in its own TMEM (256 fp32 columns per accumulator, two
// accumulators = all 512 columns).  Each CTA streams its own 128 rows of X and
// its own 128 of the tile's 256 W rows per 64-deep K chunk (32 KB per stage, as
// above), so operand bytes per output element are half the single-CTA tile's.
constexpr int kPBN = 2 * kBN;                      // output columns of a pair tile
constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPOffBars = kOffStaging + 2 * kTileBytes;   // two staged 128 x 128 halves
constexpr int kPNumBars = 2 * kStages + 5;         // full, empty, acc_full[2], acc_empty[2], drain
constexpr uint32_t kPSmemBytes = kPOffBars + kPNumBars * 8 + 16 + 1024;
static_assert(kPSmemBytes <= 227 * 1024, "pair kernel shared memory");

struct Maps {
  CUtensorMap x[kMaxRanks];  // per local rank: X [tokens, K]
  CUtensorMap w[kMaxRanks];  // per local rank: W [N, K]
};

struct Params {
  int tokens, n, k;
  int m_tiles, n_tiles, tiles, k_chunks;
  int world, rank_base, ctas_per_rank;
  int gemm_ctas;                       // CTAs 0 .. gemm_ctas - 1 of a rank run phase 1
  int owned_max;                       // partial slots per source rank
  int64_t y_stride;                    // elements
  void *y[kMaxRanks];                  // per local rank
  const void *bias[kMaxRanks];         // per local rank, [N] or null
  uint8_t *buf[kMaxRanks];             // every rank's symmetric buffer, mapped here
  int64_t off_partial, off_result, off_pflag, off_rflag, off_fix, off_fixflag;
  uint32_t *state;                     // [2]: completed calls, CTAs done in this call
  uint32_t *err;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *f) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

// OR of `v` over the 128 epilogue threads (named barrier 1): every epilogue
// thread gets the same answer, so they leave their loop together.
__device__ __forceinline__ bool epi_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

// Bounded wait until *f has reached `epoch` (modular comparison).
__device__ __forceinline__ bool wait_flag(const uint32_t *f, uint32_t epoch) {
  if (static_cast<int32_t>(ld_acquire_sys(f) - epoch) >= 0) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    __nanosleep(100);
    if (static_cast<int32_t>(ld_acquire_sys(f) - epoch) >= 0) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// Bulk copy of `bytes` from this CTA's shared memory to global memory (here: a
// peer's symmetric buffer), tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_store(void *dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(src), "r"(bytes)
               : "memory");
}
// Close the current bulk group and wait until its shared-memory source has
// been read (the staging buffer may then be refilled; the writes may still be
// in flight).
__device__ __forceinline__ void bulk_commit_wait_read() {
  asm volatile(
      "cp.async.bulk.commit_group;\n\t"
      "cp.async.bulk.wait_group.read 0;" ::
          : "memory");
}
// Wait until every bulk copy this thread issued has completed (its writes are
// performed), order them before this thread's later generic accesses, and
// issue one system-scope fence: relaxed flag stores after it publish every
// copy before it.  A system-scope fence costs microseconds on B200 across
// NVLink, so each CTA pays it once per phase rather than once per tile.
__device__ __forceinline__ void bulk_publish_fence() {
  asm volatile(
      "cp.async.bulk.wait_group 0;\n\t"
      "fence.proxy.async;\n\t"
      "fence.acq_rel.sys;" ::
          : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t *f, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *f) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t *f, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ bool wait_flag_gpu(const uint32_t *f, uint32_t epoch) {
  if (static_cast<int32_t>(ld_acquire_gpu(f) - epoch) >= 0) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if (static_cast<int32_t>(ld_acquire_gpu(f) - epoch) >= 0) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---- CTA-pair primitives ------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the object at shared::cta address `addr` in CTA
// `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Every thread of both CTAs arrives, then waits (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
// Arrive on an mbarrier of either CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
// 2-D tile load into THIS CTA's shared memory whose completion is signalled on
// an mbarrier that may live in the other CTA of the pair (`cluster_bar`, a
// shared::cluster address): both CTAs' loads complete on the leader's barrier.
// A plain load of local memory (no cross-CTA delivery of the data).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map,
                                                 uint32_t cluster_bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (both CTAs' TMEM, 256 rows) (+)= A (128 rows from each CTA) * B (N / 2
// rows from each CTA); issued by one thread of the leader CTA.
__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at shared::cta offset `bar` of every CTA in
// `cta_mask` when the pair MMAs issued so far have completed.
__device__ __forceinline__ void commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// ---- fix-up streaming ---------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The predecessors' fp32 fix-up sums of a finishing segment, streamed through
// the CTA's stage ring (idle by then: a segment with predecessors is always
// the CTA's last, and its accumulator-full signal means every MMA has read its
// operands).  Block b = q * npred + p is the 16 KB run [8 float4 groups][128
// rows] of column block q in predecessor p's slot (contiguous in the slot
// layout); it lands in ring slot b % kFixRing.  Each epilogue thread issues 8
// of its 16-byte copies, one cp.async group per block (empty past the end), so
// kFixRing blocks are in flight while earlier ones are added.
constexpr int kFixRing = 8;                          // 8 x 16 KB = the 128 KB stage ring
constexpr uint32_t kFixBlock = 8 * kBM * 16;         // 16 KB
static_assert(kFixRing * kFixBlock <= kStages * kStageBytes, "fix-up ring fits the stages");
struct FixStream {
  uint32_t ring;          // shared address of the stage ring
  const uint8_t *fix;     // this rank's fix-up region
  int first, npred;       // predecessors first .. first + npred - 1
  int step, offset;       // slot of predecessor c: c * step + offset
  int total;              // blocks: column blocks x npred
  __device__ __forceinline__ void issue(int b, int tid) const {
    if (b < total) {
      const int q = b / npred, pr = b - q * npred;
      const uint8_t *src = fix + static_cast<int64_t>((first + pr) * step + offset) * kFixBytes +
                           static_cast<int64_t>(q) * kFixBlock;
      const uint32_t dst = ring + (b % kFixRing) * kFixBlock;
#pragma unroll
      for (int i = 0; i < static_cast<int>(kFixBlock / 16) / kEpiThreads; ++i)
        cp_async16(dst + (tid + i * kEpiThreads) * 16, src + (tid + i * kEpiThreads) * 16);
    }
    cp_async_commit();
  }
  // v[32] (column block q of row `row`) += every predecessor's sum, in
  // predecessor order; all epilogue threads call it for the same q.
  __device__ __forceinline__ void add(float (&v)[32], int q, int row, int tid,
                                      const uint8_t *smem) const {
    for (int pr = 0; pr < npred; ++pr) {
      const int b = q * npred + pr;
      cp_async_wait<kFixRing - 1>();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      const float4 *blk =
          reinterpret_cast<const float4 *>(smem + (b % kFixRing) * kFixBlock) + row;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 f = blk[j * kBM];
        v[4 * j] += f.x;
        v[4 * j + 1] += f.y;
        v[4 * j + 2] += f.z;
        v[4 * j + 3] += f.w;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      issue(b + kFixRing, tid);
    }
  }
};

// One CTA's stream-K range [beg, end) of chunk units (unit = tile * kc + k
// chunk), cut into per-tile segments.  Segment j of the natural order covers
// tile t0 + j; when the first one continues a tile begun by earlier CTAs (it
// then also finishes it, as the range goes on), it is processed last.
struct Seg {
  int tile, kc0, kc1;
};
struct Sched {
  int64_t beg, end;
  int kc, n, t0;
  bool defer;
  __device__ __forceinline__ Seg get(int i) const {
    const int j = defer ? (i + 1 == n ? 0 : i + 1) : i;
    Seg s;
    s.tile = t0 + j;
    s.kc0 = j == 0 ? static_cast<int>(beg - static_cast<int64_t>(t0) * kc) : 0;
    s.kc1 = j == n - 1 ? static_cast<int>(end - static_cast<int64_t>(t0 + n - 1) * kc) : kc;
    return s;
  }
};
__device__ __forceinline__ int64_t unit_begin(int cta, int ctas, int64_t units) {
  return static_cast<int64_t>(cta) * units / ctas;
}
__device__ __forceinline__ Sched make_sched(int cta, int ctas, int64_t units, int kc) {
  Sched s;
  s.beg = unit_begin(cta, ctas, units);
  s.end = cta < ctas ? unit_begin(cta + 1, ctas, units) : s.beg;   // CTAs past `ctas`: none
  s.kc = kc;
  if (s.end <= s.beg) {
    s.n = 0;
    s.t0 = 0;
    s.defer = false;
    return s;
  }
  s.t0 = static_cast<int>(s.beg / kc);
  s.n = static_cast<int>((s.end - 1) / kc) - s.t0 + 1;
  s.defer = s.n > 1 && s.beg > static_cast<int64_t>(s.t0) * kc;
  return s;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<__half2 *>(&u));
}

// Y row-major store of 16-byte chunk `c` (0..2047) of tile (m, nt), rows >= tokens skipped.
__device__ __forceinline__ void store_y_chunk(const Params &p, void *y, int m, int nt, int c,
                                              uint4 v) {
  const int row = c >> 4;
  const int tok = m * kBM + row;
  if (tok >= p.tokens) return;
  uint8_t *dst = static_cast<uint8_t *>(y) +
                 (static_cast<int64_t>(tok) * p.y_stride + nt * kBN + (c & 15) * 8) * 2;
  *reinterpret_cast<uint4 *>(dst) = v;
}

// Phases 2 and 3 of one call, run by every thread of a CTA after its phase-1
// work: reduce the quarter tiles this rank owns (waiting for every source
// rank's partial), push them to the peers, then copy the quarters the peers
// own into Y.  Shared by the single-CTA and the CTA-pair kernels; `stage` is
// 32 KB of this CTA's shared memory.
template <typename T, int W>
__device__ __forceinline__ void exchange_phases(const Params &p, uint8_t *stage, int lr, int cta,
                                                int rank, uint32_t epoch,
                                                volatile uint32_t *abort_flag) {
  const int tid = threadIdx.x;
  constexpr int world = W;
  constexpr bool kOneShot = W == 2;
  auto fail = [&]() {
    record_error(p.err, SLOKV_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };
  // ---------------- phase 2: reduce the quarters this rank owns ----------------
  // (abort_flag is stable here: every writer has passed the barrier above, and
  // below it only changes before a __syncthreads_or that all threads read)
  if (world > 1 && !*abort_flag) {
    const T *bias = static_cast<const T *>(p.bias[lr]);
    uint8_t *own = p.buf[rank];
    const uint32_t *pflags = reinterpret_cast<const uint32_t *>(own + p.off_pflag);
    int done = 0;
    for (int u = cta;; u += p.ctas_per_rank) {
      const int slot = u / kQuarters, q = u - slot * kQuarters;
      const int tile = kOneShot ? slot : slot * world + rank;
      if (tile >= p.tiles) break;
      const int m = tile / p.n_tiles, nt = tile - (tile / p.n_tiles) * p.n_tiles;
      if (m * kBM + q * kQRows >= p.tokens) continue;   // all padding rows: nobody waits
      const bool bad =
          tid < world && !wait_flag(pflags + static_cast<int64_t>(tid) * p.owned_max + slot, epoch);
      if (__syncthreads_or(bad)) {
        if (tid == 0) fail();
        break;
      }
      // chunk cl (0..511) of the quarter: row q * 32 + cl / 16, 16-byte column cl % 16
      constexpr int kPer = (kQChunks + kThreads - 1) / kThreads;   // 3
      uint4 v[kPer][W];
#pragma unroll
      for (int b = 0; b < kPer; ++b) {
        const int cl = tid + b * kThreads;
        if (cl < kQChunks) {
          const int row = q * kQRows + (cl >> 4), cc = cl & 15;
          const int64_t off = row * 256 + ((cc ^ (row & 7)) << 4);
#pragma unroll
          for (int src = 0; src < W; ++src)
            v[b][src] = __ldcg(reinterpret_cast<const uint4 *>(
                own + p.off_partial + (static_cast<int64_t>(src) * p.owned_max + slot) * kTileBytes +
                off));
        }
      }
#pragma unroll
      for (int b = 0; b < kPer; ++b) {
        const int cl = tid + b * kThreads;
        if (cl >= kQChunks) continue;
        const int row = q * kQRows + (cl >> 4), cc = cl & 15;
        float acc[8];
        if (bias != nullptr) {
          const uint4 bv = __ldg(reinterpret_cast<const uint4 *>(bias + nt * kBN + cc * 8));
          const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack2<T>(bw[j]);
            acc[2 * j] = f.x;
            acc[2 * j + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        }
#pragma unroll
        for (int src = 0; src < W; ++src) {
          const uint32_t vw[4] = {v[b][src].x, v[b][src].y, v[b][src].z, v[b][src].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack2<T>(vw[j]);
            acc[2 * j] += f.x;
            acc[2 * j + 1] += f.y;
          }
        }
        uint4 o;
        o.x = pack2<T>(acc[0], acc[1]);
        o.y = pack2<T>(acc[2], acc[3]);
        o.z = pack2<T>(acc[4], acc[5]);
        o.w = pack2<T>(acc[6], acc[7]);
        store_y_chunk(p, p.y[lr], m, nt, row * 16 + cc, o);
        if (!kOneShot) reinterpret_cast<uint4 *>(stage)[cl] = o;     // quarter, row-major
      }
      if (kOneShot) continue;      // every rank reduced this quarter itself
      __syncthreads();
      if (tid == 0) {
        fence_proxy_async_smem();
#pragma unroll
        for (int k = 1; k < W; ++k) {
          const int peer = (rank + k) % world;
          bulk_store(p.buf[peer] + p.off_result + static_cast<int64_t>(tile) * kTileBytes +
                         q * kQBytes,
                     smem_u32(stage), kQBytes);
        }
        bulk_commit_wait_read();
      }
      ++done;
      __syncthreads();   // the staging quarter is free again
    }
    if (!kOneShot && tid == 0 && done > 0) {  // publish this CTA's reduced quarters
      bulk_publish_fence();
      int k = 0;
      for (int u = cta; k < done; u += p.ctas_per_rank) {
        const int slot = u / kQuarters, q = u - slot * kQuarters;
        const int tile = slot * world + rank;
        const int m = tile / p.n_tiles;
        if (m * kBM + q * kQRows >= p.tokens) continue;
        ++k;
#pragma unroll
        for (int j = 1; j < W; ++j) {
          const int peer = (rank + j) % world;
          st_relaxed_sys(reinterpret_cast<uint32_t *>(p.buf[peer] + p.off_rflag) +
                             tile * kQuarters + q,
                         epoch);
        }
      }
    }
  }
  __syncthreads();
  if (world > 1 && !kOneShot && !*abort_flag) {
    // ---------------- phase 3: copy the quarters owned by peers ----------------
    const uint8_t *results = p.buf[rank] + p.off_result;
    const uint32_t *rflags = reinterpret_cast<const uint32_t *>(p.buf[rank] + p.off_rflag);
    for (int i = cta;; i += p.ctas_per_rank) {
      const int nb = i / kQuarters, q = i - nb * kQuarters;
      constexpr int kPeers = W > 1 ? W - 1 : 1;      // (phase 3 only runs for W > 1)
      const int blk = nb / kPeers, r = nb - blk * kPeers;
      const int tile = blk * world + r + (r >= rank ? 1 : 0);
      if (blk * world >= p.tiles) break;
      if (tile >= p.tiles) continue;
      const int m = tile / p.n_tiles, nt = tile - (tile / p.n_tiles) * p.n_tiles;
      if (m * kBM + q * kQRows >= p.tokens) continue;
      if (__syncthreads_or(tid == 0 && !wait_flag(rflags + tile * kQuarters + q, epoch))) {
        if (tid == 0) fail();
        break;
      }
      constexpr int kPer = (kQChunks + kThreads - 1) / kThreads;
      uint4 v[kPer];
      const uint4 *src = reinterpret_cast<const uint4 *>(
          results + static_cast<int64_t>(tile) * kTileBytes + q * kQBytes);
#pragma unroll
      for (int b = 0; b < kPer; ++b) {
        const int cl = tid + b * kThreads;
        if (cl < kQChunks) v[b] = __ldcg(src + cl);
      }
#pragma unroll
      for (int b = 0; b < kPer; ++b) {
        const int cl = tid + b * kThreads;
        if (cl < kQChunks) store_y_chunk(p, p.y[lr], m, nt, q * kQChunks + cl, v[b]);
      }
    }
  }
}

// The last CTA of the call advances the epoch (nothing is reset between calls).
__device__ __forceinline__ void advance_epoch(const Params &p, uint32_t epoch) {
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.state + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.state + 1, 0u);
      __threadfence();
      atomicExch(p.state, epoch);
    }
  }
}

template <typename T, int W>
__global__ void __launch_bounds__(kThreads, 1)
    row_parallel_kernel(const __grid_constant__ Params p, const __grid_constant__ Maps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t base = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBars);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBars + kNumBars * 8);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = 2 * kStages + 2;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lr = blockIdx.x / p.ctas_per_rank;  // local (virtual) rank of this CTA
  const int cta = blockIdx.x - lr * p.ctas_per_rank;
  const int rank = p.rank_base + lr;
  constexpr int world = W;
  // two ranks: one shot (each rank pushes its partial to both and reduces every
  // tile itself, same NVLink volume as two shots and one flag round less)
  constexpr bool kOneShot = W == 2;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t *>(p.state) + 1u;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = tc::idesc_f16(kBf16, false, kBM, kBN);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(kFull + i), 1);
      mbar_init(bar(kEmpty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kAccFull + i), 1);
      mbar_init(bar(kAccEmpty + i), 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    record_error(p.err, SLOKV_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };

  // ---------------- phase 1: stream-K GEMM -> owner partial slots ----------------
  const Sched sched = make_sched(cta < p.gemm_ctas ? cta : p.gemm_ctas, p.gemm_ctas,
                                 static_cast<int64_t>(p.tiles) * p.k_chunks, p.k_chunks);
  if (warp == 4) {
    if (lane == 0) {  // TMA producer
      prefetch_tensormap(&maps.x[lr]);
      prefetch_tensormap(&maps.w[lr]);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < sched.n && !*abort_flag; ++i) {
        const Seg sg = sched.get(i);
        const int m = sg.tile / p.n_tiles, nt = sg.tile - m * p.n_tiles;
        for (int kc = sg.kc0; kc < sg.kc1; ++kc) {
          if (!mbar_wait(bar(kEmpty + s), ph ^ 1)) { fail(); break; }
          const uint32_t dst = base + s * kStageBytes;
          mbar_arrive_expect_tx(bar(kFull + s), kStageBytes);
          tma_load_2d(dst, &maps.x[lr], bar(kFull + s), kc * kBK, m * kBM);
          tma_load_2d(dst + kSlice, &maps.w[lr], bar(kFull + s), kc * kBK, nt * kBN);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {  // MMA issuer
      int s = 0;
      uint32_t ph = 0;
      for (int it = 0; it < sched.n && !*abort_flag; ++it) {
        const Seg sg = sched.get(it);
        const int acc = it & 1;
        if (!mbar_wait(bar(kAccEmpty + acc), ((it >> 1) & 1) ^ 1)) { fail(); break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + acc * kBN;
        bool ok = true;
        for (int kc = sg.kc0; kc < sg.kc1; ++kc) {
          if (!mbar_wait(bar(kFull + s), ph)) { fail(); ok = false; break; }
          tc::fence_after_sync();
          const uint32_t a = base + s * kStageBytes, b = a + kSlice;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::mma_f16_ss(d, tc::smem_desc_sw128(a + kk * 32, 16, 1024),
                           tc::smem_desc_sw128(b + kk * 32, 16, 1024), kIdesc,
                           (kc - sg.kc0) | kk);
          tc::commit(bar(kEmpty + s));
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc::commit(bar(kAccFull + acc));
      }
    }
    __syncwarp();
  } else {  // epilogue warps 0-3: row 32 * warp + lane of the tile
    const int row = warp * 32 + lane;
    uint8_t *stage = smem + kOffStaging;
    uint8_t *fix_base = p.buf[rank] + p.off_fix;
    uint32_t *fix_flags = reinterpret_cast<uint32_t *>(p.buf[rank] + p.off_fixflag);
    int pushed = 0;
    for (int it = 0; it < sched.n; ++it) {
      const Seg sg = sched.get(it);
      const int acc = it & 1;
      const bool contrib = sg.kc1 < p.k_chunks;          // the tile goes on in the next CTA
      const bool finish = !contrib && sg.kc0 > 0;         // predecessors hold its first chunks
      // all 128 threads take the same branch (epi_any), so none is left at bar 1
      if (epi_any(*abort_flag != 0)) break;
      if (epi_any(!mbar_wait(bar(kAccFull + acc), (it >> 1) & 1))) { fail(); break; }
      // predecessors: CTAs first_pred .. cta - 1 (ascending), first_pred being the
      // CTA whose range holds the tile's first chunk (unit_begin(0) = 0 ends the scan)
      int first_pred = cta;
      if (finish) {
        const int64_t tile_beg = static_cast<int64_t>(sg.tile) * p.k_chunks;
        const int64_t units = static_cast<int64_t>(p.tiles) * p.k_chunks;
        first_pred = cta - 1;
        while (unit_begin(first_pred, p.gemm_ctas, units) > tile_beg) --first_pred;
        bool bad = false;
        if (tid == 0)
          for (int c = first_pred; c < cta; ++c)
            if (!wait_flag_gpu(fix_flags + c, epoch)) { bad = true; break; }
        if (epi_any(bad)) { fail(); break; }
      }
      tc::fence_after_sync();
      // fix-up slot layout: float4 group g = 8 q + c (columns 4 g .. 4 g + 3) of
      // row `row` at float4 index g * 128 + row, so a warp's 32 rows of one
      // group are 512 contiguous bytes (coalesced stores and loads)
      float4 *my_fix =
          reinterpret_cast<float4 *>(fix_base + static_cast<int64_t>(cta) * kFixBytes) + row;
      FixStream fs{base, fix_base, first_pred, cta - first_pred, 1, 0, 4 * (cta - first_pred)};
      if (finish)
        for (int b = 0; b < kFixRing; ++b) fs.issue(b, tid);
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {  // 32 columns at a time
        uint32_t r[32];
        tc::ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + acc * kBN + q * 32, r);
        tc::wait_ld();
        if (contrib) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            my_fix[(q * 8 + c) * kBM] =
                make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                            __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
          continue;
        }
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
        if (finish) fs.add(v, q, row, tid, smem);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // four 16-byte chunks of 8 columns
          const int chunk = q * 4 + c;
          uint4 o;
          o.x = pack2<T>(v[8 * c + 0], v[8 * c + 1]);
          o.y = pack2<T>(v[8 * c + 2], v[8 * c + 3]);
          o.z = pack2<T>(v[8 * c + 4], v[8 * c + 5]);
          o.w = pack2<T>(v[8 * c + 6], v[8 * c + 7]);
          *reinterpret_cast<uint4 *>(stage + row * 256 + ((chunk ^ (row & 7)) << 4)) = o;
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kAccEmpty + acc));  // accumulator free for segment it + 2
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (contrib) {  // publish the fp32 segment sum to the finishing CTA (same GPU)
        if (tid == 0) {
          __threadfence();
          st_release_gpu(fix_flags + cta, epoch);
        }
        continue;
      }
      const int m = sg.tile / p.n_tiles, nt = sg.tile - m * p.n_tiles;
      if (world == 1) {
        for (int c = tid; c < kChunks; c += kEpiThreads) {
          const int rr = c >> 4;
          const uint4 v = *reinterpret_cast<const uint4 *>(stage + rr * 256 +
                                                            (((c & 15) ^ (rr & 7)) << 4));
          store_y_chunk(p, p.y[lr], m, nt, c, v);
        }
      } else if (tid == 0) {
        // the staged tile (kept in its swizzled layout, which the owner reads
        // back) goes to the owner's partial slot [rank][tile / world] in one copy
        // (one shot: to slot [rank][tile] of every rank)
        fence_proxy_async_smem();
        if (kOneShot) {
#pragma unroll
          for (int d = 0; d < W; ++d)
            bulk_store(p.buf[d] + p.off_partial +
                           (static_cast<int64_t>(rank) * p.owned_max + sg.tile) * kTileBytes,
                       smem_u32(stage), kTileBytes);
        } else {
          const int owner = sg.tile % world, slot = sg.tile / world;
          bulk_store(p.buf[owner] + p.off_partial +
                         (static_cast<int64_t>(rank) * p.owned_max + slot) * kTileBytes,
                     smem_u32(stage), kTileBytes);
        }
        bulk_commit_wait_read();
      }
      ++pushed;
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    if (world > 1 && tid == 0 && pushed > 0) {  // publish this CTA's partial tiles
      bulk_publish_fence();
      int k = 0;
      for (int it = 0; it < sched.n && k < pushed; ++it) {
        const Seg sg = sched.get(it);
        if (sg.kc1 < p.k_chunks) continue;
        ++k;
        if (kOneShot) {
#pragma unroll
          for (int d = 0; d < W; ++d)
            st_relaxed_sys(reinterpret_cast<uint32_t *>(p.buf[d] + p.off_pflag) +
                               static_cast<int64_t>(rank) * p.owned_max + sg.tile,
                           epoch);
        } else {
          const int owner = sg.tile % world, slot = sg.tile / world;
          st_relaxed_sys(reinterpret_cast<uint32_t *>(p.buf[owner] + p.off_pflag) +
                             static_cast<int64_t>(rank) * p.owned_max + slot,
                         epoch);
        }
      }
    }
  }
  __syncthreads();

  exchange_phases<T, W>(p, smem + kOffStaging, lr, cta, rank, epoch, abort_flag);
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
  advance_epoch(p, epoch);
}

// CTA-pair form of phase 1 (clusters of two CTAs on two SMs, cta_group::2).
// The stream-K schedule is over pair tiles (256 x 256 outputs) and pairs; both
// CTAs of a pair walk the same segments.  Per stage each CTA's TMA warp loads
// its 128 X rows and its 128 W rows into its own shared memory, both loads
// completing on the LEADER's full barrier (the leader expects both CTAs'
// bytes); the leader's MMA thread issues the M = 256, N = 256 MMAs, whose
// commits arrive on the empty / accumulator-full barriers of both CTAs.  Each
// CTA's epilogue reads its 128 rows x 256 columns from its own TMEM and
// arrives on the leader's accumulator-empty barrier (4 + 4 warps).  Outputs
// leave as two 128 x 128 tiles per CTA, so the exchange of phases 2 / 3 is the
// single-CTA kernel's.  A CTA whose 128 rows all lie past `tokens` (odd row
// tile counts) still runs the pipeline and skips only the stores.
template <typename T, int W>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    row_parallel_pair_kernel(const __grid_constant__ Params p, const __grid_constant__ Maps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t base = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kPOffBars);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kPOffBars + kPNumBars * 8);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = 2 * kStages + 2,
            kDrain = 2 * kStages + 4;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lr = blockIdx.x / p.ctas_per_rank;  // ctas_per_rank is even: a pair never straddles
  const int cta = blockIdx.x - lr * p.ctas_per_rank;
  const int rank = p.rank_base + lr;
  const uint32_t cr = cluster_ctarank();        // 0: leader (issues the MMAs), 1: peer
  const int pair = cta >> 1;
  constexpr int world = W;
  constexpr bool kOneShot = W == 2;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t *>(p.state) + 1u;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = tc::idesc_f16(kBf16, false, 2 * kBM, kPBN);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(kFull + i), 1);    // the leader's expect-tx (both CTAs' bytes)
      mbar_init(bar(kEmpty + i), 1);   // one commit of the leader
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kAccFull + i), 1);
      mbar_init(bar(kAccEmpty + i), 8);  // four epilogue warps in each CTA (leader's is used)
    }
    mbar_init(bar(kDrain), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {  // the same warp in both CTAs allocates the pair's columns
    tmem_alloc_pair(smem_u32(tmem_slot), kPTmemCols);
    tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and TMEM exist before any cross-CTA arrive or MMA
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    record_error(p.err, SLOKV_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };

  // ---------------- phase 1: stream-K GEMM over pair tiles ----------------
  const int pm_tiles = (p.m_tiles + 1) >> 1, pn_tiles = (p.n_tiles + 1) >> 1;
  const int gemm_pairs = p.gemm_ctas >> 1;
  const int64_t units = static_cast<int64_t>(pm_tiles) * pn_tiles * p.k_chunks;
  const Sched sched =
      make_sched(pair < gemm_pairs ? pair : gemm_pairs, gemm_pairs, units, p.k_chunks);
  if (warp == 4) {
    if (lane == 0) {  // TMA producer (both CTAs)
      prefetch_tensormap(&maps.x[lr]);
      prefetch_tensormap(&maps.w[lr]);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < sched.n && !*abort_flag; ++i) {
        const Seg sg = sched.get(i);
        const int pm = sg.tile / pn_tiles, pn = sg.tile - pm * pn_tiles;
        const int xrow = (2 * pm + static_cast<int>(cr)) * kBM;
        const int wrow = (2 * pn + static_cast<int>(cr)) * kBN;
        for (int kc = sg.kc0; kc < sg.kc1; ++kc) {
          if (!mbar_wait(bar(kEmpty + s), ph ^ 1)) { fail(); break; }
          const uint32_t dst = base + s * kStageBytes;
          const uint32_t full = mapa_shared(bar(kFull + s), 0);
          if (cr == 0) mbar_arrive_expect_tx(bar(kFull + s), 2 * kStageBytes);
          tma_load_2d_pair(dst, &maps.x[lr], full, kc * kBK, xrow);
          tma_load_2d_pair(dst + kSlice, &maps.w[lr], full, kc * kBK, wrow);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
      }
      // tail: wait until the MMAs have released every stage this CTA filled, so
      // no commit of the leader is still on its way to this CTA's barriers
      for (int i = 0; i < kStages && !*abort_flag; ++i) {
        if (!mbar_wait(bar(kEmpty + s), ph ^ 1)) { fail(); break; }
        if (++s == kStages) { s = 0; ph ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0 && cr == 0) {  // MMA issuer (leader only)
      int s = 0;
      uint32_t ph = 0;
      for (int it = 0; it < sched.n && !*abort_flag; ++it) {
        const Seg sg = sched.get(it);
        const int acc = it & 1;
        if (!mbar_wait(bar(kAccEmpty + acc), ((it >> 1) & 1) ^ 1)) { fail(); break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + acc * kPBN;
        bool ok = true;
        for (int kc = sg.kc0; kc < sg.kc1; ++kc) {
          if (!mbar_wait(bar(kFull + s), ph)) { fail(); ok = false; break; }
          tc::fence_after_sync();
          const uint32_t a = base + s * kStageBytes, b = a + kSlice;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16_ss_pair(d, tc::smem_desc_sw128(a + kk * 32, 16, 1024),
                            tc::smem_desc_sw128(b + kk * 32, 16, 1024), kIdesc,
                            (kc - sg.kc0) | kk);
          commit_pair(bar(kEmpty + s), 0x3);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        commit_pair(bar(kAccFull + acc), 0x3);
      }
      // every MMA issued above has completed before the pair releases TMEM
      commit_pair(bar(kDrain), 0x1);
      if (!mbar_wait(bar(kDrain), 0)) fail();
    }
    __syncwarp();
  } else {  // epilogue warps 0-3 (both CTAs): row 32 * warp + lane of this CTA's 128 rows
    const int row = warp * 32 + lane;
    uint8_t *stage = smem + kOffStaging;
    uint8_t *fix_base = p.buf[rank] + p.off_fix;
    uint32_t *fix_flags = reinterpret_cast<uint32_t *>(p.buf[rank] + p.off_fixflag);
    const uint32_t acc_empty_leader[2] = {mapa_shared(bar(kAccEmpty), 0),
                                          mapa_shared(bar(kAccEmpty + 1), 0)};
    int pushed = 0;
    for (int it = 0; it < sched.n; ++it) {
      const Seg sg = sched.get(it);
      const int acc = it & 1;
      const bool contrib = sg.kc1 < p.k_chunks;
      const bool finish = !contrib && sg.kc0 > 0;
      if (epi_any(*abort_flag != 0)) break;
      if (epi_any(!mbar_wait(bar(kAccFull + acc), (it >> 1) & 1))) { fail(); break; }
      // predecessor pairs first_pred .. pair - 1; this CTA adds the fix-up
      // slots of the same-position CTA (2 c + cr) of each
      int first_pred = pair;
      if (finish) {
        const int64_t tile_beg = static_cast<int64_t>(sg.tile) * p.k_chunks;
        first_pred = pair - 1;
        while (unit_begin(first_pred, gemm_pairs, units) > tile_beg) --first_pred;
        bool bad = false;
        if (tid == 0)
          for (int c = first_pred; c < pair; ++c)
            if (!wait_flag_gpu(fix_flags + 2 * c + cr, epoch)) { bad = true; break; }
        if (epi_any(bad)) { fail(); break; }
      }
      tc::fence_after_sync();
      // fix-up slot layout as in the single-CTA kernel (float4 group g = 8 q + c
      // of row `row` at index g * 128 + row), 64 groups for 256 columns
      float4 *my_fix =
          reinterpret_cast<float4 *>(fix_base + static_cast<int64_t>(cta) * kFixBytes) + row;
      FixStream fs{base,           fix_base, first_pred, pair - first_pred, 2, static_cast<int>(cr),
                   8 * (pair - first_pred)};
      if (finish)
        for (int b = 0; b < kFixRing; ++b) fs.issue(b, tid);
#pragma unroll 1
      for (int q = 0; q < 8; ++q) {  // 32 columns at a time; q / 4 = output half
        uint32_t r[32];
        tc::ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + acc * kPBN + q * 32, r);
        tc::wait_ld();
        if (contrib) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            my_fix[(q * 8 + c) * kBM] =
                make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                            __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
          continue;
        }
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
        if (finish) fs.add(v, q, row, tid, smem);
        uint8_t *half = stage + (q >> 2) * kTileBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // four 16-byte chunks of 8 columns
          const int chunk = (q & 3) * 4 + c;
          uint4 o;
          o.x = pack2<T>(v[8 * c + 0], v[8 * c + 1]);
          o.y = pack2<T>(v[8 * c + 2], v[8 * c + 3]);
          o.z = pack2<T>(v[8 * c + 4], v[8 * c + 5]);
          o.w = pack2<T>(v[8 * c + 6], v[8 * c + 7]);
          *reinterpret_cast<uint4 *>(half + row * 256 + ((chunk ^ (row & 7)) << 4)) = o;
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader[acc]);  // accumulator free
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (contrib) {  // publish the fp32 segment sum to the finishing pair (same GPU)
        if (tid == 0) {
          __threadfence();
          st_release_gpu(fix_flags + cta, epoch);
        }
        continue;
      }
      const int pm = sg.tile / pn_tiles, pn = sg.tile - pm * pn_tiles;
      const int m = 2 * pm + static_cast<int>(cr);
      if (m < p.m_tiles) {
        if (world == 1) {
          for (int c = tid; c < 2 * kChunks; c += kEpiThreads) {
            const int h = c / kChunks, cc = c - h * kChunks, rr = cc >> 4;
            const int nt = 2 * pn + h;
            if (nt >= p.n_tiles) continue;
            const uint4 v = *reinterpret_cast<const uint4 *>(
                stage + h * kTileBytes + rr * 256 + (((cc & 15) ^ (rr & 7)) << 4));
            store_y_chunk(p, p.y[lr], m, nt, cc, v);
          }
        } else if (tid == 0) {
          fence_proxy_async_smem();
          for (int h = 0; h < 2; ++h) {
            const int nt = 2 * pn + h;
            if (nt >= p.n_tiles) continue;
            const int tile = m * p.n_tiles + nt;
            const uint32_t src = smem_u32(stage + h * kTileBytes);
            if (kOneShot) {
#pragma unroll
              for (int d = 0; d < W; ++d)
                bulk_store(p.buf[d] + p.off_partial +
                               (static_cast<int64_t>(rank) * p.owned_max + tile) * kTileBytes,
                           src, kTileBytes);
            } else {
              const int owner = tile % world, slot = tile / world;
              bulk_store(p.buf[owner] + p.off_partial +
                             (static_cast<int64_t>(rank) * p.owned_max + slot) * kTileBytes,
                         src, kTileBytes);
            }
          }
          bulk_commit_wait_read();
        }
        ++pushed;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    if (world > 1 && tid == 0 && pushed > 0) {  // publish this CTA's partial tiles
      bulk_publish_fence();
      for (int it = 0; it < sched.n; ++it) {
        const Seg sg = sched.get(it);
        if (sg.kc1 < p.k_chunks) continue;
        const int pm = sg.tile / pn_tiles, pn = sg.tile - pm * pn_tiles;
        const int m = 2 * pm + static_cast<int>(cr);
        if (m >= p.m_tiles) continue;
        for (int h = 0; h < 2; ++h) {
          const int nt = 2 * pn + h;
          if (nt >= p.n_tiles) continue;
          const int tile = m * p.n_tiles + nt;
          if (kOneShot) {
#pragma unroll
            for (int d = 0; d < W; ++d)
              st_relaxed_sys(reinterpret_cast<uint32_t *>(p.buf[d] + p.off_pflag) +
                                 static_cast<int64_t>(rank) * p.owned_max + tile,
                             epoch);
          } else {
            const int owner = tile % world, slot = tile / world;
            st_relaxed_sys(reinterpret_cast<uint32_t *>(p.buf[owner] + p.off_pflag) +
                               static_cast<int64_t>(rank) * p.owned_max + slot,
                           epoch);
          }
        }
      }
    }
  }
  __syncthreads();

  exchange_phases<T, W>(p, smem + kOffStaging, lr, cta, rank, epoch, abort_flag);
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still arrive on its barriers
  if (warp == 0) {
    tc::fence_after_sync();
    tmem_dealloc_pair(tmem, kPTmemCols);
  }
  advance_epoch(p, epoch);
}

// ---- host side -------------------------------------------------------------

struct Layout {
  int64_t tiles_max, owned_max, off_fix, off_fixflag, off_partial, off_result, off_pflag,
      off_rflag, total;
};

inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// One rank's buffer: stream-K fix-up slots and flags (used by this GPU only),
// then, for world > 1, the partial slots [source rank][tile / world], the
// result slots [tile] and their flags (written by peers).
Layout layout(int max_tokens, int n_features, int world) {
  Layout l;
  l.tiles_max = static_cast<int64_t>((max_tokens + kBM - 1) / kBM) * (n_features / kBN);
  // (two ranks exchange one shot: every rank holds a slot for every tile)
  l.owned_max = world == 2 ? l.tiles_max : (l.tiles_max + world - 1) / world;
  l.off_fix = 0;
  l.off_fixflag = static_cast<int64_t>(kMaxCtas) * kFixBytes;
  const int64_t x = align_up(l.off_fixflag + kMaxCtas * 4, 4096);
  const bool ex = world > 1;
  const int64_t partial = ex ? static_cast<int64_t>(world) * l.owned_max * kTileBytes : 0;
  l.off_result = x + align_up(partial, 4096);
  l.off_pflag = align_up(l.off_result + (ex ? l.tiles_max * kTileBytes : 0), 4096);
  l.off_rflag = align_up(l.off_pflag + (ex ? static_cast<int64_t>(world) * l.owned_max * 4 : 0),
                         256);
  l.total = align_up(l.off_rflag + (ex ? l.tiles_max * kQuarters * 4 : 0), 4096);
  // the partial slots start at the first exchange offset
  l.off_partial = x;
  return l;
}

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

// 2-D map {K (inner), rows} with a {64, 128} box and 128-byte swizzle; rows
// past the end read as zeros.
bool encode_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dt, uint64_t k,
               uint64_t rows, uint64_t row_stride_elems) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {kBK, kBM};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

template <typename T, int W>
int launch(const Params &p, const Maps &maps, int local_ranks, cudaStream_t stream) {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(row_parallel_kernel<T, W>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) == cudaSuccess;
  });
  if (!ok) return SLOKV_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(local_ranks * p.ctas_per_rank));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, row_parallel_kernel<T, W>, p, maps) == cudaSuccess
             ? SLOKV_OK
             : SLOKV_ERR_CUDA;
}

// Co-resident clusters of two CTAs of the pair kernel on this device (clusters
// must fit a GPC, so this can be below SMs / 2); 0 if the query fails.
int pair_capacity() {
  static int cap = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    cap = 0;
    if (cudaFuncSetAttribute(row_parallel_pair_kernel<__nv_bfloat16, 1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPSmemBytes) != cudaSuccess)
      return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kPSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, row_parallel_pair_kernel<__nv_bfloat16, 1>, &cfg) ==
        cudaSuccess)
      cap = n;
    else
      cudaGetLastError();
  });
  return cap;
}

// The pair kernel is launched cooperatively where the runtime accepts a
// cooperative launch of a cluster kernel; otherwise as a plain launch whose
// grid never exceeds the co-resident cluster capacity (pair_capacity), so every
// CTA is resident and every wait of the exchange can end.
template <typename T, int W>
int launch_pair(const Params &p, const Maps &maps, int local_ranks, cudaStream_t stream) {
  static std::once_flag once;
  static bool ok = false;
  static int coop = -1;  // -1 unknown, 0 refused, 1 accepted
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(row_parallel_pair_kernel<T, W>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kPSmemBytes) == cudaSuccess;
  });
  if (!ok) return SLOKV_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(local_ranks * p.ctas_per_rank));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cap);
  if (coop != 0 && !(coop < 0 && cap != cudaStreamCaptureStatusNone)) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, row_parallel_pair_kernel<T, W>, p, maps);
    if (e == cudaSuccess) {
      coop = 1;
      return SLOKV_OK;
    }
    if (coop == 1) return SLOKV_ERR_CUDA;
    cudaGetLastError();  // a refused launch attribute leaves no sticky error
    coop = 0;
  }
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, row_parallel_pair_kernel<T, W>, p, maps) == cudaSuccess
             ? SLOKV_OK
             : SLOKV_ERR_CUDA;
}

// Grid of one call: which kernel, CTAs per rank, CTAs with GEMM work.
struct Plan {
  bool pair;
  int per_rank, gemm_ctas, ctas_per_rank, pair_capacity;
};
Plan plan_grid(int tokens, int n_features, int k_features, int world, int local_ranks) {
  const int m_tiles = (tokens + kBM - 1) / kBM, n_tiles = n_features / kBN,
            k_chunks = k_features / kBK;
  // CTA pairs (256 x 256 tiles, half the operand bytes per output, stream-K
  // over every pair) for GEMMs of at least kPairMinMacs multiply-adds; one CTA
  // per 128 x 128 tile below that.  Measured on B200 (N = 2560): the pairs'
  // main loop runs 2.3x the single-CTA tile rate, but each pair CTA drains a
  // 128 x 256 accumulator, so for decode-sized calls (T <= 512 rows per rank,
  // and T = 1024 with K = 4096) the single-CTA kernel finishes first; from
  // T = 1024 with K = 9728, or T = 2048 with K = 4096, the pairs win
  // (1.08 - 1.35x).
  Plan pl = {};
  int pair_cap = 0;
  const bool pair = m_tiles >= 2 && n_tiles >= 2 &&
                    static_cast<int64_t>(tokens) * n_features * k_features >= kPairMinMacs &&
                    (pair_cap = pair_capacity()) > 0;
  pl.pair = pair;
  pl.pair_capacity = pair_cap;
  int per_rank = (pair && 2 * pair_cap < sm_count() ? 2 * pair_cap : sm_count()) / local_ranks;
  if (per_rank > kMaxCtas) per_rank = kMaxCtas;
  if (pair) per_rank &= ~1;
  if (per_rank < (pair ? 2 : 1)) return pl;   // per_rank 0: unsupported
  pl.per_rank = per_rank;
  if (pair) {
    // stream-K over all pairs: a pair's range is at least one pair tile's K
    // loop once there are as many pair tiles as pairs, so a tile has at most
    // one predecessor; with fewer, every pair still gets >= kMinChunks chunks
    const int pair_tiles = ((m_tiles + 1) / 2) * ((n_tiles + 1) / 2);
    const int64_t by_work =
        (static_cast<int64_t>(pair_tiles) * k_chunks + kMinChunks - 1) / kMinChunks;
    const int max_pairs = per_rank / 2;
    pl.gemm_ctas = 2 * static_cast<int>(by_work < max_pairs ? by_work : max_pairs);
  } else {
    // GEMM: one CTA per tile while that keeps at least half the SMs busy (each
    // split adds an fp32 fix-up); stream-K splits of the K loops over all SMs
    // for K of 64 chunks or more (T = 512 rows: o_proj at TP 1 22.8 -> 21.0 us,
    // down_proj at TP 2 25.7 -> 21.8 us; shorter K loops lose, e.g. o_proj at
    // TP 4 11.0 vs 14.8 us) or few tiles, every CTA getting at least
    // kMinChunks K chunks.
    const int tiles = m_tiles * n_tiles;
    const int64_t units = static_cast<int64_t>(tiles) * k_chunks;
    if (k_chunks >= 64 || 2 * tiles < per_rank) {
      const int64_t by_work = (units + kMinChunks - 1) / kMinChunks;
      pl.gemm_ctas = static_cast<int>(by_work < per_rank ? by_work : per_rank);
    } else {
      pl.gemm_ctas = tiles < per_rank ? tiles : per_rank;
    }
  }
  // With an exchange every SM gets a CTA: the ones without GEMM work join the
  // reduce.
  pl.ctas_per_rank = world > 1 ? per_rank : pl.gemm_ctas;
  return pl;
}

template <typename T>
int launch_world(const Params &p, const Maps &maps, int local_ranks, bool pair,
                 cudaStream_t stream) {
  switch (p.world) {
    case 1: return pair ? launch_pair<T, 1>(p, maps, local_ranks, stream)
                        : launch<T, 1>(p, maps, local_ranks, stream);
    case 2: return pair ? launch_pair<T, 2>(p, maps, local_ranks, stream)
                        : launch<T, 2>(p, maps, local_ranks, stream);
    case 4: return pair ? launch_pair<T, 4>(p, maps, local_ranks, stream)
                        : launch<T, 4>(p, maps, local_ranks, stream);
    case 8: return pair ? launch_pair<T, 8>(p, maps, local_ranks, stream)
                        : launch<T, 8>(p, maps, local_ranks, stream);
    default: return SLOKV_ERR_UNSUPPORTED;
  }
}

}  // namespace rp
}  // namespace slokv

extern "C" size_t slokv_row_parallel_buffer_bytes(int32_t max_tokens, int32_t n_features,
                                                  int32_t world) {
  using namespace slokv::rp;
  if (max_tokens <= 0 || n_features <= 0 || n_features % kBN != 0 || world < 1 ||
      world > kMaxRanks)
    return 0;
  return static_cast<size_t>(layout(max_tokens, n_features, world).total);
}

extern "C" int slokv_row_parallel_plan(int32_t tokens, int32_t n_features, int32_t k_features,
                                       int32_t world, int32_t local_ranks, int32_t *plan) {
  using namespace slokv;
  using namespace slokv::rp;
  if (!plan || tokens <= 0 || n_features <= 0 || k_features <= 0 || world < 1 ||
      world > kMaxRanks || local_ranks < 1 || local_ranks > world)
    return SLOKV_ERR_INVALID_ARG;
  if (n_features % kBN != 0 || k_features % kBK != 0) return SLOKV_ERR_UNSUPPORTED;
  const Plan pl = plan_grid(tokens, n_features, k_features, world, local_ranks);
  plan[0] = pl.pair ? 2 : 1;
  plan[1] = pl.per_rank;
  plan[2] = pl.gemm_ctas;
  plan[3] = pl.ctas_per_rank;
  plan[4] = pl.pair_capacity;
  return pl.per_rank < 1 ? SLOKV_ERR_UNSUPPORTED : SLOKV_OK;
}

extern "C" int slokv_row_parallel_linear(
    const void *const *x, int64_t x_row_stride, const void *const *w, int64_t w_row_stride,
    const void *const *bias, void *const *y, int64_t y_row_stride, int32_t tokens,
    int32_t n_features, int32_t k_features, void *const *rank_buffers, int32_t world,
    int32_t rank_base, int32_t local_ranks, int32_t max_tokens, uint32_t *state, int32_t dtype,
    uint32_t *dev_error, void *stream) {
  using namespace slokv;
  using namespace slokv::rp;
  if (world < 1 || world > kMaxRanks || local_ranks < 1 || rank_base < 0 ||
      rank_base + local_ranks > world || tokens < 0 || max_tokens <= 0 || tokens > max_tokens ||
      n_features <= 0 || k_features <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (n_features % kBN != 0 || k_features % kBK != 0) return SLOKV_ERR_UNSUPPORTED;
  if (world != 1 && world != 2 && world != 4 && world != 8) return SLOKV_ERR_UNSUPPORTED;
  if (dtype != SLOKV_DTYPE_BF16 && dtype != SLOKV_DTYPE_F16) return SLOKV_ERR_UNSUPPORTED;
  if (tokens == 0) return SLOKV_OK;
  if (!x || !w || !y || !state || !rank_buffers) return SLOKV_ERR_INVALID_ARG;
  if (x_row_stride < k_features || w_row_stride < k_features || y_row_stride < n_features)
    return SLOKV_ERR_INVALID_ARG;
  if ((x_row_stride | w_row_stride | y_row_stride) & 7) return SLOKV_ERR_ALIGNMENT;
  Params p = {};
  Maps maps;
  const CUtensorMapDataType dt =
      dtype == SLOKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  for (int i = 0; i < local_ranks; ++i) {
    if (!x[i] || !w[i] || !y[i]) return SLOKV_ERR_INVALID_ARG;
    const uintptr_t a = reinterpret_cast<uintptr_t>(x[i]) | reinterpret_cast<uintptr_t>(w[i]) |
                        reinterpret_cast<uintptr_t>(y[i]) |
                        reinterpret_cast<uintptr_t>(bias ? bias[i] : nullptr);
    if (a & 15) return SLOKV_ERR_ALIGNMENT;
    if (!encode_2d(&maps.x[i], x[i], dt, k_features, tokens, x_row_stride) ||
        !encode_2d(&maps.w[i], w[i], dt, k_features, n_features, w_row_stride))
      return SLOKV_ERR_CUDA;
    p.y[i] = y[i];
    p.bias[i] = bias ? bias[i] : nullptr;
  }
  for (int r = 0; r < world; ++r) {
    if (!rank_buffers[r] || (reinterpret_cast<uintptr_t>(rank_buffers[r]) & 255))
      return SLOKV_ERR_INVALID_ARG;
    p.buf[r] = static_cast<uint8_t *>(rank_buffers[r]);
  }
  const Layout l = layout(max_tokens, n_features, world);
  p.tokens = tokens;
  p.n = n_features;
  p.k = k_features;
  p.m_tiles = (tokens + kBM - 1) / kBM;
  p.n_tiles = n_features / kBN;
  p.tiles = p.m_tiles * p.n_tiles;
  p.k_chunks = k_features / kBK;
  p.world = world;
  p.rank_base = rank_base;
  p.owned_max = static_cast<int>(l.owned_max);
  p.off_partial = l.off_partial;
  p.off_fix = l.off_fix;
  p.off_fixflag = l.off_fixflag;
  p.off_result = l.off_result;
  p.off_pflag = l.off_pflag;
  p.off_rflag = l.off_rflag;
  p.y_stride = y_row_stride;
  p.state = state;
  p.err = dev_error;
  const Plan plan = plan_grid(tokens, n_features, k_features, world, local_ranks);
  if (plan.per_rank < 1) return SLOKV_ERR_UNSUPPORTED;
  p.gemm_ctas = plan.gemm_ctas;
  p.ctas_per_rank = plan.ctas_per_rank;
  const bool pair = plan.pair;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == SLOKV_DTYPE_BF16 ? launch_world<__nv_bfloat16>(p, maps, local_ranks, pair, st)
                                   : launch_world<__half>(p, maps, local_ranks, pair, st);
}

// ---- symmetric buffers shared between the ranks' processes (CUDA IPC) --------

extern "C" int slokv_device_alloc(size_t bytes, void **ptr) {
  if (!ptr || bytes == 0) return SLOKV_ERR_INVALID_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return SLOKV_ERR_CUDA;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return SLOKV_ERR_CUDA;
  }
  return SLOKV_OK;
}

extern "C" int slokv_device_free(void *ptr) {
  if (!ptr) return SLOKV_OK;
  return cudaFree(ptr) == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

extern "C" int slokv_ipc_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int slokv_ipc_export(const void *ptr, void *handle_out) {
  if (!ptr || !handle_out) return SLOKV_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)) != cudaSuccess) return SLOKV_ERR_CUDA;
  memcpy(handle_out, &h, sizeof(h));
  return SLOKV_OK;
}

extern "C" int slokv_ipc_import(const void *handle, void **ptr) {
  if (!handle || !ptr) return SLOKV_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? SLOKV_OK
             : SLOKV_ERR_CUDA;
}

extern "C" int slokv_ipc_close(void *ptr) {
  if (!ptr) return SLOKV_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}
