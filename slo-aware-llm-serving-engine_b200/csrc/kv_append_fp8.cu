// Quantising paged KV append for the FP8-E4M3 cache, plus the E4M3 codec as
// stand-alone entry points.
//
// Contract (per (block, kv head), K and V separately, fp32 scale s >= 0; s == 0
// means "no nonzero value stored yet" and encodes with divisor 1, the
// "amax = 0 -> scale = 1" rule of the reference manual):
//   * the new tokens of one block in one call are adjacent in slot_mapping with
//     consecutive offsets (how the engine lays out decode and prefill slots);
//   * a = max |x| over those tokens and the head's dims; s_new = max(s_old, a / 448),
//     where s_old is the stored scale, or 0 when the run starts at offset 0 of
//     the block (a block's first token is always written at offset 0 and a
//     shared prefix block is full and never written, so a write at offset 0
//     means the page was handed to a new sequence: its stored scale is stale
//     and no caller has to clear it);
//   * if s_new > s_old > 0, the block/head's positions before the first new
//     offset are re-encoded: c' = encode(fp32(decode(c) * s_old) / s_new);
//   * new tokens: c = encode(fp32(x) / (s_new > 0 ? s_new : 1)); store s_new.
// Every multiply/divide is IEEE fp32 round-to-nearest-even (__fmul_rn,
// __fdiv_rn), so the codes are bit-identical to the CPU restatement.
//
// B200 mapping: one warp per (run of a block's new tokens, kv head, K|V); lane l
// owns dims [4l, 4l+4) of the 128-dim head, so every access is a coalesced
// 256-byte (input) or 128-byte (codes) warp transaction.  The only reduction is
// one warp max per run.
#include "common.cuh"
#include "fp8_e4m3.cuh"

namespace slokv {
namespace {

constexpr int kHeadDim = 128;

template <typename T>
__device__ __forceinline__ float4 load4(const T *p);

template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16 *p) {
  const uint2 raw = *reinterpret_cast<const uint2 *>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <>
__device__ __forceinline__ float4 load4<__half>(const __half *p) {
  const uint2 raw = *reinterpret_cast<const uint2 *>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <>
__device__ __forceinline__ float4 load4<float>(const float *p) {
  return *reinterpret_cast<const float4 *>(p);
}

__device__ __forceinline__ uint32_t encode4(float4 v, float div, bool &bad) {
  return e4m3_encode(__fdiv_rn(v.x, div), bad) | (e4m3_encode(__fdiv_rn(v.y, div), bad) << 8) |
         (e4m3_encode(__fdiv_rn(v.z, div), bad) << 16) |
         (e4m3_encode(__fdiv_rn(v.w, div), bad) << 24);
}

template <typename T>
__global__ void __launch_bounds__(256, 2) kv_append_fp8_kernel(
    const T *__restrict__ key, int64_t key_stride, const T *__restrict__ value,
    int64_t value_stride, uint8_t *__restrict__ k_codes, uint8_t *__restrict__ v_codes,
    float *__restrict__ k_scale, float *__restrict__ v_scale, const int32_t *__restrict__ slots,
    int32_t num_tokens, int32_t hkv, int32_t block_size, int32_t num_blocks, uint32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = static_cast<int64_t>(num_tokens) * hkv * 2;
  if (wid >= total) return;
  const int which = static_cast<int>(wid & 1);  // 0: K, 1: V
  const int h = static_cast<int>((wid >> 1) % hkv);
  const int i = static_cast<int>((wid >> 1) / hkv);
  const int64_t num_slots = static_cast<int64_t>(num_blocks) * block_size;

  const int32_t slot = __ldg(slots + i);
  if (slot < 0 || slot >= num_slots) {
    if (slot != -1 && lane == 0 && h == 0 && which == 0) record_error(err, SLOKV_DEVERR_SLOT_RANGE);
    return;
  }
  const int32_t blk = slot / block_size, off = slot - blk * block_size;
  if (i > 0) {
    const int32_t prev = __ldg(slots + i - 1);
    if (prev >= 0 && prev == slot - 1 && prev / block_size == blk) return;  // not a run start
  }
  int j = i + 1;
  while (j < num_tokens && j - i < block_size) {
    const int32_t sj = __ldg(slots + j);
    if (sj != slot + (j - i) || sj / block_size != blk) break;
    ++j;
  }

  const T *src = which ? value : key;
  const int64_t sstride = which ? value_stride : key_stride;
  uint8_t *codes = which ? v_codes : k_codes;
  float *scales = which ? v_scale : k_scale;
  const int64_t row = static_cast<int64_t>(hkv) * kHeadDim;  // codes per token
  const int d0 = lane * 4;

  // Runs of prefill tokens are up to a block long: the loops below keep
  // kUnroll independent loads in flight per lane instead of one.
  constexpr int kUnroll = 8;
  auto absmax4 = [](float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  };
  const T *hsrc = src + h * kHeadDim + d0;
  float amax = 0.f;
  int t = i;
  for (; t + kUnroll <= j; t += kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = load4<T>(hsrc + (t + u) * sstride);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) amax = fmaxf(amax, absmax4(v[u]));
  }
  for (; t < j; ++t) amax = fmaxf(amax, absmax4(load4<T>(hsrc + t * sstride)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));

  float *sp = scales + static_cast<int64_t>(blk) * hkv + h;
  const float s_old = off == 0 ? 0.f : *sp;   // offset 0: a freshly assigned page
  const float s_new = fmaxf(s_old, __fdiv_rn(amax, 448.0f));
  bool bad = false;
  uint8_t *base = codes + static_cast<int64_t>(blk) * block_size * row + h * kHeadDim + d0;
  if (s_new > s_old && s_old > 0.f) {
    auto reencode = [&](uint32_t c) {
      float4 v;
      v.x = __fmul_rn(e4m3_decode(c & 0xffu), s_old);
      v.y = __fmul_rn(e4m3_decode((c >> 8) & 0xffu), s_old);
      v.z = __fmul_rn(e4m3_decode((c >> 16) & 0xffu), s_old);
      v.w = __fmul_rn(e4m3_decode(c >> 24), s_old);
      return encode4(v, s_new, bad);
    };
    int p = 0;
    for (; p + kUnroll <= off; p += kUnroll) {
      uint32_t c[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) c[u] = *reinterpret_cast<const uint32_t *>(base + (p + u) * row);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        *reinterpret_cast<uint32_t *>(base + (p + u) * row) = reencode(c[u]);
    }
    for (; p < off; ++p) {
      uint32_t *cp = reinterpret_cast<uint32_t *>(base + p * row);
      *cp = reencode(*cp);
    }
  }
  const float div = s_new > 0.f ? s_new : 1.0f;
  uint8_t *dst = base + off * row;
  t = i;
  for (; t + kUnroll <= j; t += kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = load4<T>(hsrc + (t + u) * sstride);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      *reinterpret_cast<uint32_t *>(dst + (t - i + u) * row) = encode4(v[u], div, bad);
  }
  for (; t < j; ++t)
    *reinterpret_cast<uint32_t *>(dst + (t - i) * row) = encode4(load4<T>(hsrc + t * sstride), div, bad);
  __syncwarp();
  if (lane == 0) *sp = s_new;
  if (__any_sync(0xffffffffu, bad) && lane == 0) record_error(err, SLOKV_DEVERR_NONFINITE);
}

// ---- the same append in three launches, for calls with long runs ------------
//
// A prefill chunk writes runs of up to a block (256 tokens) per (block, head,
// K|V); one warp per run walks them serially.  Here one warp per token works
// on the token's 2 * hkv (head, K|V) rows: (1) each row's amax goes into a
// per-(block, head, K|V) word with atomicMax on the float bits (non-negative
// floats order like their bit patterns, so the word ends as the exact run
// amax); (2) each row derives s_new = max(s_old, amax / 448) -- the same value
// for every token of the run, s_old being 0 for a run that starts at offset 0
// -- and encodes the token; the run's first token re-encodes the block's
// earlier positions of a row whose scale grows; (3) one thread per run start
// and row stores s_new and clears the word.  Codes and scales are the
// one-launch kernel's, bit for bit.  `amax_ws` is num_blocks * hkv * 2 words,
// zero between calls.

struct RunToken {
  bool valid;       // a slot inside the pool
  bool start;       // the first token of its block's run
  int32_t blk, off; // block and position of the token
};

__device__ __forceinline__ RunToken run_token(const int32_t *slots, int i, int32_t block_size,
                                              int64_t num_slots) {
  RunToken t;
  const int32_t slot = __ldg(slots + i);
  t.valid = slot >= 0 && slot < num_slots;
  t.blk = t.valid ? slot / block_size : 0;
  t.off = t.valid ? slot - t.blk * block_size : 0;
  t.start = t.valid;
  if (t.valid && i > 0) {
    const int32_t prev = __ldg(slots + i - 1);
    if (prev >= 0 && prev == slot - 1 && prev / block_size == t.blk) t.start = false;
  }
  return t;
}

// One warp per token, looping over its 2 * hkv (head, K|V) rows four at a
// time: the token's slot is read once, the four rows' loads are in flight
// together, and lanes 0-3 issue the four rows' atomics.
template <typename T>
__global__ void __launch_bounds__(256) kv_append_fp8_amax_kernel(
    const T *__restrict__ key, int64_t key_stride, const T *__restrict__ value,
    int64_t value_stride, const int32_t *__restrict__ slots, int32_t num_tokens, int32_t hkv,
    int32_t block_size, int32_t num_blocks, uint32_t *__restrict__ amax_ws, uint32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (i >= num_tokens) return;
  const int32_t slot = __ldg(slots + i);
  if (slot < 0 || slot >= static_cast<int64_t>(num_blocks) * block_size) {
    if (slot != -1 && lane == 0) record_error(err, SLOKV_DEVERR_SLOT_RANGE);
    return;
  }
  uint32_t *words = amax_ws + static_cast<int64_t>(slot / block_size) * hkv * 2;
  const int rows = 2 * hkv;                       // row r: head r / 2, K (r even) or V
  for (int r0 = 0; r0 < rows; r0 += 4) {
    float a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = r0 + u;
      a[u] = 0.f;
      if (r < rows) {
        const T *src = ((r & 1) ? value + i * value_stride : key + i * key_stride) +
                       (r >> 1) * kHeadDim + lane * 4;
        const float4 v = load4<T>(src);
        // seeded with 0 as in the one-launch kernel: NaN elements drop out of
        // the max (fmaxf keeps the non-NaN operand), so no word holds NaN bits
        a[u] = fmaxf(fmaxf(fmaxf(0.f, fabsf(v.x)), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = fmaxf(a[u], __shfl_xor_sync(0xffffffffu, a[u], o));
    const float mine = lane == 0 ? a[0] : lane == 1 ? a[1] : lane == 2 ? a[2] : a[3];
    if (lane < 4 && r0 + lane < rows) atomicMax(words + r0 + lane, __float_as_uint(mine));
  }
}

// One warp per token over its 2 * hkv rows: s_new = max(s_old, amax / 448) of
// each row's (block, head, K|V) -- the same value for every token of the run,
// s_old being 0 for a run that starts at offset 0 -- then the token's codes;
// the run's first token re-encodes the block's earlier positions of a row
// whose scale grows.
template <typename T>
__global__ void __launch_bounds__(256, 2) kv_append_fp8_encode_kernel(
    const T *__restrict__ key, int64_t key_stride, const T *__restrict__ value,
    int64_t value_stride, uint8_t *__restrict__ k_codes, uint8_t *__restrict__ v_codes,
    const float *__restrict__ k_scale, const float *__restrict__ v_scale,
    const int32_t *__restrict__ slots, int32_t num_tokens, int32_t hkv, int32_t block_size,
    int32_t num_blocks, const uint32_t *__restrict__ amax_ws, uint32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (i >= num_tokens) return;
  const RunToken tk = run_token(slots, static_cast<int>(i), block_size,
                                static_cast<int64_t>(num_blocks) * block_size);
  if (!tk.valid) return;
  // The run starts at offset 0 (a freshly assigned page, stored scale ignored)
  // iff the token tk.off places earlier holds offset 0 of the same block: runs
  // are adjacent with consecutive offsets and a block has one run per call.
  const bool fresh = i >= tk.off && __ldg(slots + i - tk.off) ==
                                        static_cast<int64_t>(tk.blk) * block_size;
  const int64_t row = static_cast<int64_t>(hkv) * kHeadDim;
  const int d0 = lane * 4;
  const int rows = 2 * hkv;
  bool bad = false;
  for (int r0 = 0; r0 < rows; r0 += 4) {
    float4 v[4];
    float s_old[4], s_new[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = r0 + u;
      if (r >= rows) continue;
      const int h = r >> 1;
      const int64_t si = static_cast<int64_t>(tk.blk) * hkv + h;
      v[u] = load4<T>(((r & 1) ? value + i * value_stride : key + i * key_stride) +
                      h * kHeadDim + d0);
      s_old[u] = fresh ? 0.f : ((r & 1) ? v_scale : k_scale)[si];
      s_new[u] = fmaxf(s_old[u], __fdiv_rn(__uint_as_float(amax_ws[si * 2 + (r & 1)]), 448.0f));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = r0 + u;
      if (r >= rows) continue;
      uint8_t *base = ((r & 1) ? v_codes : k_codes) +
                      static_cast<int64_t>(tk.blk) * block_size * row + (r >> 1) * kHeadDim + d0;
      if (tk.start && s_new[u] > s_old[u] && s_old[u] > 0.f) {   // earlier positions
        const float so = s_old[u], sn = s_new[u];
        for (int p = 0; p < tk.off; ++p) {
          uint32_t *cp = reinterpret_cast<uint32_t *>(base + p * row);
          const uint32_t c = *cp;
          float4 w;
          w.x = __fmul_rn(e4m3_decode(c & 0xffu), so);
          w.y = __fmul_rn(e4m3_decode((c >> 8) & 0xffu), so);
          w.z = __fmul_rn(e4m3_decode((c >> 16) & 0xffu), so);
          w.w = __fmul_rn(e4m3_decode(c >> 24), so);
          *cp = encode4(w, sn, bad);
        }
      }
      *reinterpret_cast<uint32_t *>(base + tk.off * row) =
          encode4(v[u], s_new[u] > 0.f ? s_new[u] : 1.0f, bad);
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) record_error(err, SLOKV_DEVERR_NONFINITE);
}

__global__ void __launch_bounds__(256) kv_append_fp8_commit_kernel(
    float *__restrict__ k_scale, float *__restrict__ v_scale, const int32_t *__restrict__ slots,
    int32_t num_tokens, int32_t hkv, int32_t block_size, int32_t num_blocks,
    uint32_t *__restrict__ amax_ws) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= static_cast<int64_t>(num_tokens) * hkv * 2) return;
  const int which = static_cast<int>(u & 1);
  const int h = static_cast<int>((u >> 1) % hkv);
  const int i = static_cast<int>((u >> 1) / hkv);
  const RunToken tk = run_token(slots, i, block_size, static_cast<int64_t>(num_blocks) * block_size);
  if (!tk.valid || !tk.start) return;
  const int64_t si = static_cast<int64_t>(tk.blk) * hkv + h;
  float *sp = (which ? v_scale : k_scale) + si;
  *sp = fmaxf(tk.off == 0 ? 0.f : *sp, __fdiv_rn(__uint_as_float(amax_ws[si * 2 + which]), 448.0f));
  amax_ws[si * 2 + which] = 0u;
}

__global__ void e4m3_encode_kernel(const float *__restrict__ x, uint8_t *__restrict__ codes,
                                   int64_t n, uint32_t *err) {
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    codes[i] = static_cast<uint8_t>(e4m3_encode(x[i], bad));
  if (bad) record_error(err, SLOKV_DEVERR_NONFINITE);
}

__global__ void e4m3_decode_kernel(const uint8_t *__restrict__ codes, float *__restrict__ x,
                                   int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = e4m3_decode(codes[i]);
}

unsigned grid_for(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace slokv

extern "C" int slokv_kv_append_fp8(const void *key, int64_t key_row_stride, const void *value,
                                   int64_t value_row_stride, void *k_codes, void *v_codes,
                                   float *k_scale, float *v_scale, const int32_t *slot_mapping,
                                   int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                   int32_t block_size, int32_t num_blocks, int32_t in_dtype,
                                   uint32_t *dev_error, void *stream) {
  using namespace slokv;
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return SLOKV_ERR_UNSUPPORTED;
  if (num_tokens == 0) return SLOKV_OK;
  if (!key || !value || !k_codes || !v_codes || !k_scale || !v_scale || !slot_mapping)
    return SLOKV_ERR_INVALID_ARG;
  const int es = in_dtype == SLOKV_DTYPE_F32 ? 4 : 2;
  if (in_dtype != SLOKV_DTYPE_BF16 && in_dtype != SLOKV_DTYPE_F16 && in_dtype != SLOKV_DTYPE_F32)
    return SLOKV_ERR_UNSUPPORTED;
  // 4-element loads of the input and 4-byte code stores.
  if ((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value)) % (4 * es) ||
      ((key_row_stride | value_row_stride) & 3) ||
      ((reinterpret_cast<uintptr_t>(k_codes) | reinterpret_cast<uintptr_t>(v_codes)) & 3))
    return SLOKV_ERR_ALIGNMENT;
  const int64_t threads = static_cast<int64_t>(num_tokens) * num_kv_heads * 2 * 32;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto *kc = static_cast<uint8_t *>(k_codes);
  auto *vc = static_cast<uint8_t *>(v_codes);
  if (in_dtype == SLOKV_DTYPE_BF16)
    kv_append_fp8_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16 *>(key), key_row_stride,
        static_cast<const __nv_bfloat16 *>(value), value_row_stride, kc, vc, k_scale, v_scale,
        slot_mapping, num_tokens, num_kv_heads, block_size, num_blocks, dev_error);
  else if (in_dtype == SLOKV_DTYPE_F16)
    kv_append_fp8_kernel<__half><<<grid, 256, 0, st>>>(
        static_cast<const __half *>(key), key_row_stride, static_cast<const __half *>(value),
        value_row_stride, kc, vc, k_scale, v_scale, slot_mapping, num_tokens, num_kv_heads,
        block_size, num_blocks, dev_error);
  else
    kv_append_fp8_kernel<float><<<grid, 256, 0, st>>>(
        static_cast<const float *>(key), key_row_stride, static_cast<const float *>(value),
        value_row_stride, kc, vc, k_scale, v_scale, slot_mapping, num_tokens, num_kv_heads,
        block_size, num_blocks, dev_error);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

extern "C" int slokv_fp8_e4m3_encode(const float *x, uint8_t *codes, int64_t n,
                                     uint32_t *dev_error, void *stream) {
  using namespace slokv;
  if (n < 0) return SLOKV_ERR_INVALID_ARG;
  if (n == 0) return SLOKV_OK;
  if (!x || !codes) return SLOKV_ERR_INVALID_ARG;
  e4m3_encode_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, codes, n,
                                                                                 dev_error);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

extern "C" int slokv_fp8_e4m3_decode(const uint8_t *codes, float *x, int64_t n, void *stream) {
  using namespace slokv;
  if (n < 0) return SLOKV_ERR_INVALID_ARG;
  if (n == 0) return SLOKV_OK;
  if (!x || !codes) return SLOKV_ERR_INVALID_ARG;
  e4m3_decode_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, x, n);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

extern "C" size_t slokv_kv_append_fp8_runs_workspace_bytes(int32_t num_blocks,
                                                            int32_t num_kv_heads) {
  if (num_blocks <= 0 || num_kv_heads <= 0) return 0;
  return static_cast<size_t>(num_blocks) * num_kv_heads * 2 * sizeof(uint32_t);
}

extern "C" int slokv_kv_append_fp8_runs(const void *key, int64_t key_row_stride,
                                        const void *value, int64_t value_row_stride,
                                        void *k_codes, void *v_codes, float *k_scale,
                                        float *v_scale, const int32_t *slot_mapping,
                                        int32_t num_tokens, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                        int32_t in_dtype, void *workspace,
                                        size_t workspace_bytes, uint32_t *dev_error,
                                        void *stream) {
  using namespace slokv;
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return SLOKV_ERR_UNSUPPORTED;
  if (num_tokens == 0) return SLOKV_OK;
  if (!key || !value || !k_codes || !v_codes || !k_scale || !v_scale || !slot_mapping)
    return SLOKV_ERR_INVALID_ARG;
  if (!workspace ||
      workspace_bytes < slokv_kv_append_fp8_runs_workspace_bytes(num_blocks, num_kv_heads) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3))
    return SLOKV_ERR_WORKSPACE;
  const int es = in_dtype == SLOKV_DTYPE_F32 ? 4 : 2;
  if (in_dtype != SLOKV_DTYPE_BF16 && in_dtype != SLOKV_DTYPE_F16 && in_dtype != SLOKV_DTYPE_F32)
    return SLOKV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value)) % (4 * es) ||
      ((key_row_stride | value_row_stride) & 3) ||
      ((reinterpret_cast<uintptr_t>(k_codes) | reinterpret_cast<uintptr_t>(v_codes)) & 3))
    return SLOKV_ERR_ALIGNMENT;
  const int64_t units = static_cast<int64_t>(num_tokens) * num_kv_heads * 2;
  const unsigned warp_grid = static_cast<unsigned>((static_cast<int64_t>(num_tokens) * 32 + 255) / 256);
  const unsigned unit_grid = static_cast<unsigned>((units + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto *kc = static_cast<uint8_t *>(k_codes);
  auto *vc = static_cast<uint8_t *>(v_codes);
  auto *ws = static_cast<uint32_t *>(workspace);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    kv_append_fp8_amax_kernel<T><<<warp_grid, 256, 0, st>>>(
        static_cast<const T *>(key), key_row_stride, static_cast<const T *>(value),
        value_row_stride, slot_mapping, num_tokens, num_kv_heads, block_size, num_blocks, ws,
        dev_error);
    kv_append_fp8_encode_kernel<T><<<warp_grid, 256, 0, st>>>(
        static_cast<const T *>(key), key_row_stride, static_cast<const T *>(value),
        value_row_stride, kc, vc, k_scale, v_scale, slot_mapping, num_tokens, num_kv_heads,
        block_size, num_blocks, ws, dev_error);
    kv_append_fp8_commit_kernel<<<unit_grid, 256, 0, st>>>(k_scale, v_scale, slot_mapping,
                                                            num_tokens, num_kv_heads, block_size,
                                                            num_blocks, ws);
  };
  if (in_dtype == SLOKV_DTYPE_BF16)
    run(__nv_bfloat16{});
  else if (in_dtype == SLOKV_DTYPE_F16)
    run(__half{});
  else
    run(float{});
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}
