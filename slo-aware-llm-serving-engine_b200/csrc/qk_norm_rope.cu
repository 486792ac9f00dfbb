// Fused q/k RMSNorm + rotary embedding + paged append of the new K/V rows.
//
// Replaces, for one attention layer, the chain the reference runs between the
// qkv projection and attention (nanovllm/models/qwen3.py:76-86): q_norm and
// k_norm (nanovllm/layers/layernorm.py rms_forward), the rotate-half rotary
// embedding (nanovllm/layers/rotary_embedding.py) and store_kvcache
// (nanovllm/layers/attention.py:10-40).  Input is the fused qkv row
// [Hq + 2 Hkv heads x 128]; outputs are q (and optionally k) normed and
// rotated, with the normed, rotated k and the raw v written to cache row
// slot_mapping[t] (slot -1 skips, as the reference store does).
//
// Arithmetic follows the reference's op order: RMS in fp32 (sum of squares /
// 128, rsqrtf(var + eps)), the normed row rounded to the cache dtype, times the
// weight (rounded again), then rotation in fp32 of the rounded values with
// separate multiplies and adds (y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin) and a
// final rounding.  The only freedom left is the order of the 128-term sum of
// squares.
//
// B200 mapping: HBM / launch-bound elementwise work.  One warp per (token,
// head); lane l owns dims 4l .. 4l+3 (one 8-byte load), so the row is a single
// 256-byte coalesced transaction, the sum of squares is a 5-step warp
// reduction and the rotate-half partner (dim d +- 64) is lane l ^ 16.
#include "common.cuh"

namespace slokv {
namespace {

constexpr int kHeadDim = 128;
constexpr int kWarpsPerBlock = 8;

template <typename T>
struct Vec4;
template <>
struct Vec4<__nv_bfloat16> {
  __device__ __forceinline__ static float4 load(const __nv_bfloat16 *p) {
    const uint2 r = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  __device__ __forceinline__ static void store(__nv_bfloat16 *p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t *>(&a);
    r.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = r;
  }
};
template <>
struct Vec4<__half> {
  __device__ __forceinline__ static float4 load(const __half *p) {
    const uint2 r = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
  __device__ __forceinline__ static void store(__half *p, float4 v) {
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t *>(&a);
    r.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = r;
  }
};

struct NormRopeParams {
  const void *qkv;
  int64_t qkv_stride;                    // elements between token rows
  int32_t tokens, hq, hkv;
  const void *q_w, *k_w;
  float eps;
  const int64_t *positions;
  const float *cos_sin;                  // [max_position, 128]: cos[64] | sin[64]
  int32_t max_position;
  const int32_t *slots;
  void *k_cache, *v_cache;
  int64_t num_slots;
  void *q_out;
  int64_t q_out_stride;                  // elements between tokens (heads are 128 apart)
  void *k_out;
  int64_t k_out_stride;
  uint32_t *err;
};

template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    qk_norm_rope_append_kernel(const NormRopeParams p) {
  using V = Vec4<T>;
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int heads = p.hq + p.hkv;
  if (gw >= static_cast<int64_t>(p.tokens) * heads) return;
  const int t = static_cast<int>(gw / heads);
  const int hi = static_cast<int>(gw - static_cast<int64_t>(t) * heads);
  const bool is_q = hi < p.hq;
  const T *row = static_cast<const T *>(p.qkv) + t * p.qkv_stride;
  const int d0 = 4 * lane;

  // ---- RMSNorm (fp32 statistics, two roundings) ----
  float4 x = V::load(row + static_cast<int64_t>(hi) * kHeadDim + d0);
  float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss * (1.f / kHeadDim) + p.eps);
  const float4 w = V::load(static_cast<const T *>(is_q ? p.q_w : p.k_w) + d0);
  x.x = V::round(V::round(x.x * inv) * w.x);
  x.y = V::round(V::round(x.y * inv) * w.y);
  x.z = V::round(V::round(x.z * inv) * w.z);
  x.w = V::round(V::round(x.w * inv) * w.w);

  // ---- rotate-half rotary embedding: dims d and d +- 64 pair across lane ^ 16 ----
  int64_t pos = __ldg(p.positions + t);
  if (pos < 0 || pos >= p.max_position) {   // outside the rotary table: flag, clamp
    if (lane == 0) record_error(p.err, SLOKV_DEVERR_CONTEXT_LEN);
    pos = pos < 0 ? 0 : p.max_position - 1;
  }
  const float4 y = make_float4(__shfl_xor_sync(0xffffffffu, x.x, 16),
                               __shfl_xor_sync(0xffffffffu, x.y, 16),
                               __shfl_xor_sync(0xffffffffu, x.z, 16),
                               __shfl_xor_sync(0xffffffffu, x.w, 16));
  const int i0 = d0 & 63;                            // index within the half
  const float4 cs = *reinterpret_cast<const float4 *>(p.cos_sin + pos * kHeadDim + i0);
  const float4 sn = *reinterpret_cast<const float4 *>(p.cos_sin + pos * kHeadDim + 64 + i0);
  float4 r;
  if (lane < 16) {   // first half: x1 = own, x2 = partner: x1 cos - x2 sin
    r.x = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(y.x, sn.x));
    r.y = __fsub_rn(__fmul_rn(x.y, cs.y), __fmul_rn(y.y, sn.y));
    r.z = __fsub_rn(__fmul_rn(x.z, cs.z), __fmul_rn(y.z, sn.z));
    r.w = __fsub_rn(__fmul_rn(x.w, cs.w), __fmul_rn(y.w, sn.w));
  } else {           // second half: x2 = own, x1 = partner: x2 cos + x1 sin
    r.x = __fadd_rn(__fmul_rn(x.x, cs.x), __fmul_rn(y.x, sn.x));
    r.y = __fadd_rn(__fmul_rn(x.y, cs.y), __fmul_rn(y.y, sn.y));
    r.z = __fadd_rn(__fmul_rn(x.z, cs.z), __fmul_rn(y.z, sn.z));
    r.w = __fadd_rn(__fmul_rn(x.w, cs.w), __fmul_rn(y.w, sn.w));
  }

  if (is_q) {
    V::store(static_cast<T *>(p.q_out) + t * p.q_out_stride + hi * kHeadDim + d0, r);
    return;
  }
  const int hk = hi - p.hq;
  if (p.k_out != nullptr)
    V::store(static_cast<T *>(p.k_out) + t * p.k_out_stride + hk * kHeadDim + d0, r);
  const int64_t slot = __ldg(p.slots + t);
  if (slot == -1) return;
  if (slot < -1 || slot >= p.num_slots) {
    if (lane == 0) record_error(p.err, SLOKV_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t crow = slot * p.hkv * kHeadDim + hk * kHeadDim + d0;
  V::store(static_cast<T *>(p.k_cache) + crow, r);
  // v: raw copy of this head's row
  const uint2 vv = *reinterpret_cast<const uint2 *>(
      row + static_cast<int64_t>(p.hq + p.hkv + hk) * kHeadDim + d0);
  *reinterpret_cast<uint2 *>(static_cast<T *>(p.v_cache) + crow) = vv;
}

}  // namespace
}  // namespace slokv

extern "C" int slokv_qk_norm_rope_append(
    const void *qkv, int64_t qkv_row_stride, int32_t num_tokens, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, const void *q_weight, const void *k_weight, float eps,
    const int64_t *positions, const float *cos_sin, int32_t max_position,
    const int32_t *slot_mapping, void *k_cache, void *v_cache, int64_t num_slots, void *q_out,
    int64_t q_out_row_stride, void *k_out, int64_t k_out_row_stride, int32_t dtype,
    uint32_t *dev_error, void *stream) {
  using namespace slokv;
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_position <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (num_tokens == 0) return SLOKV_OK;
  if (head_dim != kHeadDim) return SLOKV_ERR_UNSUPPORTED;
  if (dtype != SLOKV_DTYPE_BF16 && dtype != SLOKV_DTYPE_F16) return SLOKV_ERR_UNSUPPORTED;
  if (!qkv || !q_weight || !k_weight || !positions || !cos_sin || !slot_mapping || !k_cache ||
      !v_cache || !q_out || num_slots <= 0)
    return SLOKV_ERR_INVALID_ARG;
  // 8-byte vectors of 2-byte elements: rows, heads and weights 8-byte aligned;
  // the cos/sin table 16-byte aligned (float4 reads).
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q_out) |
                         reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(k_cache) |
                         reinterpret_cast<uintptr_t>(v_cache) |
                         reinterpret_cast<uintptr_t>(q_weight) |
                         reinterpret_cast<uintptr_t>(k_weight);
  if ((ptrs & 7u) || (reinterpret_cast<uintptr_t>(cos_sin) & 15u)) return SLOKV_ERR_ALIGNMENT;
  if ((qkv_row_stride | q_out_row_stride | (k_out ? k_out_row_stride : 0)) & 3)
    return SLOKV_ERR_ALIGNMENT;
  NormRopeParams p;
  p.qkv = qkv;
  p.qkv_stride = qkv_row_stride;
  p.tokens = num_tokens;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.q_w = q_weight;
  p.k_w = k_weight;
  p.eps = eps;
  p.positions = positions;
  p.cos_sin = cos_sin;
  p.max_position = max_position;
  p.slots = slot_mapping;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.num_slots = num_slots;
  p.q_out = q_out;
  p.q_out_stride = q_out_row_stride;
  p.k_out = k_out;
  p.k_out_stride = k_out_row_stride;
  p.err = dev_error;
  const int64_t warps = static_cast<int64_t>(num_tokens) * (num_q_heads + num_kv_heads);
  const int64_t blocks = (warps + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > 0x7fffffff) return SLOKV_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == SLOKV_DTYPE_BF16)
    qk_norm_rope_append_kernel<__nv_bfloat16>
        <<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, st>>>(p);
  else
    qk_norm_rope_append_kernel<__half>
        <<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}
