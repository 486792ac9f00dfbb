// Paged KV append: scatter each step's new K/V rows into the block pool through
// slot_mapping.  Replaces the Triton store_kvcache kernel of the reference
// (nanovllm/layers/attention.py:10-40): same semantics (slot == -1 skips the
// token; cache row `slot` receives num_kv_heads * head_dim contiguous
// elements), bit copy for any element width.
//
// B200 design: the copy is pure HBM traffic (2 KB of K + 2 KB of V per token at
// Qwen3-4B TP1), so every thread moves one 16-byte vector of K and one of V,
// consecutive threads cover consecutive vectors of a row (fully coalesced
// 512-byte warp transactions), and a grid-stride loop keeps several vectors in
// flight per thread for the large mixed-batch case (up to 16K tokens).
#include "common.cuh"

namespace slokv {
namespace {

template <typename Vec>
__global__ void __launch_bounds__(256) kv_append_kernel(
    const char *__restrict__ key, int64_t key_stride, const char *__restrict__ value,
    int64_t value_stride, char *__restrict__ k_cache, char *__restrict__ v_cache,
    const int32_t *__restrict__ slots, int32_t num_tokens, int32_t chunks, int64_t row_bytes,
    int64_t num_slots, uint32_t *err) {
  const int64_t total = static_cast<int64_t>(num_tokens) * chunks;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    const int32_t n = static_cast<int32_t>(i / chunks);
    const int32_t c = static_cast<int32_t>(i - static_cast<int64_t>(n) * chunks);
    const int64_t slot = __ldg(slots + n);
    if (slot == -1) continue;
    if (slot < -1 || slot >= num_slots) {
      if (c == 0) record_error(err, SLOKV_DEVERR_SLOT_RANGE);
      continue;
    }
    const int64_t off = static_cast<int64_t>(c) * sizeof(Vec);
    const Vec kv = *reinterpret_cast<const Vec *>(key + n * key_stride + off);
    const Vec vv = *reinterpret_cast<const Vec *>(value + n * value_stride + off);
    *reinterpret_cast<Vec *>(k_cache + slot * row_bytes + off) = kv;
    *reinterpret_cast<Vec *>(v_cache + slot * row_bytes + off) = vv;
  }
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

template <typename Vec>
int launch(const void *key, int64_t ks, const void *value, int64_t vs, void *kc, void *vc,
           const int32_t *slots, int32_t n, int64_t row_bytes, int64_t num_slots, uint32_t *err,
           cudaStream_t stream) {
  const int32_t chunks = static_cast<int32_t>(row_bytes / sizeof(Vec));
  const int64_t total = static_cast<int64_t>(n) * chunks;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  kv_append_kernel<Vec><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const char *>(key), ks, static_cast<const char *>(value), vs,
      static_cast<char *>(kc), static_cast<char *>(vc), slots, n, chunks, row_bytes, num_slots,
      err);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}

}  // namespace
}  // namespace slokv

extern "C" int slokv_kv_append(const void *key, int64_t key_row_stride, const void *value,
                               int64_t value_row_stride, void *k_cache, void *v_cache,
                               const int32_t *slot_mapping, int32_t num_tokens,
                               int32_t row_elems, int32_t elem_bytes, int64_t num_slots,
                               uint32_t *dev_error, void *stream) {
  using namespace slokv;
  if (num_tokens < 0 || row_elems <= 0 || num_slots < 0) return SLOKV_ERR_INVALID_ARG;
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4) return SLOKV_ERR_UNSUPPORTED;
  if (num_tokens == 0) return SLOKV_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return SLOKV_ERR_INVALID_ARG;
  const int64_t row_bytes = static_cast<int64_t>(row_elems) * elem_bytes;
  const int64_t ks = key_row_stride * elem_bytes, vs = value_row_stride * elem_bytes;
  // Widest vector every address and stride allows.
  uint64_t bits = static_cast<uint64_t>(row_bytes) | static_cast<uint64_t>(ks) |
                  static_cast<uint64_t>(vs) | reinterpret_cast<uintptr_t>(key) |
                  reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(k_cache) |
                  reinterpret_cast<uintptr_t>(v_cache);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((bits & 15u) == 0)
    return launch<int4>(key, ks, value, vs, k_cache, v_cache, slot_mapping, num_tokens, row_bytes,
                        num_slots, dev_error, s);
  if ((bits & 7u) == 0)
    return launch<uint2>(key, ks, value, vs, k_cache, v_cache, slot_mapping, num_tokens,
                         row_bytes, num_slots, dev_error, s);
  if ((bits & 3u) == 0)
    return launch<uint32_t>(key, ks, value, vs, k_cache, v_cache, slot_mapping, num_tokens,
                            row_bytes, num_slots, dev_error, s);
  if ((bits & 1u) == 0)
    return launch<uint16_t>(key, ks, value, vs, k_cache, v_cache, slot_mapping, num_tokens,
                            row_bytes, num_slots, dev_error, s);
  return launch<uint8_t>(key, ks, value, vs, k_cache, v_cache, slot_mapping, num_tokens,
                         row_bytes, num_slots, dev_error, s);
}

extern "C" const char *slokv_status_string(int status) {
  switch (status) {
    case SLOKV_OK: return "ok";
    case SLOKV_ERR_INVALID_ARG: return "invalid argument";
    case SLOKV_ERR_ALIGNMENT: return "pointer or stride not aligned as required";
    case SLOKV_ERR_UNSUPPORTED: return "unsupported dtype or geometry";
    case SLOKV_ERR_CUDA: return "CUDA runtime error";
    case SLOKV_ERR_WORKSPACE: return "workspace missing or too small";
    case SLOKV_ERR_SCRATCH_LIMIT:
      return "geometry needs more than the fixed scratch of the allocation-free entry point";
    default: return "unknown status";
  }
}

extern "C" int slokv_abi_version(void) { return 3; }
