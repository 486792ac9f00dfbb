// Block-pool page copy for prefix sharing (copy-on-write of a shared tail
// block), preemption by swap (gather pages into a compact buffer, scatter them
// back) and snapshot/restore.  The reference's only device page copy is
// `pool[:, :, page].copy_(saved[:, :, j])` over every (K|V, layer) plane
// (diagnostics/online_token_replay/tensors.py:34-43); this kernel performs all
// pages x planes of such a copy in one launch.
//
// Pure HBM traffic: each CTA moves 16 KB units (256 threads x 4 x 16-byte
// vectors, all four loads issued before the stores), grid-strided over
// pages x planes x units so one launch saturates the copy bandwidth.
#include "common.cuh"

namespace slokv {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int64_t kUnitBytes = static_cast<int64_t>(kThreads) * kVecPerThread * 16;

__global__ void __launch_bounds__(kThreads) kv_block_copy_kernel(
    const char *__restrict__ src, int64_t src_plane, int64_t src_page,
    const int32_t *__restrict__ src_ids, int32_t src_cap, char *__restrict__ dst,
    int64_t dst_plane, int64_t dst_page, const int32_t *__restrict__ dst_ids, int32_t dst_cap,
    int32_t num_pages, int32_t num_planes, int64_t page_bytes, int64_t units_per_page,
    uint32_t *err) {
  const int64_t total = static_cast<int64_t>(num_pages) * num_planes * units_per_page;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    const int64_t unit = u % units_per_page;
    const int64_t pp = u / units_per_page;
    const int32_t plane = static_cast<int32_t>(pp % num_planes);
    const int32_t i = static_cast<int32_t>(pp / num_planes);
    const int64_t s = src_ids ? static_cast<int64_t>(__ldg(src_ids + i)) : i;
    const int64_t d = dst_ids ? static_cast<int64_t>(__ldg(dst_ids + i)) : i;
    if (s < 0 || d < 0) continue;
    if (s >= src_cap || d >= dst_cap) {
      if (threadIdx.x == 0 && unit == 0 && plane == 0) record_error(err, SLOKV_DEVERR_BLOCK_RANGE);
      continue;
    }
    const char *sp = src + plane * src_plane + s * src_page;
    char *dp = dst + plane * dst_plane + d * dst_page;
    const int64_t off0 = unit * kUnitBytes;
    int4 v[kVecPerThread];
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t off = off0 + (static_cast<int64_t>(k) * kThreads + threadIdx.x) * 16;
      if (off < page_bytes) v[k] = __ldcs(reinterpret_cast<const int4 *>(sp + off));
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t off = off0 + (static_cast<int64_t>(k) * kThreads + threadIdx.x) * 16;
      if (off < page_bytes) __stcs(reinterpret_cast<int4 *>(dp + off), v[k]);
    }
  }
}

}  // namespace
}  // namespace slokv

extern "C" int slokv_kv_block_copy(const void *src, int64_t src_plane_stride_bytes,
                                   int64_t src_page_stride_bytes, const int32_t *src_ids,
                                   int32_t src_capacity, void *dst,
                                   int64_t dst_plane_stride_bytes, int64_t dst_page_stride_bytes,
                                   const int32_t *dst_ids, int32_t dst_capacity,
                                   int32_t num_pages, int32_t num_planes, int64_t page_bytes,
                                   uint32_t *dev_error, void *stream) {
  using namespace slokv;
  if (num_pages < 0 || num_planes < 0 || page_bytes < 0 || src_capacity < 0 || dst_capacity < 0)
    return SLOKV_ERR_INVALID_ARG;
  if (num_pages == 0 || num_planes == 0 || page_bytes == 0) return SLOKV_OK;
  if (!src || !dst) return SLOKV_ERR_INVALID_ARG;
  const uint64_t bits = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                        static_cast<uint64_t>(src_plane_stride_bytes) |
                        static_cast<uint64_t>(src_page_stride_bytes) |
                        static_cast<uint64_t>(dst_plane_stride_bytes) |
                        static_cast<uint64_t>(dst_page_stride_bytes) |
                        static_cast<uint64_t>(page_bytes);
  if (bits & 15u) return SLOKV_ERR_ALIGNMENT;
  const int64_t units = (page_bytes + kUnitBytes - 1) / kUnitBytes;
  const int64_t total = static_cast<int64_t>(num_pages) * num_planes * units;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = static_cast<int64_t>(sms) * 8;
  if (grid > total) grid = total;
  kv_block_copy_kernel<<<static_cast<unsigned>(grid), kThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char *>(src), src_plane_stride_bytes, src_page_stride_bytes, src_ids,
      src_capacity, static_cast<char *>(dst), dst_plane_stride_bytes, dst_page_stride_bytes,
      dst_ids, dst_capacity, num_pages, num_planes, page_bytes, units, dev_error);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}
