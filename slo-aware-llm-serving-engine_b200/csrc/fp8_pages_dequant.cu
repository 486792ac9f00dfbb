// Dequantise the FP8-E4M3 pool pages that a batch of prefill rows reads into a
// bf16/f16 page buffer, so prefix-cache (paged) prefill over an FP8 pool runs on
// the tcgen05 prefill kernel unchanged.
//
// Row r of the batch reads keys 0 .. k_len_r - 1 through block_tables[r]; its
// page p (p < pages_per_row, p * block_size < k_len_r) is written to buffer page
// r * pages_per_row + p in f16: K as its unscaled code values (E4M3 is a subset
// of f16, so exact) with the page's K scale kept beside it -- the prefill
// multiplies the logits by it, as the FP8 decode does, instead of rounding
// code * scale (|k| up to the block amax) to 10 bits -- and V as
// decode(code) * scale (fp32 product, the oracle's dequantisation) rounded to
// f16.  Pages past a row's keys are not touched (the prefill never reads them);
// a block id outside the pool fills its buffer page with zeros (scale 0) and
// sets SLOKV_DEVERR_BLOCK_RANGE.
//
// B200 mapping: streaming HBM work (1 byte in, 2 bytes out per element).  One
// thread per 16 codes of a page (one 16-byte load per plane, two 16-byte stores),
// consecutive threads on consecutive bytes, grid-stride over all pages.
#include "common.cuh"
#include "fp8_e4m3.cuh"

namespace slokv {
namespace {

constexpr int kHeadDim = 128;

struct DequantParams {
  const uint8_t *k_codes, *v_codes;
  int64_t k_block_stride, v_block_stride;   // bytes (= elements) between pages
  const float *k_scale, *v_scale;           // [num_blocks, hkv]
  int32_t num_blocks, block_size, hkv;
  const int32_t *tables;
  int64_t table_stride;
  int32_t max_blocks;
  const int32_t *cu_k;
  int32_t rows, width;                      // pages_per_row
  __half *dst_k, *dst_v;
  float *dst_k_scale;                       // [rows * width, hkv]
  uint32_t *err;
};

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void dequant16(const uint4 codes, float scale, __half *dst) {
  const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = __fmul_rn(e4m3_decode(w[i] & 0xffu), scale);
    const float b = __fmul_rn(e4m3_decode((w[i] >> 8) & 0xffu), scale);
    const float c = __fmul_rn(e4m3_decode((w[i] >> 16) & 0xffu), scale);
    const float d = __fmul_rn(e4m3_decode(w[i] >> 24), scale);
    out[2 * i] = pack2(a, b);
    out[2 * i + 1] = pack2(c, d);
  }
  reinterpret_cast<uint4 *>(dst)[0] = make_uint4(out[0], out[1], out[2], out[3]);
  reinterpret_cast<uint4 *>(dst)[1] = make_uint4(out[4], out[5], out[6], out[7]);
}

__global__ void __launch_bounds__(256) fp8_pages_dequant_kernel(const DequantParams p) {
  const int64_t page_elems = static_cast<int64_t>(p.block_size) * p.hkv * kHeadDim;
  const int64_t units = page_elems / 16;                 // 16 codes per thread step
  const int64_t total = static_cast<int64_t>(p.rows) * p.width * units;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += step) {
    const int64_t slot = u / units;
    const int64_t e0 = (u - slot * units) * 16;          // element offset in the page
    const int r = static_cast<int>(slot / p.width);
    const int pg = static_cast<int>(slot - static_cast<int64_t>(r) * p.width);
    const int k_len = __ldg(p.cu_k + r + 1) - __ldg(p.cu_k + r);
    if (static_cast<int64_t>(pg) * p.block_size >= k_len) continue;
    __half *dk = p.dst_k + slot * page_elems + e0;
    __half *dv = p.dst_v + slot * page_elems + e0;
    // the first chunk of each head of the page's first token carries the scale
    const bool head_lead = e0 < static_cast<int64_t>(p.hkv) * kHeadDim && e0 % kHeadDim == 0;
    const int32_t blk =
        pg < p.max_blocks ? __ldg(p.tables + static_cast<int64_t>(r) * p.table_stride + pg) : -1;
    if (blk < 0 || blk >= p.num_blocks) {
      if (e0 == 0) record_error(p.err, SLOKV_DEVERR_BLOCK_RANGE);
      if (head_lead) p.dst_k_scale[slot * p.hkv + e0 / kHeadDim] = 0.f;
      const uint4 z = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4 *>(dk)[0] = z;
      reinterpret_cast<uint4 *>(dk)[1] = z;
      reinterpret_cast<uint4 *>(dv)[0] = z;
      reinterpret_cast<uint4 *>(dv)[1] = z;
      continue;
    }
    const int h = static_cast<int>((e0 / kHeadDim) % p.hkv);
    const int64_t si = static_cast<int64_t>(blk) * p.hkv + h;
    const uint4 ck = *reinterpret_cast<const uint4 *>(p.k_codes + blk * p.k_block_stride + e0);
    const uint4 cv = *reinterpret_cast<const uint4 *>(p.v_codes + blk * p.v_block_stride + e0);
    if (head_lead) p.dst_k_scale[slot * p.hkv + h] = __ldg(p.k_scale + si);
    dequant16(ck, 1.f, dk);
    dequant16(cv, __ldg(p.v_scale + si), dv);
  }
}

int sm_count_dq() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

}  // namespace
}  // namespace slokv

extern "C" int slokv_fp8_pages_dequant(const void *k_codes, const void *v_codes,
                                       int64_t k_block_stride, int64_t v_block_stride,
                                       const float *k_scale, const float *v_scale,
                                       int32_t num_blocks, int32_t block_size,
                                       int32_t num_kv_heads, int32_t head_dim,
                                       const int32_t *block_tables, int64_t block_table_stride,
                                       int32_t max_blocks_per_seq, const int32_t *cu_seqlens_k,
                                       int32_t num_rows, int32_t pages_per_row, void *dst_k,
                                       void *dst_v, float *dst_k_scale, uint32_t *dev_error,
                                       void *stream) {
  using namespace slokv;
  if (num_rows < 0 || pages_per_row < 0 || num_blocks <= 0 || block_size <= 0 ||
      num_kv_heads <= 0 || max_blocks_per_seq <= 0)
    return SLOKV_ERR_INVALID_ARG;
  if (num_rows == 0 || pages_per_row == 0) return SLOKV_OK;
  if (head_dim != kHeadDim) return SLOKV_ERR_UNSUPPORTED;
  if (!k_codes || !v_codes || !k_scale || !v_scale || !block_tables || !cu_seqlens_k || !dst_k ||
      !dst_v || !dst_k_scale)
    return SLOKV_ERR_INVALID_ARG;
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(k_codes) |
                         reinterpret_cast<uintptr_t>(v_codes) | reinterpret_cast<uintptr_t>(dst_k) |
                         reinterpret_cast<uintptr_t>(dst_v);
  if ((ptrs & 15u) || ((k_block_stride | v_block_stride) & 15)) return SLOKV_ERR_ALIGNMENT;
  DequantParams p;
  p.k_codes = static_cast<const uint8_t *>(k_codes);
  p.v_codes = static_cast<const uint8_t *>(v_codes);
  p.k_block_stride = k_block_stride;
  p.v_block_stride = v_block_stride;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.hkv = num_kv_heads;
  p.tables = block_tables;
  p.table_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.cu_k = cu_seqlens_k;
  p.rows = num_rows;
  p.width = pages_per_row;
  p.dst_k = static_cast<__half *>(dst_k);
  p.dst_v = static_cast<__half *>(dst_v);
  p.dst_k_scale = dst_k_scale;
  p.err = dev_error;
  const int64_t units = static_cast<int64_t>(num_rows) * pages_per_row * block_size *
                        num_kv_heads * kHeadDim / 16;
  int64_t blocks = (units + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_dq()) * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  fp8_pages_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SLOKV_OK : SLOKV_ERR_CUDA;
}
