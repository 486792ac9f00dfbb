// E4M3FN (OCP FP8, finite-only, max 448) codec used by the quantised KV cache.
//
// Semantics follow the reference engine's exact CPU encoder
// (benchmarks/v0/probe_quant_support.py:24-56): nearest representable value,
// ties to the even code, magnitude saturated at 448, sign kept (-0 -> 0x80);
// non-finite input has no code (the reference raises; here the caller's error
// word is flagged and the NaN code 0x7F is stored).
//
// Encoding (derived from the format): the 127 non-negative codes are monotonic
// and every binade holds 8 of them, so for 0 <= m < 448 with binade exponent
// e = max(floor(log2 m), -6):  code = 8 (e + 7) + rint(m * 2^(3 - e)) - 8.
// m * 2^(3-e) is an exact power-of-two scaling, rint() is the hardware
// round-to-nearest-even, and a mantissa that rounds up to 16 carries into the
// next binade's first code; e = -6 covers the subnormal codes (quantum 2^-9).
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace slokv {

__device__ __forceinline__ uint32_t e4m3_encode(float t, bool &nonfinite) {
  const uint32_t bits = __float_as_uint(t);
  const uint32_t sign = (bits >> 24) & 0x80u;
  const float mag = __uint_as_float(bits & 0x7fffffffu);
  if (!(mag <= 3.402823466e38f)) {  // NaN or infinity
    nonfinite = true;
    return sign | 0x7fu;
  }
  if (mag >= 448.0f) return sign | 126u;
  int e = static_cast<int>((__float_as_uint(mag) >> 23) & 0xffu) - 127;
  if (e < -6) e = -6;
  const float pow2 = __uint_as_float(static_cast<uint32_t>(127 + 3 - e) << 23);
  const float q = __fmul_rn(mag, pow2);
  const int r = static_cast<int>(rintf(q));
  return sign | static_cast<uint32_t>((e + 7) * 8 + r - 8);
}

__device__ __forceinline__ float e4m3_decode(uint32_t code) {
  const uint32_t sign = (code & 0x80u) << 24;
  const uint32_t e = (code >> 3) & 0xfu, m = code & 7u;
  if (e == 15u && m == 7u) return __uint_as_float(0x7fc00000u | sign);
  if (e == 0u) return __uint_as_float(__float_as_uint(static_cast<float>(m) * 0.001953125f) | sign);
  return __uint_as_float(sign | ((e + 120u) << 23) | (m << 20));
}

// Two E4M3 codes (low byte = first) -> f16x2 (low half = first), exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_codes) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
      static_cast<__nv_fp8x2_storage_t>(two_codes & 0xffffu), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

}  // namespace slokv
