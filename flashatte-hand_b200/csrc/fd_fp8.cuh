// fd_fp8.cuh - e4m3 helpers shared by the FP8-cache kernels.
//
// A value x is carried through an e4m3 tensor-core product as three e4m3
// parts, x ~= p0 + p1 / 16 + p2 / 256: p0 = rn(x), p1 = rn(16 (x - p0)),
// p2 = rn(16 (16 (x - p0) - p1)).  Each part adds about four significant
// bits, so the sum keeps about twelve (a 16-bit query row is reproduced to
// within its own rounding), and the parts are placed side by side in the
// UMMA N dimension where they cost nothing (a tcgen05.mma takes the same
// time for any N up to 64).  Callers scale x so its magnitude sits below the
// e4m3 maximum (448) and well above its smallest subnormal (2^-9).
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace fd {

__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  return static_cast<uint32_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t v) {
  const __half2_raw r =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v & 0xFFFFu), __NV_E4M3);
  return __half22float2(__half2(r));
}

// Parts of a pair (a, b): w[k] holds part k of a in its low byte, of b in the next.
__device__ __forceinline__ void e4m3_split2(float a, float b, uint32_t (&w)[3]) {
  w[0] = e4m3x2(a, b);
  float2 f = e4m3x2_to_float2(w[0]);
  a = (a - f.x) * 16.f;
  b = (b - f.y) * 16.f;
  w[1] = e4m3x2(a, b);
  f = e4m3x2_to_float2(w[1]);
  a = (a - f.x) * 16.f;
  b = (b - f.y) * 16.f;
  w[2] = e4m3x2(a, b);
}

// Parts of 16 consecutive values: part k as 16 bytes in out[k].
__device__ __forceinline__ void e4m3_split16(const float (&x)[16], uint4 (&out)[3]) {
  uint32_t w[8][3];
#pragma unroll
  for (int i = 0; i < 8; ++i) e4m3_split2(x[2 * i], x[2 * i + 1], w[i]);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    out[k].x = w[0][k] | (w[1][k] << 16);
    out[k].y = w[2][k] | (w[3][k] << 16);
    out[k].z = w[4][k] | (w[5][k] << 16);
    out[k].w = w[6][k] | (w[7][k] << 16);
  }
}

}  // namespace fd
