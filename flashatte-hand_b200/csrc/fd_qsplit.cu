// fd_qsplit.cu - query rows as three e4m3 parts for the e4m3-cache kernel.
//
// With an e4m3 K cache the QK product runs as kind::f8f6f4 UMMAs, whose two
// operands must both be 8-bit.  Each 16-bit query row is therefore scaled by
// a power of two (so its largest magnitude lands in [128, 256), below the
// e4m3 maximum of 448) and split into three e4m3 parts (fd_fp8.cuh) that the
// kernel multiplies side by side and recombines in fp32; the power of two is
// undone exactly by its inverse, stored per row.  The reference has no FP8
// path; this is the query half of the FP8 KV-cache extension of its decode.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fd_fp8.cuh"
#include "fd_kernels.h"

namespace fd {

namespace {

constexpr int kSplitThreads = 128;  // 16 rows x 8 threads x 16 dims

template <typename T> __device__ __forceinline__ float load_f32(const T* p);
template <> __device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <> __device__ __forceinline__ float load_f32<__half>(const __half* p) {
  return __half2float(*p);
}

// One CTA per (sequence b, KV head kvh): rows r = qi * group + g.
template <typename T>
__global__ void __launch_bounds__(kSplitThreads)
    split_query_kernel(const T* __restrict__ q, int seqlen_q, int num_heads, int group,
                       uint8_t* __restrict__ q8, float* __restrict__ q_inv) {
  const int bk = blockIdx.x;  // b * Hkv + kvh
  const int hkv = num_heads / group;
  const int b = bk / hkv, kvh = bk - b * hkv;
  const int r = threadIdx.x >> 3;
  const int d0 = (threadIdx.x & 7) * 16;
  const int qi = r / group, g = r - qi * group;
  const bool valid = qi < seqlen_q;
  float x[16];
  float mx = 0.f;
  if (valid) {
    const T* src = q + ((static_cast<int64_t>(b) * seqlen_q + qi) * num_heads + kvh * group + g) *
                           kHeadDim + d0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      x[i] = load_f32(src + i);
      mx = fmaxf(mx, fabsf(x[i]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = 0.f;
  }
  // row maximum over the row's 8 threads (consecutive lanes)
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
  // s = 2^k with mx * s in [128, 256): k = 7 - floor(log2 mx), clamped to the
  // normal range; rows of zeros (and padding rows) keep s = 1.
  int k = 0;
  if (mx > 0.f && mx <= 3.0e38f) {
    const int e = ((__float_as_int(mx) >> 23) & 0xff) - 127;
    k = 7 - e;
    k = k < -126 ? -126 : (k > 126 ? 126 : k);
  }
  const float s = __int_as_float((k + 127) << 23);
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] *= s;
  uint4 parts[3];
  e4m3_split16(x, parts);
  uint8_t* dst = q8 + static_cast<int64_t>(bk) * (3 * kMaxGroup * kHeadDim) + r * kHeadDim + d0;
#pragma unroll
  for (int p = 0; p < 3; ++p)
    *reinterpret_cast<uint4*>(dst + p * kMaxGroup * kHeadDim) = parts[p];
  if ((threadIdx.x & 7) == 0)
    q_inv[static_cast<int64_t>(bk) * kMaxGroup + r] = valid ? __int_as_float((127 - k) << 23) : 0.f;
}

}  // namespace

cudaError_t launch_split_query(const void* q, int dtype, int batch, int seqlen_q, int num_heads,
                               int num_heads_k, uint8_t* q8, float* q_inv, cudaStream_t stream) {
  const int64_t blocks = static_cast<int64_t>(batch) * num_heads_k;
  if (blocks <= 0) return cudaSuccess;
  const int group = num_heads / num_heads_k;
  if (dtype == 0)
    split_query_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), kSplitThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(q), seqlen_q, num_heads, group, q8, q_inv);
  else
    split_query_kernel<__half><<<static_cast<unsigned>(blocks), kSplitThreads, 0, stream>>>(
        static_cast<const __half*>(q), seqlen_q, num_heads, group, q8, q_inv);
  return cudaGetLastError();
}

}  // namespace fd
