// fd_xgpu.cu - second half of the cross-GPU split-KV step: merge the parts
// every rank pushed into this rank's exchange buffer over NVLink.
//
// Each rank's decode kernel (fd_decode_sm100.cu, exchange mode) stores its
// partial (O, ln-LSE) for every output row straight into every rank's
// exchange buffer through peer mappings, and the last of its CTAs stores the
// step's epoch into each rank's flag for it.  This kernel waits (bounded)
// until all flags of the current buffer half read the epoch, then merges the
// parts with LSE weights — the reference's split combine
// (submission-oj/best_flashattn_kvcache_decode.cu:956-1037) with the splits
// on different GPUs, and the data moved by the producing kernel itself rather
// than by a separate collective.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fd_kernels.h"
#include "fd_ptx.cuh"

namespace fd {

namespace {

constexpr int kCombineThreads = 128;

template <typename O> __device__ __forceinline__ O from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// One CTA per output row r = (b * sq + qi) * hq + h; LSE rows are laid out
// (b * hq + h) * sq + qi as in the decode kernel.
template <typename OutT>
__global__ void __launch_bounds__(kCombineThreads)
    exchange_combine_kernel(const float* __restrict__ parts, int64_t part_stride, int64_t lse_off,
                            const uint32_t* flags, int world, uint32_t epoch, int sq, int hq,
                            OutT* __restrict__ out, float* __restrict__ lse_out, int* err,
                            unsigned long long timeout_ns) {
  __shared__ int ready;
  const int tid = threadIdx.x;
  if (tid == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < world && ok; ++j) {
      while (ld_acquire_sys_u32(flags + j) != epoch) {
        if (globaltimer_ns() - t0 > timeout_ns) {
          ok = 0;
          report_status(err, kStatusTimeout);
          break;
        }
      }
    }
    ready = ok;
  }
  __syncthreads();
  if (!ready) return;

  const int64_t r = blockIdx.x;
  const int64_t per_b = static_cast<int64_t>(sq) * hq;
  const int64_t b = r / per_b;
  const int64_t rem = r - b * per_b;
  const int64_t qi = rem / hq, h = rem - qi * hq;
  const int64_t li = (b * hq + h) * sq + qi;
  const float neg_inf = -__int_as_float(0x7f800000);
  const float log2e = 1.4426950408889634f;
  float mx = neg_inf;
  for (int j = 0; j < world; ++j) mx = fmaxf(mx, __ldcg(parts + j * part_stride + lse_off + li));
  float den = 0.f;
  float w[kMaxExchangeRanks];
#pragma unroll
  for (int j = 0; j < kMaxExchangeRanks; ++j) {
    w[j] = 0.f;
    if (j < world) {
      const float lj = __ldcg(parts + j * part_stride + lse_off + li);
      w[j] = lj == neg_inf ? 0.f : fast_exp2((lj - mx) * log2e);
      den += w[j];
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = tid; d < kHeadDim; d += kCombineThreads) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxExchangeRanks; ++j)
      if (j < world && w[j] > 0.f) acc = fmaf(w[j], __ldcg(parts + j * part_stride + r * kHeadDim + d), acc);
    out[r * kHeadDim + d] = from_f32<OutT>(acc * inv);
  }
  if (lse_out != nullptr && tid == 0)
    lse_out[li] = den > 0.f ? mx + fast_log2(den) * 0.69314718055994531f : neg_inf;
}

}  // namespace

cudaError_t launch_exchange_combine(const float* parts, int64_t part_stride, int64_t lse_off,
                                    const uint32_t* flags, int world, uint32_t epoch, int64_t rows,
                                    int sq, int hq, void* out, int out_dtype, float* lse_out,
                                    int* err, unsigned long long timeout_ns, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(rows));
  switch (out_dtype) {
    case 0:
      exchange_combine_kernel<__nv_bfloat16><<<grid, kCombineThreads, 0, stream>>>(
          parts, part_stride, lse_off, flags, world, epoch, sq, hq,
          static_cast<__nv_bfloat16*>(out), lse_out, err, timeout_ns);
      break;
    case 1:
      exchange_combine_kernel<__half><<<grid, kCombineThreads, 0, stream>>>(
          parts, part_stride, lse_off, flags, world, epoch, sq, hq, static_cast<__half*>(out),
          lse_out, err, timeout_ns);
      break;
    default:
      exchange_combine_kernel<float><<<grid, kCombineThreads, 0, stream>>>(
          parts, part_stride, lse_off, flags, world, epoch, sq, hq, static_cast<float*>(out),
          lse_out, err, timeout_ns);
      break;
  }
  return cudaGetLastError();
}

}  // namespace fd
