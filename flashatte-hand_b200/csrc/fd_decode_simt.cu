// fd_decode_simt.cu - CUDA-core decode kernel for the shapes the tensor-core
// path does not take (head dim other than 128, more than 16 query heads per
// KV head, page sizes that are not a multiple of 16, unaligned pointers), and
// the stand-alone LSE combine kernel used after a cross-GPU exchange.
//
// The SIMT kernel plays the role of the reference's paged_decode_fallback_
// kernel (submission-oj/best_flashattn_kvcache_decode.cu:233-371): one CTA per
// (sequence, query head), same edge rules (length <= 0 writes zeros, length 1
// returns the single V row), but warp-parallel over tokens instead of one
// block reduction per token, any head dim in {32, 64, 128, 256}, any group
// size and page size, fp32 online softmax in the log2 domain.  A page id
// inside a sequence's range that is outside the pool reads as zero rows and
// is reported in the device status word (FD_ERR_BAD_PAGE).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fd_kernels.h"
#include "fd_ptx.cuh"

namespace fd {

namespace {

constexpr int kSimtWarps = 4;

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename O> __device__ __forceinline__ O from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Vec {
  T v[VEC];
};

template <typename T, typename OutT, int VEC>
__global__ void __launch_bounds__(32 * kSimtWarps)
    decode_simt_kernel(const SimtParams p) {
  constexpr int D = 32 * VEC;
  __shared__ float sm_m[kSimtWarps], sm_l[kSimtWarps];
  __shared__ float sm_o[kSimtWarps][D];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bqh = blockIdx.x;  // (b, qi, h), h fastest: q/out row index
  const int h = bqh % p.num_heads;
  const int bq = bqh / p.num_heads;
  const int qi = bq % p.seqlen_q;
  const int b = bq / p.seqlen_q;
  const int kvh = h / p.group;
  const float neg_inf = -__int_as_float(0x7f800000);

  const int stored = p.seqlens[b];
  const int64_t want = static_cast<int64_t>(stored < 0 ? 0 : stored) + p.len_add;
  const int64_t max_len = p.bt_stride * static_cast<int64_t>(p.page);
  const int64_t cap = max_len < 0x7fffffff ? max_len : 0x7fffffff;
  int len = static_cast<int>(want > cap ? cap : want);
  // bottom-right causal mask: query token qi sits at position L - sq + qi
  if (p.causal) len = len - (p.seqlen_q - 1 - qi);
  if (len < 0) len = 0;

  const T* q = reinterpret_cast<const T*>(p.q) + static_cast<int64_t>(bqh) * D + lane * VEC;
  const T* kc = reinterpret_cast<const T*>(p.k);
  const T* vc = reinterpret_cast<const T*>(p.v);
  const int32_t* bt = p.block_table + static_cast<int64_t>(b) * p.bt_stride;

  float qf[VEC];
  {
    const Vec<T, VEC> qv = *reinterpret_cast<const Vec<T, VEC>*>(q);
#pragma unroll
    for (int i = 0; i < VEC; ++i) qf[i] = to_f32(qv.v[i]) * p.scale_log2;
  }
  float m = neg_inf, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;

  for (int t = warp; t < len; t += kSimtWarps) {
    const int64_t page = bt[t / p.page];
    const bool in_pool = page >= 0 && page < p.num_blocks;  // out-of-pool ids read as zero rows
    if (!in_pool && lane == 0) report_status(p.err, kStatusBadPage);
    const int64_t row = ((page * p.page + (t % p.page)) * p.num_heads_k + kvh) * D + lane * VEC;
    Vec<T, VEC> kv, vv;
    if (in_pool) {
      kv = *reinterpret_cast<const Vec<T, VEC>*>(kc + row);
      vv = *reinterpret_cast<const Vec<T, VEC>*>(vc + row);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) { kv.v[i] = from_f32<T>(0.f); vv.v[i] = from_f32<T>(0.f); }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) s = fmaf(qf[i], to_f32(kv.v[i]), s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float m_new = fmaxf(m, s);
    const float alpha = fast_exp2(m - m_new);
    const float pe = fast_exp2(s - m_new);
    l = fmaf(l, alpha, pe);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(acc[i], alpha, pe * to_f32(vv.v[i]));
    m = m_new;
  }

  if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
  for (int i = 0; i < VEC; ++i) sm_o[warp][lane * VEC + i] = acc[i];
  __syncthreads();

  float mx = neg_inf;
#pragma unroll
  for (int w = 0; w < kSimtWarps; ++w) mx = fmaxf(mx, sm_m[w]);
  float den = 0.f;
  float wts[kSimtWarps];
#pragma unroll
  for (int w = 0; w < kSimtWarps; ++w) {
    wts[w] = sm_m[w] == neg_inf ? 0.f : fast_exp2(sm_m[w] - mx);
    den = fmaf(wts[w], sm_l[w], den);
  }
  OutT* out = reinterpret_cast<OutT*>(p.out) + static_cast<int64_t>(bqh) * D;
  for (int d = threadIdx.x; d < D; d += 32 * kSimtWarps) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kSimtWarps; ++w) o = fmaf(wts[w], sm_o[w][d], o);
    out[d] = from_f32<OutT>(den > 0.f ? o / den : 0.f);
  }
  if (p.lse != nullptr && threadIdx.x == 0)
    p.lse[(static_cast<int64_t>(b) * p.num_heads + h) * p.seqlen_q + qi] =
        den > 0.f ? (mx + fast_log2(den)) * 0.69314718055994531f : neg_inf;
}

// out[r] = sum_j w_j o_j[r] / sum_j w_j with w_j = exp(lse_j - max lse),
// parts with lse = -inf weigh zero (their O is never read).  Part j of O
// starts at part_o + j * o_stride, part j of LSE at part_lse + j * l_stride.
template <typename OutT>
__global__ void __launch_bounds__(128)
    combine_lse_kernel(const float* __restrict__ part_o, int64_t o_stride,
                       const float* __restrict__ part_lse, int64_t l_stride, int64_t n_parts,
                       int64_t head_dim, OutT* __restrict__ out, float* __restrict__ lse_out) {
  const int64_t r = blockIdx.x;
  const float neg_inf = -__int_as_float(0x7f800000);
  const float log2e = 1.4426950408889634f;
  float mx = neg_inf;
  for (int64_t j = 0; j < n_parts; ++j) mx = fmaxf(mx, part_lse[j * l_stride + r]);
  float den = 0.f;
  for (int64_t j = 0; j < n_parts; ++j) {
    const float lj = part_lse[j * l_stride + r];
    den += lj == neg_inf ? 0.f : fast_exp2((lj - mx) * log2e);
  }
  for (int64_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t j = 0; j < n_parts; ++j) {
      const float lj = part_lse[j * l_stride + r];
      if (lj == neg_inf) continue;
      acc = fmaf(fast_exp2((lj - mx) * log2e), part_o[j * o_stride + r * head_dim + d], acc);
    }
    out[r * head_dim + d] = from_f32<OutT>(den > 0.f ? acc / den : 0.f);
  }
  if (lse_out != nullptr && threadIdx.x == 0)
    lse_out[r] = den > 0.f ? mx + fast_log2(den) * 0.69314718055994531f : neg_inf;
}

template <typename T, typename OutT>
cudaError_t launch_simt_typed(const SimtParams& p, cudaStream_t stream) {
  const int grid = p.batch * p.seqlen_q * p.num_heads;
  switch (p.head_dim) {
    case 32: decode_simt_kernel<T, OutT, 1><<<grid, 32 * kSimtWarps, 0, stream>>>(p); break;
    case 64: decode_simt_kernel<T, OutT, 2><<<grid, 32 * kSimtWarps, 0, stream>>>(p); break;
    case 128: decode_simt_kernel<T, OutT, 4><<<grid, 32 * kSimtWarps, 0, stream>>>(p); break;
    case 256: decode_simt_kernel<T, OutT, 8><<<grid, 32 * kSimtWarps, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_simt(const SimtParams& p, int dtype, bool out_fp32, cudaStream_t stream) {
  if (dtype == 0)
    return out_fp32 ? launch_simt_typed<__nv_bfloat16, float>(p, stream)
                    : launch_simt_typed<__nv_bfloat16, __nv_bfloat16>(p, stream);
  return out_fp32 ? launch_simt_typed<__half, float>(p, stream)
                  : launch_simt_typed<__half, __half>(p, stream);
}

cudaError_t launch_combine_lse(const float* part_o, int64_t o_stride, const float* part_lse,
                               int64_t l_stride, int64_t n_parts, int64_t rows, int64_t head_dim,
                               void* out, int out_dtype, float* lse_out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(rows));
  switch (out_dtype) {
    case 0:
      combine_lse_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(
          part_o, o_stride, part_lse, l_stride, n_parts, head_dim, static_cast<__nv_bfloat16*>(out),
          lse_out);
      break;
    case 1:
      combine_lse_kernel<__half><<<grid, 128, 0, stream>>>(part_o, o_stride, part_lse, l_stride,
                                                           n_parts, head_dim,
                                                           static_cast<__half*>(out), lse_out);
      break;
    default:
      combine_lse_kernel<float><<<grid, 128, 0, stream>>>(part_o, o_stride, part_lse, l_stride,
                                                          n_parts, head_dim,
                                                          static_cast<float*>(out), lse_out);
      break;
  }
  return cudaGetLastError();
}

}  // namespace fd
