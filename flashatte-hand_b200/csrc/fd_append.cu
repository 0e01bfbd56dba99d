// fd_append.cu - write a decode step's new keys/values into the paged cache.
//
// flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens,
// block_table, ...) first stores k / v [B, seqlen_new, Hkv, D] at positions
// cache_seqlens[b] .. cache_seqlens[b] + seqlen_new - 1 of each sequence and
// then attends over cache_seqlens[b] + seqlen_new keys.  The reference's
// evaluator calls it with k = v = None (scripts/evaluate_flashattn_submission.py
// :233-239), so its submissions never append; this is the adjacent step of a
// real decode loop.  One CTA per new (sequence, token) row copies the row's
// Hkv heads of K and V (Hkv * D elements each, contiguous in both the source
// and the cache row) with 16-byte vector accesses.  A row whose position has
// no page (past the block table, or a page id outside the pool) is skipped and
// counted, so a short table never turns into an out-of-bounds store.  For an
// e4m3 cache the 16-bit rows are quantised with per-KV-head scales.
#include <cuda_runtime.h>

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fd_fp8.cuh"
#include "fd_kernels.h"
#include "fd_ptx.cuh"

namespace fd {

namespace {

constexpr int kAppendThreads = 128;

__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }

__global__ void __launch_bounds__(kAppendThreads)
    append_kv_kernel(const AppendParams p) {
  const int row = blockIdx.x;  // b * seqlen_new + t
  const int b = row / p.seqlen_new;
  const int t = row - b * p.seqlen_new;
  const int stored = p.seqlens[b];
  const int64_t pos = static_cast<int64_t>(stored < 0 ? 0 : stored) + t;
  const int64_t page_idx = pos / p.page;
  int64_t pg = -1;
  if (page_idx < p.bt_stride) pg = p.block_table[static_cast<int64_t>(b) * p.bt_stride + page_idx];
  if (pg < 0 || pg >= p.num_blocks) {
    if (threadIdx.x == 0 && p.skipped != nullptr) atomicAdd(p.skipped, 1);
    // a page id in the table that is not in the pool is the caller's error
    if (threadIdx.x == 0 && page_idx < p.bt_stride) report_status(p.err, kStatusBadPage);
    return;
  }
  const int64_t row_bytes = static_cast<int64_t>(p.num_heads_k) * p.head_dim * p.elem_bytes;
  const int64_t dst_off = (pg * p.page + pos % p.page) * row_bytes;
  const int64_t src_off = static_cast<int64_t>(row) * row_bytes;
  const uint8_t* ks = static_cast<const uint8_t*>(p.k_new) + src_off;
  const uint8_t* vs = static_cast<const uint8_t*>(p.v_new) + src_off;
  uint8_t* kd = static_cast<uint8_t*>(p.k_cache) + dst_off;
  uint8_t* vd = static_cast<uint8_t*>(p.v_cache) + dst_off;
  const bool vec = ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs) |
                     reinterpret_cast<uintptr_t>(kd) | reinterpret_cast<uintptr_t>(vd) |
                     static_cast<uintptr_t>(row_bytes)) & 15u) == 0;
  if (vec) {
    const int64_t n = row_bytes / 16;
    for (int64_t i = threadIdx.x; i < n; i += kAppendThreads) {
      reinterpret_cast<uint4*>(kd)[i] = __ldg(reinterpret_cast<const uint4*>(ks) + i);
      reinterpret_cast<uint4*>(vd)[i] = __ldg(reinterpret_cast<const uint4*>(vs) + i);
    }
  } else {
    const int64_t n = row_bytes / 2;  // 16-bit elements
    for (int64_t i = threadIdx.x; i < n; i += kAppendThreads) {
      reinterpret_cast<uint16_t*>(kd)[i] = reinterpret_cast<const uint16_t*>(ks)[i];
      reinterpret_cast<uint16_t*>(vd)[i] = reinterpret_cast<const uint16_t*>(vs)[i];
    }
  }
}

// e4m3 cache: each new 16-bit value x of KV head h is stored as
// e4m3(x / scale[h]) (round to nearest even, saturating at +-448).  Same row
// placement and skipping as above; one thread per 8 consecutive values.
template <typename T>
__global__ void __launch_bounds__(kAppendThreads)
    append_kv_e4m3_kernel(const AppendParams p) {
  const int row = blockIdx.x;
  const int b = row / p.seqlen_new;
  const int t = row - b * p.seqlen_new;
  const int stored = p.seqlens[b];
  const int64_t pos = static_cast<int64_t>(stored < 0 ? 0 : stored) + t;
  const int64_t page_idx = pos / p.page;
  int64_t pg = -1;
  if (page_idx < p.bt_stride) pg = p.block_table[static_cast<int64_t>(b) * p.bt_stride + page_idx];
  if (pg < 0 || pg >= p.num_blocks) {
    if (threadIdx.x == 0 && p.skipped != nullptr) atomicAdd(p.skipped, 1);
    // a page id in the table that is not in the pool is the caller's error
    if (threadIdx.x == 0 && page_idx < p.bt_stride) report_status(p.err, kStatusBadPage);
    return;
  }
  const int64_t row_elems = static_cast<int64_t>(p.num_heads_k) * p.head_dim;
  const int64_t dst_off = (pg * p.page + pos % p.page) * row_elems;
  const int64_t src_off = static_cast<int64_t>(row) * row_elems;
  for (int64_t i = threadIdx.x * 8; i < row_elems; i += kAppendThreads * 8) {
    const int h = static_cast<int>(i / p.head_dim);
    const float sk = p.k_scale[h], sv = p.v_scale[h];
    const T* kn = static_cast<const T*>(p.k_new) + src_off + i;
    const T* vn = static_cast<const T*>(p.v_new) + src_off + i;
    uint32_t kw[4], vw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kw[j] = e4m3x2(to_float(kn[2 * j]) / sk, to_float(kn[2 * j + 1]) / sk);
      vw[j] = e4m3x2(to_float(vn[2 * j]) / sv, to_float(vn[2 * j + 1]) / sv);
    }
    uint8_t* kd = static_cast<uint8_t*>(p.k_cache) + dst_off + i;
    uint8_t* vd = static_cast<uint8_t*>(p.v_cache) + dst_off + i;
    *reinterpret_cast<uint2*>(kd) = make_uint2(kw[0] | (kw[1] << 16), kw[2] | (kw[3] << 16));
    *reinterpret_cast<uint2*>(vd) = make_uint2(vw[0] | (vw[1] << 16), vw[2] | (vw[3] << 16));
  }
}

}  // namespace

cudaError_t launch_append_kv_e4m3(const AppendParams& p, int src_dtype, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.batch) * p.seqlen_new;
  if (rows <= 0) return cudaSuccess;
  if (src_dtype == 0)
    append_kv_e4m3_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), kAppendThreads, 0, stream>>>(p);
  else
    append_kv_e4m3_kernel<__half><<<static_cast<unsigned>(rows), kAppendThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_append_kv(const AppendParams& p, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.batch) * p.seqlen_new;
  if (rows <= 0) return cudaSuccess;
  append_kv_kernel<<<static_cast<unsigned>(rows), kAppendThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace fd
