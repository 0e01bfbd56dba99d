// fd_noalloc.cu - fd_decode_paged_noalloc: the decode entry point for callers
// that must not allocate device memory.
//
// Who needs it: a host process whose framework allocator has already
// reserved nearly all of the GPU's memory (a cudaMalloc from this library
// would then fail, or fragment that pool), and serving loops that allocate
// everything at start-up and forbid allocation afterwards so a request can
// never stall on, or fail in, the allocator.  Those callers still pass their
// inputs and outputs; the only memory this library would otherwise allocate
// is the split-KV scratch (partial O / LSE and arrival counters).
//
// Here that scratch is a fixed array in the library's device image
// (kNoAllocScratchBytes per GPU that loads the library, held until the
// process exits).  Host code cannot use the array's name as a device
// address, so the first call on each device looks the address up with
// cudaGetSymbolAddress while that device is current and keeps it.  Errors a
// kernel meets are reported in the device status word that fd_device_status
// reads, as for every other entry point.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/flashdecode.h"
#include "fd_kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchAddress {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t status = cudaSuccess;
};
ScratchAddress g_scratch_addr[kMaxDevices];

// Device address of g_noalloc_scratch on `dev` (the current device).
void* scratch_address(int dev, cudaError_t* status) {
  ScratchAddress& s = g_scratch_addr[dev];
  std::call_once(s.once, [&s] { s.status = cudaGetSymbolAddress(&s.ptr, g_noalloc_scratch); });
  *status = s.status;
  return s.status == cudaSuccess ? s.ptr : nullptr;
}

}  // namespace

extern "C" int fd_decode_paged_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       void* out, float* lse, const int32_t* cache_seqlens,
                                       const int32_t* block_table, int64_t block_table_stride,
                                       int64_t batch_size, int64_t num_heads,
                                       int64_t num_heads_k, int64_t headdim,
                                       int64_t page_block_size, int64_t num_blocks, int dtype,
                                       int out_dtype, float softmax_scale, int64_t max_seqlen_k,
                                       void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fd::report_error(FD_ERR_CUDA, "no current CUDA device");
  cudaError_t status = cudaSuccess;
  void* scratch = scratch_address(dev, &status);
  if (scratch == nullptr)
    return fd::report_error(FD_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s",
                            cudaGetErrorString(status));
  // Shapes the CUDA-core kernel takes (other head dims, wide groups,
  // unaligned pointers, short launches) use no split scratch at all: they
  // are never refused for its size.  (Invalid arguments are left to
  // fd_decode_paged to report.)
  const bool uses_scratch =
      num_heads > 0 && num_heads_k > 0 && num_heads % num_heads_k == 0 &&
      !fd::is_short_launch(block_table_stride, page_block_size, max_seqlen_k) &&
      fd::uses_tensor_core_path(q, k_cache, v_cache, headdim, num_heads / num_heads_k,
                                page_block_size);
  if (uses_scratch) {
    const size_t need = fd_decode_workspace_size(batch_size, num_heads, num_heads_k, headdim);
    if (need > kNoAllocScratchBytes)
      return fd::report_error(FD_ERR_WORKSPACE,
                              "this shape needs %zu bytes of split scratch; the no-allocation entry "
                              "point has a fixed %zu-byte area (use fd_decode_paged with a caller "
                              "workspace instead)",
                              need, kNoAllocScratchBytes);
    // Every call shares the area and finds the previous call's contents: clear
    // the part that must start at zero (launch epoch and arrival counters).
    if (need > 0) {
      const size_t head = fd::workspace_layout(
          batch_size < fd::kMaxBatchPerLaunch ? batch_size : fd::kMaxBatchPerLaunch, num_heads_k,
          num_heads / num_heads_k, 0).lse_off;
      const cudaError_t e = cudaMemsetAsync(scratch, 0, head, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess)
        return fd::report_error(FD_ERR_CUDA, "clearing scratch: %s", cudaGetErrorString(e));
    }
  }
  return fd_decode_paged(q, k_cache, v_cache, out, lse, cache_seqlens, block_table,
                         block_table_stride, batch_size, num_heads, num_heads_k, headdim,
                         page_block_size, num_blocks, dtype, out_dtype, softmax_scale,
                         max_seqlen_k, scratch, kNoAllocScratchBytes, stream);
}
