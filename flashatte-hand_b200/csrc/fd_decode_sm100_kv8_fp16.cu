// fd_decode_sm100_kv8_fp16.cu - e4m3 K/V cache, __half queries, __half output
// instantiations of the tensor-core decode kernel (see fd_decode_sm100.cuh).
#include "fd_decode_sm100.cuh"

namespace fd {

cudaError_t launch_sm100_kv8_fp16(const TensorMaps& m, const DecodeParams& p, int grid,
                              cudaStream_t stream) {
  return launch_ncol_kv8<__half, __half>(m, p, grid, stream);
}

}  // namespace fd
