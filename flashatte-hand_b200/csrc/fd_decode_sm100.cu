// fd_decode_sm100.cu - host-side pieces of the tensor-core decode kernel:
// shared-memory size, workspace carve-up and the dtype dispatch to the
// instantiations in fd_decode_sm100_[kv8_]{bf16,fp16}[_f32].cu (split so nvcc
// compiles them in parallel).
#include "fd_decode_sm100.cuh"

namespace fd {

size_t sm100_smem_bytes() { return static_cast<size_t>(Geo<false>::kSmemBytes); }

WorkspaceLayout workspace_layout(int64_t batch_per_launch, int64_t num_heads_k, int64_t qrows,
                                 int grid_max) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  const size_t pairs = static_cast<size_t>(batch_per_launch * num_heads_k);
  const size_t slots = pairs + static_cast<size_t>(grid_max);
  WorkspaceLayout w;
  w.epoch_off = 0;     // two 64-bit words, see DecodeParams::epoch_word
  w.done_off = 64;     // cross-GPU exchange: finished-CTA count
  w.tickets_off = 128; // one 64-bit arrival counter per (sequence, KV head) pair
  w.lse_off = up(w.tickets_off + pairs * 8);
  w.o_off = w.lse_off + up(slots * qrows * 4);
  w.total = w.o_off + up(slots * qrows * kHeadDim * 4);
  return w;
}

cudaError_t launch_decode_sm100(const TensorMaps& m, const DecodeParams& p, int dtype,
                                bool out_fp32, int grid, cudaStream_t stream) {
  if (dtype == 0)
    return out_fp32 ? launch_sm100_bf16_f32(m, p, grid, stream) : launch_sm100_bf16(m, p, grid, stream);
  return out_fp32 ? launch_sm100_fp16_f32(m, p, grid, stream) : launch_sm100_fp16(m, p, grid, stream);
}

cudaError_t launch_decode_sm100_kv8(const TensorMaps& m, const DecodeParams& p, int q_dtype,
                                    bool out_fp32, int grid, cudaStream_t stream) {
  if (q_dtype == 0)
    return out_fp32 ? launch_sm100_kv8_bf16_f32(m, p, grid, stream)
                    : launch_sm100_kv8_bf16(m, p, grid, stream);
  return out_fp32 ? launch_sm100_kv8_fp16_f32(m, p, grid, stream)
                  : launch_sm100_kv8_fp16(m, p, grid, stream);
}

}  // namespace fd
