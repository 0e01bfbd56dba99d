// fd_kernels.h - host-visible launch interface of the device kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fd {

constexpr int kHeadDim = 128;          // head dim of the tensor-core path
constexpr int kTileTokens = 128;       // KV tokens per pipeline stage (UMMA M of Q.K^T)
constexpr int kMaxGroup = 16;          // query heads per KV head (UMMA N, padded)
constexpr int kMaxBatchPerLaunch = 512;   // sequences per launch (schedule lives in smem)
constexpr int kMaxExchangeRanks = 8;   // GPUs of one node in a cross-GPU split-KV exchange
constexpr int kSm100Threads = 256;     // warps 0/6 TMA, warps 1/7 MMA (PV/QK), warps 2-5 softmax/epilogue

// Per-launch parameters of the tensor-core kernel (tensor maps travel as
// separate __grid_constant__ arguments).
struct DecodeParams {
  void* out;                  // [B, seqlen_q, Hq, 128] of OutT
  float* lse;                 // [B, Hq, seqlen_q] natural log, nullable
  const int32_t* seqlens;     // [B]
  const int32_t* block_table; // [B, bt_stride]
  int64_t bt_stride;
  int batch, num_heads, num_heads_k, group, page, chunk;
  int seqlen_q, causal;       // query tokens per sequence; bottom-right causal mask
  int qrows;                  // seqlen_q * group query rows per (sequence, KV head)
  float scale_log2;           // softmax_scale * log2(e)
  float* part_o;              // [slots, group, 128] fp32 (normalised partial O)
  float* part_lse;            // [slots, group] log2-domain partial LSE
  // [batch * num_heads_k] arrival counters of split pairs: bits [12, 64) the
  // launch epoch, bits [0, 12) the arrivals seen in it.  The CTA that merges
  // a pair clears its counter, so a launch that completes leaves them all 0.
  unsigned long long* tickets;
  int* err;                   // the device's status word (first error a kernel met)
  unsigned long long timeout_ns;
  // Launch epoch kept on the device (workspace): [0] the epoch the next
  // launch uses (1 .. 2^52 - 1; 0 in a zeroed workspace), [1] the launch's
  // epoch-tagged count of CTAs that have read it; the last of them advances
  // [0] and clears [1].  A launch replayed from a CUDA graph therefore gets a
  // fresh epoch like any other launch.
  unsigned long long* epoch_word;
  int64_t num_blocks;         // pages in the K/V pool: block_table ids must lie in [0, num_blocks)
  // Cross-GPU split-KV exchange (xworld > 0): instead of out/lse, every
  // result row goes as fp32 O and ln-LSE to each rank's exchange part
  // xpart[j] (O at [row*128 + d], LSE at [xlse_off + lse row]); the CTA that
  // finishes last on this GPU then stores xepoch to each rank's flag xflag[j].
  int xworld;
  float* xpart[kMaxExchangeRanks];
  uint32_t* xflag[kMaxExchangeRanks];
  int64_t xlse_off;
  uint32_t xepoch;
  uint32_t* xdone;            // count of finished CTAs (workspace, zeroed before the launch)
  int pdl;                    // launch with a programmatic dependency on the previous kernel
  int len_add;                // keys appended this step: attended length = max(seqlens[b], 0) + len_add
  int cost_tile, cost_seg;    // split cost model: fixed cost per tile and per pair, in
                              // units where a full tile's K/V bytes cost 8
  int cost_floor;             // least cost of a pair (its per-pair part is raised to reach it)
  int align_tiles;            // pair-aligned split when B * Hkv <= grid and every
                              // sequence has at most this many tiles (0: never)
  // e4m3 K/V only: dequantisation scales per KV head (K = k8 * k_scale[h],
  // V = v8 * v_scale[h]) and the 16-bit query [B, seqlen_q, Hq, 128], which
  // the kernel splits into e4m3 parts itself.
  const float* k_scale;
  const float* v_scale;
  const void* q;
};

struct SimtParams {
  const void* q; const void* k; const void* v;
  void* out; float* lse;
  const int32_t* seqlens; const int32_t* block_table;
  int64_t bt_stride;
  int batch, num_heads, num_heads_k, group, head_dim, page;
  int seqlen_q, causal;
  int64_t num_blocks;
  float scale_log2;
  int len_add;  // as DecodeParams::len_add
  int* err;     // the device's status word (FD_ERR_BAD_PAGE on an out-of-pool page id)
};

// New keys/values written into the paged cache before attention
// (flash_attn_with_kvcache's k / v arguments): row t of sequence b goes to
// position max(seqlens[b], 0) + t.
struct AppendParams {
  const void* k_new; const void* v_new;  // [B, seqlen_new, Hkv, D]
  void* k_cache; void* v_cache;          // [num_blocks, page, Hkv, D]
  const int32_t* seqlens; const int32_t* block_table;
  int64_t bt_stride, num_blocks;
  int batch, seqlen_new, num_heads_k, head_dim, page, elem_bytes;
  int* skipped;  // nullable: incremented per (b, t) row that had no page to go to
  int* err;      // the device's status word (FD_ERR_BAD_PAGE on an out-of-pool page id)
  const float* k_scale;  // e4m3 cache only: per-KV-head quantisation scales
  const float* v_scale;
};
cudaError_t launch_append_kv(const AppendParams& p, cudaStream_t stream);
// 16-bit new rows (src_dtype 0 bf16, 1 fp16) into an e4m3 cache: x / scale[h], head_dim % 8 == 0.
cudaError_t launch_append_kv_e4m3(const AppendParams& p, int src_dtype, cudaStream_t stream);

// Workspace carve-up for the tensor-core kernel: [epoch_off, lse_off) must
// be zero before the workspace's first use (the kernel keeps it consistent
// afterwards); the partials after it need no initial value.
struct WorkspaceLayout {
  size_t epoch_off, done_off, tickets_off, lse_off, o_off, total;
};
WorkspaceLayout workspace_layout(int64_t batch_per_launch, int64_t num_heads_k, int64_t qrows,
                                 int grid_max);

// TMA descriptors of one launch: q [B, sq, Hq, 128] (box 64 x group x sq), K and
// V caches [num_blocks, page, Hkv, 128] with `chunk`-token boxes for full
// tiles and 16-token boxes for a sequence's last partial tile.
struct TensorMaps {
  CUtensorMap q, k, v, k16, v16;
};

// Per-dtype instantiations of the tensor-core kernel (one translation unit each).
cudaError_t launch_sm100_bf16(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_bf16_f32(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_fp16(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_fp16_f32(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
// e4m3 K/V cache, query of type bf16 / fp16 (read through DecodeParams::q;
// tm.q is not used), output of the query type or fp32.
cudaError_t launch_sm100_kv8_bf16(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_kv8_bf16_f32(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_kv8_fp16(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);
cudaError_t launch_sm100_kv8_fp16_f32(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream);

// Launchers.  dtype: 0 bf16, 1 fp16; out_fp32 selects an fp32 output.
cudaError_t launch_decode_sm100(const TensorMaps& m, const DecodeParams& p, int dtype,
                                bool out_fp32, int grid, cudaStream_t stream);
// e4m3 K/V cache; q_dtype (0 bf16, 1 fp16) is the query's and the 16-bit output's type.
cudaError_t launch_decode_sm100_kv8(const TensorMaps& m, const DecodeParams& p, int q_dtype,
                                    bool out_fp32, int grid, cudaStream_t stream);
cudaError_t launch_decode_simt(const SimtParams& p, int dtype, bool out_fp32, cudaStream_t stream);
cudaError_t launch_combine_lse(const float* part_o, int64_t o_stride, const float* part_lse,
                               int64_t l_stride, int64_t n_parts, int64_t rows, int64_t head_dim,
                               void* out, int out_dtype, float* lse_out, cudaStream_t stream);

// Cross-GPU split-KV exchange: merge the `world` parts of this rank's
// exchange buffer half once every rank's flag in it reads `epoch` (bounded
// wait; on expiry *err = FD_ERR_DEVICE_TIMEOUT and nothing is written).
cudaError_t launch_exchange_combine(const float* parts, int64_t part_stride, int64_t lse_off,
                                    const uint32_t* flags, int world, uint32_t epoch, int64_t rows,
                                    int sq, int hq, void* out, int out_dtype, float* lse_out,
                                    int* err, unsigned long long timeout_ns, cudaStream_t stream);

cudaError_t launch_bounded_wait_probe(unsigned long long budget_ns, int* status,
                                      unsigned long long* waited_ns, cudaStream_t stream);

size_t sm100_smem_bytes();

// Device status word codes (match FD_ERR_DEVICE_TIMEOUT / FD_ERR_BAD_PAGE).
constexpr int kStatusTimeout = 5;
constexpr int kStatusBadPage = 6;

// Address of the current device's status word (a __device__ int inside this
// library, looked up once per device); nullptr if the lookup failed.
int* device_status_word();

// Whether a 16-bit decode is short enough (every sequence at most
// FD_SIMT_MAX_TOKENS long, bounded by the block table's width times the
// page or by max_seqlen_k when given) to run on the CUDA-core kernel, whose
// latency chain is shorter than the tensor-core pipeline's fill.
bool is_short_launch(int64_t block_table_stride, int64_t page_block_size, int64_t max_seqlen_k);

// Whether a 16-bit decode of this shape runs on the tensor-core kernel (and so
// uses split scratch) rather than the CUDA-core kernel, which needs none.
bool uses_tensor_core_path(const void* q, const void* k_cache, const void* v_cache,
                           int64_t headdim, int64_t qrows, int64_t page_block_size);

// Record `code` and a printf-style message as this thread's last error (what
// fd_last_error / fd_last_error_message report) and return `code`.
int report_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

}  // namespace fd
