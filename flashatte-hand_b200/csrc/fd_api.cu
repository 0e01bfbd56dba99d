// fd_api.cu - the C ABI (include/flashdecode.h): argument checks, kernel
// choice, tensor-map encoding, workspace ownership, error reporting.
//
// Host dispatch replaces the reference's run_kernel body
// (submission-oj/best_flashattn_kvcache_decode.cu:1186-1426): instead of a
// fixed split table chosen from (batch, max length) and a grow-only static
// workspace shared by every device and stream, the split is decided on the
// device from cache_seqlens (stream-K ranges, see fd_decode_sm100.cu) and the
// workspace is either the caller's or a library-owned buffer per (device,
// stream), so calls on different streams never share split scratch.  Errors
// a kernel meets (a bounded wait that ran out, a page id outside the pool)
// go to one status word per device inside this library, read and cleared by
// fd_device_status whichever workspace the call used.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/flashdecode.h"
#include "fd_kernels.h"
#include "fd_trace.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;  // 1 s per in-kernel wait
constexpr int kDefaultCostTile = 2;
constexpr int kDefaultCostSeg = 12;
// e4m3 caches: a tile carries half the bytes for the same fixed work, and a
// pair also pays the in-kernel query split.  Swept on config 3's skewed
// lengths (log-uniform 16 .. 32768): the 16-bit weights left CTAs with many
// short sequences overloaded (295 us); these give 198 us.
constexpr int kDefaultCostTile8 = 8;
constexpr int kDefaultCostSeg8 = 48;
// Least cost of a pair (see CostModel in fd_decode_sm100.cuh): a pair of a
// tile or two is a latency chain (query load, QK, softmax, PV, finish) that
// the ring cannot hide behind streaming, so its share of a CTA's range is
// raised to 40 units (four full tiles).  Measured on one B200 against no
// floor: config 3's 8-way batch shard 65.4 -> 54.4 us, its 4-way shard
// 97.1 -> 90.9 us, contest B=64 L=2048 41.6 -> 37.3 us and B=32 L=4096
// 59.2 -> 54.2 us; pairs of four tiles or more (config 5, config 2) keep
// their cost and their times.  A larger seg for every pair gains about as
// much on config 3 but slows the page-16 config 5 mixes.
constexpr int kDefaultCostFloor = 40;
constexpr int kDefaultCostFloor8 = 0;
// Pair-aligned split (one whole (sequence, KV head) pair per CTA) for
// launches with no more pairs than SMs and no sequence longer than this
// many 128-token tiles (see the schedule set-up in fd_decode_sm100.cuh).
constexpr int kDefaultAlignTiles = 16;
// Short launches on the CUDA-core kernel (see simt_max_tokens).
constexpr int kDefaultSimtMaxTokens = 64;

thread_local int t_last_error = FD_OK;
thread_local char t_last_msg[256] = "ok";

int set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int set_error(int code, const char* fmt, ...) {
  t_last_error = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_msg, sizeof(t_last_msg), fmt, ap);
  va_end(ap);
  return code;
}

int set_ok() {
  t_last_error = FD_OK;
  std::strcpy(t_last_msg, "ok");
  return FD_OK;
}

// ----------------------------------------------------------------- driver
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Status word of each device: the first error a kernel of this library met
// since fd_device_status last read it (kStatusTimeout, kStatusBadPage).
__device__ int g_device_status;

// Library-owned workspace of one stream (streams passing workspace = NULL).
// cudaStreamPerThread names a different stream in every host thread, so its
// workspaces are also keyed by thread.
struct StreamWorkspace {
  cudaStream_t stream;
  std::thread::id thread;
  void* ptr;
  size_t bytes;
};

struct DeviceState {
  std::mutex mu;
  int num_sms = 0;
  std::vector<StreamWorkspace> ws;       // the current workspace of each stream
  std::vector<StreamWorkspace> retired;  // outgrown ones (graphs may still use them)
  cudaStream_t zero_stream = nullptr;    // non-blocking: clears new workspaces
  std::once_flag status_once;
  int* status = nullptr;               // device address of g_device_status
};
DeviceState g_dev[kMaxDevices];

int device_sms(int dev) {
  DeviceState& s = g_dev[dev];
  std::lock_guard<std::mutex> lk(s.mu);
  if (s.num_sms == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    s.num_sms = n;
  }
  return s.num_sms;
}

// Device address of the status word on `dev` (the current device): the
// symbol's name is only a host-side stand-in, so it is looked up once per
// device while that device is current.
int* status_word(int dev) {
  DeviceState& s = g_dev[dev];
  std::call_once(s.status_once, [&s] {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) s.status = static_cast<int*>(p);
  });
  return s.status;
}

// Library-owned workspace of (`dev`, `stream`): grow-only, zero-filled when
// allocated, kept until the process exits.  A workspace that a larger call
// outgrows is retired rather than freed, since a CUDA graph captured on the
// stream may still use it.  A stream that is being captured gets its
// workspace too: the allocation and the clearing are made under the relaxed
// capture mode on an internal stream that is not captured, so nothing of
// them enters the graph.
void* internal_workspace(int dev, size_t bytes, cudaStream_t stream, const char** why) {
  DeviceState& s = g_dev[dev];
  std::lock_guard<std::mutex> lk(s.mu);
  const std::thread::id tid =
      stream == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id();
  StreamWorkspace* e = nullptr;
  for (StreamWorkspace& w : s.ws)
    if (w.stream == stream && w.thread == tid) e = &w;
  if (e != nullptr && e->bytes >= bytes) return e->ptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (stream != nullptr && cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    *why = "cannot query the stream's capture status";
    return nullptr;
  }
  const bool capturing = cs != cudaStreamCaptureStatusNone;
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  if (capturing) cudaThreadExchangeStreamCaptureMode(&mode);
  void* p = nullptr;
  cudaError_t err = cudaSuccess;
  if (s.zero_stream == nullptr) err = cudaStreamCreateWithFlags(&s.zero_stream, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaMalloc(&p, bytes);
  if (err == cudaSuccess) err = cudaMemsetAsync(p, 0, bytes, s.zero_stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s.zero_stream);
  if (capturing) cudaThreadExchangeStreamCaptureMode(&mode);
  if (err != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    *why = "cannot allocate or clear the workspace";
    return nullptr;
  }
  if (e != nullptr) {
    s.retired.push_back(*e);
    e->ptr = p;
    e->bytes = bytes;
  } else {
    s.ws.push_back(StreamWorkspace{stream, tid, p, bytes});
  }
  return p;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Sequences per launch.  The kernel keeps per-sequence cost prefix sums in
// int32 and divides cost positions in 32 bits, so a launch's cost line (per
// sequence at most per_seq_cost, or the pair-aligned split's per-pair cost,
// times Hkv) times (grid + 1) must stay below 2^32.  0: not even one fits.
int64_t seqs_per_launch(int64_t per_seq_cost, int64_t aligned_cost, int64_t hkv, int sms) {
  const int64_t c = per_seq_cost > aligned_cost ? per_seq_cost : aligned_cost;
  const int64_t line = c * hkv * (static_cast<int64_t>(sms) + 1);
  if (c > INT32_MAX || line > static_cast<int64_t>(UINT32_MAX)) return 0;
  int64_t n = static_cast<int64_t>(UINT32_MAX) / line;
  if (n > INT32_MAX / c) n = INT32_MAX / c;
  return n < fd::kMaxBatchPerLaunch ? n : fd::kMaxBatchPerLaunch;
}

int esize(int dtype) { return dtype == FD_DTYPE_FP32 ? 4 : 2; }

// Tuning knobs (FD_TMA_CHUNK, FD_COST_TILE / FD_COST_SEG / FD_COST_FLOOR and
// their e4m3 twins, FD_ALIGN_TILES, FD_SIMT_MAX_TOKENS, FD_PDL, FD_WAIT_TIMEOUT_NS) are read from the
// environment only when
// FD_DEBUG_KNOBS=1: without that switch a caller's environment cannot change
// the schedule or the timeouts of the operator.
const char* knob(const char* name) {
  static const bool enabled = [] {
    const char* e = std::getenv("FD_DEBUG_KNOBS");
    return e != nullptr && std::strcmp(e, "1") == 0;
  }();
  return enabled ? std::getenv(name) : nullptr;
}

// Tokens per TMA box for full tiles: the largest of 128/64/32/16 dividing the
// page (a box never crosses a page).  FD_TMA_CHUNK lowers it (tuning knob).
int pick_chunk(int64_t page) {
  static const int cap = [] {
    const char* e = knob("FD_TMA_CHUNK");
    const int v = e != nullptr ? std::atoi(e) : 128;
    return (v == 16 || v == 32 || v == 64) ? v : 128;
  }();
  for (int c = cap; c >= 16; c /= 2)
    if (page % c == 0) return c;
  return 0;
}

CUresult encode(CUtensorMap* m, int dtype, int rank, const void* base, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box) {
  const cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  return encode_fn()(m,
                     dtype == FD_DTYPE_E4M3   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                     : dtype == FD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims, strides, box,
                     estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     // a 16-bit K/V row of one head is 256 contiguous bytes, an e4m3
                     // row 128: promoting an e4m3 fetch to 256 B would drag in the
                     // neighbouring head's row (1.5x the DRAM reads, measured)
                     dtype == FD_DTYPE_E4M3 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                            : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// K and V tensor maps ([num_blocks, page, Hkv, 128] caches; boxes of `chunk`
// tokens for full tiles and 16 for partial ones).  Encoding a map is pure host
// work that costs about as much as a small decode call, and a decode loop
// passes the same caches every step, so each thread keeps the maps of its
// last call and re-encodes only when pointers or shape change.
struct KvMapKey {
  const void* k;
  const void* v;
  int64_t hkv, page, nblk;
  int dtype, chunk;
  bool operator==(const KvMapKey& o) const {
    return k == o.k && v == o.v && hkv == o.hkv && page == o.page && nblk == o.nblk &&
           dtype == o.dtype && chunk == o.chunk;
  }
};

CUresult kv_maps(fd::TensorMaps& m, int dtype, const void* k, const void* v, int64_t hkv,
                 int64_t page, int64_t nblk, int chunk) {
  thread_local KvMapKey key{};
  thread_local CUtensorMap cached[4];
  thread_local bool valid = false;
  const KvMapKey want{k, v, hkv, page, nblk, dtype, chunk};
  if (!(valid && key == want)) {
    const bool e4m3 = dtype == FD_DTYPE_E4M3;
    const cuuint64_t es = e4m3 ? 1 : 2;
    const cuuint64_t dims[4] = {128, (cuuint64_t)hkv, (cuuint64_t)page, (cuuint64_t)nblk};
    const cuuint64_t strides[3] = {128 * es, (cuuint64_t)hkv * 128 * es,
                                   (cuuint64_t)(page * hkv) * 128 * es};
    // 16-bit rows are loaded as two 64-dim halves, e4m3 rows whole
    const cuuint32_t bx = e4m3 ? 128 : 64;
    const cuuint32_t box[4] = {bx, 1, (cuuint32_t)chunk, 1};
    const cuuint32_t box16[4] = {bx, 1, 16, 1};
    valid = false;
    CUresult r = encode(&cached[0], dtype, 4, k, dims, strides, box);
    if (r == CUDA_SUCCESS) r = encode(&cached[1], dtype, 4, v, dims, strides, box);
    if (r == CUDA_SUCCESS) r = encode(&cached[2], dtype, 4, k, dims, strides, box16);
    if (r == CUDA_SUCCESS) r = encode(&cached[3], dtype, 4, v, dims, strides, box16);
    if (r != CUDA_SUCCESS) return r;
    key = want;
    valid = true;
  }
  m.k = cached[0];
  m.v = cached[1];
  m.k16 = cached[2];
  m.v16 = cached[3];
  return CUDA_SUCCESS;
}

// Split cost model (units: a full tile's K/V bytes = 8): fixed cost per
// tile and per (sequence, KV head) pair.  FD_COST_TILE / FD_COST_SEG override
// them for 16-bit caches, FD_COST_TILE8 / FD_COST_SEG8 for e4m3 caches.
int env_int(const char* name, int dflt, int lo, int hi) {
  const char* e = knob(name);
  if (e == nullptr) return dflt;
  const long x = std::strtol(e, nullptr, 10);
  return (x >= lo && x <= hi) ? static_cast<int>(x) : dflt;
}
int cost_tile(bool kv8 = false) {
  static const int v = env_int("FD_COST_TILE", kDefaultCostTile, 0, 64);
  static const int v8 = env_int("FD_COST_TILE8", kDefaultCostTile8, 0, 64);
  return kv8 ? v8 : v;
}
int cost_seg(bool kv8 = false) {
  static const int v = env_int("FD_COST_SEG", kDefaultCostSeg, 1, 256);
  static const int v8 = env_int("FD_COST_SEG8", kDefaultCostSeg8, 1, 256);
  return kv8 ? v8 : v;
}

int cost_floor(bool kv8 = false) {
  static const int v = env_int("FD_COST_FLOOR", kDefaultCostFloor, 0, 1024);
  static const int v8 = env_int("FD_COST_FLOOR8", kDefaultCostFloor8, 0, 1024);
  return kv8 ? v8 : v;
}
// Largest per-pair part (`lead`) of any pair under the cost model.
int64_t max_lead(bool kv8 = false) {
  const int floor = cost_floor(kv8);
  return cost_seg(kv8) > floor ? cost_seg(kv8) : floor;
}

int align_tiles() {
  static const int v = env_int("FD_ALIGN_TILES", kDefaultAlignTiles, 0, 4096);
  return v;
}

// Launches whose sequences are all at most this many tokens long (bounded by
// the block table's width times the page, or by max_seqlen_k when given) run
// on the CUDA-core kernel: its one CTA per query head has a shorter latency
// chain than the tensor-core pipeline's fill, and the few kilobytes of K/V
// such a launch reads stay in L2 (FD_SIMT_MAX_TOKENS).
int simt_max_tokens() {
  static const int v = env_int("FD_SIMT_MAX_TOKENS", kDefaultSimtMaxTokens, 0, 1 << 20);
  return v;
}

// Programmatic dependent launch of the decode kernel (FD_PDL=0 turns it off):
// its prologue may overlap the previous kernel on the stream; it reads no
// input before that kernel has completed.
bool pdl_enabled() {
  static const bool v = env_int("FD_PDL", 1, 0, 1) != 0;
  return v;
}

unsigned long long timeout_ns() {
  static unsigned long long v = [] {
    const char* e = knob("FD_WAIT_TIMEOUT_NS");
    if (e != nullptr) {
      const unsigned long long x = std::strtoull(e, nullptr, 10);
      if (x > 0) return x;
    }
    return kDefaultTimeoutNs;
  }();
  return v;
}

}  // namespace

namespace fd {
int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return status_word(dev);
}

bool is_short_launch(int64_t block_table_stride, int64_t page_block_size, int64_t max_seqlen_k) {
  const int64_t table_tokens = block_table_stride * page_block_size;
  const int64_t bound =
      max_seqlen_k > 0 && max_seqlen_k < table_tokens ? max_seqlen_k : table_tokens;
  return bound <= simt_max_tokens();
}

bool uses_tensor_core_path(const void* q, const void* k_cache, const void* v_cache,
                           int64_t headdim, int64_t qrows, int64_t page_block_size) {
  return headdim == kHeadDim && qrows <= kMaxGroup && pick_chunk(page_block_size) > 0 &&
         aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && encode_fn() != nullptr;
}

int report_error(int code, const char* fmt, ...) {
  t_last_error = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_msg, sizeof(t_last_msg), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace fd

extern "C" {

const char* fd_version(void) { return "flashdecode-sm100 0.1.0"; }

int fd_last_error(void) { return t_last_error; }

const char* fd_last_error_message(void) { return t_last_msg; }

const char* fd_error_string(int code) {
  switch (code) {
    case FD_OK: return "ok";
    case FD_ERR_INVALID_ARG: return "invalid argument";
    case FD_ERR_UNSUPPORTED: return "unsupported configuration";
    case FD_ERR_WORKSPACE: return "workspace missing or too small";
    case FD_ERR_CUDA: return "CUDA error";
    case FD_ERR_DEVICE_TIMEOUT: return "in-kernel wait timed out";
    case FD_ERR_BAD_PAGE: return "page id outside the KV pool";
    default: return "unknown error";
  }
}

size_t fd_decode_workspace_size_mq(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                   int64_t num_heads_k, int64_t headdim) {
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0 || num_heads_k <= 0 ||
      num_heads % num_heads_k != 0)
    return 0;
  (void)headdim;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return 0;
  const int sms = device_sms(dev);
  if (sms <= 0) return 0;
  const int64_t nb = batch_size < fd::kMaxBatchPerLaunch ? batch_size : fd::kMaxBatchPerLaunch;
  return fd::workspace_layout(nb, num_heads_k, seqlen_q * (num_heads / num_heads_k), sms).total;
}

size_t fd_decode_workspace_size(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                                int64_t headdim) {
  return fd_decode_workspace_size_mq(batch_size, 1, num_heads, num_heads_k, headdim);
}

}  // extern "C"

namespace {

// Exchange-mode arguments of one cross-GPU split-KV step (see fd_xgpu.cu).
struct ExchangeArgs {
  int world;
  float* part[fd::kMaxExchangeRanks];
  uint32_t* flag[fd::kMaxExchangeRanks];
  int64_t lse_off;
  uint32_t epoch;
};

int decode_impl(const void* q, const void* k_cache, const void* v_cache, void* out, float* lse,
                const int32_t* cache_seqlens, const int32_t* block_table,
                int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                int64_t num_heads_k, int64_t headdim, int64_t page_block_size, int64_t num_blocks,
                int dtype, int out_dtype, float softmax_scale, int causal, int64_t max_seqlen_k,
                int len_add, void* workspace, size_t workspace_bytes, void* stream,
                const ExchangeArgs* xa, int** err_word) {
  fd::TraceRange trace("decode");
  if (xa != nullptr) out = xa->part[0];  // results go to the exchange parts
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr ||
      cache_seqlens == nullptr || block_table == nullptr)
    return set_error(FD_ERR_INVALID_ARG, "null tensor pointer");
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0 || num_heads_k <= 0 ||
      page_block_size <= 0 || num_blocks <= 0 || block_table_stride <= 0)
    return set_error(FD_ERR_INVALID_ARG,
                     "sizes must be positive (batch=%lld heads=%lld kv_heads=%lld page=%lld "
                     "num_blocks=%lld bt_stride=%lld)",
                     (long long)batch_size, (long long)num_heads, (long long)num_heads_k,
                     (long long)page_block_size, (long long)num_blocks,
                     (long long)block_table_stride);
  if (num_heads % num_heads_k != 0)
    return set_error(FD_ERR_INVALID_ARG, "num_heads %lld not a multiple of num_heads_k %lld",
                     (long long)num_heads, (long long)num_heads_k);
  if (dtype != FD_DTYPE_BF16 && dtype != FD_DTYPE_FP16)
    return set_error(FD_ERR_INVALID_ARG, "dtype must be bf16 or fp16");
  if (out_dtype != dtype && out_dtype != FD_DTYPE_FP32)
    return set_error(FD_ERR_INVALID_ARG, "out_dtype must equal dtype or be fp32");
  if (!std::isfinite(softmax_scale))
    return set_error(FD_ERR_INVALID_ARG, "softmax_scale must be finite");
  if (headdim != 32 && headdim != 64 && headdim != 128 && headdim != 256)
    return set_error(FD_ERR_UNSUPPORTED, "head dim %lld not in {32, 64, 128, 256}",
                     (long long)headdim);
  if (batch_size * seqlen_q * num_heads > INT32_MAX || seqlen_q > 65535 || num_blocks > INT32_MAX ||
      page_block_size > INT32_MAX || num_heads > 65535)
    return set_error(FD_ERR_UNSUPPORTED, "size exceeds 32-bit index range");

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(FD_ERR_CUDA, "no current CUDA device");
  int* status = status_word(dev);
  if (status == nullptr) return set_error(FD_ERR_CUDA, "cannot find the device status word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int group = static_cast<int>(num_heads / num_heads_k);
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  const bool out_fp32 = out_dtype == FD_DTYPE_FP32;
  const int chunk = pick_chunk(page_block_size);
  const int64_t qrows = seqlen_q * group;

  const bool short_launch =
      xa == nullptr && fd::is_short_launch(block_table_stride, page_block_size, max_seqlen_k);
  const bool tensor_core_path =
      !short_launch &&
      fd::uses_tensor_core_path(q, k_cache, v_cache, headdim, qrows, page_block_size);
  if (xa != nullptr && (!tensor_core_path || batch_size > fd::kMaxBatchPerLaunch))
    return set_error(FD_ERR_UNSUPPORTED,
                     "cross-GPU exchange needs the tensor-core path and at most %d sequences",
                     fd::kMaxBatchPerLaunch);
  if (!tensor_core_path) {
    fd::SimtParams sp;
    sp.q = q; sp.k = k_cache; sp.v = v_cache; sp.out = out; sp.lse = lse;
    sp.seqlens = cache_seqlens; sp.block_table = block_table; sp.bt_stride = block_table_stride;
    sp.batch = static_cast<int>(batch_size); sp.num_heads = static_cast<int>(num_heads);
    sp.num_heads_k = static_cast<int>(num_heads_k); sp.group = group;
    sp.head_dim = static_cast<int>(headdim); sp.page = static_cast<int>(page_block_size);
    sp.seqlen_q = static_cast<int>(seqlen_q); sp.causal = causal ? 1 : 0;
    sp.num_blocks = num_blocks; sp.scale_log2 = scale_log2; sp.len_add = len_add;
    sp.err = status;
    const int vec = static_cast<int>(headdim / 32) * 2;  // bytes per lane load
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
         reinterpret_cast<uintptr_t>(v_cache)) % vec != 0)
      return set_error(FD_ERR_UNSUPPORTED, "q/k/v not aligned to %d bytes", vec);
    const cudaError_t e = fd::launch_decode_simt(sp, dtype, out_fp32, st);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "simt launch: %s", cudaGetErrorString(e));
    return set_ok();
  }

  const int sms = device_sms(dev);
  if (sms <= 0) return set_error(FD_ERR_CUDA, "cannot query SM count");
  const int64_t nb_max = batch_size < fd::kMaxBatchPerLaunch ? batch_size : fd::kMaxBatchPerLaunch;
  const fd::WorkspaceLayout wl = fd::workspace_layout(nb_max, num_heads_k, qrows, sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (ws == nullptr) {
    const char* why = "";
    ws = static_cast<uint8_t*>(internal_workspace(dev, wl.total, st, &why));
    if (ws == nullptr) return set_error(FD_ERR_WORKSPACE, "%zu-byte workspace: %s", wl.total, why);
  } else if (workspace_bytes < wl.total) {
    return set_error(FD_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes,
                     wl.total);
  } else if (!aligned16(ws)) {
    return set_error(FD_ERR_WORKSPACE, "workspace not 16-byte aligned");
  }

  const int es = esize(dtype);
  const int64_t kv_max = block_table_stride * page_block_size;
  const int64_t len_bound =
      max_seqlen_k > 0 ? (max_seqlen_k < kv_max ? max_seqlen_k : kv_max) : kv_max;
  const int64_t tiles_bound = len_bound > 0 ? (len_bound + fd::kTileTokens - 1) / fd::kTileTokens : 1;

  fd::TensorMaps maps;
  {
    const CUresult r = kv_maps(maps, dtype, k_cache, v_cache, num_heads_k, page_block_size,
                               num_blocks, chunk);
    if (r != CUDA_SUCCESS) return set_error(FD_ERR_CUDA, "K/V tensor map encode failed (%d)", (int)r);
  }

  // Bound the batch of one launch so the kernel's cost arithmetic fits.
  const int64_t per_seq_cost =
      max_lead() + ((kv_max + fd::kTileTokens - 1) / fd::kTileTokens + 1) *
                       (8 + static_cast<int64_t>(cost_tile()));
  const int64_t per_launch = seqs_per_launch(
      per_seq_cost, max_lead() + static_cast<int64_t>(align_tiles()) * (8 + cost_tile()) + 1,
      num_heads_k, sms);
  if (per_launch == 0) return set_error(FD_ERR_UNSUPPORTED, "sequence too long");
  if (xa != nullptr && per_launch < batch_size)
    return set_error(FD_ERR_UNSUPPORTED, "cross-GPU exchange: the batch does not fit one launch");
  for (int64_t b0 = 0; b0 < batch_size; b0 += per_launch) {
    const int64_t nb = batch_size - b0 < per_launch ? batch_size - b0 : per_launch;
    {
      // q [nb, sq, Hq, 128]: box = 64 dims x group heads x all sq tokens of one sequence
      const uint8_t* qb = static_cast<const uint8_t*>(q) + b0 * seqlen_q * num_heads * 128 * es;
      const cuuint64_t dims[4] = {128, (cuuint64_t)num_heads, (cuuint64_t)seqlen_q, (cuuint64_t)nb};
      const cuuint64_t strides[3] = {(cuuint64_t)(128 * es), (cuuint64_t)(num_heads * 128 * es),
                                     (cuuint64_t)(seqlen_q * num_heads * 128 * es)};
      const cuuint32_t box[4] = {64, (cuuint32_t)group, (cuuint32_t)seqlen_q, 1};
      // same per-thread reuse as the K/V maps: the query buffer is usually
      // the same from step to step
      thread_local const void* q_key_ptr = nullptr;
      thread_local int64_t q_key[5] = {0, 0, 0, 0, 0};
      thread_local CUtensorMap q_cached;
      const int64_t want[5] = {num_heads, seqlen_q, nb, group, dtype};
      CUresult r = CUDA_SUCCESS;
      if (q_key_ptr != qb || std::memcmp(q_key, want, sizeof(want)) != 0) {
        q_key_ptr = nullptr;
        r = encode(&q_cached, dtype, 4, qb, dims, strides, box);
        if (r == CUDA_SUCCESS) {
          q_key_ptr = qb;
          std::memcpy(q_key, want, sizeof(want));
        }
      }
      maps.q = q_cached;
      if (r != CUDA_SUCCESS) return set_error(FD_ERR_CUDA, "Q tensor map encode failed (%d)", (int)r);
    }
    fd::DecodeParams p;
    p.out = static_cast<uint8_t*>(out) + b0 * seqlen_q * num_heads * 128 * esize(out_dtype);
    p.lse = lse != nullptr ? lse + b0 * num_heads * seqlen_q : nullptr;
    p.seqlens = cache_seqlens + b0;
    p.block_table = block_table + b0 * block_table_stride;
    p.bt_stride = block_table_stride;
    p.batch = static_cast<int>(nb);
    p.num_heads = static_cast<int>(num_heads);
    p.num_heads_k = static_cast<int>(num_heads_k);
    p.group = group;
    p.seqlen_q = static_cast<int>(seqlen_q);
    p.causal = causal ? 1 : 0;
    p.qrows = static_cast<int>(qrows);
    p.page = static_cast<int>(page_block_size);
    p.chunk = chunk;
    p.scale_log2 = scale_log2;
    p.err = status;
    p.tickets = reinterpret_cast<unsigned long long*>(ws + wl.tickets_off);
    p.part_lse = reinterpret_cast<float*>(ws + wl.lse_off);
    p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
    p.timeout_ns = timeout_ns();
    p.epoch_word = reinterpret_cast<unsigned long long*>(ws + wl.epoch_off);
    p.num_blocks = num_blocks;
    p.align_tiles = align_tiles();
    p.cost_tile = cost_tile();
    p.cost_seg = cost_seg();
    p.cost_floor = cost_floor();
    p.xworld = 0;
    p.pdl = (xa == nullptr && pdl_enabled()) ? 1 : 0;
    p.len_add = len_add;
    if (xa != nullptr) {
      p.xworld = xa->world;
      for (int j = 0; j < fd::kMaxExchangeRanks; ++j) {
        p.xpart[j] = j < xa->world ? xa->part[j] : nullptr;
        p.xflag[j] = j < xa->world ? xa->flag[j] : nullptr;
      }
      p.xlse_off = xa->lse_off;
      p.xepoch = xa->epoch;
      p.xdone = reinterpret_cast<uint32_t*>(ws + wl.done_off);
      const cudaError_t ez = cudaMemsetAsync(p.xdone, 0, sizeof(uint32_t), st);
      if (ez != cudaSuccess) return set_error(FD_ERR_CUDA, "clear done counter: %s", cudaGetErrorString(ez));
    }
    if (err_word != nullptr) *err_word = status;
    const int64_t work_bound = nb * num_heads_k * tiles_bound;
    const int grid = static_cast<int>(work_bound < sms ? work_bound : sms);
    const cudaError_t e = fd::launch_decode_sm100(maps, p, dtype, out_fp32, grid, st);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "sm100 launch: %s", cudaGetErrorString(e));
  }
  return set_ok();
}

// One cross-GPU split-KV step (see fd_decode_paged_xgpu in the header):
// this rank's exchange arguments for `step`, then `decode(xa, err)` (the
// decode kernel in exchange mode, fp32 parts to every rank), then the merge
// of all ranks' parts into out / lse on this rank.
template <typename Decode>
int xgpu_step(int64_t batch_size, int64_t seqlen_q, int64_t num_heads, int rank, int world,
              void* const* xbufs, uint64_t step, void* out, int out_dtype, float* lse,
              void* stream, Decode&& decode) {
  fd::TraceRange trace("exchange");
  if (xbufs == nullptr || out == nullptr) return set_error(FD_ERR_INVALID_ARG, "null pointer");
  if (world < 1 || world > fd::kMaxExchangeRanks || rank < 0 || rank >= world)
    return set_error(FD_ERR_INVALID_ARG, "rank %d / world %d", rank, world);
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0)
    return set_error(FD_ERR_INVALID_ARG, "sizes must be positive");
  for (int j = 0; j < world; ++j)
    if (xbufs[j] == nullptr) return set_error(FD_ERR_INVALID_ARG, "exchange buffer %d is null", j);
  const int64_t rows = batch_size * seqlen_q * num_heads;
  const int64_t part = ((rows * (fd::kHeadDim + 1) + 63) / 64) * 64;
  const int half = static_cast<int>(step & 1);
  // Buffer: [flags half 0 | flags half 1 | parts half 0 | parts half 1],
  // flags 256 B per half (one u32 per rank), parts world * `part` floats.
  ExchangeArgs xa;
  xa.world = world;
  xa.lse_off = rows * fd::kHeadDim;
  xa.epoch = static_cast<uint32_t>(step % 0x7FFFFFFFull) + 1u;
  for (int j = 0; j < world; ++j) {
    uint8_t* base = static_cast<uint8_t*>(xbufs[j]);
    xa.flag[j] = reinterpret_cast<uint32_t*>(base + half * 256) + rank;
    xa.part[j] = reinterpret_cast<float*>(base + 512) + (static_cast<int64_t>(half) * world + rank) * part;
  }
  int* err = nullptr;
  const int st = decode(&xa, &err);
  if (st != FD_OK) return st;
  uint8_t* mine = static_cast<uint8_t*>(xbufs[rank]);
  const float* parts = reinterpret_cast<const float*>(mine + 512) + static_cast<int64_t>(half) * world * part;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(mine + half * 256);
  const cudaError_t e = fd::launch_exchange_combine(
      parts, part, rows * fd::kHeadDim, flags, world, xa.epoch, rows, static_cast<int>(seqlen_q),
      static_cast<int>(num_heads), out, out_dtype, lse, err, timeout_ns(),
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "exchange combine: %s", cudaGetErrorString(e));
  return set_ok();
}

}  // namespace

extern "C" {

int fd_decode_paged_mq(const void* q, const void* k_cache, const void* v_cache, void* out,
                       float* lse, const int32_t* cache_seqlens, const int32_t* block_table,
                       int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                       int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                       int64_t page_block_size, int64_t num_blocks, int dtype, int out_dtype,
                       float softmax_scale, int causal, int64_t max_seqlen_k, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return decode_impl(q, k_cache, v_cache, out, lse, cache_seqlens, block_table, block_table_stride,
                     batch_size, seqlen_q, num_heads, num_heads_k, headdim, page_block_size,
                     num_blocks, dtype, out_dtype, softmax_scale, causal, max_seqlen_k, 0, workspace,
                     workspace_bytes, stream, nullptr, nullptr);
}

size_t fd_xgpu_buffer_size(int64_t batch_size, int64_t seqlen_q, int64_t num_heads, int world) {
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0 || world <= 0 ||
      world > fd::kMaxExchangeRanks)
    return 0;
  const int64_t rows = batch_size * seqlen_q * num_heads;
  const int64_t part = ((rows * (fd::kHeadDim + 1) + 63) / 64) * 64;  // floats, 256 B aligned
  return 2 * 256 + 2 * static_cast<size_t>(world) * part * sizeof(float);
}

int fd_xgpu_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes == 0)
    return set_error(FD_ERR_INVALID_ARG, "null pointer or zero size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    return set_error(FD_ERR_CUDA, "exchange buffer: %s", cudaGetErrorString(e));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return set_ok();
}

int fd_xgpu_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return set_error(FD_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "open peer buffer: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_xgpu_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "close peer buffer: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_xgpu_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "free exchange buffer: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_decode_paged_xgpu(const void* q, const void* k_cache, const void* v_cache,
                         const int32_t* cache_seqlens, const int32_t* block_table,
                         int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                         int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                         int64_t page_block_size, int64_t num_blocks, int dtype, int out_dtype,
                         float softmax_scale, int causal, int64_t max_seqlen_k, int rank,
                         int world, void* const* xbufs, uint64_t step, void* out, float* lse,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (out_dtype != dtype && out_dtype != FD_DTYPE_FP32)
    return set_error(FD_ERR_INVALID_ARG, "out_dtype must equal dtype or be fp32");
  return xgpu_step(batch_size, seqlen_q, num_heads, rank, world, xbufs, step, out, out_dtype, lse,
                   stream, [&](const ExchangeArgs* xa, int** err) {
                     return decode_impl(q, k_cache, v_cache, nullptr, nullptr, cache_seqlens,
                                        block_table, block_table_stride, batch_size, seqlen_q,
                                        num_heads, num_heads_k, headdim, page_block_size,
                                        num_blocks, dtype, FD_DTYPE_FP32, softmax_scale, causal,
                                        max_seqlen_k, 0, workspace, workspace_bytes, stream, xa,
                                        err);
                   });
}

int fd_append_kv_paged(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int32_t* cache_seqlens, const int32_t* block_table,
                       int64_t block_table_stride, int64_t batch_size, int64_t seqlen_new,
                       int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                       int64_t num_blocks, int dtype, void* stream) {
  fd::TraceRange trace("append");
  if (k_new == nullptr || v_new == nullptr || k_cache == nullptr || v_cache == nullptr ||
      cache_seqlens == nullptr || block_table == nullptr)
    return set_error(FD_ERR_INVALID_ARG, "null tensor pointer");
  if (batch_size <= 0 || seqlen_new <= 0 || num_heads_k <= 0 || headdim <= 0 ||
      page_block_size <= 0 || num_blocks <= 0 || block_table_stride <= 0)
    return set_error(FD_ERR_INVALID_ARG, "sizes must be positive");
  if (dtype != FD_DTYPE_BF16 && dtype != FD_DTYPE_FP16)
    return set_error(FD_ERR_INVALID_ARG, "dtype must be bf16 or fp16");
  if (seqlen_new > 65535 || batch_size * seqlen_new > INT32_MAX || page_block_size > INT32_MAX ||
      num_heads_k * headdim > INT32_MAX)
    return set_error(FD_ERR_UNSUPPORTED, "size exceeds 32-bit index range");
  fd::AppendParams ap;
  ap.k_new = k_new; ap.v_new = v_new; ap.k_cache = k_cache; ap.v_cache = v_cache;
  ap.seqlens = cache_seqlens; ap.block_table = block_table;
  ap.bt_stride = block_table_stride; ap.num_blocks = num_blocks;
  ap.batch = static_cast<int>(batch_size); ap.seqlen_new = static_cast<int>(seqlen_new);
  ap.num_heads_k = static_cast<int>(num_heads_k); ap.head_dim = static_cast<int>(headdim);
  ap.page = static_cast<int>(page_block_size); ap.elem_bytes = esize(dtype);
  ap.skipped = nullptr;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return set_error(FD_ERR_CUDA, "no current CUDA device");
    ap.err = status_word(dev);
    if (ap.err == nullptr) return set_error(FD_ERR_CUDA, "cannot find the device status word");
  }
  ap.k_scale = nullptr;
  ap.v_scale = nullptr;
  const cudaError_t e = fd::launch_append_kv(ap, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "append launch: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_decode_paged_kvappend(const void* q, void* k_cache, void* v_cache, const void* k_new,
                             const void* v_new, void* out, float* lse,
                             const int32_t* cache_seqlens, const int32_t* block_table,
                             int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                             int64_t seqlen_new, int64_t num_heads, int64_t num_heads_k,
                             int64_t headdim, int64_t page_block_size, int64_t num_blocks,
                             int dtype, int out_dtype, float softmax_scale, int causal,
                             int64_t max_seqlen_k, void* workspace, size_t workspace_bytes,
                             void* stream) {
  // Check what the attention half would reject before the cache is written.
  if (q == nullptr || out == nullptr) return set_error(FD_ERR_INVALID_ARG, "null tensor pointer");
  if (seqlen_q <= 0 || num_heads <= 0 || num_heads_k <= 0 || num_heads % num_heads_k != 0)
    return set_error(FD_ERR_INVALID_ARG, "bad head counts or seqlen_q");
  if (headdim != 32 && headdim != 64 && headdim != 128 && headdim != 256)
    return set_error(FD_ERR_UNSUPPORTED, "head dim %lld not in {32, 64, 128, 256}",
                     (long long)headdim);
  if (out_dtype != dtype && out_dtype != FD_DTYPE_FP32)
    return set_error(FD_ERR_INVALID_ARG, "out_dtype must equal dtype or be fp32");
  if (!std::isfinite(softmax_scale))
    return set_error(FD_ERR_INVALID_ARG, "softmax_scale must be finite");
  if (batch_size * seqlen_q * num_heads > INT32_MAX || seqlen_q > 65535 || num_heads > 65535)
    return set_error(FD_ERR_UNSUPPORTED, "size exceeds 32-bit index range");
  if (workspace != nullptr &&
      workspace_bytes < fd_decode_workspace_size_mq(batch_size, seqlen_q, num_heads, num_heads_k,
                                                    headdim))
    return set_error(FD_ERR_WORKSPACE, "workspace too small");
  const int st = fd_append_kv_paged(k_new, v_new, k_cache, v_cache, cache_seqlens, block_table,
                                    block_table_stride, batch_size, seqlen_new, num_heads_k,
                                    headdim, page_block_size, num_blocks, dtype, stream);
  if (st != FD_OK) return st;
  return decode_impl(q, k_cache, v_cache, out, lse, cache_seqlens, block_table, block_table_stride,
                     batch_size, seqlen_q, num_heads, num_heads_k, headdim, page_block_size,
                     num_blocks, dtype, out_dtype, softmax_scale, causal, max_seqlen_k,
                     static_cast<int>(seqlen_new), workspace, workspace_bytes, stream, nullptr,
                     nullptr);
}

// e4m3 K/V cache (see fd_decode_paged_fp8 in the header): one launch of the
// e4m3 tensor-core kernel per kMaxBatchPerLaunch sequences; the kernel splits
// the 16-bit query rows into e4m3 parts itself.  Same workspace as the
// 16-bit path.

static int check_kv8_args(const void* q, const void* k_cache, const void* v_cache,
                          const float* k_scale, const float* v_scale, const void* out,
                          const int32_t* cache_seqlens, const int32_t* block_table,
                          int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                          int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                          int64_t page_block_size, int64_t num_blocks, int q_dtype, int out_dtype,
                          float softmax_scale) {
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || k_scale == nullptr ||
      v_scale == nullptr || out == nullptr || cache_seqlens == nullptr || block_table == nullptr)
    return set_error(FD_ERR_INVALID_ARG, "null pointer");
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0 || num_heads_k <= 0 ||
      page_block_size <= 0 || num_blocks <= 0 || block_table_stride <= 0)
    return set_error(FD_ERR_INVALID_ARG, "sizes must be positive");
  if (num_heads % num_heads_k != 0)
    return set_error(FD_ERR_INVALID_ARG, "num_heads %lld not a multiple of num_heads_k %lld",
                     (long long)num_heads, (long long)num_heads_k);
  if (q_dtype != FD_DTYPE_BF16 && q_dtype != FD_DTYPE_FP16)
    return set_error(FD_ERR_INVALID_ARG, "query dtype must be bf16 or fp16");
  if (out_dtype != q_dtype && out_dtype != FD_DTYPE_FP32)
    return set_error(FD_ERR_INVALID_ARG, "out_dtype must equal the query dtype or be fp32");
  if (!std::isfinite(softmax_scale))
    return set_error(FD_ERR_INVALID_ARG, "softmax_scale must be finite");
  if (batch_size * seqlen_q * num_heads > INT32_MAX || seqlen_q > 65535 || num_blocks > INT32_MAX ||
      page_block_size > INT32_MAX || num_heads > 65535)
    return set_error(FD_ERR_UNSUPPORTED, "size exceeds 32-bit index range");
  if (headdim != fd::kHeadDim)
    return set_error(FD_ERR_UNSUPPORTED, "e4m3 cache: head dim must be 128 (got %lld)",
                     (long long)headdim);
  if (seqlen_q * (num_heads / num_heads_k) > fd::kMaxGroup)
    return set_error(FD_ERR_UNSUPPORTED, "e4m3 cache: seqlen_q * group must be <= %d", fd::kMaxGroup);
  if (pick_chunk(page_block_size) == 0)
    return set_error(FD_ERR_UNSUPPORTED, "e4m3 cache: page size must be a multiple of 16");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(FD_ERR_UNSUPPORTED, "e4m3 cache: q/k/v must be 16-byte aligned");
  if (encode_fn() == nullptr) return set_error(FD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  return FD_OK;
}

static int decode_kv8_impl(const void* q, const void* k_cache, const void* v_cache,
                           const float* k_scale, const float* v_scale, void* out, float* lse,
                           const int32_t* cache_seqlens, const int32_t* block_table,
                           int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                           int64_t num_heads, int64_t num_heads_k, int64_t page_block_size,
                           int64_t num_blocks, int q_dtype, int out_dtype, float softmax_scale,
                           int causal, int64_t max_seqlen_k, int len_add, void* workspace,
                           size_t workspace_bytes, void* stream,
                           const ExchangeArgs* xa = nullptr, int** err_word = nullptr) {
  fd::TraceRange trace("decode_e4m3");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(FD_ERR_CUDA, "no current CUDA device");
  int* status = status_word(dev);
  if (status == nullptr) return set_error(FD_ERR_CUDA, "cannot find the device status word");
  if (xa != nullptr && batch_size > fd::kMaxBatchPerLaunch)
    return set_error(FD_ERR_UNSUPPORTED, "cross-GPU exchange takes at most %d sequences",
                     fd::kMaxBatchPerLaunch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int group = static_cast<int>(num_heads / num_heads_k);
  const int64_t qrows = seqlen_q * group;
  const int chunk = pick_chunk(page_block_size);
  const int sms = device_sms(dev);
  if (sms <= 0) return set_error(FD_ERR_CUDA, "cannot query SM count");
  const int64_t nb_max = batch_size < fd::kMaxBatchPerLaunch ? batch_size : fd::kMaxBatchPerLaunch;
  const fd::WorkspaceLayout wl = fd::workspace_layout(nb_max, num_heads_k, qrows, sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (ws == nullptr) {
    const char* why = "";
    ws = static_cast<uint8_t*>(internal_workspace(dev, wl.total, st, &why));
    if (ws == nullptr) return set_error(FD_ERR_WORKSPACE, "%zu-byte workspace: %s", wl.total, why);
  } else if (workspace_bytes < wl.total) {
    return set_error(FD_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, wl.total);
  } else if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
    return set_error(FD_ERR_WORKSPACE, "workspace not 256-byte aligned");
  }
  const int64_t kv_max = block_table_stride * page_block_size;
  const int64_t len_bound =
      max_seqlen_k > 0 ? (max_seqlen_k < kv_max ? max_seqlen_k : kv_max) : kv_max;
  const int64_t tiles_bound = len_bound > 0 ? (len_bound + fd::kTileTokens - 1) / fd::kTileTokens : 1;
  fd::TensorMaps maps;
  {
    // e4m3 rows: one 128-byte row per (token, KV head)
    const CUresult r = kv_maps(maps, FD_DTYPE_E4M3, k_cache, v_cache, num_heads_k,
                               page_block_size, num_blocks, chunk);
    if (r != CUDA_SUCCESS) return set_error(FD_ERR_CUDA, "K/V tensor map encode failed (%d)", (int)r);
  }
  const int64_t per_seq_cost =
      max_lead(true) + ((kv_max + fd::kTileTokens - 1) / fd::kTileTokens + 1) *
                       (8 + static_cast<int64_t>(cost_tile(true)));
  const int64_t per_launch = seqs_per_launch(
      per_seq_cost,
      max_lead(true) + static_cast<int64_t>(align_tiles()) * (8 + cost_tile(true)) + 1,
      num_heads_k, sms);
  if (per_launch == 0) return set_error(FD_ERR_UNSUPPORTED, "sequence too long");
  if (xa != nullptr && per_launch < batch_size)
    return set_error(FD_ERR_UNSUPPORTED, "cross-GPU exchange: the batch does not fit one launch");
  const int es = esize(q_dtype);
  std::memset(&maps.q, 0, sizeof(maps.q));  // the e4m3 kernel reads the query through p.q
  for (int64_t b0 = 0; b0 < batch_size; b0 += per_launch) {
    const int64_t nb = batch_size - b0 < per_launch ? batch_size - b0 : per_launch;
    const uint8_t* qb = static_cast<const uint8_t*>(q) + b0 * seqlen_q * num_heads * 128 * es;
    fd::DecodeParams p{};
    p.out = static_cast<uint8_t*>(out) + b0 * seqlen_q * num_heads * 128 * esize(out_dtype);
    p.lse = lse != nullptr ? lse + b0 * num_heads * seqlen_q : nullptr;
    p.seqlens = cache_seqlens + b0;
    p.block_table = block_table + b0 * block_table_stride;
    p.bt_stride = block_table_stride;
    p.batch = static_cast<int>(nb);
    p.num_heads = static_cast<int>(num_heads);
    p.num_heads_k = static_cast<int>(num_heads_k);
    p.group = group;
    p.seqlen_q = static_cast<int>(seqlen_q);
    p.causal = causal ? 1 : 0;
    p.qrows = static_cast<int>(qrows);
    p.page = static_cast<int>(page_block_size);
    p.chunk = chunk;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;
    p.err = status;
    p.tickets = reinterpret_cast<unsigned long long*>(ws + wl.tickets_off);
    p.part_lse = reinterpret_cast<float*>(ws + wl.lse_off);
    p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
    p.timeout_ns = timeout_ns();
    p.epoch_word = reinterpret_cast<unsigned long long*>(ws + wl.epoch_off);
    p.num_blocks = num_blocks;
    p.align_tiles = align_tiles();
    p.cost_tile = cost_tile(true);
    p.cost_seg = cost_seg(true);
    p.cost_floor = cost_floor(true);
    p.xworld = 0;
    p.pdl = (xa == nullptr && pdl_enabled()) ? 1 : 0;
    p.len_add = len_add;
    p.k_scale = k_scale;
    p.v_scale = v_scale;
    p.q = qb;
    if (xa != nullptr) {
      p.xworld = xa->world;
      for (int j = 0; j < fd::kMaxExchangeRanks; ++j) {
        p.xpart[j] = j < xa->world ? xa->part[j] : nullptr;
        p.xflag[j] = j < xa->world ? xa->flag[j] : nullptr;
      }
      p.xlse_off = xa->lse_off;
      p.xepoch = xa->epoch;
      p.xdone = reinterpret_cast<uint32_t*>(ws + wl.done_off);
      const cudaError_t ez = cudaMemsetAsync(p.xdone, 0, sizeof(uint32_t), st);
      if (ez != cudaSuccess) return set_error(FD_ERR_CUDA, "clear done counter: %s", cudaGetErrorString(ez));
    }
    if (err_word != nullptr) *err_word = status;
    const int64_t work_bound = nb * num_heads_k * tiles_bound;
    const int grid = static_cast<int>(work_bound < sms ? work_bound : sms);
    const cudaError_t e = fd::launch_decode_sm100_kv8(maps, p, q_dtype, out_dtype == FD_DTYPE_FP32, grid, st);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "sm100 e4m3 launch: %s", cudaGetErrorString(e));
  }
  return set_ok();
}

size_t fd_decode_workspace_size_fp8(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                    int64_t num_heads_k, int64_t headdim) {
  if (batch_size <= 0 || seqlen_q <= 0 || num_heads <= 0 || num_heads_k <= 0 ||
      num_heads % num_heads_k != 0 || headdim != fd::kHeadDim)
    return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return 0;
  const int sms = device_sms(dev);
  if (sms <= 0) return 0;
  const int64_t nb = batch_size < fd::kMaxBatchPerLaunch ? batch_size : fd::kMaxBatchPerLaunch;
  return fd::workspace_layout(nb, num_heads_k, seqlen_q * (num_heads / num_heads_k), sms).total;
}

int fd_decode_paged_fp8_xgpu(const void* q, const void* k_cache, const void* v_cache,
                             const float* k_scale, const float* v_scale,
                             const int32_t* cache_seqlens, const int32_t* block_table,
                             int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                             int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                             int64_t page_block_size, int64_t num_blocks, int q_dtype,
                             int out_dtype, float softmax_scale, int causal, int64_t max_seqlen_k,
                             int rank, int world, void* const* xbufs, uint64_t step, void* out,
                             float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  const int st = check_kv8_args(q, k_cache, v_cache, k_scale, v_scale, out, cache_seqlens,
                                block_table, block_table_stride, batch_size, seqlen_q, num_heads,
                                num_heads_k, headdim, page_block_size, num_blocks, q_dtype,
                                out_dtype, softmax_scale);
  if (st != FD_OK) return st;
  return xgpu_step(batch_size, seqlen_q, num_heads, rank, world, xbufs, step, out, out_dtype, lse,
                   stream, [&](const ExchangeArgs* xa, int** err) {
                     return decode_kv8_impl(q, k_cache, v_cache, k_scale, v_scale, nullptr, nullptr,
                                            cache_seqlens, block_table, block_table_stride,
                                            batch_size, seqlen_q, num_heads, num_heads_k,
                                            page_block_size, num_blocks, q_dtype, FD_DTYPE_FP32,
                                            softmax_scale, causal, max_seqlen_k, 0, workspace,
                                            workspace_bytes, stream, xa, err);
                   });
}

int fd_append_kv_paged_fp8(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                           const float* k_scale, const float* v_scale,
                           const int32_t* cache_seqlens, const int32_t* block_table,
                           int64_t block_table_stride, int64_t batch_size, int64_t seqlen_new,
                           int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                           int64_t num_blocks, int src_dtype, void* stream) {
  fd::TraceRange trace("append_e4m3");
  if (k_new == nullptr || v_new == nullptr || k_cache == nullptr || v_cache == nullptr ||
      k_scale == nullptr || v_scale == nullptr || cache_seqlens == nullptr || block_table == nullptr)
    return set_error(FD_ERR_INVALID_ARG, "null pointer");
  if (batch_size <= 0 || seqlen_new <= 0 || num_heads_k <= 0 || headdim <= 0 ||
      page_block_size <= 0 || num_blocks <= 0 || block_table_stride <= 0)
    return set_error(FD_ERR_INVALID_ARG, "sizes must be positive");
  if (src_dtype != FD_DTYPE_BF16 && src_dtype != FD_DTYPE_FP16)
    return set_error(FD_ERR_INVALID_ARG, "new rows must be bf16 or fp16");
  if (headdim % 8 != 0 || (reinterpret_cast<uintptr_t>(k_cache) & 7u) != 0 ||
      (reinterpret_cast<uintptr_t>(v_cache) & 7u) != 0)
    return set_error(FD_ERR_UNSUPPORTED, "e4m3 append: head dim must be a multiple of 8, caches 8-byte aligned");
  if (seqlen_new > 65535 || batch_size * seqlen_new > INT32_MAX || page_block_size > INT32_MAX ||
      num_heads_k * headdim > INT32_MAX)
    return set_error(FD_ERR_UNSUPPORTED, "size exceeds 32-bit index range");
  fd::AppendParams ap;
  ap.k_new = k_new; ap.v_new = v_new; ap.k_cache = k_cache; ap.v_cache = v_cache;
  ap.seqlens = cache_seqlens; ap.block_table = block_table;
  ap.bt_stride = block_table_stride; ap.num_blocks = num_blocks;
  ap.batch = static_cast<int>(batch_size); ap.seqlen_new = static_cast<int>(seqlen_new);
  ap.num_heads_k = static_cast<int>(num_heads_k); ap.head_dim = static_cast<int>(headdim);
  ap.page = static_cast<int>(page_block_size); ap.elem_bytes = 1;
  ap.skipped = nullptr;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return set_error(FD_ERR_CUDA, "no current CUDA device");
    ap.err = status_word(dev);
    if (ap.err == nullptr) return set_error(FD_ERR_CUDA, "cannot find the device status word");
  }
  ap.k_scale = k_scale;
  ap.v_scale = v_scale;
  const cudaError_t e = fd::launch_append_kv_e4m3(ap, src_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "e4m3 append launch: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_decode_paged_fp8(const void* q, void* k_cache, void* v_cache, const float* k_scale,
                        const float* v_scale, const void* k_new, const void* v_new,
                        int64_t seqlen_new, void* out, float* lse, const int32_t* cache_seqlens,
                        const int32_t* block_table, int64_t block_table_stride,
                        int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                        int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                        int64_t num_blocks, int q_dtype, int out_dtype, float softmax_scale,
                        int causal, int64_t max_seqlen_k, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int st = check_kv8_args(q, k_cache, v_cache, k_scale, v_scale, out, cache_seqlens, block_table,
                          block_table_stride, batch_size, seqlen_q, num_heads, num_heads_k,
                          headdim, page_block_size, num_blocks, q_dtype, out_dtype, softmax_scale);
  if (st != FD_OK) return st;
  if ((k_new == nullptr) != (v_new == nullptr))
    return set_error(FD_ERR_INVALID_ARG, "k_new and v_new must be given together");
  int len_add = 0;
  if (k_new != nullptr) {
    if (seqlen_new <= 0 || seqlen_new > 65535)
      return set_error(FD_ERR_INVALID_ARG, "seqlen_new out of range");
    if (workspace != nullptr &&
        workspace_bytes < fd_decode_workspace_size_fp8(batch_size, seqlen_q, num_heads, num_heads_k,
                                                       headdim))
      return set_error(FD_ERR_WORKSPACE, "workspace too small");
    st = fd_append_kv_paged_fp8(k_new, v_new, k_cache, v_cache, k_scale, v_scale, cache_seqlens,
                                block_table, block_table_stride, batch_size, seqlen_new,
                                num_heads_k, headdim, page_block_size, num_blocks, q_dtype, stream);
    if (st != FD_OK) return st;
    len_add = static_cast<int>(seqlen_new);
  }
  return decode_kv8_impl(q, k_cache, v_cache, k_scale, v_scale, out, lse, cache_seqlens,
                         block_table, block_table_stride, batch_size, seqlen_q, num_heads,
                         num_heads_k, page_block_size, num_blocks, q_dtype, out_dtype,
                         softmax_scale, causal, max_seqlen_k, len_add, workspace, workspace_bytes,
                         stream);
}

int fd_decode_paged(const void* q, const void* k_cache, const void* v_cache, void* out, float* lse,
                    const int32_t* cache_seqlens, const int32_t* block_table,
                    int64_t block_table_stride, int64_t batch_size, int64_t num_heads,
                    int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                    int64_t num_blocks, int dtype, int out_dtype, float softmax_scale,
                    int64_t max_seqlen_k, void* workspace, size_t workspace_bytes, void* stream) {
  return fd_decode_paged_mq(q, k_cache, v_cache, out, lse, cache_seqlens, block_table,
                            block_table_stride, batch_size, 1, num_heads, num_heads_k, headdim,
                            page_block_size, num_blocks, dtype, out_dtype, softmax_scale, 0,
                            max_seqlen_k, workspace, workspace_bytes, stream);
}

void run_kernel(const void* q, const void* k_cache_paged, const void* v_cache_paged, void* output,
                const int32_t* cache_seqlens, const int32_t* block_table, int64_t batch_size,
                int64_t seqlen_k, int64_t seqlen_q, int64_t num_heads, int64_t num_heads_k,
                int64_t headdim, int64_t page_block_size, int64_t num_blocks, int64_t causal) {
  if (batch_size <= 0 || num_blocks <= 0 || headdim <= 0 || seqlen_q <= 0) {
    set_error(FD_ERR_INVALID_ARG, "batch_size, num_blocks and headdim must be positive");
    return;
  }
  const int64_t bt_stride = num_blocks / batch_size;  // reference: blocks_per_batch
  if (bt_stride <= 0) {
    set_error(FD_ERR_INVALID_ARG, "num_blocks %lld < batch_size %lld", (long long)num_blocks,
              (long long)batch_size);
    return;
  }
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(headdim)));
  fd_decode_paged_mq(q, k_cache_paged, v_cache_paged, output, nullptr, cache_seqlens, block_table,
                     bt_stride, batch_size, seqlen_q, num_heads, num_heads_k, headdim,
                     page_block_size, num_blocks, FD_DTYPE_BF16, FD_DTYPE_BF16, scale,
                     causal != 0 ? 1 : 0, seqlen_k, nullptr, 0, nullptr);
}

int fd_combine_lse(const float* part_o, int64_t part_o_stride, const float* part_lse,
                   int64_t part_lse_stride, int64_t n_parts, int64_t rows, int64_t headdim,
                   void* out, int out_dtype, float* lse_out, void* stream) {
  fd::TraceRange trace("combine_lse");
  if (part_o == nullptr || part_lse == nullptr || out == nullptr)
    return set_error(FD_ERR_INVALID_ARG, "null pointer");
  if (n_parts <= 0 || rows < 0 || headdim <= 0 || rows > INT32_MAX)
    return set_error(FD_ERR_INVALID_ARG, "bad sizes");
  if (part_o_stride == 0) part_o_stride = rows * headdim;
  if (part_lse_stride == 0) part_lse_stride = rows;
  if (part_o_stride < rows * headdim || part_lse_stride < rows)
    return set_error(FD_ERR_INVALID_ARG, "part strides overlap the parts");
  if (out_dtype != FD_DTYPE_BF16 && out_dtype != FD_DTYPE_FP16 && out_dtype != FD_DTYPE_FP32)
    return set_error(FD_ERR_INVALID_ARG, "bad out_dtype");
  const cudaError_t e =
      fd::launch_combine_lse(part_o, part_o_stride, part_lse, part_lse_stride, n_parts, rows,
                             headdim, out, out_dtype, lse_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "combine launch: %s", cudaGetErrorString(e));
  return set_ok();
}

int fd_selftest_bounded_wait(uint64_t budget_ns, uint64_t* waited_ns) {
  int* d_status = nullptr;
  unsigned long long* d_waited = nullptr;
  if (cudaMalloc(&d_status, sizeof(int)) != cudaSuccess)
    return set_error(FD_ERR_CUDA, "cudaMalloc failed");
  if (cudaMalloc(&d_waited, sizeof(unsigned long long)) != cudaSuccess) {
    cudaFree(d_status);
    return set_error(FD_ERR_CUDA, "cudaMalloc failed");
  }
  int status = -1;
  unsigned long long waited = 0;
  cudaError_t e = fd::launch_bounded_wait_probe(budget_ns, d_status, d_waited, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&status, d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess)
    e = cudaMemcpy(&waited, d_waited, sizeof(waited), cudaMemcpyDeviceToHost);
  cudaFree(d_status);
  cudaFree(d_waited);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "probe: %s", cudaGetErrorString(e));
  if (waited_ns != nullptr) *waited_ns = waited;
  if (status == FD_ERR_DEVICE_TIMEOUT)
    return set_error(FD_ERR_DEVICE_TIMEOUT, "bounded wait gave up after %llu ns", waited);
  return set_ok();
}

int fd_device_status(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(FD_ERR_CUDA, "no current CUDA device");
  if (cudaDeviceSynchronize() != cudaSuccess)
    return set_error(FD_ERR_CUDA, "device synchronize failed");
  int* w = status_word(dev);
  if (w == nullptr) return set_error(FD_ERR_CUDA, "cannot find the device status word");
  int word = 0;
  if (cudaMemcpy(&word, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_error(FD_ERR_CUDA, "cannot read device status");
  if (word == 0) return set_ok();
  const int zero = 0;
  if (cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return set_error(FD_ERR_CUDA, "cannot clear device status");
  if (word == FD_ERR_BAD_PAGE)
    return set_error(FD_ERR_BAD_PAGE,
                     "a block_table entry inside a sequence's length was outside [0, num_blocks) "
                     "(those rows were read as zeros)");
  if (word == FD_ERR_DEVICE_TIMEOUT)
    return set_error(FD_ERR_DEVICE_TIMEOUT, "a bounded in-kernel wait ran out");
  return set_error(word, "device reported status %d", word);
}

size_t fd_library_workspace_bytes(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  DeviceState& s = g_dev[dev];
  std::lock_guard<std::mutex> lk(s.mu);
  size_t total = 0;
  for (const StreamWorkspace& w : s.ws) total += w.bytes;
  for (const StreamWorkspace& w : s.retired) total += w.bytes;
  return total;
}

}  // extern "C"
