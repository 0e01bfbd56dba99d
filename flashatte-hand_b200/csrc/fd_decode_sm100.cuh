// fd_decode_sm100.cuh - persistent split-KV paged decode kernel for B200
// (device code and launch templates; fd_decode_sm100_*.cu instantiate it).
//
// Work decomposition (replaces the reference's fixed split table and
// per-split grid, submission-oj/best_flashattn_kvcache_decode.cu:1039-1076,
// :1381-1418, and its balanced page ranges :664-671): every (sequence b,
// KV head) pair is a row of 128-token tiles; the rows are laid end to end
// (b-major, then KV head) and the line is cut into contiguous ranges of
// equal estimated cost (K/V bytes of each tile + a fixed cost per tile + a
// fixed cost per pair), one per persistent CTA.  A CTA walks its range
// segment by segment (a segment = the part of one pair inside the range).
// A pair that lies inside one CTA is written straight to the output; a pair
// cut by range boundaries leaves one normalised partial (O, log2-LSE) per
// segment and the CTA that finishes last merges them (replaces the separate
// combine launch, best :956-1037, :1420-1425).
//
// Per tile the CTA runs, warp-specialised:
//   warps 0,6 TMA producers: gather the tile's K (warp 0, with the group's
//             query rows) and V (warp 6) rows page by page through
//             block_table into 3-deep shared-memory rings (128B-swizzled,
//             two 64-dim halves); a sequence's last, partial tile is fetched
//             in 16-token boxes covering only its valid rows.
//   warp 7    tcgen05 issuer for S^T[tok, head] = K . Q^T (M=128 tokens,
//             N=16 heads, K=128 dims) into TMEM;
//   warp 1    tcgen05 issuer for O^T[dim, head] = V^T . P^T (M=128 dims,
//             N=2x16 heads, K=128 tokens) into TMEM, and TMEM owner.
//   warps 2-5 softmax + epilogue: thread = TMEM lane = token row for S and
//             head-dim for O; fp32 online softmax in the log2 domain (the
//             reference's convention, best :541-578), P written to shared
//             memory for the second UMMA, per-tile O folded into registers.
// One KV byte is read from HBM exactly once; the arithmetic runs on the
// tensor cores so the SM's issue slots stay free for the memory pipeline.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "fd_kernels.h"
#include "fd_fp8.cuh"
#include "fd_ptx.cuh"

namespace fd {

namespace {

// Stage / buffer geometry, by K/V element type (and, for e4m3, query rows).
//   16-bit K/V: a 128-token K or V tile is two 64-dim halves of 128 B rows
//   (16 KB each, 128B-swizzled); the group's query rows ride in each stage;
//   P is two 16-bit parts (hi = round(P), lo = round(P - hi)) side by side in
//   the UMMA N dimension, so summing V.hi and V.lo keeps P's fp32 precision.
//   e4m3 K/V: one 128 B row holds all 128 dims, a tile is 16 KB; each stage
//   carries the query rows as three e4m3 parts (48 rows of 128 B, split by
//   the K producer warp) and P is split into three e4m3 parts the same way
//   (see the softmax warps).  Four stages up to 8 query rows, five at 16
//   (more softmax work per tile wants a deeper ring; with less, a fifth
//   stage only adds requests in flight to a saturated memory system:
//   measured 3 % slower).
// S^T tiles rotate through three TMEM buffers, P and O^T through two.  PV(i)
// may overwrite O buffer i%2 once P(i) is written, since each softmax thread
// loads O(i-2) before it writes P(i): the O buffers need no "empty" barrier.
template <bool KV8, int NCOL = kMaxGroup> struct Geo {
  static constexpr int kStages = KV8 ? (NCOL <= 8 ? 4 : 5) : 3;
  static constexpr int kHalfBytes = kTileTokens * 128;              // 128 rows x 128 B
  static constexpr int kOperandBytes = KV8 ? kHalfBytes : 2 * kHalfBytes;  // one K or V tile
  static constexpr int kParts = KV8 ? 3 : 2;                        // P (and Q) parts
  static constexpr int kQSlotBytes = KV8 ? 3 * kMaxGroup * 128 : 2 * kMaxGroup * 128;
  static constexpr int kStageBytes = 2 * kOperandBytes + kQSlotBytes;
  static constexpr int kPBufBytes = KV8 ? kTileTokens * 3 * kMaxGroup : kTileTokens * 2 * kMaxGroup * 2;
  static constexpr int kSCols = KV8 ? 3 * kMaxGroup : kMaxGroup;    // TMEM columns of one S^T tile
  static constexpr int kOCols = KV8 ? 3 * kMaxGroup : 2 * kMaxGroup;  // of one O^T tile
  static constexpr int kSBufs = 3;
  static constexpr int kTmemCols = KV8 ? 256 : 128;
  // e4m3: inverse query-row scales, one slot per segment, from the K producer
  // to the softmax warps (q_full barrier per slot).  The producer runs at most
  // kStages + kSBufs tiles ahead of the softmax, so 16 slots never overrun.
  static constexpr int kQRing = KV8 ? 16 : 0;
  static_assert(kQRing == 0 || kQRing > kStages + kSBufs, "query-scale ring too short");
  // e4m3: the 16-bit query rows of a segment (16 x 256 B), fetched one
  // segment ahead by a bulk copy into one of two buffers
  static constexpr int kQRawBufs = KV8 ? 2 : 0;
  static constexpr int kQRawBytes = kMaxGroup * kHeadDim * 2;
  // kfull/kempty/vfull/vempty per stage, s_full/s_empty per S buffer,
  // p_full/o_full x2, q_full per query-scale slot, qraw_full per raw buffer
  static constexpr int kNumBars = 4 * kStages + 2 * kSBufs + 4 + kQRing + kQRawBufs;
  // Shared-memory carve-up, offsets from a 1024-byte aligned base.
  static constexpr int kOffStages = 0;
  static constexpr int kOffP = kOffStages + kStages * kStageBytes;
  static constexpr int kOffQRaw = kOffP + 2 * kPBufBytes;
  static constexpr int kOffBars = kOffQRaw + kQRawBufs * kQRawBytes;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;           // tmem slot, abort, last flag
  static constexpr int kOffRed = (kOffMisc + 64 + 15) & ~15;         // [2][4][16] floats tile maxima
  static constexpr int kOffFin = kOffRed + 2 * 4 * kMaxGroup * 4;    // [2][4][16] floats row sums
  static constexpr int kOffQInv = kOffFin + 2 * 4 * kMaxGroup * 4;   // [kQRing][16] floats
  static constexpr int kOffPrefix = kOffQInv + kQRing * kMaxGroup * 4;  // [B+1] pair-cost prefix sums
  static constexpr int kOffLens = kOffPrefix + (kMaxBatchPerLaunch + 1) * 4;  // [B] clamped lengths
  static constexpr int kSmemUsed = kOffLens + kMaxBatchPerLaunch * 4;
  static constexpr int kSmemBytes = kSmemUsed + 1024;                // slack for 1024-B alignment
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
  static_assert(kStageBytes % 1024 == 0 && kOffP % 1024 == 0, "swizzled tiles need 1 KB alignment");
  static_assert(kSBufs * kSCols + 2 * kOCols <= kTmemCols, "TMEM columns");
  // TMEM columns: S^T buffer b at kSCols * b, O^T buffer b after the S buffers.
  static __device__ __forceinline__ uint32_t col_s(int b) { return static_cast<uint32_t>(b * kSCols); }
  static __device__ __forceinline__ uint32_t col_o(int b) {
    return static_cast<uint32_t>(kSBufs * kSCols + b * kOCols);
  }
};
constexpr int kQkWarp = 7;  // issues QK; warp 1 issues PV
constexpr int kVProducerWarp = 6;

// Arrival counter of a split (sequence, KV head) pair, and of the grid:
// bits [12, 64) hold the launch epoch, bits [0, 12) the arrivals seen in that
// epoch (at most one per CTA, and a launch has at most 4095 CTAs).  Epochs run
// 1 .. 2^52 - 1 and then start again at 1, so a counter can only be mistaken
// for the current launch's after 2^52 - 1 launches on one workspace (centuries
// of back-to-back calls).  Only a launch that stopped early (a bounded wait
// ran out) leaves a counter behind: the CTA that merges a pair clears its
// counter and the last CTA to arrive clears the grid counter, so a launch
// that completes leaves every counter at zero.  The first arrival of a launch
// stamps the epoch with one compare-and-swap; every arrival that sees the
// stamp counts itself with one fetch-and-add, so the tens of CTAs sharing one
// long sequence's pair, finishing together, do not queue on a compare-and-swap
// loop.  Returns true for the pair's last arrival.
constexpr int kTicketCountBits = 12;
constexpr unsigned long long kTicketCountMask = (1ull << kTicketCountBits) - 1ull;
constexpr unsigned long long kEpochMax = (1ull << (64 - kTicketCountBits)) - 1ull;
__device__ __forceinline__ bool ticket_arrive(unsigned long long* t, unsigned long long epoch, int nseg) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(t);
  for (;;) {
    if ((cur >> kTicketCountBits) == epoch) {
      const unsigned long long old = atomicAdd(t, 1ull);
      return (old & kTicketCountMask) + 1ull == static_cast<unsigned long long>(nseg);
    }
    const unsigned long long prev = atomicCAS(t, cur, (epoch << kTicketCountBits) | 1ull);
    if (prev == cur) return nseg == 1;
    cur = prev;
  }
}

// UMMA shared-memory descriptor (tcgen05 matrix descriptor): start address,
// leading/stride byte offsets (16-byte units), version 1, layout type.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                               uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}
constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSw128 = 2;

// UMMA instruction descriptor for kind::f16 with an fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, bool a_mn_major, bool b_mn_major,
                                                  int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// UMMA instruction descriptor for kind::f8f6f4, both operands e4m3 (format
// code 0), fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(bool a_mn_major, bool b_mn_major, int m,
                                                       int n) {
  return (1u << 4) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// split2(a, b): hi = round-to-nearest 16-bit pair of (a, b), lo = the same
// rounding of the residuals (a - hi.x, b - hi.y); hi + lo carries ~16 more
// mantissa bits than hi alone.
template <typename T> struct DType;
template <> struct DType<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  static __device__ __forceinline__ float2 unpack2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};
template <> struct DType<__half> {
  static constexpr bool kBf16 = false;
  static __device__ __forceinline__ float2 unpack2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  static __device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};

template <typename O> __device__ __forceinline__ O to_out(float x);
template <> __device__ __forceinline__ float to_out<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half to_out<__half>(float x) { return __float2half_rn(x); }

// ---------------------------------------------------------------- schedule
// Work is split in cost space.  In units where the K/V bytes of a full
// 128-token tile cost kFullTile = 8, a tile also costs `tile_fixed` (its
// fixed QK / softmax / PV work), a sequence's partial last tile costs its
// 16-token boxes instead of 8, and every (sequence, KV head) pair costs
// `seg` once (its set-up and epilogue), raised where needed so that no pair
// costs less than `floor` (a pair of a few tiles is a latency chain that
// the ring cannot hide behind streaming).  This per-pair part is the pair's
// `lead`: its first tile starts at the pair's start and tile j >= 1 at
// start + lead + j * full.  Pairs are laid end to end (b-major, then KV
// head); CTA c takes the tiles whose start cost lies in [C*c/G, C*(c+1)/G).
// Every tile belongs to exactly one CTA; a pair spread over several CTAs is
// merged by the last of them.
constexpr int kFullTile = 8;

struct CostModel {
  int tile_fixed, seg, floor;
  __device__ __forceinline__ int full() const { return kFullTile + tile_fixed; }
  // cost of the tiles of one pair of a sequence of `len` tokens
  __device__ __forceinline__ int tiles_cost(int len) const {
    const int n_full = len / kTileTokens, rem = len % kTileTokens;
    return n_full * full() + ((rem > 0 || len == 0) ? (rem + 15) / 16 + tile_fixed : 0);
  }
  __device__ __forceinline__ int lead(int len) const {
    const int raised = floor - tiles_cost(len);
    return raised > seg ? raised : seg;
  }
  __device__ __forceinline__ int pair_cost(int len) const { return lead(len) + tiles_cost(len); }
  // upper bound of any pair's lead
  __device__ __forceinline__ int max_lead() const { return floor > seg ? floor : seg; }
};

__device__ __forceinline__ int seq_tiles(int len) {
  return len > 0 ? (len + kTileTokens - 1) / kTileTokens : 1;
}

// Divisions of the schedule, in 32 bits: the host caps a launch's batch so
// that its cost line times (grid + 1) stays below 2^32 (all the schedule's
// cost positions, and a position times the grid, fit in 32 bits).  A 64-bit
// integer division is a long software sequence, and these run, cold, on
// every CTA's path to its first load.
__device__ __forceinline__ int64_t div_u32(int64_t a, int64_t b) {
  return static_cast<int64_t>(static_cast<uint32_t>(a) / static_cast<uint32_t>(b));
}
__device__ __forceinline__ int64_t ceil_div_u32(int64_t a, int64_t b) { return div_u32(a + b - 1, b); }

// One segment of a CTA's work: tiles tile0 .. tile0+ntiles-1 of pair (b, kvh).
struct Segment {
  int b, kvh, pair;
  int tile0, ntiles;
  int seqlen;
  int nseg, cfirst;  // how many CTAs share this pair, and the first of them
};

struct Schedule {
  const int* cost_prefix;  // [B+1] per-pair cost prefix over sequences (smem)
  const int* lens;         // [B] sequence lengths, clamped to [0, max_len] (smem)
  int64_t max_len, total;  // total = Hkv * cost_prefix[B]
  int batch, hkv, grid;
  // Pair-aligned split (align_m > 0): every pair costs align_cost and CTA c
  // takes the whole pairs [align_m * c, align_m * (c + 1)).
  int align_m;
  int64_t align_cost;
  CostModel cm;

  __device__ __forceinline__ int len_of(int b) const { return lens[b]; }
  __device__ __forceinline__ int64_t range_start(int c) const {
    if (align_m > 0) {
      const int64_t pairs = static_cast<int64_t>(batch) * hkv;
      const int64_t first_pair = static_cast<int64_t>(align_m) * c;
      return align_cost * (first_pair < pairs ? first_pair : pairs);
    }
    return div_u32(total * c, grid);
  }
  // CTA whose range holds cost position s: largest c with range_start(c) <= s
  // (cost split only: the pair-aligned split cuts no pair, so it never asks)
  __device__ __forceinline__ int cta_of(int64_t s) const {
    return static_cast<int>(div_u32((s + 1) * grid + total - 1, total) - 1);
  }
  __device__ __forceinline__ int64_t pair_start(int pair) const {
    const int b = pair / hkv, kvh = pair - b * hkv;
    return static_cast<int64_t>(hkv) * cost_prefix[b] +
           static_cast<int64_t>(kvh) * (cost_prefix[b + 1] - cost_prefix[b]);
  }
  // start of tile j of the pair that starts at cp and has lead `lead`
  __device__ __forceinline__ int64_t tile_start(int64_t cp, int lead, int j) const {
    return j == 0 ? cp : cp + lead + static_cast<int64_t>(j) * cm.full();
  }
  // Segment of `pair` from tile j0 on, cut at range end e1; false if no tile
  // of the pair at or after j0 starts before e1.  Integer work here is 32-bit
  // except for pairs split across CTAs (rare), where cta_of is evaluated.
  __device__ __forceinline__ bool make(int pair, int j0, int64_t e1, Segment& s) const {
    const int b = pair / hkv;
    const int len = len_of(b);
    const int n = seq_tiles(len);
    const int lead = cm.lead(len);
    const int64_t cp = pair_start(pair);
    if (j0 >= n || tile_start(cp, lead, j0) >= e1) return false;
    // last tile with start < e1: j <= ceil((e1 - cp - lead) / full) - 1
    const int64_t x64 = e1 - cp - lead;
    int jmax = 0;
    if (x64 > 0) {
      const int x = x64 < 0x7fffffff ? static_cast<int>(x64) : 0x7fffffff;
      jmax = (x + cm.full() - 1) / cm.full() - 1;
    }
    if (jmax > n - 1) jmax = n - 1;
    s.b = b;
    s.kvh = pair - b * hkv;
    s.pair = pair;
    s.tile0 = j0;
    s.ntiles = jmax - j0 + 1;
    s.seqlen = len;
    if (j0 == 0 && jmax == n - 1) {  // the whole pair lies in this range
      s.nseg = 1;
      s.cfirst = -1;
    } else {
      s.cfirst = cta_of(cp);
      s.nseg = cta_of(tile_start(cp, lead, n - 1)) - s.cfirst + 1;
    }
    return true;
  }
  // First segment of CTA c (false if the CTA has no tile).
  __device__ __forceinline__ bool first(int c, Segment& s) const {
    if (c >= grid) return false;
    const int64_t e0 = range_start(c), e1 = range_start(c + 1);
    int lo = 0, hi = batch - 1;  // largest b with hkv * prefix[b] <= e0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(hkv) * cost_prefix[mid] <= e0) lo = mid; else hi = mid - 1;
    }
    const int pc = cost_prefix[lo + 1] - cost_prefix[lo];
    int kvh = static_cast<int>(div_u32(e0 - static_cast<int64_t>(hkv) * cost_prefix[lo], pc));
    kvh = kvh < hkv - 1 ? kvh : hkv - 1;
    const int pair = lo * hkv + kvh;
    const int64_t cp = pair_start(pair);
    int j0 = 0;
    if (e0 > cp) {
      const int64_t x = e0 - cp - cm.lead(len_of(lo));
      j0 = static_cast<int>(x > 0 ? ceil_div_u32(x, cm.full()) : 1);
      if (j0 < 1) j0 = 1;
    }
    if (make(pair, j0, e1, s)) return true;
    return pair + 1 < batch * hkv && make(pair + 1, 0, e1, s);
  }
  // Segment after `s` within the range that ends at cost e1.
  __device__ __forceinline__ bool next(const Segment& s, int64_t e1, Segment& nx) const {
    if (s.tile0 + s.ntiles < seq_tiles(s.seqlen)) return false;  // range ended inside the pair
    return s.pair + 1 < batch * hkv && make(s.pair + 1, 0, e1, nx);
  }
};

// ---------------------------------------------------------------- e4m3 query
// With an e4m3 K cache the QK product runs as kind::f8f6f4 UMMAs, whose
// operands must both be 8-bit.  Each 16-bit query row is scaled by a power of
// two 2^k that brings its largest magnitude into [128, 256) (below the e4m3
// maximum 448) and split into three e4m3 parts x = p0 + p1/16 + p2/256
// (fd_fp8.cuh); the kernel multiplies the parts side by side, recombines S in
// fp32 and undoes 2^k exactly.  The K producer warp does this once per
// segment for the NCOL rows the kernel reads (r = qi * group + g): lane l
// holds row r = l / (32 / NCOL), 4 NCOL dims from 4 NCOL (l % (32 / NCOL)).
template <int NCOL> struct QuerySplitMap {
  static constexpr int kLanesPerRow = 32 / NCOL;         // 8, 4, 2
  static constexpr int kDims = kHeadDim / kLanesPerRow;  // 16, 32, 64
  static constexpr int kChunks = kDims / 16;             // 16-dim e4m3 chunks per part
  static constexpr int kRaw = kDims / 8;                 // 16-byte pieces of the 16-bit row
};

// Lane 0: bulk-copy the segment's query rows r = qi * group + g (256 B each)
// into `dst` (row r at r * 256), completing on `bar`.  The group's rows of one
// query token are adjacent heads, so one copy per token.
template <typename T, bool MULTI>
__device__ __forceinline__ void fetch_query_rows(const DecodeParams& p, int b, int kvh, int qrows,
                                                 uint8_t* dst, uint64_t* bar) {
  const int sq = MULTI ? p.seqlen_q : 1;
  const uint32_t row_bytes = kHeadDim * 2;
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(qrows) * row_bytes);
  const T* base = static_cast<const T*>(p.q) +
                  (static_cast<int64_t>(b) * sq * p.num_heads + kvh * p.group) * kHeadDim;
  for (int qi = 0; qi < sq; ++qi)
    bulk_load(dst + qi * p.group * row_bytes, base + static_cast<int64_t>(qi) * p.num_heads * kHeadDim,
              p.group * row_bytes, bar);
}

// The lane's 4 NCOL query values from the staged rows, zeros for rows
// r >= qrows.
template <int NCOL>
__device__ __forceinline__ void read_query_rows(const uint8_t* rows, int qrows, int lane,
                                                uint4 (&raw)[QuerySplitMap<NCOL>::kRaw]) {
  using M = QuerySplitMap<NCOL>;
  const int r = lane / M::kLanesPerRow, sub = lane % M::kLanesPerRow;
  const uint4* src = reinterpret_cast<const uint4*>(rows + r * (kHeadDim * 2) + sub * (M::kDims * 2));
#pragma unroll
  for (int i = 0; i < M::kRaw; ++i) raw[i] = r < qrows ? src[i] : make_uint4(0, 0, 0, 0);
}

template <typename T> __device__ __forceinline__ void unpack8(const uint4& w, float2 (&f)[4]) {
  f[0] = DType<T>::unpack2(w.x);
  f[1] = DType<T>::unpack2(w.y);
  f[2] = DType<T>::unpack2(w.z);
  f[3] = DType<T>::unpack2(w.w);
}

// Scale and split the lane's values (all 32 lanes call this together):
// part[j][k] = part k of the lane's dims 16 j .. 16 j + 15.  Returns 2^-k,
// the inverse of the row's scale.
template <typename T, int NCOL>
__device__ __forceinline__ float split_query_rows(const uint4 (&raw)[QuerySplitMap<NCOL>::kRaw],
                                                  uint4 (&part)[QuerySplitMap<NCOL>::kChunks][3]) {
  using M = QuerySplitMap<NCOL>;
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < M::kRaw; ++i) {
    float2 f[4];
    unpack8<T>(raw[i], f);
#pragma unroll
    for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fmaxf(fabsf(f[e].x), fabsf(f[e].y)));
  }
#pragma unroll
  for (int o = 1; o < M::kLanesPerRow; o <<= 1)  // the row's other lanes (adjacent)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // 2^k with mx 2^k in [128, 256): k = 7 - floor(log2 mx), clamped to the
  // normal range; rows of zeros keep k = 0.
  int k = 0;
  if (mx > 0.f && mx <= 3.0e38f) {
    const int e = ((__float_as_int(mx) >> 23) & 0xff) - 127;
    k = 7 - e;
    k = k < -126 ? -126 : (k > 126 ? 126 : k);
  }
  const float sc = __int_as_float((k + 127) << 23);
#pragma unroll
  for (int j = 0; j < M::kChunks; ++j) {
    float x[16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float2 f[4];
      unpack8<T>(raw[2 * j + h], f);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[8 * h + 2 * e] = f[e].x * sc;
        x[8 * h + 2 * e + 1] = f[e].y * sc;
      }
    }
    e4m3_split16(x, part[j]);
  }
  return __int_as_float((127 - k) << 23);
}

__device__ __forceinline__ bool lane0_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                           uint64_t budget, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait_bounded(bar, parity, abort_flag, budget) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// MULTI = false: one query token per sequence, no causal mask (plain decode).
// MULTI = true: seqlen_q query tokens, optional bottom-right causal mask.
template <typename T, typename OutT, int NCOL, bool MULTI, bool XCHG, bool KV8>
__global__ void __launch_bounds__(kSm100Threads, 1)
    decode_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_k16,
                        const __grid_constant__ CUtensorMap tm_v16, const DecodeParams p) {
  using G = Geo<KV8, NCOL>;
  // 16-bit P.V uses N = 2*NL columns: NL hi parts then NL lo parts of P.
  // NCOL query rows are computed per (sequence, KV head); the 16-bit P
  // layout holds NL >= 8 columns per part (a UMMA needs N >= 16), the
  // columns past NCOL being zero.
  constexpr int NL = NCOL < 8 ? 8 : NCOL;
  constexpr int kPvN = 2 * NL;
  constexpr int kPGroupBytes = (kPvN / 8) * 128;  // one 8-token group of P rows
  constexpr int kPGroupBytes8 = 3 * 128;           // the same for the three e4m3 parts of P
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  // Stage s: K tile at +0, V tile at +32 KB, query rows at +64 KB.
  uint8_t* stages = smem + G::kOffStages;
  uint8_t* pbufs = smem + G::kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kOffBars);
  // The K ring (K tile + query rows) and the V ring share the stage slots
  // but fill and drain independently: K is free once QK has run, V once P.V has.
  uint64_t* kfull = bars;                 // [G::kStages] K + query rows landed
  uint64_t* kempty = kfull + G::kStages;     // [G::kStages] QK of the tile done
  uint64_t* vfull = kempty + G::kStages;     // [G::kStages] V landed
  uint64_t* vempty = vfull + G::kStages;     // [G::kStages] P.V of the tile done
  uint64_t* s_full = vempty + G::kStages;    // [G::kSBufs] S^T in TMEM
  uint64_t* s_empty = s_full + G::kSBufs;    // [G::kSBufs] S^T read by the softmax warps
  uint64_t* p_full = s_empty + G::kSBufs;    // [2] P written
  uint64_t* o_full = p_full + 2;          // [2] O^T in TMEM
  uint64_t* q_full = o_full + 2;          // [G::kQRing] inverse query-row scales written
  uint64_t* qraw_full = q_full + G::kQRing;  // [G::kQRawBufs] raw query rows landed
  uint8_t* qraw_buf = smem + G::kOffQRaw;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + G::kOffMisc + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + G::kOffMisc + 8);
  // Tiles of this CTA, published by the producer once its walk is done.
  volatile int* tiles_total = reinterpret_cast<volatile int*>(smem + G::kOffMisc + 12);
  // This launch's epoch (see DecodeParams::epoch_word), read once by thread 0.
  unsigned long long* launch_epoch = reinterpret_cast<unsigned long long*>(smem + G::kOffMisc + 16);
  float* red = reinterpret_cast<float*>(smem + G::kOffRed);
  float* fin = reinterpret_cast<float*>(smem + G::kOffFin);
  float* qinv_ring = reinterpret_cast<float*>(smem + G::kOffQInv);
  int* prefix = reinterpret_cast<int*>(smem + G::kOffPrefix);
  int* lens = reinterpret_cast<int*>(smem + G::kOffLens);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int batch = p.batch;
  const int hkv = p.num_heads_k;
  const int group = p.group;
  const int sq = MULTI ? p.seqlen_q : 1;  // query tokens per sequence
  const int qrows = p.qrows;   // query rows per (sequence, KV head): sq * group <= 16
  const uint64_t budget = p.timeout_ns;
  const int64_t max_len = p.bt_stride * static_cast<int64_t>(p.page);

  // ------------------------------------------------------------ prologue
  // Nothing below reads global memory before pdl_wait_prerequisites(): the
  // barrier set-up, TMEM allocation and shared-memory clearing may overlap
  // the previous kernel on the stream when the launch allows it.
  if (tid == 0) pdl_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    for (int i = 0; i < G::kSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    for (int i = 0; i < G::kQRing; ++i) mbar_init(&q_full[i], 1);
    for (int i = 0; i < G::kQRawBufs; ++i) mbar_init(&qraw_full[i], 1);
    *abort_flag = 0;
    *last_flag = 0;
    *tiles_total = 0x7fffffff;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, G::kTmemCols);
  // Zero the stages' query areas (rows >= qrows stay zero: the query TMA
  // writes rows < qrows only) and the P buffers (columns >= qrows stay zero).
  for (int s = 0; s < G::kStages; ++s) {
    uint4* z = reinterpret_cast<uint4*>(stages + s * G::kStageBytes + 2 * G::kOperandBytes);
    for (int i = tid; i < G::kQSlotBytes / 16; i += kSm100Threads) z[i] = make_uint4(0, 0, 0, 0);
  }
  {
    uint4* z = reinterpret_cast<uint4*>(pbufs);
    for (int i = tid; i < 2 * G::kPBufBytes / 16; i += kSm100Threads) z[i] = make_uint4(0, 0, 0, 0);
  }
  const CostModel cm{p.cost_tile, p.cost_seg, p.cost_floor};
  pdl_wait_prerequisites();
  // The epoch load is issued here and consumed after the sequence lengths'
  // loads, so the two round trips overlap.
  unsigned long long epoch_ld = 0;
  if (tid == 0) epoch_ld = *reinterpret_cast<volatile unsigned long long*>(p.epoch_word);
  // Pair-aligned split (below): whole pairs per CTA when every sequence has
  // at most align_tiles / m tiles, m = pairs per CTA = ceil(B * Hkv / grid).
  const int64_t n_pairs = static_cast<int64_t>(batch) * hkv;
  const int align_m = static_cast<int>(ceil_div_u32(n_pairs, gridDim.x));
  const int align_max_tiles = p.align_tiles / align_m;
  bool short_pairs = true;  // every sequence of this thread has at most align_max_tiles tiles
  for (int b = tid; b < batch; b += kSm100Threads) {
    const int stored = __ldg(p.seqlens + b);
    // keys cached before this step plus the ones it appended
    const int64_t want = static_cast<int64_t>(stored < 0 ? 0 : stored) + p.len_add;
    const int64_t cap = max_len < 0x7fffffff ? max_len : 0x7fffffff;
    const int len = static_cast<int>(want > cap ? cap : want);
    lens[b] = len;
    prefix[b + 1] = cm.pair_cost(len);
    short_pairs = short_pairs && seq_tiles(len) <= align_max_tiles;
  }
  if (tid == 0) {
    prefix[0] = 0;
    *launch_epoch = epoch_ld & kEpochMax;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  short_pairs = __syncthreads_and(short_pairs) != 0;
  tc_fence_after();
  // Pair-aligned split: when every CTA's share is short — m = ceil(B * Hkv /
  // grid) whole pairs of at most align_tiles / m tiles each, so at most
  // align_tiles tiles per CTA — each CTA takes m whole pairs: no pair is
  // cut, so no partial, arrival counter or merge lengthens a launch whose
  // whole time is its latency chain.  Every pair then costs the same
  // `aligned_cost` (more than its tiles' starts need: lead + (align_tiles - 1)
  // full tiles) and range c is exactly pairs [m c, m (c + 1)).
  const bool aligned = short_pairs && align_max_tiles > 0;
  const int aligned_cost = cm.max_lead() + p.align_tiles * cm.full() + 1;
  if (warp == 0) {  // inclusive scan of pair costs -> exclusive prefix sums
    int carry = 0;
    for (int base = 1; base <= batch; base += 32) {
      const int idx = base + lane;
      int v = idx <= batch ? (aligned ? aligned_cost : prefix[idx]) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      v += carry;
      if (idx <= batch) prefix[idx] = v;
      carry = __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();

  const uint32_t tmem = *tmem_slot;
  const int cta = blockIdx.x;
  Schedule sched;
  sched.cost_prefix = prefix;
  sched.lens = lens;
  sched.max_len = max_len;
  sched.total = static_cast<int64_t>(hkv) * prefix[batch];
  sched.batch = batch;
  sched.hkv = hkv;
  sched.cm = cm;
  // Each CTA's cost range is longer than the costliest tile (lead + full), so
  // every range holds at least one tile start: no CTA inside a pair's span is
  // empty, which the nseg count relies on.  CTAs past that (the host sized
  // the grid from an upper bound) have nothing to do.
  sched.align_m = aligned ? align_m : 0;
  sched.align_cost = aligned_cost;
  if (aligned) {
    sched.grid = static_cast<int>(ceil_div_u32(n_pairs, align_m));
  } else {
    const int64_t g = div_u32(sched.total, cm.max_lead() + cm.full() + 1);
    sched.grid = static_cast<int>(g < 1 ? 1 : (g < gridDim.x ? g : gridDim.x));
  }
  const int64_t range_end = sched.range_start(cta + 1);

  if (warp == 0 || warp == kVProducerWarp) {
    // ---------------------------------------------------------- TMA producers
    // Warp 0 issues the K boxes and the group's query rows of each stage,
    // warp 6 its V boxes; both arrive on the stage's `full` barrier.  Two
    // issuing warps halve the per-stage TMA issue time, which matters for
    // small pages (16-token boxes: 16 per operand per tile).
    const bool is_v = warp == kVProducerWarp;
    if (lane == 0) {
      if (is_v) {
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_v16);
      } else {
        if constexpr (!KV8) tma_prefetch_desc(&tm_q);  // e4m3: no query map
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_k16);
      }
    }
    uint64_t* ring_full = is_v ? vfull : kfull;
    uint64_t* ring_empty = is_v ? vempty : kempty;
    const CUtensorMap* map_full = is_v ? &tm_v : &tm_k;
    const CUtensorMap* map_tail = is_v ? &tm_v16 : &tm_k16;
    const int operand_off = is_v ? G::kOperandBytes : 0;
    // 16-bit query rows ride with K (two halves of qrows x 128 B); the e4m3
    // query parts are stored into the stage by this warp instead
    const uint32_t extra_tx = (is_v || KV8) ? 0u : 2u * qrows * 128u;
    constexpr uint32_t kRowTx = KV8 ? 128u : 256u;  // K or V bytes per token
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const int chunk = p.chunk;  // tokens per TMA box of a full tile; never crosses a page
    const int nchunks = kTileTokens / chunk;
    int64_t it = 0;
    bool ok = true;
    Segment s;
    bool have = sched.first(cta, s);
    // e4m3 (warp 0): the segment's 16-bit query rows, bulk-copied one
    // segment ahead into qraw_buf, and their e4m3 parts (split_query_rows).
    using QM = QuerySplitMap<NCOL>;
    [[maybe_unused]] uint4 qpart[QM::kChunks][3];
    if constexpr (KV8) {
      if (!is_v && have && lane == 0) fetch_query_rows<T, MULTI>(p, s.b, s.kvh, qrows, qraw_buf, &qraw_full[0]);
    }
    for (int64_t sgo = 0; have && ok; ++sgo) {
      Segment nx;
      const bool have_nx = sched.next(s, range_end, nx);
      if constexpr (KV8) {
        if (!is_v) {
          const int rb = static_cast<int>(sgo & 1);
          ok = mbar_wait_bounded(&qraw_full[rb], static_cast<uint32_t>((sgo >> 1) & 1), abort_flag, budget);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          uint4 qraw[QM::kRaw];
          read_query_rows<NCOL>(qraw_buf + rb * G::kQRawBytes, qrows, lane, qraw);
          const float qinv = split_query_rows<T, NCOL>(qraw, qpart);
          __syncwarp();  // buffer rb ^ 1 was read a segment ago; refill it
          if (have_nx && lane == 0)
            fetch_query_rows<T, MULTI>(p, nx.b, nx.kvh, qrows, qraw_buf + (rb ^ 1) * G::kQRawBytes,
                                       &qraw_full[rb ^ 1]);
          // Slot sgo % kQRing was last read by the softmax warps for segment
          // sgo - kQRing, which began more than kStages + kSBufs tiles ago.
          const int slot = static_cast<int>(sgo % G::kQRing);
          const int qr = lane / QM::kLanesPerRow;
          if (lane % QM::kLanesPerRow == 0) qinv_ring[slot * kMaxGroup + qr] = qr < qrows ? qinv : 0.f;
          __syncwarp();
          if (lane == 0) mbar_arrive(&q_full[slot]);
        }
      }
      const int32_t* bt_row = p.block_table + static_cast<int64_t>(s.b) * p.bt_stride;
      for (int t = 0; t < s.ntiles; ++t, ++it) {
        const int tok0 = (s.tile0 + t) * kTileTokens;
        const int valid_rows = s.seqlen - tok0;
        // Full tile: `nchunks` boxes of `chunk` tokens.  Last partial tile:
        // 16-token boxes over the valid rows only.
        const bool tail = valid_rows < kTileTokens;
        const int box = tail ? 16 : chunk;
        const int nbox = tail ? (valid_rows > 0 ? (valid_rows + 15) / 16 : 0) : nchunks;
        const int pos = tok0 + lane * box;
        const bool need = lane < nbox;
        // Issued before the wait for the stage and first used after it, so the
        // page-table round trip overlaps the wait.  With 16-token pages a tile
        // reads eight new entries; checking them here, before the wait, put
        // that round trip on the producer's path (config 5 ran 8 % slower,
        // 10 % with an e4m3 cache).
        int page_id = 0;
        if (need) page_id = __ldg(bt_row + pos / p.page);
        const int stage = static_cast<int>(it % G::kStages);
        ok = lane0_wait(&ring_empty[stage], static_cast<uint32_t>((it / G::kStages) & 1) ^ 1u,
                        abort_flag, budget, lane);
        if (!ok) break;
        uint8_t* sdst = stages + stage * G::kStageBytes;
        if constexpr (KV8) {
          // A stage already holds this segment's query parts unless its
          // previous tile (it - kStages) belonged to an earlier segment.
          if (!is_v && t < G::kStages) {
            // The query parts, as rows part * 16 + r of 128 B laid out as a
            // 128B-swizzled TMA box would leave them: 16-byte chunk c of row R
            // at chunk c ^ (R & 7).  Rows r >= NCOL are never read back from
            // S.  Ordered before the `full` arrival below.
            uint8_t* qdst = sdst + 2 * G::kOperandBytes;
            const int r = lane / QM::kLanesPerRow, sub = lane % QM::kLanesPerRow;
#pragma unroll
            for (int k = 0; k < 3; ++k) {
              const int row = k * kMaxGroup + r;
#pragma unroll
              for (int j = 0; j < QM::kChunks; ++j) {
                const int c = sub * QM::kChunks + j;
                *reinterpret_cast<uint4*>(qdst + row * 128 + ((c ^ (row & 7)) << 4)) = qpart[j][k];
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
          }
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&ring_full[stage], static_cast<uint32_t>(nbox * box) * kRowTx + extra_tx);
          if constexpr (!KV8) {
            if (!is_v) {
              // rows qi * group + g: query token qi, head kvh * group + g
              uint8_t* qdst = sdst + 2 * G::kOperandBytes;
              tma_load_4d(&tm_q, &ring_full[stage], qdst, 0, s.kvh * group, 0, s.b, pol_keep);
              tma_load_4d(&tm_q, &ring_full[stage], qdst + G::kQSlotBytes / 2, 64, s.kvh * group, 0,
                          s.b, pol_keep);
            }
          }
        }
        __syncwarp();
        if (need) {
          if (page_id < 0 || page_id >= p.num_blocks) {
            // A page id inside the sequence's range that is not in the pool:
            // report it and fetch a box that lies wholly past the pool
            // instead, which the tensor copy fills with zeros (no access
            // outside the cache; those keys score 0 and their values add 0).
            report_status(p.err, kStatusBadPage);
            page_id = static_cast<int>(p.num_blocks);
          }
          const int off = pos % p.page;
          const CUtensorMap* m = tail ? map_tail : map_full;
          uint8_t* dst = sdst + operand_off + lane * box * 128;
          tma_load_4d(m, &ring_full[stage], dst, 0, s.kvh, off, page_id, pol_stream);
          if constexpr (!KV8)
            tma_load_4d(m, &ring_full[stage], dst + G::kHalfBytes, 64, s.kvh, off, page_id, pol_stream);
        }
        __syncwarp();
      }
      s = nx;
      have = have_nx;
    }
    if (!is_v && lane == 0) {
      *tiles_total = static_cast<int>(it);
      // Every CTA has read this launch's epoch before it counts itself here;
      // the last to count hands the next launch a new one (1 .. 2^52 - 1; a
      // zeroed workspace starts at 0, consistent with its zeroed counters)
      // and clears the count; the next launch reads both only after this
      // grid has completed.  Done after the last load is issued, the round
      // trips overlap the drain of the ring, and CTAs arrive spread over
      // their different finishing times.
      const unsigned long long e = *launch_epoch;
      if (ticket_arrive(p.epoch_word + 1, e, static_cast<int>(gridDim.x))) {
        p.epoch_word[0] = e % kEpochMax + 1ull;
        p.epoch_word[1] = 0ull;
      }
    }
  } else if (warp == 1 || warp == kQkWarp) {
    // ---------------------------------------------------------- UMMA issuers
    // A tcgen05.mma of M = 128, K = 16 occupies the tensor pipe ~48 cycles
    // whatever N (up to 64), and the issuing thread stalls until it is taken,
    // so one tile's 16 UMMAs keep an issuing thread busy for ~0.4 us.  Two
    // warps issue: warp 7 runs QK(i) once K(i) has landed and S buffer i%3
    // is drained; warp 1 runs P.V(i) once P(i) is written and V(i) has landed
    // (P(i) also means O buffer i%2 is drained).  While one waits on its
    // barriers the other's UMMAs keep the pipe busy.  Tiles 0 .. ntiles-1 of
    // this CTA's range; the count is known once the producer has walked it.
    const bool is_qk = warp == kQkWarp;
    // Lane 0: wait for the phase; 1 = completed, 0 = tile idx does not exist
    // (the range holds fewer tiles), -1 = gave up (timeout or abort).
    auto issue_wait = [&](uint64_t* bar, uint32_t parity, int64_t idx) -> int {
      uint64_t t0 = 0;
      uint32_t spins = 0;
      while (true) {
        if (mbar_try_wait(bar, parity)) return 1;
        if (idx >= *tiles_total) return 0;
        if (((++spins) & 63u) == 0u) {
          if (*abort_flag) return -1;
          const uint64_t now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > budget) {
            *abort_flag = 1;
            return -1;
          }
        }
      }
    };
    constexpr bool kBf16 = DType<T>::kBf16;
    constexpr uint32_t idesc_qk = make_idesc(kBf16, false, false, 128, kMaxGroup);
    constexpr uint32_t idesc_pv = make_idesc(kBf16, true, true, 128, kPvN);
    constexpr uint32_t idesc_qk8 = make_idesc_e4m3(false, false, 128, 3 * kMaxGroup);
    constexpr uint32_t idesc_pv8 = make_idesc_e4m3(true, true, 128, 3 * kMaxGroup);
    for (int64_t i = 0;; ++i) {
      int st = 1;
      if (lane == 0) {
        const int stage = static_cast<int>(i % G::kStages);
        const uint32_t ring_ph = static_cast<uint32_t>((i / G::kStages) & 1);
        if (is_qk) {
          const int sb = static_cast<int>(i % G::kSBufs);
          st = issue_wait(&kfull[stage], ring_ph, i);
          if (st == 1) st = issue_wait(&s_empty[sb], static_cast<uint32_t>(((i / G::kSBufs) & 1) ^ 1), i);
          if (st == 1) {
            tc_fence_after();
            const uint32_t kaddr = smem_u32(stages + stage * G::kStageBytes);
            const uint32_t qaddr = kaddr + 2 * G::kOperandBytes;
            if constexpr (KV8) {
#pragma unroll
              for (int j = 0; j < kHeadDim / 32; ++j) {
                // A = e4m3 K tile, K-major 128B swizzle: one 128 B row holds all
                // 128 dims; the 32-dim step j moves 32 B inside the row.  B = the
                // 48 rows of query parts, same layout.
                const uint64_t a = make_sdesc(kaddr + j * 32, 16, 1024, kLayoutSw128);
                const uint64_t b = make_sdesc(qaddr + j * 32, 16, 1024, kLayoutSw128);
                umma_f8(tmem + G::col_s(sb), a, b, idesc_qk8, j > 0 ? 1u : 0u);
              }
            } else {
#pragma unroll
              for (int j = 0; j < kHeadDim / 16; ++j) {
                // A = K tile, K-major 128B swizzle: 8-row groups 1 KB apart; the
                // 16-dim step j moves 32 B inside a 128 B row, 64-dim halves 16 KB apart.
                const uint64_t a =
                    make_sdesc(kaddr + (j >> 2) * G::kHalfBytes + (j & 3) * 32, 16, 1024, kLayoutSw128);
                const uint64_t b = make_sdesc(qaddr + (j >> 2) * (G::kQSlotBytes / 2) + (j & 3) * 32, 16,
                                              1024, kLayoutSw128);
                umma_f16(tmem + G::col_s(sb), a, b, idesc_qk, j > 0 ? 1u : 0u);
              }
            }
            umma_commit(&s_full[sb]);
            umma_commit(&kempty[stage]);
          }
        } else {
          const int pb = static_cast<int>(i & 1);
          st = issue_wait(&p_full[pb], static_cast<uint32_t>((i >> 1) & 1), i);
          if (st == 1) st = issue_wait(&vfull[stage], ring_ph, i);
          if (st == 1) {
            tc_fence_after();
            const uint32_t vaddr = smem_u32(stages + stage * G::kStageBytes + G::kOperandBytes);
            const uint32_t paddr = smem_u32(pbufs + pb * G::kPBufBytes);
            if constexpr (KV8) {
#pragma unroll
              for (int j = 0; j < kTileTokens / 32; ++j) {
                // A = e4m3 V^T: MN-major, 128B swizzle, all 128 dims in one 128 B
                // row (one swizzle atom along M), 8-token groups 1 KB apart (SBO).
                const uint64_t a = make_sdesc(vaddr + j * 4096, G::kOperandBytes, 1024, kLayoutSw128);
                // B = [P0 | P1 | P2]^T: MN-major, no swizzle; 16-column core
                // matrices 128 B apart (SBO), 8-token groups 384 B apart (LBO).
                const uint64_t b = make_sdesc(paddr + j * 4 * kPGroupBytes8, kPGroupBytes8, 128, kLayoutNone);
                umma_f8(tmem + G::col_o(pb), a, b, idesc_pv8, j > 0 ? 1u : 0u);
              }
            } else {
#pragma unroll
              for (int j = 0; j < kTileTokens / 16; ++j) {
                // A = V^T: MN-major (head-dim contiguous), 128B swizzle; the two
                // 64-dim halves are 16 KB apart (LBO), 8-token groups 1 KB apart (SBO).
                const uint64_t a = make_sdesc(vaddr + j * 2048, G::kHalfBytes, 1024, kLayoutSw128);
                // B = [P_hi | P_lo]^T: MN-major (heads contiguous), no swizzle;
                // 8-column core matrices 128 B apart (SBO), 8-token groups kPGroupBytes apart (LBO).
                const uint64_t b = make_sdesc(paddr + j * 2 * kPGroupBytes, kPGroupBytes, 128, kLayoutNone);
                umma_f16(tmem + G::col_o(pb), a, b, idesc_pv, j > 0 ? 1u : 0u);
              }
            }
            umma_commit(&o_full[pb]);
            umma_commit(&vempty[stage]);
          }
        }
      }
      st = __shfl_sync(0xffffffffu, st, 0);
      if (st != 1) break;
    }
  } else {
    // ---------------------------------------------------------- softmax warps
    // One flat loop over the CTA's tiles.  Iteration i runs the softmax of
    // tile i, then folds in O of tile i-1.  When tile i opens a new segment,
    // O of the previous segment's last tile arrives in that same iteration
    // and the previous segment is finished there, so the P.V round trip of a
    // segment's last tile overlaps the next segment's first softmax.
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;  // token row of S, head-dim index of O
    const int d = row;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float neg_inf = -__int_as_float(0x7f800000);
    const int hq = p.num_heads;
    OutT* out = reinterpret_cast<OutT*>(p.out);
    struct State {
      float m[NCOL], l[NCOL], o[NCOL], a[NCOL];
    };
    auto reset = [&](State& st) {
#pragma unroll
      for (int h = 0; h < NCOL; ++h) {
        st.m[h] = neg_inf;
        st.l[h] = 0.f;
        st.o[h] = 0.f;
        st.a[h] = 0.f;
      }
    };
    // O^T of tile i (hi + lo halves) for this thread's head-dim row.
    auto load_o = [&](int64_t i, float (&ov)[NCOL]) {
      const int pb = static_cast<int>(i & 1);
      mbar_wait_bounded(&o_full[pb], static_cast<uint32_t>((i >> 1) & 1), abort_flag, budget);
      tc_fence_after();
      if constexpr (KV8) {
        // three parts of P, 16 columns apart: O = O0 + O1 / 16 + O2 / 256
        if constexpr (NCOL == kMaxGroup) {
          // 16 rows: one part at a time (same sums, 32 fewer live registers)
          uint32_t r0[NCOL];
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb), r0);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < NCOL; ++h) ov[h] = __uint_as_float(r0[h]);
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb) + kMaxGroup, r0);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < NCOL; ++h) ov[h] = fmaf(__uint_as_float(r0[h]), 1.f / 16.f, ov[h]);
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb) + 2 * kMaxGroup, r0);
          tmem_wait_ld();
          tc_fence_before();  // orders these loads before the next P arrival (frees the O buffer)
#pragma unroll
          for (int h = 0; h < NCOL; ++h) ov[h] = fmaf(__uint_as_float(r0[h]), 1.f / 256.f, ov[h]);
        } else {
          uint32_t r0[NCOL], r1[NCOL], r2[NCOL];
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb), r0);
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb) + kMaxGroup, r1);
          tmem_ld_cols<NCOL>(lane_addr + G::col_o(pb) + 2 * kMaxGroup, r2);
          tmem_wait_ld();
          tc_fence_before();  // orders this load before the next P arrival (frees the O buffer)
#pragma unroll
          for (int h = 0; h < NCOL; ++h)
            ov[h] = fmaf(__uint_as_float(r2[h]), 1.f / 256.f,
                         fmaf(__uint_as_float(r1[h]), 1.f / 16.f, __uint_as_float(r0[h])));
        }
      } else {
        uint32_t r[kPvN];
        if constexpr (NL == 8) tmem_ld_x16(lane_addr + G::col_o(pb), r); else tmem_ld_x32(lane_addr + G::col_o(pb), r);
        tmem_wait_ld();
        tc_fence_before();  // orders this load before the next P arrival (frees the O buffer)
#pragma unroll
        for (int h = 0; h < NCOL; ++h) ov[h] = __uint_as_float(r[h]) + __uint_as_float(r[NL + h]);
      }
    };
    // Segment epilogue: direct output, or partial + (last arrival) merge.
    int fin_buf = 0;
    // `scratch`: a P buffer no P.V is reading (used when merging a split pair).
    auto finish = [&](const Segment& sg, const State& st, uint8_t* scratch) {
      float* fb = fin + fin_buf * (4 * kMaxGroup);
      fin_buf ^= 1;
#pragma unroll
      for (int h = 0; h < NCOL; ++h) {
        float v = st.l[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) fb[quad * kMaxGroup + h] = v;
      }
      named_bar_sync(1, 128);
      float l_tot[NCOL];
#pragma unroll
      for (int h = 0; h < NCOL; ++h)
        l_tot[h] = (fb[h] + fb[kMaxGroup + h]) + (fb[2 * kMaxGroup + h] + fb[3 * kMaxGroup + h]);
      // column h = query row (qi, g): token qi of the sequence's sq new
      // tokens, query head kvh * group + g
      auto out_index = [&](int h) {
        const int qi = MULTI ? h / group : 0, g = h - qi * group;
        return ((static_cast<int64_t>(sg.b) * sq + qi) * hq + sg.kvh * group + g) * kHeadDim + d;
      };
      auto lse_index = [&](int h) {
        const int qi = MULTI ? h / group : 0, g = h - qi * group;
        return (static_cast<int64_t>(sg.b) * hq + sg.kvh * group + g) * sq + qi;
      };
      // Result writers: the output (and LSE), or, in a cross-GPU exchange,
      // this rank's part in every rank's exchange buffer.
      auto put_o = [&](int64_t oi, float v) {
        if constexpr (XCHG) {
          for (int j = 0; j < p.xworld; ++j) p.xpart[j][oi] = v;
        } else {
          out[oi] = to_out<OutT>(v);
        }
      };
      auto put_lse = [&](int64_t li, float v) {
        if constexpr (XCHG) {
          for (int j = 0; j < p.xworld; ++j) p.xpart[j][p.xlse_off + li] = v;
        } else if (p.lse != nullptr) {
          p.lse[li] = v;
        }
      };
      // e4m3 V: O carries 256 P (see the P split) times the stored V
      const float osc = KV8 ? __ldg(p.v_scale + sg.kvh) * (1.f / 256.f) : 1.f;
      if (sg.nseg == 1) {
#pragma unroll
        for (int h = 0; h < NCOL; ++h) {
          if (h < qrows) {
            const float v = l_tot[h] > 0.f ? st.o[h] * osc / l_tot[h] : 0.f;
            put_o(out_index(h), v);
            if (d == h)
              put_lse(lse_index(h),
                      l_tot[h] > 0.f ? (st.m[h] + fast_log2(l_tot[h])) * 0.69314718055994531f : neg_inf);
          }
        }
        return;
      }
      const int64_t slot = static_cast<int64_t>(cta) + sg.pair;
      float* po = p.part_o + slot * qrows * kHeadDim + d;
#pragma unroll
      for (int h = 0; h < NCOL; ++h) {
        if (h < qrows) {
          po[h * kHeadDim] = l_tot[h] > 0.f ? st.o[h] * osc / l_tot[h] : 0.f;
          if (d == h) p.part_lse[slot * qrows + h] = l_tot[h] > 0.f ? st.m[h] + fast_log2(l_tot[h]) : neg_inf;
        }
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (d == 0) {
        int is_last = 0;
        if (!*abort_flag) is_last = ticket_arrive(p.tickets + sg.pair, *launch_epoch, sg.nseg) ? 1 : 0;
        // Every segment of the pair has counted itself: clear the counter for
        // later launches (nothing else touches it in this one).
        if (is_last) *reinterpret_cast<volatile unsigned long long*>(p.tickets + sg.pair) = 0ull;
        *last_flag = is_last;
      }
      named_bar_sync(1, 128);
      const int merge = *last_flag;
      named_bar_sync(1, 128);  // last_flag is reused by the next split segment
      if (!merge) return;
      __threadfence();
      const int64_t sbase = static_cast<int64_t>(sg.cfirst) + sg.pair;
      // The pair's nseg x qrows partial LSEs are contiguous: stage them in a
      // free P buffer with one parallel load, so the per-head weights come
      // from shared memory and only the independent partial-O loads remain.
      const int nl = sg.nseg * qrows;
      float* sl = reinterpret_cast<float*>(scratch);
      const bool staged = nl <= G::kPBufBytes / 4;
      if (staged) {
        for (int i = d; i < nl; i += 128) sl[i] = __ldcg(p.part_lse + sbase * qrows + i);
        named_bar_sync(1, 128);
      }
      // A warp covers a 128-dim row with 16-byte loads (lane l: dims 4l..4l+3);
      // warp w merges rows w, w+4, ...  The segments are taken in batches:
      // each thread issues the loads of a whole batch (8 16-byte loads,
      // kBatch segments x its kRows rows) before it uses any of them, so a
      // pair cut into tens of segments (a long sequence spread over many
      // CTAs) merges in a few L2 round trips.
      auto lse_of = [&](int j, int h) {
        return staged ? sl[j * qrows + h] : __ldcg(p.part_lse + (sbase + j) * qrows + h);
      };
      constexpr int kRows = (NCOL + 3) / 4;  // rows per thread
      constexpr int kBatch = 8 / kRows;      // segments per batch of loads
      const int lane4 = d & 31, rg = d >> 5;
      float mx[kRows], den[kRows], acc[kRows][4];
#pragma unroll
      for (int k = 0; k < kRows; ++k) {
        mx[k] = neg_inf;
        den[k] = 0.f;
        acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
      }
      for (int j = 0; j < sg.nseg; ++j) {
#pragma unroll
        for (int k = 0; k < kRows; ++k)
          if (rg + 4 * k < qrows) mx[k] = fmaxf(mx[k], lse_of(j, rg + 4 * k));
      }
      const float* po4 = p.part_o + sbase * qrows * kHeadDim + 4 * lane4;
      for (int j0 = 0; j0 < sg.nseg; j0 += kBatch) {
        float4 o[kBatch][kRows];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
#pragma unroll
          for (int k = 0; k < kRows; ++k) {
            const int h = rg + 4 * k, j = j0 + u;
            o[u][k] = (j < sg.nseg && h < qrows)
                          ? __ldcg(reinterpret_cast<const float4*>(
                                po4 + (static_cast<int64_t>(j) * qrows + h) * kHeadDim))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
#pragma unroll
          for (int k = 0; k < kRows; ++k) {
            const int h = rg + 4 * k, j = j0 + u;
            if (j < sg.nseg && h < qrows) {
              const float lj = lse_of(j, h);
              const float wj = lj == neg_inf ? 0.f : fast_exp2(lj - mx[k]);  // empty parts hold O = 0
              acc[k][0] = fmaf(wj, o[u][k].x, acc[k][0]);
              acc[k][1] = fmaf(wj, o[u][k].y, acc[k][1]);
              acc[k][2] = fmaf(wj, o[u][k].z, acc[k][2]);
              acc[k][3] = fmaf(wj, o[u][k].w, acc[k][3]);
              den[k] += wj;
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kRows; ++k) {
        const int h = rg + 4 * k;
        if (h < qrows) {
          const float inv = den[k] > 0.f ? 1.f / den[k] : 0.f;
          const int64_t base = out_index(h) - d + 4 * lane4;
#pragma unroll
          for (int e = 0; e < 4; ++e) put_o(base + e, acc[k][e] * inv);
          if (lane4 == 0)
            put_lse(lse_index(h),
                    den[k] > 0.f ? (mx[k] + fast_log2(den[k])) * 0.69314718055994531f : neg_inf);
        }
      }
    };

    // Per query row h = (qi, g): how many of the sequence's last keys it may
    // not see (0 unless causal): key t is visible iff t < L + coff[h].
    int coff[NCOL];
#pragma unroll
    for (int h = 0; h < NCOL; ++h) coff[h] = (MULTI && p.causal) ? (h / group) - (sq - 1) : 0;

    // e4m3 K: per query row of the segment, softmax scale (log2) x K scale x
    // the inverse of the row's query-part scale
    float qf[KV8 ? NCOL : 1];
    State cur, prev;
    reset(cur);
    reset(prev);
    Segment seg{}, prev_seg{};
    int t = 0;
    int64_t it = 0;
    int64_t sgo = 0;  // segment ordinal (slot of the query-scale ring)
    for (bool have = sched.first(cta, seg); have; ++it, ++t) {
      bool prev_open = false;
      if (t == seg.ntiles) {  // next segment, if the range has one
        Segment nx;
        if (!sched.next(seg, range_end, nx)) break;
        prev_seg = seg;
        seg = nx;
        ++sgo;
        t = 0;
        prev = cur;
        reset(cur);
        prev_open = true;
      }
      if constexpr (KV8) {
        if (t == 0) {
          const float ks = __ldg(p.k_scale + seg.kvh) * p.scale_log2;
          const int slot = static_cast<int>(sgo % G::kQRing);
          mbar_wait_bounded(&q_full[slot], static_cast<uint32_t>((sgo / G::kQRing) & 1), abort_flag, budget);
          const float* qi = qinv_ring + slot * kMaxGroup;
#pragma unroll
          for (int h = 0; h < NCOL; ++h) qf[h] = ks * qi[h];
        }
      }
      // ---- softmax of tile `it`
      const int sb = static_cast<int>(it & 1);  // P buffer and max-exchange slot
      const int stage = static_cast<int>(it % G::kStages);
      {
        const int sbuf = static_cast<int>(it % G::kSBufs);
        mbar_wait_bounded(&s_full[sbuf], static_cast<uint32_t>((it / G::kSBufs) & 1), abort_flag, budget);
      }
      tc_fence_after();
      uint32_t r[NCOL];
      float s8[KV8 ? NCOL : 1];
      {
        const uint32_t cs = G::col_s(static_cast<int>(it % G::kSBufs));
        if constexpr (KV8) {
          // three parts of the query, 16 columns apart: S = S0 + S1 / 16 + S2 / 256
          if constexpr (NCOL == kMaxGroup) {
            // 16 rows: one part at a time (same sums, 32 fewer live registers)
            tmem_ld_cols<NCOL>(lane_addr + cs, r);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < NCOL; ++h) s8[h] = __uint_as_float(r[h]);
            tmem_ld_cols<NCOL>(lane_addr + cs + kMaxGroup, r);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < NCOL; ++h) s8[h] = fmaf(__uint_as_float(r[h]), 1.f / 16.f, s8[h]);
            tmem_ld_cols<NCOL>(lane_addr + cs + 2 * kMaxGroup, r);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < NCOL; ++h) s8[h] = fmaf(__uint_as_float(r[h]), 1.f / 256.f, s8[h]);
          } else {
            uint32_t r1[NCOL], r2[NCOL];
            tmem_ld_cols<NCOL>(lane_addr + cs, r);
            tmem_ld_cols<NCOL>(lane_addr + cs + kMaxGroup, r1);
            tmem_ld_cols<NCOL>(lane_addr + cs + 2 * kMaxGroup, r2);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < NCOL; ++h)
              s8[h] = fmaf(__uint_as_float(r2[h]), 1.f / 256.f,
                           fmaf(__uint_as_float(r1[h]), 1.f / 16.f, __uint_as_float(r[h])));
          }
        } else {
          tmem_ld_cols<NCOL>(lane_addr + cs, r);
          tmem_wait_ld();
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[it % G::kSBufs]);

      const int tok0 = (seg.tile0 + t) * kTileTokens;
      const int valid_rows = seg.seqlen - tok0;  // may exceed 128; <=0 only for empty sequences
      const bool valid = row < valid_rows;
      float sv[NCOL];
      float* red_t = red + (it & 1) * (4 * kMaxGroup);
#pragma unroll
      for (int h = 0; h < NCOL; ++h) {
        // causal: query row h sees keys up to its own position L - sq + qi
        const bool vis = MULTI ? row < valid_rows + coff[h] : valid;
        if constexpr (KV8)
          sv[h] = vis ? s8[h] * qf[h] : neg_inf;
        else
          sv[h] = vis ? __uint_as_float(r[h]) * p.scale_log2 : neg_inf;
        const float wm = warp_max_f32(sv[h]);
        if (lane == 0) red_t[quad * kMaxGroup + h] = wm;
      }
      named_bar_sync(1, 128);
      float pv[NCOL], alpha[NCOL];
#pragma unroll
      for (int h = 0; h < NCOL; ++h) {
        const float tmax = fmaxf(fmaxf(red_t[h], red_t[kMaxGroup + h]),
                                 fmaxf(red_t[2 * kMaxGroup + h], red_t[3 * kMaxGroup + h]));
        const float m_new = fmaxf(cur.m[h], tmax);
        const float m_use = m_new == neg_inf ? 0.f : m_new;
        alpha[h] = fast_exp2(cur.m[h] - m_use);
        pv[h] = (h < qrows) ? fast_exp2(sv[h] - m_use) : 0.f;
        cur.l[h] = fmaf(cur.l[h], alpha[h], pv[h]);
        cur.m[h] = m_new;
      }
      if (valid_rows < kTileTokens && !valid &&
          mbar_wait_bounded(&vfull[stage], static_cast<uint32_t>((it / G::kStages) & 1), abort_flag, budget)) {
        // Rows past the sequence end: stale or never-written data must not
        // reach P.V (0 * NaN), so zero this token's V row in the stage, after
        // the tile's V copy (whose last box may cover the row) has landed.
        uint4* vrow0 = reinterpret_cast<uint4*>(stages + stage * G::kStageBytes + G::kOperandBytes + row * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) vrow0[i] = make_uint4(0, 0, 0, 0);
        if constexpr (!KV8) {
          uint4* vrow1 = reinterpret_cast<uint4*>(stages + stage * G::kStageBytes + G::kOperandBytes + G::kHalfBytes + row * 128);
#pragma unroll
          for (int i = 0; i < 8; ++i) vrow1[i] = make_uint4(0, 0, 0, 0);
        }
      }
      if constexpr (KV8) {
        // This token's row of [P0 | P1 | P2], the e4m3 parts of 256 P (scaled
        // so small probabilities stay above the e4m3 subnormal range):
        // 16-column chunks 128 B apart.
        uint8_t* prow = pbufs + sb * G::kPBufBytes + (row >> 3) * kPGroupBytes8 + (row & 7) * 16;
        uint32_t w[8][3];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (2 * i < NCOL) {
            e4m3_split2(pv[2 * i] * 256.f, pv[2 * i + 1] * 256.f, w[i]);
          } else {
            w[i][0] = w[i][1] = w[i][2] = 0u;
          }
        }
#pragma unroll
        for (int k = 0; k < 3; ++k)
          *reinterpret_cast<uint4*>(prow + k * 128) =
              make_uint4(w[0][k] | (w[1][k] << 16), w[2][k] | (w[3][k] << 16),
                         w[4][k] | (w[5][k] << 16), w[6][k] | (w[7][k] << 16));
      } else {
        // This token's row of [P_hi | P_lo]: 8-column chunks 128 B apart.
        uint8_t* prow = pbufs + sb * G::kPBufBytes + (row >> 3) * kPGroupBytes + (row & 7) * 16;
#pragma unroll
        for (int c = 0; c < NL / 8; ++c) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (8 * c + 2 * j < NCOL) {
              DType<T>::split2(pv[8 * c + 2 * j], pv[8 * c + 2 * j + 1], hw[j], lw[j]);
            } else {
              hw[j] = lw[j] = 0u;
            }
          }
          *reinterpret_cast<uint4*>(prow + c * 128) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(prow + (NL / 8 + c) * 128) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[sb]);

      // ---- O of tile it-1
      if (it > 0) {
        float ov[NCOL];
        load_o(it - 1, ov);
        if (prev_open) {
#pragma unroll
          for (int h = 0; h < NCOL; ++h) prev.o[h] = fmaf(prev.o[h], prev.a[h], ov[h]);
          // P.V(it-1) is done, so its P buffer is free until tile it+1's softmax
          finish(prev_seg, prev, pbufs + ((it + 1) & 1) * G::kPBufBytes);
        } else {
#pragma unroll
          for (int h = 0; h < NCOL; ++h) cur.o[h] = fmaf(cur.o[h], cur.a[h], ov[h]);
        }
      }
#pragma unroll
      for (int h = 0; h < NCOL; ++h) cur.a[h] = alpha[h];
    }
    if (it > 0) {
      float ov[NCOL];
      load_o(it - 1, ov);
#pragma unroll
      for (int h = 0; h < NCOL; ++h) cur.o[h] = fmaf(cur.o[h], cur.a[h], ov[h]);
      finish(seg, cur, pbufs);  // every P.V is done
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (XCHG && tid == 0 && !*abort_flag) {
    // After the CTA barrier, one system-scope fence publishes the CTA's
    // exchange writes; the CTA that finishes last on this GPU then tells
    // every rank that this rank's part is complete (the host zeroes xdone
    // before each launch).
    __threadfence_system();
    if (atomicAdd(p.xdone, 1u) == gridDim.x - 1u) {
      __threadfence_system();
      for (int j = 0; j < p.xworld; ++j) st_release_sys_u32(p.xflag[j], p.xepoch);
    }
  }
  if (*abort_flag) {
    if (tid == 0) {
      report_status(p.err, kStatusTimeout);
      // Let any copy or MMA still in flight land before the CTA's shared
      // memory and TMEM are released (bounded: 2 ms).
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 2000000ull) {
      }
    }
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

template <typename T, typename OutT, int NCOL, bool MULTI, bool XCHG = false, bool KV8 = false>
cudaError_t launch_typed(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream) {
  using G = Geo<KV8, NCOL>;
  auto kern = decode_sm100_kernel<T, OutT, NCOL, MULTI, XCHG, KV8>;
  // The attribute is per device; setting it again is harmless.
  static unsigned long long configured = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if ((__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & bit) == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, bit, __ATOMIC_RELEASE);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kSm100Threads);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, m.q, m.k, m.v, m.k16, m.v16, p);
}

// e4m3 K/V; T is the query type (the kernel splits its rows into e4m3 parts).
template <typename T, typename OutT>
cudaError_t launch_ncol_kv8(const TensorMaps& m, const DecodeParams& p, int grid,
                            cudaStream_t stream) {
  const bool multi = p.seqlen_q > 1 || p.causal;
  if constexpr (std::is_same<OutT, float>::value) {
    if (p.xworld > 0) {  // cross-GPU exchange: fp32 parts to every rank
      if (p.qrows <= 8)
        return multi ? launch_typed<T, float, 8, true, true, true>(m, p, grid, stream)
                     : launch_typed<T, float, 8, false, true, true>(m, p, grid, stream);
      return multi ? launch_typed<T, float, 16, true, true, true>(m, p, grid, stream)
                   : launch_typed<T, float, 16, false, true, true>(m, p, grid, stream);
    }
  }
  if (p.qrows <= 4)
    return multi ? launch_typed<T, OutT, 4, true, false, true>(m, p, grid, stream)
                 : launch_typed<T, OutT, 4, false, false, true>(m, p, grid, stream);
  if (p.qrows <= 8)
    return multi ? launch_typed<T, OutT, 8, true, false, true>(m, p, grid, stream)
                 : launch_typed<T, OutT, 8, false, false, true>(m, p, grid, stream);
  return multi ? launch_typed<T, OutT, 16, true, false, true>(m, p, grid, stream)
               : launch_typed<T, OutT, 16, false, false, true>(m, p, grid, stream);
}

template <typename T, typename OutT>
cudaError_t launch_ncol(const TensorMaps& m, const DecodeParams& p, int grid, cudaStream_t stream) {
  const bool multi = p.seqlen_q > 1 || p.causal;
  if constexpr (std::is_same<OutT, float>::value) {
    if (p.xworld > 0) {  // cross-GPU exchange: fp32 parts to every rank
      if (p.qrows <= 8)
        return multi ? launch_typed<T, float, 8, true, true>(m, p, grid, stream)
                     : launch_typed<T, float, 8, false, true>(m, p, grid, stream);
      return multi ? launch_typed<T, float, 16, true, true>(m, p, grid, stream)
                   : launch_typed<T, float, 16, false, true>(m, p, grid, stream);
    }
  }
  if (p.qrows <= 4)
    return multi ? launch_typed<T, OutT, 4, true>(m, p, grid, stream)
                 : launch_typed<T, OutT, 4, false>(m, p, grid, stream);
  if (p.qrows <= 8)
    return multi ? launch_typed<T, OutT, 8, true>(m, p, grid, stream)
                 : launch_typed<T, OutT, 8, false>(m, p, grid, stream);
  return multi ? launch_typed<T, OutT, 16, true>(m, p, grid, stream)
               : launch_typed<T, OutT, 16, false>(m, p, grid, stream);
}

}  // namespace

}  // namespace fd
