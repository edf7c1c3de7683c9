// Block-sparse prefill of the indexed gated FFN on tcgen05 tensor cores (sm_100a).
//
// Tokens come in tiles of 128 rows and records in blocks of 64 (a block id b
// stands for records [64b, 64b + 64), the expansion of
// clustering/block_layout.py:61-64).  Tile t uses the blocks listed for it:
//   y[r] = sum over records n of the blocks of r's tile of silu(g_n . x_r) (u_n . x_r) d_n.
// The reference computes each tile with runtime/ffn.py:20-39 on the expanded
// ids (three gathers and three GEMMs per tile).
//
// A call runs groups of up to four tiles (512 tokens); a group is two launches:
//  plan     one CTA: per-block tile masks from the per-tile block lists; each
//           tile's ascending block list; the gate/up work units (a pair of
//           blocks against each tile that uses them, the units of one pair
//           adjacent) with the prefix of their costs; every CTA's stream-K
//           ranges.
//  prefill  one persistent CTA per SM (cooperative launch), two phases split by
//           a grid barrier:
//   1. gate/up: per unit (a tile and one or two of its blocks),
//      A[tok, 64b .. 64b+63] = silu(X G_b^T) * (X U_b^T): M = 128 tokens,
//      N = 128 per block (64 gate + 64 up records), K = hidden in chunks of 64.
//   2. down: per unit (tile t, 256 hidden outputs), y = A[tile, blocks] D[blocks, h]:
//      M = 128 tokens, N = 256, K = 64 records per block of the tile.
//  Both phases are balanced stream-K style: the cost-weighted sequence of
//  (unit, K step) iterations is cut into one contiguous range per CTA, so a
//  unit may be split between consecutive CTAs.  The CTA that runs a unit's
//  first K step finishes it: a CTA whose range starts inside a unit writes its
//  fp32 accumulators to its slot and raises a flag; the finishing CTA, which
//  reaches the unit at the end of its own range, adds them before the
//  activation (phase 1) or the output (phase 2).
//
// Operands move by tiled TMA (128-byte swizzle, no multicast) through a 4-stage
// shared-memory ring; two threads (in two warps) load the weight boxes and one
// the activation boxes (all three arrive on the stage's barrier), one thread issues the
// MMAs, four warps read TMEM (two 256-column accumulator buffers, so the
// epilogue of one unit overlaps the MMAs of the next).  Every wait is bounded (2 s) and reports
// QCC_DEV_TIMEOUT through the workspace status word.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <mutex>

#include "qcc_common.cuh"
#include "qcc_host.h"
#include "qcc_tc.cuh"

namespace qcc {

namespace {

constexpr int kTile = 128;                // tokens per tile (MMA M)
constexpr int kBlock = 64;                // records per block
constexpr int kRowBytes = 128;            // one 128-byte swizzled row: a gate/up K step (64 16-bit or 32 fp32 elements)
constexpr int kHRange = 256;              // hidden outputs per down unit (MMA N)
constexpr int kMaxTiles = 4;
constexpr int kMasks = (1 << kMaxTiles) - 1;  // non-empty tile masks of a block
constexpr int kGroupTokens = kTile * kMaxTiles;
constexpr int kStages = 4;
// warp 1: MMA, warps 2-5: TMEM readers, warps 0, 6 and 7: TMA producers.  A
// thread issuing tiled TMA copies back to back spends ~0.25 us per ring
// iteration plus ~0.1 us per box (measured: 6 boxes of 64 rows from L2 in
// 0.79 us), so each ring iteration is loaded in full by one producer and the
// three take turns: iteration i belongs to producer i % 3.
constexpr int kThreads = 256;
constexpr int kProducerWarp[3] = {0, 6, 7};
constexpr int kProducers = 3;
constexpr int kFirstReader = 2, kReaders = 4;  // warps 2-5 read TMEM (warp w: lanes 32*(w%4) .. +31)
constexpr int kPlanThreads = 1024;
constexpr uint32_t kBox64 = 64 * 128;     // [64 rows x 128 bytes]: 8 KB
constexpr uint32_t kBox128 = 128 * 128;   // [128 rows x 128 bytes]: 16 KB
constexpr uint32_t kStageBytes = 48 * 1024;
constexpr int kSmemList = 2048;           // down steps staged in shared memory
constexpr int kPlanUnits = 4096;          // gate/up units the plan kernel keeps in shared memory
constexpr int kPlanListBlocks = 4096;     // blocks up to which the plan keeps its pairing sequence in shared memory
constexpr int kMaxPlanGrid = 256;         // prefill CTAs the plan computes ranges for (one per SM)
constexpr uint32_t kControlBytes = 12 * 1024;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + kControlBytes + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = 256;        // one accumulator buffer
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kMaxBlocks = (1 << 15) - 1;  // block ids fit the 15-bit fields of a unit word (0x7FFF: none)
constexpr int kMaxDownUnits = 512;        // tiles x 256-wide hidden ranges (hidden <= 32768)
constexpr size_t kSlotFloats = 128 * 256; // one CTA's partial accumulators
constexpr int kMaxContrib = 16;           // CTAs that may hand partial sums to one unit's finishing CTA
constexpr int kPairCost = 3, kSingleCost = 4;  // stream-K cost of one gate/up chunk of a block pair / single block
constexpr int kSplitTarget = 8;           // ranges are at least 1/8 of the largest unit's cost

// Workspace header (int32 words).
constexpr int kHdrStatus = 0;
constexpr int kHdrUnits = 1;
constexpr int kHdrCost = 2;               // total gate/up cost
constexpr int kHdrEpoch = 3;              // incremented by every plan launch
constexpr int kHdrArrive = 4;             // grid-barrier counter, reset by every plan launch
constexpr int kHdrTileCount = 8;          // [kMaxTiles] blocks per tile
constexpr size_t kHeaderBytes = 256;

// Stream-K ranges of one CTA for both phases (index 0: gate/up, 1: down),
// [(lo_u, lo_k), (hi_u, hi_k)), and the CTAs that hand partial sums to the
// unit this CTA finishes last.  Written by the plan kernel.
struct alignas(16) Ranges {
  int lo_u[2], lo_k[2], hi_u[2], hi_k[2];
  int n_contrib[2];
  int contrib[2][kMaxContrib];
  int pad[2];
};
static_assert(sizeof(Ranges) % 16 == 0, "ranges record");

struct Control {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint64_t steps_ready;    // the down-step list below is filled
  uint32_t tmem_base;
  int abort;
  int epoch;
  Ranges r;
  int steps[kSmemList];    // (down unit << 16) | block of each of this CTA's down steps, in order
  int n_steps;             // down steps of this CTA (entries of `steps` valid: min(n_steps, kSmemList))
};
static_assert(sizeof(Control) <= kControlBytes, "control block");
static_assert(offsetof(Control, r) % 16 == 0, "the ranges record is copied with 16-byte accesses");
static_assert(kProducerWarp[1] >= kFirstReader + kReaders && kProducerWarp[2] > kProducerWarp[1] &&
                  kProducerWarp[2] * 32 < kThreads && kProducerWarp[0] == 0,
              "warp roles");

struct PrefillArgs {
  int32_t* header;
  const int32_t* units;
  const int32_t* unit_prefix;  // [n_units + 1] exclusive cost prefix
  const int32_t* tile_list;    // [kMaxTiles][n_blocks]
  const uint8_t* block_masks;  // [n_blocks] bit t: tile t uses the block
  const Ranges* ranges;        // [gridDim.x]
  int n_blocks;
  int n_chunks;                // gate/up K steps
  int n_hranges;               // down units per tile
  int hidden;
  int n_tokens;                // rows of this group
  int n_tiles;
  void* abuf;                  // activations: 16-bit, or fp32 for fp32 records
  int64_t ld_abuf;
  float* partials;             // [gridDim.x][kSlotFloats]
  int32_t* flags1;             // [gridDim.x]
  int32_t* flags2;             // [gridDim.x]
  void* y;
  int64_t ldy;
  int y_dtype;
  int y_vec;                   // 16-byte stores allowed
};

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  const uint32_t a = smem_addr(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// Bounded wait for one phase of `bar`.  Returns false when another role has
// aborted or when the limit passed (then it records the timeout).
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      *abort_flag = 1;
      atomicOr(status, QCC_DEV_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool warp_wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                int* status) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(bar, parity, abort_flag, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ int ld_acquire(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Lane 0 of the warp waits (bounded) until flags[list[i]] == epoch for every
// i < n; all lanes get the result.
__device__ __forceinline__ bool warp_wait_flags(const int32_t* flags, const int* list, int n, int epoch,
                                                volatile int* abort_flag, int* status) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t start = global_timer_ns();
    for (int i = 0; i < n && ok; ++i) {
      while (ld_acquire(flags + list[i]) != epoch) {
        if (*abort_flag || global_timer_ns() - start > kWaitLimitNs) {
          if (!*abort_flag) atomicOr(status, QCC_DEV_TIMEOUT);
          *abort_flag = 1;
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ void drain_loads(Control* ctl, uint32_t issued) {
  const uint32_t first = issued > static_cast<uint32_t>(kStages) ? issued - kStages : 0u;
  for (uint32_t i = first; i < issued; ++i) mbar_wait_bounded(&ctl->full[i % kStages], (i / kStages) & 1u, kWaitLimitNs);
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Named barrier of the four TMEM-reading warps.
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.f + __expf(-g)); }

// Per operand format (kFmtF16 / kFmtBF16 / kFmtTF32): element bytes, the
// elements of a 128-byte row (a gate/up K step, and the records of one down
// step), and the down rows' boxes per 256-wide hidden range.  fp32 records
// take the down phase in half blocks: a step of 32 records keeps the stage at
// 48 KB (16 KB of activations, 32 KB of down rows in eight [32 x 32] boxes).
template <int kFmt>
struct Fmt {
  static constexpr int kEs = kFmt == kFmtTF32 ? 4 : 2;
  static constexpr int kRow = kRowBytes / kEs;            // 64 or 32
  static constexpr int kStepsPerBlock = kBlock / kRow;    // down steps per block: 1 or 2
  static constexpr int kDownBoxes = kHRange / kRow;       // 4 or 8
  static constexpr uint32_t kDownBox = kRow * kRowBytes;  // bytes of one down box: 8 KB or 4 KB
  static constexpr int kMmaK = 32 / kEs;                  // elements per MMA K step (32 bytes)
};

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (kBf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Gate/up unit word: tile << 30 | second block << 15 | first block (second
// block 0x7FFF: none).  A unit is one 128-token tile against the gate and up
// rows of one or two of its blocks (MMA N = 128 per block).
constexpr int kNoBlock = 0x7FFF;
__device__ __forceinline__ int unit_tile(int unit) { return static_cast<int>(static_cast<uint32_t>(unit) >> 30); }
__device__ __forceinline__ int unit_block(int unit, int j) { return j == 0 ? unit & 0x7FFF : (unit >> 15) & 0x7FFF; }
__device__ __forceinline__ int unit_blocks(int unit) { return ((unit >> 15) & 0x7FFF) == kNoBlock ? 1 : 2; }

// ---------------------------------------------------------------------------
// Stream-K ranges.
// ---------------------------------------------------------------------------

// Phase 1: (unit, chunk) at cost position p.  A chunk of a block pair costs
// kPairCost, a chunk of a single block kSingleCost: per-CTA stamps measured
// 0.154 and 0.202 us per ring iteration (the ring is latency-bound, so a
// single block's iteration is not cheaper than a pair's).
__device__ void locate_gate_up(const int* units, const int* prefix, int n_units, int total, int64_t p, int* u,
                               int* k) {
  if (p >= total || n_units == 0) {
    *u = n_units;
    *k = 0;
    return;
  }
  int lo = 0, hi = n_units - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (prefix[mid] <= p)
      lo = mid;
    else
      hi = mid - 1;
  }
  *u = lo;
  *k = static_cast<int>((p - prefix[lo]) / (unit_blocks(units[lo]) == 2 ? kPairCost : kSingleCost));
}

// Phase 2: (unit, step) at position p; units without steps share their
// prefix with the next unit, and the search lands on the one with steps.
__device__ void locate_down(const int* prefix, int n_units, int64_t p, int* u, int* k) {
  const int total = prefix[n_units];
  if (p >= total || n_units == 0) {
    *u = n_units;
    *k = 0;
    return;
  }
  int lo = 0, hi = n_units - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (prefix[mid] <= p)
      lo = mid;
    else
      hi = mid - 1;
  }
  *u = lo;
  *k = static_cast<int>(p - prefix[lo]);
}

// Number of ranges actually used: at most the grid, and few enough that a
// range covers at least 1/kSplitTarget of the costliest unit (so no unit is
// shared by more than about kSplitTarget + 1 CTAs).
__device__ __forceinline__ int effective_ranges(int64_t total, int64_t unit_max, int grid) {
  if (total <= 0 || unit_max <= 0) return 1;
  int64_t cap = total * kSplitTarget / unit_max;
  if (cap > grid) cap = grid;
  return cap < 1 ? 1 : static_cast<int>(cap);
}

// Range of CTA i out of g and the CTAs with non-empty ranges that hand partial
// sums to its last unit.  Returns false if that needs more than kMaxContrib.
template <typename Bound>
__device__ bool range_of(int i, int g, Bound bound, Ranges* r, int ph) {
  r->n_contrib[ph] = 0;
  if (i >= g) {
    bound(g, &r->lo_u[ph], &r->lo_k[ph]);
    r->hi_u[ph] = r->lo_u[ph];
    r->hi_k[ph] = r->lo_k[ph];
    return true;
  }
  bound(i, &r->lo_u[ph], &r->lo_k[ph]);
  bound(i + 1, &r->hi_u[ph], &r->hi_k[ph]);
  const int hi_u = r->hi_u[ph], hi_k = r->hi_k[ph];
  if (hi_k == 0 || (hi_u == r->lo_u[ph] && r->lo_k[ph] > 0)) return true;  // last segment complete or not a head
  int u1 = hi_u, k1 = hi_k;  // start of range j
  for (int j = i + 1; j < g; ++j) {
    const int u = u1, k = k1;
    if (u != hi_u || k == 0) break;
    bound(j + 1, &u1, &k1);
    if (u1 == u && k1 == k) continue;  // empty range
    if (r->n_contrib[ph] == kMaxContrib) return false;
    r->contrib[ph][r->n_contrib[ph]++] = j;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Plan.  One CTA: per-block tile masks, each tile's ascending block list, the
// gate/up units (words as above) and their cost prefix, then the stream-K
// ranges of every CTA of the prefill grid.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kPlanThreads)
    prefill_plan_kernel(const int32_t* __restrict__ tile_blocks, const int32_t* __restrict__ tile_offsets,
                        int n_tiles, int n_blocks, int n_chunks, int n_hranges, int steps_per_block, int grid,
                        int32_t* __restrict__ header,
                        int32_t* __restrict__ units, int32_t* __restrict__ unit_prefix,
                        int32_t* __restrict__ tile_list, int32_t* __restrict__ seq_global,
                        uint32_t* __restrict__ block_masks, Ranges* __restrict__ ranges) {
  extern __shared__ __align__(16) uint32_t words[];  // one mask byte per block, the staged units / prefix, the pairs
  __shared__ int scratch[64];
  __shared__ int s_down[kMaxDownUnits + 1];
  __shared__ int s_tile_count[kMaxTiles];
  __shared__ int s_off[kMaxTiles + 1];
  __shared__ int s_fail;
  __shared__ int s_epoch;
  __shared__ int s_bu[2][kMaxPlanGrid + 1], s_bk[2][kMaxPlanGrid + 1];  // stream-K range boundaries
  __shared__ int s_group[kMasks + 1];  // start of each tile mask's group in the pairing sequence
  // The prefill launch that follows may be scheduled now; it waits for this
  // grid to complete before it reads anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x;
  const int n_words = (n_blocks + 3) / 4;
  const int cap = min(2 * n_blocks + 8, kPlanUnits);
  int* s_units = reinterpret_cast<int*>(words + n_words);
  int* s_prefix = s_units + cap;
  // The pairing sequence of the gate/up units (below): in shared memory up to
  // kPlanListBlocks blocks, else in the workspace.
  int* seq = n_blocks <= kPlanListBlocks ? s_prefix + cap + 1 : seq_global;
  for (int i = tid; i < n_words; i += blockDim.x) words[i] = 0u;
  if (tid == 0) {
    s_fail = 0;
    s_epoch = header[kHdrEpoch];  // read now, not in the serial section below
  }
  if (tid <= n_tiles) s_off[tid] = __ldg(tile_offsets + tid);
  __syncthreads();
  bool bad = false, sorted_offsets = true;
  for (int t = 0; t < n_tiles; ++t)
    if (s_off[t] < 0 || s_off[t + 1] < s_off[t]) sorted_offsets = false;
  if (sorted_offsets) {
    // Every tile's block ids in one pass (all loads in flight at once).
    for (int j = s_off[0] + tid; j < s_off[n_tiles]; j += blockDim.x) {
      int t = 0;
      while (t + 1 < n_tiles && j >= s_off[t + 1]) ++t;
      const int b = __ldg(tile_blocks + j);
      if (b >= 0 && b < n_blocks)
        atomicOr(&words[b >> 2], (1u << t) << (8 * (b & 3)));
      else
        bad = true;
    }
  } else {
    for (int t = 0; t < n_tiles; ++t) {
      const int begin = s_off[t], end = s_off[t + 1];
      if (begin < 0 || end < begin) {
        bad = true;
        continue;
      }
      for (int j = begin + tid; j < end; j += blockDim.x) {
        const int b = __ldg(tile_blocks + j);
        if (b >= 0 && b < n_blocks)
          atomicOr(&words[b >> 2], (1u << t) << (8 * (b & 3)));
        else
          bad = true;
      }
    }
  }
  if (bad) atomicOr(header + kHdrStatus, QCC_DEV_ID_RANGE);
  __syncthreads();
  for (int i = tid; i < n_words; i += blockDim.x) block_masks[i] = words[i];
  const uint8_t* mask = reinterpret_cast<const uint8_t*>(words);
  const int chunk = (n_blocks + blockDim.x - 1) / blockDim.x;
  const int lo = min(n_blocks, tid * chunk);
  const int hi = min(n_blocks, lo + chunk);
  // Each tile's blocks in ascending order: the four tiles' counts go through
  // two scans, two tiles per 32-bit word (a count fits 16 bits: n_blocks <=
  // kMaxBlocks < 2^15).
  static_assert(kMaxTiles == 4 && kMaxBlocks <= 65535, "packed tile counts");
  int c01 = 0, c23 = 0;
  for (int i = lo; i < hi; ++i) {
    const int m = mask[i];
    c01 += (m & 1) | (((m >> 1) & 1) << 16);
    c23 += ((m >> 2) & 1) | (((m >> 3) & 1) << 16);
  }
  int tot01, tot23;
  const int p01 = block_exclusive_scan(c01, scratch, &tot01);
  const int p23 = block_exclusive_scan(c23, scratch, &tot23);
  int pos_t[kMaxTiles] = {p01 & 0xFFFF, p01 >> 16, p23 & 0xFFFF, p23 >> 16};
  for (int i = lo; i < hi; ++i) {
    const int m = mask[i];
#pragma unroll
    for (int t = 0; t < kMaxTiles; ++t)
      if (t < n_tiles && ((m >> t) & 1)) {
        tile_list[t * n_blocks + pos_t[t]] = i;
        ++pos_t[t];
      }
  }
  if (tid == 0) {
    const int tots[kMaxTiles] = {tot01 & 0xFFFF, tot01 >> 16, tot23 & 0xFFFF, tot23 >> 16};
    for (int t = 0; t < kMaxTiles; ++t) s_tile_count[t] = t < n_tiles ? tots[t] : 0;
  }
  __syncthreads();  // tile lists and counts visible to the block
  // Gate/up units.  The blocks that any tile uses are put in one sequence,
  // grouped by their tile mask (the groups in Gray-code order of the mask, so
  // that neighbouring groups differ in one tile; ascending ids inside a
  // group), and consecutive blocks of the sequence form the pairs.  A pair
  // makes one unit for each tile that uses either of its blocks, and those
  // units are adjacent: the tiles sharing a block run it on neighbouring CTAs a
  // few K steps apart, so all but the first read its rows from L2.  (Pairing
  // each tile's own blocks instead re-read shared blocks from DRAM: 329 MB of
  // gate/up reads against 212 MB unique on a 512-token call.)  A tile that
  // uses only one block of a pair -- only at a group boundary -- computes the
  // other block's activations too, which nothing reads.  An odd block left
  // over makes single-block units at the end.  Warp w counts and then places
  // the blocks of mask gray(w + 1).
  {
    const int warp = tid >> 5, lane = tid & 31;
    static_assert(kPlanThreads / 32 >= kMasks, "one warp per tile mask");
    const int mv = (warp + 1) ^ ((warp + 1) >> 1);
    if (warp < kMasks) {
      int cnt = 0;
      for (int b0 = 0; b0 < n_blocks; b0 += 32) {
        const int b = b0 + lane;
        cnt += __popc(__ballot_sync(0xffffffffu, b < n_blocks && mask[b] == mv));
      }
      if (lane == 0) s_group[warp] = cnt;
    }
    __syncthreads();
    if (tid == 0) {
      int o = 0;
      for (int g = 0; g < kMasks; ++g) {
        const int c = s_group[g];
        s_group[g] = o;
        o += c;
      }
      s_group[kMasks] = o;
    }
    __syncthreads();
    if (warp < kMasks) {
      int pos = s_group[warp];
      for (int b0 = 0; b0 < n_blocks; b0 += 32) {
        const int b = b0 + lane;
        const bool hit = b < n_blocks && mask[b] == mv;
        const uint32_t bal = __ballot_sync(0xffffffffu, hit);
        if (hit) seq[pos + __popc(bal & ((1u << lane) - 1u))] = b;
        pos += __popc(bal);
      }
    }
    __syncthreads();
  }
  const int n_union = s_group[kMasks];
  const int n_pairs = n_union / 2;
  const int single_mask = (n_union & 1) ? mask[seq[n_union - 1]] : 0;
  const int pchunk = (n_pairs + blockDim.x - 1) / blockDim.x;
  const int p_lo = min(n_pairs, tid * pchunk);
  const int p_hi = min(n_pairs, p_lo + pchunk);
  int mine = 0;
  for (int q = p_lo; q < p_hi; ++q) mine += __popc(mask[seq[2 * q]] | mask[seq[2 * q + 1]]);
  int pair_units;
  int pos = block_exclusive_scan(mine, scratch, &pair_units);
  // Cost prefix: kPairCost per chunk for a pair unit, kSingleCost for a single.
  for (int q = p_lo; q < p_hi; ++q) {
    const int b1 = seq[2 * q], b2 = seq[2 * q + 1];
    const int tm = mask[b1] | mask[b2];
#pragma unroll
    for (int t = 0; t < kMaxTiles; ++t) {
      if (!((tm >> t) & 1)) continue;
      const int word = static_cast<int>((static_cast<uint32_t>(t) << 30) | (static_cast<uint32_t>(b2) << 15) |
                                        static_cast<uint32_t>(b1));
      const int run = kPairCost * pos * n_chunks;
      units[pos] = word;
      unit_prefix[pos] = run;
      if (pos < cap) {
        s_units[pos] = word;
        s_prefix[pos] = run;
      }
      ++pos;
    }
  }
  const int total_units = pair_units + __popc(single_mask);
  const int total1 = (kPairCost * pair_units + kSingleCost * (total_units - pair_units)) * n_chunks;
  if (tid == 0) {
    int q = pair_units;
    for (int t = 0; t < kMaxTiles; ++t) {
      if (!((single_mask >> t) & 1)) continue;
      const int word = static_cast<int>((static_cast<uint32_t>(t) << 30) |
                                        (static_cast<uint32_t>(kNoBlock) << 15) |
                                        static_cast<uint32_t>(seq[n_union - 1]));
      const int run = (kPairCost * pair_units + kSingleCost * (q - pair_units)) * n_chunks;
      units[q] = word;
      unit_prefix[q] = run;
      if (q < cap) {
        s_units[q] = word;
        s_prefix[q] = run;
      }
      ++q;
    }
    for (int t = 0; t < kMaxTiles; ++t) header[kHdrTileCount + t] = t < n_tiles ? s_tile_count[t] : 0;
    header[kHdrUnits] = total_units;
    header[kHdrCost] = total1;
    unit_prefix[total_units] = total1;
    if (total_units < cap) s_prefix[total_units] = total1;
    header[kHdrEpoch] = s_epoch + 1;
    header[kHdrArrive] = 0;
  }
  // Down units: v = range * n_tiles + tile, steps = blocks of the tile; their
  // step prefix in closed form, one thread per unit.
  for (int v = tid; v <= n_hranges * n_tiles; v += blockDim.x) {
    const int part = v % n_tiles;
    int tot = 0, pre = 0;
    for (int t = 0; t < n_tiles; ++t) {
      tot += s_tile_count[t];
      if (t < part) pre += s_tile_count[t];
    }
    s_down[v] = ((v / n_tiles) * tot + pre) * steps_per_block;
  }
  __syncthreads();
  // Ranges of every CTA of the prefill grid.
  const bool staged = total_units < cap;
  const int* u_arr = staged ? s_units : units;
  const int* p_arr = staged ? s_prefix : unit_prefix;
  const int g1 = effective_ranges(total1, static_cast<int64_t>(max(kPairCost, kSingleCost)) * n_chunks, grid);
  const int n_down = n_hranges * n_tiles;
  const int total2 = s_down[n_down];
  int max_steps = 0;
  for (int t = 0; t < n_tiles; ++t) max_steps = max(max_steps, s_tile_count[t] * steps_per_block);
  const int g2 = effective_ranges(total2, max_steps, grid);
  // Every range boundary once, in parallel (phase 1 on threads 0..g1, phase 2
  // on threads kPlanThreads/2..): the per-CTA pass below only reads them.
  if (tid <= g1) {
    int u, k;
    locate_gate_up(u_arr, p_arr, total_units, total1, static_cast<int64_t>(tid) * total1 / g1, &u, &k);
    s_bu[0][tid] = u;
    s_bk[0][tid] = k;
  }
  if (tid >= kPlanThreads / 2 && tid - kPlanThreads / 2 <= g2) {
    const int j = tid - kPlanThreads / 2;
    int u, k;
    locate_down(s_down, n_down, static_cast<int64_t>(j) * total2 / g2, &u, &k);
    s_bu[1][j] = u;
    s_bk[1][j] = k;
  }
  __syncthreads();
  for (int i = tid; i < grid; i += blockDim.x) {
    Ranges r;
    auto bound1 = [&](int j, int* u, int* k) {
      *u = s_bu[0][j];
      *k = s_bk[0][j];
    };
    auto bound2 = [&](int j, int* u, int* k) {
      *u = s_bu[1][j];
      *k = s_bk[1][j];
    };
    const bool ok = range_of(i, g1, bound1, &r, 0) & range_of(i, g2, bound2, &r, 1);
    if (!ok) s_fail = 1;
    r.pad[0] = r.pad[1] = 0;
    ranges[i] = r;
  }
  __syncthreads();
  if (tid == 0 && s_fail) atomicOr(header + kHdrStatus, QCC_DEV_TIMEOUT);
}

// idx-th unit of a CTA's range in processing order, or -1 past the end: a
// first segment that continues another CTA's unit goes first (it hands over
// partial sums), then the units in between, then an unfinished last segment
// (this CTA completes that unit with the partial sums of the CTAs running its
// later steps, which those CTAs produce first, so they are in by then).
// Taking the last segment second instead left its epilogue waiting on the
// partials for the whole of the middle units, and those ran ~40 % slower
// per step meanwhile.
__device__ __forceinline__ int seg_unit(const Ranges& r, int ph, int idx, int n_units) {
  const int lo_u = r.lo_u[ph], lo_k = r.lo_k[ph], hi_u = r.hi_u[ph], hi_k = r.hi_k[ph];
  const bool c = lo_k > 0 && lo_u < n_units;
  const bool h = hi_k > 0 && !(hi_u == lo_u && lo_k > 0) && hi_u < n_units;
  if (c) {
    if (idx == 0) return lo_u;
    --idx;
  }
  const int mid_lo = c ? lo_u + 1 : lo_u;
  const int mid_hi = min(h ? hi_u : hi_u + 1, n_units);
  if (idx < mid_hi - mid_lo) return mid_lo + idx;
  idx -= max(mid_hi - mid_lo, 0);
  return h && idx == 0 ? hi_u : -1;
}

// Segment [ks, ke) of unit u inside [lo, hi); returns false if empty.
__device__ __forceinline__ bool segment(int u, int lo_u, int lo_k, int hi_u, int hi_k, int steps, int* ks, int* ke) {
  *ks = u == lo_u ? lo_k : 0;
  *ke = u == hi_u ? hi_k : steps;
  return *ks < *ke;
}

// ---------------------------------------------------------------------------
// The prefill kernel.
// ---------------------------------------------------------------------------

template <int kFmt>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_records, const __grid_constant__ CUtensorMap tm_down,
                   const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_abuf,
                   const PrefillArgs a) {
  using F = Fmt<kFmt>;
  constexpr bool kBf16 = kFmt == kFmtBF16;
  // Launched as a programmatic dependent of the plan kernel: the grid may be
  // scheduled while the plan runs, and waits here for it to complete.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  Control* ctl = reinterpret_cast<Control*>(smem + kStages * kStageBytes);
  volatile int* abort_flag = &ctl->abort;
  int* status = a.header + kHdrStatus;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->full[s], 1);  // the iteration's producer arrives with its bytes
      mbar_init(&ctl->empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&ctl->acc_full[j], 1);
      mbar_init(&ctl->acc_empty[j], 4);  // one arrival per TMEM-reading warp
    }
    mbar_init(&ctl->drain, 1);
    mbar_init(&ctl->steps_ready, 1);
    ctl->abort = 0;
    ctl->epoch = a.header[kHdrEpoch];
    fence_barrier_init();
  }
  {
    // This CTA's ranges, computed by the plan kernel.
    const int4* src = reinterpret_cast<const int4*>(a.ranges + blockIdx.x);
    int4* dst = reinterpret_cast<int4*>(&ctl->r);
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(Ranges) / 16); i += blockDim.x) dst[i] = src[i];
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = ctl->tmem_base;
  const int epoch = ctl->epoch;
  const int n_units = a.header[kHdrUnits];
  const int n_down = a.n_hranges * a.n_tiles;
  if (warp == kFirstReader) {
    // This CTA's down steps in order, staged for the TMA thread.
    int n = 0;
    for (int si = 0, v; (v = seg_unit(ctl->r, 1, si, n_down)) >= 0; ++si) {
      const int t = v % a.n_tiles;
      int ks, ke;
      if (!segment(v, ctl->r.lo_u[1], ctl->r.lo_k[1], ctl->r.hi_u[1], ctl->r.hi_k[1], a.header[kHdrTileCount + t] * F::kStepsPerBlock, &ks, &ke))
        continue;
      for (int j = ks + lane; j < ke; j += 32)
        if (n + (j - ks) < kSmemList)
          ctl->steps[n + (j - ks)] = (v << 16) | a.tile_list[t * a.n_blocks + j / F::kStepsPerBlock];
      n += ke - ks;
    }
    __syncwarp();
    if (lane == 0) {
      ctl->n_steps = n;
      mbar_arrive(&ctl->steps_ready);
    }
  }

  // Per-role pipeline state, carried from phase 1 into phase 2.
  uint32_t it = 0;  // producer / MMA: ring iterations
  uint32_t ut = 0;  // MMA / TMEM readers: accumulator buffers used

  // ------------------------------ phase 1 ------------------------------
  const int producer = warp == kProducerWarp[0] ? 0 : warp == kProducerWarp[1] ? 1 : warp == kProducerWarp[2] ? 2 : -1;
  if (producer >= 0 && lane == 0) {
    // x box of the unit's tile (A) and the gate and up rows of its one or two
    // blocks (B).  Rows of a block that several tiles use stay in L2 for the
    // other tiles' units (which run on neighbouring CTAs); rows of a block
    // that one tile uses are read once.
    if (producer == 0) {
      tma_prefetch_map(&tm_records);
      tma_prefetch_map(&tm_down);
      tma_prefetch_map(&tm_x);
      tma_prefetch_map(&tm_abuf);
    }
    const uint64_t keep = policy_evict_last(), stream = policy_evict_first();
    for (int si = 0, u; (u = seg_unit(ctl->r, 0, si, n_units)) >= 0 && !*abort_flag; ++si) {
      int ks, ke;
      if (!segment(u, ctl->r.lo_u[0], ctl->r.lo_k[0], ctl->r.hi_u[0], ctl->r.hi_k[0], a.n_chunks, &ks, &ke)) continue;
      const int unit = a.units[u];
      const int t = unit_tile(unit);
      const int nb = unit_blocks(unit);
      const int b1 = unit_block(unit, 0), b2 = nb == 2 ? unit_block(unit, 1) : b1;
      const uint64_t pol1 = __popc(a.block_masks[b1]) > 1 ? keep : stream;
      const uint64_t pol2 = __popc(a.block_masks[b2]) > 1 ? keep : stream;
      for (int kc = ks; kc < ke; ++kc, ++it) {
        if (static_cast<int>(it % kProducers) != producer) continue;
        const int s = it % kStages;
        if (!wait_phase(&ctl->empty[s], ((it / kStages) & 1u) ^ 1u, abort_flag, status)) break;
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&ctl->full[s], (1 + nb) * kBox128);
        tma_load_2d_hint(st, &tm_x, kc * F::kRow, t * kTile, &ctl->full[s], keep);
        tma_load_3d_hint(st + kBox128, &tm_records, kc * F::kRow, 0, b1 * kBlock, &ctl->full[s], pol1);
        tma_load_3d_hint(st + kBox128 + kBox64, &tm_records, kc * F::kRow, 1, b1 * kBlock, &ctl->full[s], pol1);
        if (nb == 2) {
          tma_load_3d_hint(st + 2 * kBox128, &tm_records, kc * F::kRow, 0, b2 * kBlock, &ctl->full[s], pol2);
          tma_load_3d_hint(st + 2 * kBox128 + kBox64, &tm_records, kc * F::kRow, 1, b2 * kBlock, &ctl->full[s], pol2);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // One MMA per 32-byte K step: M = 128 tokens, N = 128 per block (256 for a
    // block pair).
    constexpr uint32_t idesc1 = idesc_f32acc(128, 128, kFmt, false, false);
    constexpr uint32_t idesc2 = idesc_f32acc(128, 256, kFmt, false, false);
    for (int si = 0, u; (u = seg_unit(ctl->r, 0, si, n_units)) >= 0 && !*abort_flag; ++si) {
      int ks, ke;
      if (!segment(u, ctl->r.lo_u[0], ctl->r.lo_k[0], ctl->r.hi_u[0], ctl->r.hi_k[0], a.n_chunks, &ks, &ke)) continue;
      const uint32_t idesc = unit_blocks(a.units[u]) == 2 ? idesc2 : idesc1;
      const uint32_t j = ut & 1u;
      if (!wait_phase(&ctl->acc_empty[j], ((ut >> 1) & 1u) ^ 1u, abort_flag, status)) break;
      tc_fence_after_sync();
      const uint32_t d0 = tmem + j * kAccCols;
      bool ok = true;
      for (int kc = ks; kc < ke; ++kc, ++it) {
        const int s = it % kStages;
        if (!wait_phase(&ctl->full[s], (it / kStages) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t st = smem_addr(smem + s * kStageBytes);
        const uint64_t a_desc = smem_desc_sw128(st, 16, 1024);            // x tile, K-major
        const uint64_t b_desc = smem_desc_sw128(st + kBox128, 16, 1024);  // gate/up rows, K-major
#pragma unroll
        for (int kk = 0; kk < kRowBytes / 32; ++kk) {
          if constexpr (kFmt == kFmtTF32)
            tc_mma_tf32(d0, a_desc + 2u * kk, b_desc + 2u * kk, idesc, (kc > ks || kk > 0) ? 1u : 0u);
          else
            tc_mma_f16(d0, a_desc + 2u * kk, b_desc + 2u * kk, idesc, (kc > ks || kk > 0) ? 1u : 0u);
        }
        tc_commit(&ctl->empty[s]);
      }
      if (!ok) break;
      tc_commit(&ctl->acc_full[j]);
      ++ut;
    }
  } else if (warp >= kFirstReader && warp < kFirstReader + kReaders) {
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 = token rows of the tile
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    for (int si = 0, u; (u = seg_unit(ctl->r, 0, si, n_units)) >= 0; ++si) {
      int ks, ke;
      if (!segment(u, ctl->r.lo_u[0], ctl->r.lo_k[0], ctl->r.hi_u[0], ctl->r.hi_k[0], a.n_chunks, &ks, &ke)) continue;
      const int unit = a.units[u];
      const int t = unit_tile(unit);
      const int nt = unit_blocks(unit);  // accumulator column groups of 128: one per block
      const uint32_t j = ut & 1u;
      if (!warp_wait_phase(&ctl->acc_full[j], (ut >> 1) & 1u, abort_flag, status)) break;
      tc_fence_after_sync();
      const uint32_t col0 = lane_base + j * kAccCols;
      if (ks > 0) {
        // Not this unit's first K steps: hand the accumulators to the CTA that finishes it.
        // Column-quad-major slot (float4 of columns 4m..4m+3 at m * 128 + row):
        // the 32 rows of a warp store 512 contiguous bytes per instruction.
        float4* slot = reinterpret_cast<float4*>(a.partials + static_cast<size_t>(blockIdx.x) * kSlotFloats);
        for (int i = 0; i < nt; ++i) {
          float4* dst = slot + static_cast<size_t>(i) * 32 * 128 + row;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_load32(col0 + i * 128u + c * 32u, v);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              __stcg(dst + (c * 8 + e) * 128, make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]));
          }
        }
        __threadfence();
        epilogue_sync();
        if (threadIdx.x == 64) atomicExch(a.flags1 + blockIdx.x, epoch);
      } else {
        const bool wait_others = ke < a.n_chunks;
        if (wait_others)
          warp_wait_flags(a.flags1, ctl->r.contrib[0], ctl->r.n_contrib[0], epoch, abort_flag, status);
        for (int i = 0; i < nt; ++i) {
          const int b = unit_block(unit, i);
          const int64_t dst_off = static_cast<int64_t>(t * kTile + row) * a.ld_abuf + static_cast<int64_t>(b) * kBlock;
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float g[32], v[32];
            // One contributor (the usual case): its partials are requested
            // before the TMEM loads, so the two latencies overlap.
            const bool one = wait_others && ctl->r.n_contrib[0] == 1;
            float4 pg[8], pu[8];
            if (one) {
              const float4* p =
                  reinterpret_cast<const float4*>(a.partials + static_cast<size_t>(ctl->r.contrib[0][0]) * kSlotFloats) +
                  static_cast<size_t>(i) * 32 * 128 + row;
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                pg[e] = __ldcg(p + (c * 8 + e) * 128);
                pu[e] = __ldcg(p + (16 + c * 8 + e) * 128);
              }
            }
            tmem_load32(col0 + i * 128u + c * 32u, g);
            tmem_load32(col0 + i * 128u + 64u + c * 32u, v);
            if (one) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                g[4 * e] += pg[e].x, g[4 * e + 1] += pg[e].y, g[4 * e + 2] += pg[e].z, g[4 * e + 3] += pg[e].w;
                v[4 * e] += pu[e].x, v[4 * e + 1] += pu[e].y, v[4 * e + 2] += pu[e].z, v[4 * e + 3] += pu[e].w;
              }
            } else if (wait_others) {
              for (int ci = 0; ci < ctl->r.n_contrib[0]; ++ci) {
                const float4* p = reinterpret_cast<const float4*>(
                                      a.partials + static_cast<size_t>(ctl->r.contrib[0][ci]) * kSlotFloats) +
                                  static_cast<size_t>(i) * 32 * 128 + row;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float4 pg = __ldcg(p + (c * 8 + e) * 128);
                  const float4 pu = __ldcg(p + (16 + c * 8 + e) * 128);
                  g[4 * e] += pg.x, g[4 * e + 1] += pg.y, g[4 * e + 2] += pg.z, g[4 * e + 3] += pg.w;
                  v[4 * e] += pu.x, v[4 * e + 1] += pu.y, v[4 * e + 2] += pu.z, v[4 * e + 3] += pu.w;
                }
              }
            }
            if constexpr (kFmt == kFmtTF32) {
              float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(a.abuf) + dst_off + c * 32);
#pragma unroll
              for (int e = 0; e < 8; ++e)
                d4[e] = make_float4(silu(g[4 * e]) * v[4 * e], silu(g[4 * e + 1]) * v[4 * e + 1],
                                    silu(g[4 * e + 2]) * v[4 * e + 2], silu(g[4 * e + 3]) * v[4 * e + 3]);
            } else {
              uint32_t w[16];
#pragma unroll
              for (int e = 0; e < 16; ++e)
                w[e] = pack2<kBf16>(silu(g[2 * e]) * v[2 * e], silu(g[2 * e + 1]) * v[2 * e + 1]);
              uint4* d4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.abuf) + dst_off + c * 32);
#pragma unroll
              for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
            }
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->acc_empty[j]);
      ++ut;
    }
    // Activations written with generic stores are read by TMA in phase 2.
    fence_proxy_async_global();
  }

  // --------------------------- grid barrier ----------------------------
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.header + kHdrArrive, 1);
    const uint64_t start = global_timer_ns();
    while (ld_acquire(a.header + kHdrArrive) < static_cast<int>(gridDim.x)) {
      if (global_timer_ns() - start > kWaitLimitNs) {
        ctl->abort = 1;
        atomicOr(status, QCC_DEV_TIMEOUT);
        break;
      }
    }
    fence_proxy_async_global();
  }
  __syncthreads();

  // ------------------------------ phase 2 ------------------------------
  const int staged = min(ctl->n_steps, kSmemList);
  if (producer >= 0 && lane == 0) {
    // The tile's activations of the step's records (A) and their down rows
    // for the unit's 256 hidden outputs (B).  Down rows of a block that
    // several tiles use are read by each of their units of the same hidden
    // range: kept in L2, as in phase 1.
    const uint64_t keep = policy_evict_last(), stream = policy_evict_first();
    int si = 0;  // position in this CTA's step sequence
    for (int sv = 0, v; (v = seg_unit(ctl->r, 1, sv, n_down)) >= 0 && !*abort_flag; ++sv) {
      const int t = v % a.n_tiles, r = v / a.n_tiles;
      int ks, ke;
      if (!segment(v, ctl->r.lo_u[1], ctl->r.lo_k[1], ctl->r.hi_u[1], ctl->r.hi_k[1],
                   a.header[kHdrTileCount + t] * F::kStepsPerBlock, &ks, &ke))
        continue;
      for (int step = ks; step < ke; ++step, ++it, ++si) {
        if (static_cast<int>(it % kProducers) != producer) continue;
        const int b = si < staged ? (ctl->steps[si] & 0xFFFF) : a.tile_list[t * a.n_blocks + step / F::kStepsPerBlock];
        const int r0 = b * kBlock + (step % F::kStepsPerBlock) * F::kRow;  // first record of the step
        const int s = it % kStages;
        if (!wait_phase(&ctl->empty[s], ((it / kStages) & 1u) ^ 1u, abort_flag, status)) break;
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&ctl->full[s], kBox128 + F::kDownBoxes * F::kDownBox);
        tma_load_2d_hint(st, &tm_abuf, r0, t * kTile, &ctl->full[s], keep);
        const uint64_t pol = __popc(a.block_masks[b]) > 1 ? keep : stream;
        for (int qq = 0; qq < F::kDownBoxes; ++qq)
          tma_load_3d_hint(st + kBox128 + qq * F::kDownBox, &tm_down, r * kHRange + qq * F::kRow, 2, r0, &ctl->full[s],
                           pol);
      }
    }
    // Every copy of the last iterations has landed before the CTA exits.
    if (producer == 0) drain_loads(ctl, it);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_f32acc(128, 256, kFmt, false, true);
    for (int sv = 0, v; (v = seg_unit(ctl->r, 1, sv, n_down)) >= 0 && !*abort_flag; ++sv) {
      const int t = v % a.n_tiles;
      int ks, ke;
      if (!segment(v, ctl->r.lo_u[1], ctl->r.lo_k[1], ctl->r.hi_u[1], ctl->r.hi_k[1], a.header[kHdrTileCount + t] * F::kStepsPerBlock, &ks, &ke))
        continue;
      const uint32_t j = ut & 1u;
      if (!wait_phase(&ctl->acc_empty[j], ((ut >> 1) & 1u) ^ 1u, abort_flag, status)) break;
      tc_fence_after_sync();
      const uint32_t d0 = tmem + j * kAccCols;
      bool ok = true;
      for (int step = ks; step < ke; ++step, ++it) {
        const int s = it % kStages;
        if (!wait_phase(&ctl->full[s], (it / kStages) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t st = smem_addr(smem + s * kStageBytes);
        const uint64_t a_desc = smem_desc_sw128(st, 16, 1024);          // activations, K-major
        // Down rows, hidden-major (MN-major B): fp32 rows take the 32-byte-atom swizzle.
        const uint64_t b_desc = kFmt == kFmtTF32 ? smem_desc_sw128_atom32(st + kBox128, F::kDownBox, 512)
                                                 : smem_desc_sw128(st + kBox128, F::kDownBox, 1024);
        constexpr uint32_t kBStep = F::kMmaK * kRowBytes / 16;  // K rows of one MMA, in descriptor units
#pragma unroll
        for (int kk = 0; kk < kRowBytes / 32; ++kk) {
          if constexpr (kFmt == kFmtTF32)
            tc_mma_tf32(d0, a_desc + 2u * kk, b_desc + kBStep * kk, idesc, (step > ks || kk > 0) ? 1u : 0u);
          else
            tc_mma_f16(d0, a_desc + 2u * kk, b_desc + kBStep * kk, idesc, (step > ks || kk > 0) ? 1u : 0u);
        }
        tc_commit(&ctl->empty[s]);
      }
      if (!ok) break;
      tc_commit(&ctl->acc_full[j]);
      ++ut;
    }
  } else if (warp >= kFirstReader && warp < kFirstReader + kReaders) {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const size_t y_es = a.y_dtype == QCC_DTYPE_F32 ? 4 : 2;
    for (int sv = 0, v; (v = seg_unit(ctl->r, 1, sv, n_down)) >= 0; ++sv) {
      const int t = v % a.n_tiles, r = v / a.n_tiles;
      int ks, ke;
      const int steps = a.header[kHdrTileCount + t] * F::kStepsPerBlock;
      if (!segment(v, ctl->r.lo_u[1], ctl->r.lo_k[1], ctl->r.hi_u[1], ctl->r.hi_k[1], steps, &ks, &ke)) continue;
      const uint32_t j = ut & 1u;
      if (!warp_wait_phase(&ctl->acc_full[j], (ut >> 1) & 1u, abort_flag, status)) break;
      tc_fence_after_sync();
      const uint32_t col0 = lane_base + j * kAccCols;
      if (ks > 0) {
        // Column-quad-major slot, as in phase 1.
        float4* dst = reinterpret_cast<float4*>(a.partials + static_cast<size_t>(blockIdx.x) * kSlotFloats) + row;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          float vv[32];
          tmem_load32(col0 + c * 32u, vv);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            __stcg(dst + (c * 8 + e) * 128, make_float4(vv[4 * e], vv[4 * e + 1], vv[4 * e + 2], vv[4 * e + 3]));
        }
        __threadfence();
        epilogue_sync();
        if (threadIdx.x == 64) atomicExch(a.flags2 + blockIdx.x, epoch);
      } else {
        const bool wait_others = ke < steps;
        if (wait_others)
          warp_wait_flags(a.flags2, ctl->r.contrib[1], ctl->r.n_contrib[1], epoch, abort_flag, status);
        const int tok = t * kTile + row;
        const bool row_ok = tok < a.n_tokens;
        uint8_t* yrow = static_cast<uint8_t*>(a.y) + static_cast<size_t>(tok) * a.ldy * y_es;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          float vv[32];
          tmem_load32(col0 + c * 32u, vv);
          if (wait_others) {
            for (int ci = 0; ci < ctl->r.n_contrib[1]; ++ci) {
              const float4* p =
                  reinterpret_cast<const float4*>(a.partials + static_cast<size_t>(ctl->r.contrib[1][ci]) * kSlotFloats) + row;
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float4 pv = __ldcg(p + (c * 8 + e) * 128);
                vv[4 * e] += pv.x, vv[4 * e + 1] += pv.y, vv[4 * e + 2] += pv.z, vv[4 * e + 3] += pv.w;
              }
            }
          }
          const int h0 = r * kHRange + c * 32;
          if (!row_ok || h0 >= a.hidden) continue;
          if (a.y_vec && h0 + 32 <= a.hidden) {
            if (a.y_dtype == QCC_DTYPE_F32) {
              float4* d4 = reinterpret_cast<float4*>(yrow + static_cast<size_t>(h0) * 4);
#pragma unroll
              for (int e = 0; e < 8; ++e) d4[e] = make_float4(vv[4 * e], vv[4 * e + 1], vv[4 * e + 2], vv[4 * e + 3]);
            } else {
              uint32_t w[16];
#pragma unroll
              for (int e = 0; e < 16; ++e)
                w[e] = a.y_dtype == QCC_DTYPE_BF16 ? pack2<true>(vv[2 * e], vv[2 * e + 1])
                                                   : pack2<false>(vv[2 * e], vv[2 * e + 1]);
              uint4* d4 = reinterpret_cast<uint4*>(yrow + static_cast<size_t>(h0) * 2);
#pragma unroll
              for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (h0 + e < a.hidden) store_as(a.y, static_cast<int64_t>(tok) * a.ldy + h0 + e, a.y_dtype, vv[e]);
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->acc_empty[j]);
      ++ut;
    }
    // Tiles without blocks: their rows are zero.  Spread over the grid by (tile, range).
    for (int v = blockIdx.x; v < n_down; v += gridDim.x) {
      const int t = v % a.n_tiles, r = v / a.n_tiles;
      if (a.header[kHdrTileCount + t] * F::kStepsPerBlock != 0) continue;
      const int tok = t * kTile + row;
      if (tok >= a.n_tokens) continue;
      for (int h = r * kHRange; h < min(a.hidden, (r + 1) * kHRange); ++h)
        store_as(a.y, static_cast<int64_t>(tok) * a.ldy + h, a.y_dtype, 0.f);
    }
  }

  // ------------------------------ teardown -----------------------------
  if (warp == 1 && lane == 0) {
    tc_commit(&ctl->drain);
    mbar_wait_bounded(&ctl->drain, 0, kWaitLimitNs);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// Tensor map (bf16, fp16 or fp32) with the 128-byte swizzle; dims / strides innermost first.
bool make_map(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims, const uint64_t* strides,
              const uint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_tiled();
  if (fn == nullptr) return false;
  const uint32_t elem[3] = {1, 1, 1};
  const CUtensorMapDataType type = dtype == QCC_DTYPE_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : dtype == QCC_DTYPE_F16  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUresult r = fn(map, type,
                        rank, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct PrefillLayout {
  int n_blocks = 0, grid = 0;
  int64_t npad = 0;
  size_t units = 0, prefix = 0, tile_list = 0, seq = 0, masks = 0, ranges = 0, flags1 = 0, flags2 = 0, abuf = 0, partials = 0,
         total = 0;
};

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

PrefillLayout prefill_layout(int64_t n_records, int num_sms) {
  PrefillLayout l;
  l.n_blocks = static_cast<int>((n_records + kBlock - 1) / kBlock);
  l.grid = num_sms;
  l.npad = static_cast<int64_t>(l.n_blocks) * kBlock;
  size_t off = kHeaderBytes;
  l.units = off;  // at most one unit per tile for every pair of blocks, rounded up: 2 * n_blocks + 2
  off = round_up(off + (2 * static_cast<size_t>(l.n_blocks) + 8) * 4, 256);
  l.prefix = off;
  off = round_up(off + (2 * static_cast<size_t>(l.n_blocks) + 9) * 4, 256);
  l.tile_list = off;
  off = round_up(off + static_cast<size_t>(kMaxTiles) * l.n_blocks * 4, 256);
  l.seq = off;  // the plan's pairing sequence when it does not fit in shared memory
  off = round_up(off + static_cast<size_t>(l.n_blocks) * 4, 256);
  l.masks = off;  // one tile-mask byte per block
  off = round_up(off + static_cast<size_t>(l.n_blocks) + 4, 256);
  l.ranges = off;
  off = round_up(off + static_cast<size_t>(l.grid) * sizeof(Ranges), 256);
  l.flags1 = off;
  off = round_up(off + static_cast<size_t>(l.grid) * 4, 256);
  l.flags2 = off;
  off = round_up(off + static_cast<size_t>(l.grid) * 4, 1024);
  l.abuf = off;
  off = round_up(off + static_cast<size_t>(kGroupTokens) * l.npad * 4, 1024);  // fp32 activations at most
  l.partials = off;
  off += static_cast<size_t>(l.grid) * kSlotFloats * 4;
  l.total = round_up(off, 256);
  return l;
}

}  // namespace

}  // namespace qcc

extern "C" size_t qcc_prefill_workspace_bytes(int64_t n_records, int hidden) {
  if (n_records <= 0 || hidden <= 0) return 0;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return 0;
  const qcc::DeviceInfo& info = qcc::device_info(device);
  return qcc::prefill_layout(n_records, info.num_sms).total;
}

extern "C" size_t qcc_prefill_workspace_status_offset(void) { return 0; }

extern "C" int qcc_indexed_ffn_prefill(const void* x, int64_t ldx, int n_tokens, int hidden, const void* packed,
                                       int64_t n_records, int dtype, const int32_t* tile_blocks,
                                       const int32_t* tile_offsets, void* workspace, size_t workspace_bytes, void* y,
                                       int64_t ldy, int y_dtype, cudaStream_t stream) {
  using namespace qcc;
  if (dtype != QCC_DTYPE_BF16 && dtype != QCC_DTYPE_F16 && dtype != QCC_DTYPE_F32) return QCC_ERR_DTYPE;
  if (!valid_dtype(y_dtype)) return QCC_ERR_DTYPE;
  if (n_tokens < 0 || hidden <= 0 || n_records <= 0 || ldx < hidden || ldy < hidden) return QCC_ERR_SHAPE;
  if (n_records > static_cast<int64_t>(kMaxBlocks) * kBlock) return QCC_ERR_UNSUPPORTED;
  if ((hidden + kHRange - 1) / kHRange * kMaxTiles > kMaxDownUnits) return QCC_ERR_UNSUPPORTED;
  if (n_tokens == 0) return QCC_OK;
  if (x == nullptr || packed == nullptr || tile_blocks == nullptr || tile_offsets == nullptr || workspace == nullptr ||
      y == nullptr)
    return QCC_ERR_INVALID_ARGUMENT;
  // TMA: 16-byte aligned bases and row strides.
  const int es = dtype_bytes(dtype);
  const int row_elems = kRowBytes / es;  // elements of a 128-byte row: the boxes' inner extent
  if (!aligned16(x) || !aligned16(packed) || !aligned16(workspace) || (ldx * es) % 16 != 0) return QCC_ERR_ALIGNMENT;
  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const DeviceInfo& info = device_info(device);
  const PrefillLayout l = prefill_layout(n_records, info.num_sms);
  if (workspace_bytes < l.total) return QCC_ERR_WORKSPACE;
  if (info.max_smem_optin < static_cast<int>(kSmemBytes) || l.grid > kMaxPlanGrid) return QCC_ERR_UNSUPPORTED;
  const int hp = hidden_pad(hidden, dtype);
  uint8_t* ws = static_cast<uint8_t*>(workspace);

  PrefillArgs args{};
  args.header = reinterpret_cast<int32_t*>(ws);
  args.units = reinterpret_cast<int32_t*>(ws + l.units);
  args.unit_prefix = reinterpret_cast<int32_t*>(ws + l.prefix);
  args.tile_list = reinterpret_cast<int32_t*>(ws + l.tile_list);
  args.block_masks = ws + l.masks;
  args.ranges = reinterpret_cast<const Ranges*>(ws + l.ranges);
  args.n_blocks = l.n_blocks;
  args.n_chunks = (hidden + row_elems - 1) / row_elems;
  args.n_hranges = (hidden + kHRange - 1) / kHRange;
  args.hidden = hidden;
  args.abuf = ws + l.abuf;
  args.ld_abuf = l.npad;
  args.partials = reinterpret_cast<float*>(ws + l.partials);
  args.flags1 = reinterpret_cast<int32_t*>(ws + l.flags1);
  args.flags2 = reinterpret_cast<int32_t*>(ws + l.flags2);
  args.ldy = ldy;
  args.y_dtype = y_dtype;
  const size_t y_es = static_cast<size_t>(dtype_bytes(y_dtype));
  args.y_vec = aligned16(y) && (static_cast<size_t>(ldy) * y_es) % 16 == 0;

  // Records as a 3-D tensor {hidden_pad, segment (gate, up, down), record}:
  // gate/up boxes of 64 records, down boxes of one down step's records (read
  // MN-major by the MMA: fp32 ones with the 32-byte-atom swizzle that
  // kind::tf32 requires for an MN-major operand).
  CUtensorMap tm_records, tm_down, tm_abuf;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(hp), 3, static_cast<uint64_t>(n_records)};
    const uint64_t strides[2] = {static_cast<uint64_t>(hp) * es, static_cast<uint64_t>(hp) * 3 * es};
    const uint32_t box[3] = {static_cast<uint32_t>(row_elems), 1, 64};
    const uint32_t down_box[3] = {static_cast<uint32_t>(row_elems), 1, static_cast<uint32_t>(row_elems)};
    if (!make_map(&tm_records, dtype, 3, packed, dims, strides, box) ||
        !make_map(&tm_down, dtype, 3, packed, dims, strides, down_box,
                  dtype == QCC_DTYPE_F32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B))
      return QCC_ERR_UNSUPPORTED;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(l.npad), static_cast<uint64_t>(kGroupTokens)};
    const uint64_t strides[1] = {static_cast<uint64_t>(l.npad) * es};
    const uint32_t box[2] = {static_cast<uint32_t>(row_elems), 128};
    if (!make_map(&tm_abuf, dtype, 2, args.abuf, dims, strides, box)) return QCC_ERR_UNSUPPORTED;
  }
  const void* kernel = dtype == QCC_DTYPE_BF16  ? reinterpret_cast<const void*>(prefill_kernel<kFmtBF16>)
                       : dtype == QCC_DTYPE_F16 ? reinterpret_cast<const void*>(prefill_kernel<kFmtF16>)
                                                : reinterpret_cast<const void*>(prefill_kernel<kFmtTF32>);
  if (!ensure_max_dynamic_smem(reinterpret_cast<const void*>(prefill_plan_kernel), device) ||
      !ensure_max_dynamic_smem(kernel, device))
    return QCC_ERR_CUDA;
  const size_t plan_smem =
      round_up(static_cast<size_t>(l.n_blocks), 4) +
      (2 * static_cast<size_t>(std::min(2 * l.n_blocks + 8, kPlanUnits)) + 1) * 4 +
      (l.n_blocks <= kPlanListBlocks ? static_cast<size_t>(l.n_blocks) * 4 : 0);
  const uint8_t* xb = static_cast<const uint8_t*>(x);
  uint8_t* yb = static_cast<uint8_t*>(y);

  clear_stale_error();
  for (int g0 = 0; g0 < n_tokens; g0 += kGroupTokens) {
    const int rows = std::min(kGroupTokens, n_tokens - g0);
    args.n_tokens = rows;
    args.n_tiles = (rows + kTile - 1) / kTile;
    args.y = yb + static_cast<size_t>(g0) * ldy * y_es;
    CUtensorMap tm_x;
    {
      const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(rows)};
      const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * es};
      const uint32_t box[2] = {static_cast<uint32_t>(row_elems), 128};
      if (!make_map(&tm_x, dtype, 2, xb + static_cast<size_t>(g0) * ldx * es, dims, strides, box))
        return QCC_ERR_UNSUPPORTED;
    }
    prefill_plan_kernel<<<1, kPlanThreads, plan_smem, stream>>>(
        tile_blocks, tile_offsets + g0 / kTile, args.n_tiles, l.n_blocks, args.n_chunks, args.n_hranges,
        kBlock / row_elems, l.grid,
        args.header, const_cast<int32_t*>(args.units), const_cast<int32_t*>(args.unit_prefix),
        const_cast<int32_t*>(args.tile_list), reinterpret_cast<int32_t*>(ws + l.seq),
        reinterpret_cast<uint32_t*>(ws + l.masks), const_cast<Ranges*>(args.ranges));
    if (!launch_ok()) return QCC_ERR_CUDA;
    // Every CTA must be resident at once (grid barrier, cross-CTA flags).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(l.grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    // Cooperative (grid barrier between the phases) and a programmatic
    // dependent of the plan kernel (its launch overlaps the plan).
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    void* kargs[] = {&tm_records, &tm_down, &tm_x, &tm_abuf, &args};
    if (!cuda_ok(cudaLaunchKernelExC(&cfg, kernel, kargs))) return QCC_ERR_CUDA;
  }
  return QCC_OK;
}
