// Block-sparse prefill of the indexed gated FFN on tcgen05 tensor cores (sm_100a).
//
// Tokens come in tiles of 128 rows and records in blocks of 64 (a block id b
// stands for records [64b, 64b + 64), the expansion of
// clustering/block_layout.py:61-64).  Tile t uses the blocks listed for it:
//   y[r] = sum over records n of the blocks of r's tile of silu(g_n . x_r) (u_n . x_r) d_n.
// The reference computes each tile with runtime/ffn.py:20-39 on the expanded
// ids (three gathers and three GEMMs per tile).
//
// A call runs groups of up to four tiles (512 tokens); each group is four
// launches:
//  plan      one CTA: per-block tile masks from the per-tile block lists, the
//            gate/up work units (a block with one or two of its tiles) and the
//            union of blocks with their masks.
//  gate/up   persistent; per unit A[tok, 64b .. 64b+63] = silu(X G_b^T) * (X U_b^T)
//            for the unit's tiles: M = 128 tokens, N = 128 (64 gate + 64 up
//            records), K = hidden in 64-wide chunks.  A block used by three or
//            four tiles is two units that run side by side, so the second
//            read of its gate/up rows usually hits L2.
//  down      y^T[h, tok] = sum over blocks of D_b[h, n] A[tok, n]: M = 128 hidden
//            rows of one chunk, N = 128 tokens of a tile, K = 64 records of a
//            block.  The accumulators of all four tiles live in TMEM (512
//            columns).  The union is split S ways per hidden chunk so that the
//            grid fills the GPU; each CTA writes an fp32 partial.
//  reduce    sums the S partials in a fixed order and writes y (only when S > 1).
//
// Operands move by tiled TMA (128-byte swizzle, no multicast) through a 4-stage
// shared-memory ring; one thread issues the loads, one thread issues the
// MMAs, four warps read TMEM.  Every wait is bounded (2 s) and reports
// QCC_DEV_TIMEOUT through the workspace status word.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "qcc_common.cuh"
#include "qcc_host.h"
#include "qcc_tc.cuh"

namespace qcc {

namespace {

constexpr int kTile = 128;                // tokens per tile
constexpr int kBlock = 64;                // records per block
constexpr int kChunk = 64;                // hidden elements per K chunk (one 128-byte swizzled row)
constexpr int kMaxTiles = 4;              // tiles per group: 4 x 128 TMEM columns
constexpr int kGroupTokens = kTile * kMaxTiles;
constexpr int kHChunk = 128;              // hidden rows per down-projection CTA
constexpr int kMaxSplits = 4;
constexpr int kStages = 4;
constexpr int kThreads = 192;             // warp 0: TMA, warp 1: MMA, warps 2-5: TMEM readers
constexpr int kPlanThreads = 1024;
constexpr uint32_t kHalfBox = 64 * 128;   // [64 rows x 64 elements] of 16-bit: 8 KB
constexpr uint32_t kTileBox = 128 * 128;  // [128 rows x 64 elements]: 16 KB
constexpr uint32_t kStageBytes = 2 * kHalfBox + 2 * kTileBox;  // 48 KB
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 256 + 1024;  // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kMaxBlocks = 1 << 16;       // byte map of the plan kernel in shared memory

// Workspace header (int32 words).
constexpr int kHdrStatus = 0;
constexpr int kHdrUnits = 1;
constexpr int kHdrUnion = 2;
constexpr size_t kHeaderBytes = 256;

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
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

// The same wait for a whole warp: lane 0 polls, every lane gets the result.
__device__ __forceinline__ bool warp_wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                int* status) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(bar, parity, abort_flag, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Waits, without regard to an abort, for the loads of the last issued stages
// so that no copy is still writing shared memory when the CTA exits.
__device__ __forceinline__ void drain_loads(Barriers* bars, uint32_t issued) {
  const uint32_t first = issued > static_cast<uint32_t>(kStages) ? issued - kStages : 0u;
  for (uint32_t i = first; i < issued; ++i) mbar_wait_bounded(&bars->full[i % kStages], (i / kStages) & 1u, kWaitLimitNs);
}

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.f + __expf(-g)); }

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

// Unit word: block << 8 | first tile << 4 | second tile (0xF: none).
// Union word: block << 8 | tile mask.
__global__ void __launch_bounds__(kPlanThreads)
    prefill_plan_kernel(const int32_t* __restrict__ tile_blocks, const int32_t* __restrict__ tile_offsets,
                        int n_tiles, int n_blocks, int32_t* __restrict__ header, int32_t* __restrict__ units,
                        int32_t* __restrict__ unions) {
  extern __shared__ __align__(16) uint32_t words[];  // one mask byte per block
  __shared__ int scratch[64];
  const int tid = threadIdx.x;
  const int n_words = (n_blocks + 3) / 4;
  for (int i = tid; i < n_words; i += blockDim.x) words[i] = 0u;
  __syncthreads();
  bool bad = false;
  for (int t = 0; t < n_tiles; ++t) {
    const int begin = __ldg(tile_offsets + t);
    const int end = __ldg(tile_offsets + t + 1);
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
  if (bad) atomicOr(header + kHdrStatus, QCC_DEV_ID_RANGE);
  __syncthreads();
  const uint8_t* mask = reinterpret_cast<const uint8_t*>(words);
  const int chunk = (n_blocks + blockDim.x - 1) / blockDim.x;
  const int lo = min(n_blocks, tid * chunk);
  const int hi = min(n_blocks, lo + chunk);
  int n_union = 0, n_units = 0;
  for (int i = lo; i < hi; ++i) {
    const int m = mask[i];
    if (m != 0) {
      ++n_union;
      n_units += (__popc(m) + 1) / 2;
    }
  }
  int total_union, total_units;
  int pos_union = block_exclusive_scan(n_union, scratch, &total_union);
  int pos_units = block_exclusive_scan(n_units, scratch, &total_units);
  for (int i = lo; i < hi; ++i) {
    const int m = mask[i];
    if (m == 0) continue;
    unions[pos_union++] = (i << 8) | m;
    int tl[kMaxTiles];
    int c = 0;
#pragma unroll
    for (int t = 0; t < kMaxTiles; ++t)
      if ((m >> t) & 1) tl[c++] = t;
    for (int p = 0; p < c; p += 2) units[pos_units++] = (i << 8) | (tl[p] << 4) | (p + 1 < c ? tl[p + 1] : 0xF);
  }
  if (tid == 0) {
    header[kHdrUnits] = total_units;
    header[kHdrUnion] = total_union;
  }
}

// Common prologue of the tensor-core kernels: barriers, TMEM allocation.
__device__ __forceinline__ Barriers* setup(uint8_t* smem) {
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&bars->acc_full[j], 1);
      mbar_init(&bars->acc_empty[j], 4);  // one arrival per TMEM-reading warp
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  return bars;
}

// Common end: every MMA has completed before TMEM is released.
__device__ __forceinline__ void teardown(Barriers* bars, bool mma_thread) {
  if (mma_thread) {
    tc_commit(&bars->drain);
    mbar_wait_bounded(&bars->drain, 0, kWaitLimitNs);
  }
  tc_fence_before_sync();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after_sync();
    tmem_dealloc(bars->tmem_base, kTmemCols);
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_gate_up_kernel(const __grid_constant__ CUtensorMap tm_records, const __grid_constant__ CUtensorMap tm_x,
                           int n_chunks, int32_t* __restrict__ header, const int32_t* __restrict__ units,
                           uint16_t* __restrict__ abuf, int64_t ld_abuf) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  Barriers* bars = setup(smem);
  volatile int* abort_flag = &bars->abort;
  int* status = header + kHdrStatus;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_units = header[kHdrUnits];
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&tm_records);
      tma_prefetch_map(&tm_x);
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const int unit = units[u];
        const int b = unit >> 8;
        const int ta = (unit >> 4) & 0xF;
        const int tb = unit & 0xF;
        const int nt = tb == 0xF ? 1 : 2;
        const uint32_t bytes = 2 * kHalfBox + nt * kTileBox;
        bool ok = true;
        for (int kc = 0; kc < n_chunks; ++kc, ++it) {
          const int s = it % kStages;
          if (!wait_phase(&bars->empty[s], ((it / kStages) & 1u) ^ 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], bytes);
          tma_load_3d(st, &tm_records, kc * kChunk, 0, b * kBlock, &bars->full[s]);
          tma_load_3d(st + kHalfBox, &tm_records, kc * kChunk, 1, b * kBlock, &bars->full[s]);
          tma_load_2d(st + 2 * kHalfBox, &tm_x, kc * kChunk, ta * kTile, &bars->full[s]);
          if (nt == 2) tma_load_2d(st + 2 * kHalfBox + kTileBox, &tm_x, kc * kChunk, tb * kTile, &bars->full[s]);
        }
        if (!ok) break;
      }
      drain_loads(bars, it);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, 128, kBf16, false, false);
      uint32_t it = 0, ut = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ut) {
        const int unit = units[u];
        const int nt = (unit & 0xF) == 0xF ? 1 : 2;
        const uint32_t j = ut & 1u;
        if (!wait_phase(&bars->acc_empty[j], ((ut >> 1) & 1u) ^ 1u, abort_flag, status)) break;
        tc_fence_after_sync();
        const uint32_t d0 = tmem + j * 256u;
        bool ok = true;
        for (int kc = 0; kc < n_chunks; ++kc, ++it) {
          const int s = it % kStages;
          if (!wait_phase(&bars->full[s], (it / kStages) & 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t st = smem_addr(smem + s * kStageBytes);
          const uint64_t b_desc = smem_desc_sw128(st, 16, 1024);
          for (int i = 0; i < nt; ++i) {
            const uint64_t a_desc = smem_desc_sw128(st + 2 * kHalfBox + i * kTileBox, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < kChunk / 16; ++kk)
              tc_mma_f16(d0 + i * 128u, a_desc + 2u * kk, b_desc + 2u * kk, idesc, (kc | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&bars->empty[s]);
        }
        if (!ok) break;
        tc_commit(&bars->acc_full[j]);
      }
    }
  } else {
    // TMEM readers: warp w may read lanes 32*(w%4) .. +31 = token rows of the tile.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t ut = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ut) {
      const int unit = units[u];
      const int b = unit >> 8;
      const int ta = (unit >> 4) & 0xF;
      const int tb = unit & 0xF;
      const int nt = tb == 0xF ? 1 : 2;
      const uint32_t j = ut & 1u;
      if (!warp_wait_phase(&bars->acc_full[j], (ut >> 1) & 1u, abort_flag, status)) break;
      tc_fence_after_sync();
      for (int i = 0; i < nt; ++i) {
        const int t = i == 0 ? ta : tb;
        const uint32_t col0 = tmem + (static_cast<uint32_t>(q * 32) << 16) + j * 256u + i * 128u;
        uint16_t* dst = abuf + static_cast<int64_t>(t * kTile + row) * ld_abuf + static_cast<int64_t>(b) * kBlock;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float g[32], v[32];
          tmem_load32(col0 + c * 32, g);
          tmem_load32(col0 + 64 + c * 32, v);
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            w[e] = pack2<kBf16>(silu(g[2 * e]) * v[2 * e], silu(g[2 * e + 1]) * v[2 * e + 1]);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[j]);
    }
  }
  teardown(bars, warp == 1 && lane == 0);
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_down_kernel(const __grid_constant__ CUtensorMap tm_records, const __grid_constant__ CUtensorMap tm_abuf,
                        int32_t* __restrict__ header, const int32_t* __restrict__ unions, int n_hchunks, int splits,
                        int hidden, int n_tokens, float* __restrict__ partials, int64_t ld_part, void* __restrict__ y,
                        int64_t ldy, int y_dtype) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  Barriers* bars = setup(smem);
  volatile int* abort_flag = &bars->abort;
  int* status = header + kHdrStatus;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int hc = blockIdx.x % n_hchunks;
  const int split = blockIdx.x / n_hchunks;
  const int n_union = header[kHdrUnion];
  const int e_begin = static_cast<int>(static_cast<int64_t>(split) * n_union / splits);
  const int e_end = static_cast<int>(static_cast<int64_t>(split + 1) * n_union / splits);
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&tm_records);
      tma_prefetch_map(&tm_abuf);
      uint32_t it = 0;
      bool ok = true;
      for (int e = e_begin; e < e_end && ok; ++e) {
        const int word = unions[e];
        const int b = word >> 8;
        int m = word & 0xF;
        while (m != 0 && ok) {
          const int t0 = __ffs(m) - 1;
          m &= m - 1;
          const int t1 = m != 0 ? __ffs(m) - 1 : -1;
          if (t1 >= 0) m &= m - 1;
          const int s = it % kStages;
          if (!wait_phase(&bars->empty[s], ((it / kStages) & 1u) ^ 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], 2 * kHalfBox + (t1 >= 0 ? 2 : 1) * kTileBox);
          tma_load_3d(st, &tm_records, hc * kHChunk, 2, b * kBlock, &bars->full[s]);
          tma_load_3d(st + kHalfBox, &tm_records, hc * kHChunk + 64, 2, b * kBlock, &bars->full[s]);
          tma_load_2d(st + 2 * kHalfBox, &tm_abuf, b * kBlock, t0 * kTile, &bars->full[s]);
          if (t1 >= 0) tma_load_2d(st + 2 * kHalfBox + kTileBox, &tm_abuf, b * kBlock, t1 * kTile, &bars->full[s]);
          ++it;
        }
      }
      drain_loads(bars, it);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, 128, kBf16, true, false);
      uint32_t it = 0, started = 0;
      bool ok = true;
      for (int e = e_begin; e < e_end && ok; ++e) {
        int m = unions[e] & 0xF;
        while (m != 0) {
          const int t0 = __ffs(m) - 1;
          m &= m - 1;
          const int t1 = m != 0 ? __ffs(m) - 1 : -1;
          if (t1 >= 0) m &= m - 1;
          const int s = it % kStages;
          if (!wait_phase(&bars->full[s], (it / kStages) & 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t st = smem_addr(smem + s * kStageBytes);
          // D slice: MN-major, 64 hidden rows per 128-byte line, second 64 rows kHalfBox further.
          const uint64_t a_desc = smem_desc_sw128(st, kHalfBox, 1024);
          for (int i = 0; i < (t1 >= 0 ? 2 : 1); ++i) {
            const int t = i == 0 ? t0 : t1;
            const uint64_t b_desc = smem_desc_sw128(st + 2 * kHalfBox + i * kTileBox, 16, 1024);
            const uint32_t acc = (started >> t) & 1u;
#pragma unroll
            for (int kk = 0; kk < kBlock / 16; ++kk)
              tc_mma_f16(tmem + t * 128u, a_desc + 128u * kk, b_desc + 2u * kk, idesc, (acc | kk) != 0 ? 1u : 0u);
            started |= 1u << t;
          }
          tc_commit(&bars->empty[s]);
          ++it;
        }
      }
      tc_commit(&bars->acc_full[0]);
    }
  } else {
    const int q = warp & 3;
    const int hl = q * 32 + lane;  // TMEM lane = hidden row of the chunk
    const int h = hc * kHChunk + hl;
    uint32_t started = 0;
    for (int e = e_begin; e < e_end; ++e) started |= unions[e] & 0xF;
    const bool ready = warp_wait_phase(&bars->acc_full[0], 0, abort_flag, status);
    tc_fence_after_sync();
    const int n_tiles = (n_tokens + kTile - 1) / kTile;
    float* part = partials + static_cast<int64_t>(split) * kGroupTokens * ld_part;
    for (int t = 0; t < n_tiles && ready; ++t) {
      const bool have = (started >> t) & 1u;
      for (int c = 0; c < kTile / 32; ++c) {
        float v[32];
        if (have) {
          tmem_load32(tmem + (static_cast<uint32_t>(q * 32) << 16) + t * 128u + c * 32u, v);
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = 0.f;
        }
        if (h < hidden) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int tok = t * kTile + c * 32 + k;
            if (tok < n_tokens) {
              if (splits == 1)
                store_as(y, static_cast<int64_t>(tok) * ldy + h, y_dtype, v[k]);
              else
                part[static_cast<int64_t>(tok) * ld_part + h] = v[k];
            }
          }
        }
      }
    }
  }
  teardown(bars, warp == 1 && lane == 0);
}

// y = sum of the S partials (fixed order), converted to the output type.
__global__ void __launch_bounds__(256)
    prefill_reduce_kernel(const float* __restrict__ partials, int64_t ld_part, int splits, int n_tokens, int hidden,
                          void* __restrict__ y, int64_t ldy, int y_dtype) {
  const int64_t total = static_cast<int64_t>(n_tokens) * hidden;
  const int64_t plane = static_cast<int64_t>(kGroupTokens) * ld_part;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / hidden;
    const int64_t h = i - tok * hidden;
    const int64_t off = tok * ld_part + h;
    float acc = __ldcg(partials + off);
    for (int s = 1; s < splits; ++s) acc += __ldcg(partials + s * plane + off);
    store_as(y, tok * ldy + h, y_dtype, acc);
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

// 16-bit tensor map with the 128-byte swizzle; dims / strides innermost first.
bool make_map(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims, const uint64_t* strides,
              const uint32_t* box) {
  auto fn = encode_tiled();
  if (fn == nullptr) return false;
  const uint32_t elem[3] = {1, 1, 1};
  const CUresult r = fn(map, dtype == QCC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        rank, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct PrefillLayout {
  int n_blocks = 0, n_hchunks = 0, splits = 1;
  int64_t npad = 0, ld_part = 0;
  size_t units = 0, unions = 0, abuf = 0, partials = 0, total = 0;
};

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

PrefillLayout prefill_layout(int64_t n_records, int hidden, int num_sms) {
  PrefillLayout l;
  l.n_blocks = static_cast<int>((n_records + kBlock - 1) / kBlock);
  l.n_hchunks = (hidden + kHChunk - 1) / kHChunk;
  l.splits = std::max(1, std::min(kMaxSplits, num_sms / std::max(1, l.n_hchunks)));
  l.npad = static_cast<int64_t>(l.n_blocks) * kBlock;
  l.ld_part = round_up(static_cast<size_t>(hidden), 4);
  size_t off = kHeaderBytes;
  l.units = off;
  off = round_up(off + 2 * static_cast<size_t>(l.n_blocks) * 4, 256);
  l.unions = off;
  off = round_up(off + static_cast<size_t>(l.n_blocks) * 4, 1024);
  l.abuf = off;
  off = round_up(off + static_cast<size_t>(kGroupTokens) * l.npad * 2, 1024);
  l.partials = off;
  if (l.splits > 1) off += static_cast<size_t>(l.splits) * kGroupTokens * l.ld_part * 4;
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
  return qcc::prefill_layout(n_records, hidden, info.num_sms).total;
}

extern "C" size_t qcc_prefill_workspace_status_offset(void) { return 0; }

extern "C" int qcc_indexed_ffn_prefill(const void* x, int64_t ldx, int n_tokens, int hidden, const void* packed,
                                       int64_t n_records, int dtype, const int32_t* tile_blocks,
                                       const int32_t* tile_offsets, void* workspace, size_t workspace_bytes, void* y,
                                       int64_t ldy, int y_dtype, cudaStream_t stream) {
  using namespace qcc;
  if (dtype != QCC_DTYPE_BF16 && dtype != QCC_DTYPE_F16) return valid_dtype(dtype) ? QCC_ERR_UNSUPPORTED : QCC_ERR_DTYPE;
  if (!valid_dtype(y_dtype)) return QCC_ERR_DTYPE;
  if (n_tokens < 0 || hidden <= 0 || n_records <= 0 || ldx < hidden || ldy < hidden) return QCC_ERR_SHAPE;
  if (n_records > static_cast<int64_t>(kMaxBlocks) * kBlock) return QCC_ERR_UNSUPPORTED;
  if (n_tokens == 0) return QCC_OK;
  if (x == nullptr || packed == nullptr || tile_blocks == nullptr || tile_offsets == nullptr || workspace == nullptr ||
      y == nullptr)
    return QCC_ERR_INVALID_ARGUMENT;
  // TMA: 16-byte aligned bases and row strides.
  if (!aligned16(x) || !aligned16(packed) || !aligned16(workspace) || (ldx * 2) % 16 != 0) return QCC_ERR_ALIGNMENT;
  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const DeviceInfo& info = device_info(device);
  const PrefillLayout l = prefill_layout(n_records, hidden, info.num_sms);
  if (workspace_bytes < l.total) return QCC_ERR_WORKSPACE;
  const int hp = hidden_pad(hidden, dtype);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* header = reinterpret_cast<int32_t*>(ws);
  int32_t* units = reinterpret_cast<int32_t*>(ws + l.units);
  int32_t* unions = reinterpret_cast<int32_t*>(ws + l.unions);
  uint16_t* abuf = reinterpret_cast<uint16_t*>(ws + l.abuf);
  float* partials = reinterpret_cast<float*>(ws + l.partials);

  // Records as a 3-D tensor {hidden_pad, segment (gate, up, down), record}.
  CUtensorMap tm_records, tm_abuf;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(hp), 3, static_cast<uint64_t>(n_records)};
    const uint64_t strides[2] = {static_cast<uint64_t>(hp) * 2, static_cast<uint64_t>(hp) * 6};
    const uint32_t box[3] = {64, 1, 64};
    if (!make_map(&tm_records, dtype, 3, packed, dims, strides, box)) return QCC_ERR_UNSUPPORTED;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(l.npad), static_cast<uint64_t>(kGroupTokens)};
    const uint64_t strides[1] = {static_cast<uint64_t>(l.npad) * 2};
    const uint32_t box[2] = {64, 128};
    if (!make_map(&tm_abuf, dtype, 2, abuf, dims, strides, box)) return QCC_ERR_UNSUPPORTED;
  }
  const void* fns[4] = {reinterpret_cast<const void*>(prefill_plan_kernel),
                        dtype == QCC_DTYPE_BF16 ? reinterpret_cast<const void*>(prefill_gate_up_kernel<true>)
                                                : reinterpret_cast<const void*>(prefill_gate_up_kernel<false>),
                        dtype == QCC_DTYPE_BF16 ? reinterpret_cast<const void*>(prefill_down_kernel<true>)
                                                : reinterpret_cast<const void*>(prefill_down_kernel<false>),
                        reinterpret_cast<const void*>(prefill_reduce_kernel)};
  for (const void* fn : fns)
    if (!ensure_max_dynamic_smem(fn, device)) return QCC_ERR_CUDA;
  if (info.max_smem_optin < static_cast<int>(kSmemBytes)) return QCC_ERR_UNSUPPORTED;
  const size_t plan_smem = round_up(static_cast<size_t>(l.n_blocks), 4);
  const int n_chunks = (hidden + kChunk - 1) / kChunk;
  const int units_grid = std::max(1, std::min(info.num_sms, 2 * l.n_blocks));
  const int down_grid = l.n_hchunks * l.splits;
  const uint8_t* xb = static_cast<const uint8_t*>(x);
  uint8_t* yb = static_cast<uint8_t*>(y);
  const size_t y_esize = static_cast<size_t>(dtype_bytes(y_dtype));

  clear_stale_error();
  for (int g0 = 0; g0 < n_tokens; g0 += kGroupTokens) {
    const int rows = std::min(kGroupTokens, n_tokens - g0);
    const int n_tiles = (rows + kTile - 1) / kTile;
    CUtensorMap tm_x;
    {
      const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(rows)};
      const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * 2};
      const uint32_t box[2] = {64, 128};
      if (!make_map(&tm_x, dtype, 2, xb + static_cast<size_t>(g0) * ldx * 2, dims, strides, box))
        return QCC_ERR_UNSUPPORTED;
    }
    void* yg = yb + static_cast<size_t>(g0) * ldy * y_esize;
    prefill_plan_kernel<<<1, kPlanThreads, plan_smem, stream>>>(tile_blocks, tile_offsets + g0 / kTile, n_tiles,
                                                                l.n_blocks, header, units, unions);
    if (!launch_ok()) return QCC_ERR_CUDA;
    if (dtype == QCC_DTYPE_BF16)
      prefill_gate_up_kernel<true><<<units_grid, kThreads, kSmemBytes, stream>>>(tm_records, tm_x, n_chunks, header,
                                                                                 units, abuf, l.npad);
    else
      prefill_gate_up_kernel<false><<<units_grid, kThreads, kSmemBytes, stream>>>(tm_records, tm_x, n_chunks, header,
                                                                                  units, abuf, l.npad);
    if (!launch_ok()) return QCC_ERR_CUDA;
    if (dtype == QCC_DTYPE_BF16)
      prefill_down_kernel<true><<<down_grid, kThreads, kSmemBytes, stream>>>(
          tm_records, tm_abuf, header, unions, l.n_hchunks, l.splits, hidden, rows, partials, l.ld_part, yg, ldy,
          y_dtype);
    else
      prefill_down_kernel<false><<<down_grid, kThreads, kSmemBytes, stream>>>(
          tm_records, tm_abuf, header, unions, l.n_hchunks, l.splits, hidden, rows, partials, l.ld_part, yg, ldy,
          y_dtype);
    if (!launch_ok()) return QCC_ERR_CUDA;
    if (l.splits > 1) {
      const int64_t total = static_cast<int64_t>(rows) * hidden;
      const int grid = static_cast<int>(std::min<int64_t>(4 * info.num_sms, (total + 255) / 256));
      prefill_reduce_kernel<<<grid, 256, 0, stream>>>(partials, l.ld_part, l.splits, rows, hidden, yg, ldy, y_dtype);
      if (!launch_ok()) return QCC_ERR_CUDA;
    }
  }
  return QCC_OK;
}
