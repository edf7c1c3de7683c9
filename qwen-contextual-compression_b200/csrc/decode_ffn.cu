// Fused indexed gated FFN for decode / small batches (sm_100a).
//
// Two launches replace the reference's two kernels
// (runtime/cuda_indexed.py:23-26 gate_up_* then down_*), split differently:
//
// 1. indexed_ffn_decode_kernel: each CTA owns a contiguous run of the
//    selected-id list, streams the selected neurons' packed records
//    [gate_row | up_row | down_col] from HBM into a shared-memory ring with
//    one non-multicast bulk copy per record (mbarrier completion), computes
//    g = G_j.x, u = U_j.x with fp32 accumulation, a_j = silu(g) * u, and
//    accumulates a_j * D_j into a per-thread fp32 slice of y held in
//    registers.  At the end the CTA stores its partial y row (fp32) to the
//    workspace and exits: no CTA waits for another.
// 2. decode_reduce_kernel (a programmatic dependent of the first): each CTA
//    sums one column slice of y over all partial rows in a fixed order and
//    writes it in the output dtype -- or, with several ranks, stores its
//    column sums into every rank's exchange buffer and adds the ranks' sums
//    in rank order.  No atomics touch y, so the result is bit-reproducible
//    for a given grid.
//
// Because decode CTAs exit as soon as their records are done, the SMs they
// free take the next launch's CTAs while slower CTAs still stream.  With
// QCC_IDS_READY the next decode starts its record copies right away, before
// it waits for the launches ahead of it; only x is read after that wait.
//
// Compute thread t of a CTA owns the 8-element hidden slots v = t + k * n
// (k < VPT, n compute threads): it holds x[b, 8v:8v+8] and the partial
// y[b, 8v:8v+8] in registers, reads the matching 16-byte pieces of every
// staged record, and all partial dot products meet in one warp-shuffle +
// shared-memory reduction per group of R records (one named barrier of the
// compute warps per group).  A producer warp issues the record copies.

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "qcc_common.cuh"
#include "qcc_host.h"
#include "qcc_tc.cuh"

namespace qcc {

namespace {

// Workspace header: status word (offset 0), the reduce launch's departure
// counter (offset 8, used with several ranks), padding.
constexpr int kWorkspaceHeader = 256;
constexpr int kMaxGrid = 160;          // decode CTAs (one per SM) whose partial rows the workspace holds
constexpr int kRowLoads = (kMaxGrid + 31) / 32;  // partial rows per lane in the reduce
constexpr int kMaxStages = 16;      // ring slots (mbarriers) for the gate|up-only and down-only passes
constexpr int kMaxStagesFull = 8;   // ring slots when whole records stream (registers of the first ids)
constexpr int kMaxThreads = 320;  // compute threads: 10 warps; hidden 5120 = two 8-element slots per thread
constexpr int kMaxBlock = kMaxThreads + 32;  // plus the producer warp
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any bulk-copy wait, default exchange bound
constexpr int kMaxRanks = 8;
// Cross-rank exchange buffer: a 256-byte header -- the launches that used
// this buffer (u32 at offset 0) and the exchange wait bound in ns (u64 at
// offset 8, 0 = 2 s) -- then three slots, each holding one region of column
// sums per rank, [3 slots][world][slot_words] float4.  slot_words follows
// from the buffer's size, so the slots never move when the batch of a call
// changes.  Every word starts as the empty mark (the bits of -0.0f).  A
// writer stores its sums (with -0.0 turned into +0.0); a reader waits until
// no word of a sum is the empty mark, then marks it empty again.  The data is
// its own flag: no fences, no separate flag round trip.
// Launch e of a buffer uses slot e % 3.  A rank starts launch e + 3 only
// after finishing launch e + 2, which needed every rank's launch-(e + 2)
// sums, and each rank wrote those after its own launch e had ended: so every
// owner has read and re-marked slot e % 3 before any rank writes it again.
// The counter lives in the buffer, not in the per-stream workspace, so that
// several layers (buffers) interleaved on one stream each step through the
// three slots in turn.
constexpr uint32_t kEmptyMark = 0x80000000u;
constexpr int kXchgSlots = 3;
constexpr int kXchgHeader = 256;
constexpr int kXchgLimitOffset = 8;

// Stores and polls of exchange words: relaxed at system scope, so the store
// reaches the peer's memory without a fence and every poll reads it anew.
__device__ __forceinline__ void st_relaxed_sys(uint4* p, uint4 v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_sys(const uint4* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ bool has_empty_mark(uint4 w) {
  return w.x == kEmptyMark || w.y == kEmptyMark || w.z == kEmptyMark || w.w == kEmptyMark;
}

// What one launch of the record-streaming kernel computes.
constexpr int kModeFull = 0;    // y over the records: gate / up dot products, activation, down
constexpr int kModeGateUp = 1;  // activations (and scores) only: gate | up parts of the records, no y
constexpr int kModeDown = 2;    // y from given activations: down parts of the records only

struct DecodeArgs {
  const void* x;
  int64_t ldx;
  const uint8_t* packed;
  int64_t record_bytes;
  int64_t n_records;
  int hidden;
  int hidden_pad;
  const void* ids;
  int ids64;
  int ids_ready;  // ids / count / mask may be read before the preceding launches finish
  const uint8_t* token_mask;
  int mask_shift;  // token b uses bit mask_shift + b of its token_mask byte
  int n_ids;
  const int32_t* n_ids_dev;
  unsigned int* status;
  float4* partials;  // [slices][gridDim.x][part_per] float4 (slice-major partial rows)
  int part_per;      // float4 columns per reduce slice
  void* a_out;
  int64_t lda;
  int a_dtype;
  int stages;
  int id_cap;          // capacity of the shared id cache (>= ids per CTA)
  int64_t ring_bytes;  // stages * record_bytes (16-byte multiple)
  int x_vec;           // x rows are 16-byte aligned with hidden % 8 == 0: vector loads
  // Shard range (id_lo >= 0): the ids are global and ascending, and only
  // those in [id_lo, id_hi) -- one contiguous run of the list -- are used,
  // rebased by id_lo.  id_lo < 0: the ids are already local.
  int64_t id_lo;
  int64_t id_hi;
  // Part of each record that is streamed (bytes from the record start, size).
  int64_t copy_offset;
  int copy_bytes;
  // kModeGateUp outputs, indexed by the record's (local) id: activation
  // [B, ld_act_out] fp32 and, when score_out is set, |activation| * col_w[id]
  // (col_w null: |activation|).
  float* act_out;
  int64_t ld_act_out;
  float* score_out;
  int64_t ld_score;
  const float* col_w;
  // kModeDown input: activation [B, ld_act_in] in act_in_dtype, read at the
  // record's (local) id.
  const void* act_in;
  int64_t ld_act_in;
  int act_in_dtype;
};

struct ReduceArgs {
  const float4* partials;  // [slices][rows][per]
  int rows;                // partial rows (the decode grid)
  int per;                 // float4 columns per slice (one slice per CTA)
  int nvec;                // B * hidden_pad / 4
  int seg;                 // hidden_pad
  int hidden;
  void* y_out;
  int64_t ldy;
  int y_dtype;
  const float* y_in;  // optional fp32 [B, ld_in] added to the result
  int64_t ld_in;
  unsigned int* status;
  unsigned int* depart;  // CTAs done with this launch (several ranks only; the last resets it)
  // Cross-rank sum (world > 1): each CTA's column sums go to every rank's
  // exchange buffer; y is the sum over ranks in rank order.
  int world;
  int rank;
  int64_t slot_words;  // float4 words of one (slot, rank) region
  unsigned int* epoch;  // launch counter in this rank's exchange header (advanced by the last CTA)
  const unsigned long long* wait_limit;  // this rank's exchange wait bound (ns, 0 = default)
  uint8_t* xchg[kMaxRanks];  // column-sum slots of all ranks' exchange buffers, own included
};

// Id j of the list; with no list (ids null) the records themselves, in order.
__device__ __forceinline__ int64_t load_id(const DecodeArgs& a, int j) {
  if (a.ids == nullptr) return j;
  return a.ids64 ? __ldg(reinterpret_cast<const long long*>(a.ids) + j)
                 : static_cast<int64_t>(__ldg(reinterpret_cast<const int32_t*>(a.ids) + j));
}

__device__ __forceinline__ float load_as_f32(const void* base, int64_t idx, int dtype) {
  if (dtype == QCC_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  if (dtype == QCC_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  return __ldg(reinterpret_cast<const float*>(base) + idx);
}

__host__ __device__ constexpr int next_pow2(int v) { return v <= 1 ? 1 : 2 * next_pow2((v + 1) / 2); }

// Multi-value warp reduction: V (a power of two <= 32) per-lane values in,
// the warp total of value (lane / (32 / V)) out.  Each butterfly level halves
// the number of live values, so V values cost log2(32) + V - 1 shuffles
// instead of 5 * V.
template <int V>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[V], int lane) {
  static_assert(V >= 1 && V <= 32 && (V & (V - 1)) == 0, "V must be a power of two <= 32");
  int off = 16;
#pragma unroll
  for (int n = V; n > 1; n >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
  return v[0];
}

// Barrier 1 over the first n threads of the CTA (the compute warps; the
// producer warp does not take part) that also ORs a predicate across them.
__device__ __forceinline__ bool compute_barrier_or(bool v, int n) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(n)
      : "memory");
  return r != 0;
}

// Shared-memory layout after the record ring (host mirrors it in tail_bytes):
//   filled mbarriers [kMaxStages] | consumed mbarriers [kMaxStages] |
//   warp partials [2][VP][32] f32 | flag [4] i32 (flag[0]: the consumers gave
//   up) | ids [id_cap] i32 | token bits [id_cap] u8
//
// DN (whole records only): the down slices are read from the ring when the
// group is finished, one iteration later, and the group's slots are refilled
// after that (instead of holding the slices in registers and refilling at
// once).  Frees the registers that two records per group need at 3-4 tokens,
// at the cost of R fewer records in flight.
template <typename T, int B, int VPT, int R, int MODE, bool DN>
__global__ void __launch_bounds__(kMaxBlock, 1) indexed_ffn_decode_kernel(const DecodeArgs a) {
  static_assert(!DN || MODE == kModeFull, "down slices from the ring: whole records only");
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kVals = 2 * R * B;          // partial sums per group: (gate, up) x records x tokens
  constexpr int VP = next_pow2(kVals);      // padded to a power of two for the butterfly
  constexpr int kLanesPer = 32 / VP;        // lanes holding one value after the butterfly
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  // The last warp is the producer: it issues the record copies, the others
  // (nthreads compute threads) consume them.
  const int nthreads = blockDim.x - 32;
  const int nwarps = nthreads >> 5;
  const bool producer = warp == nwarps;
  const int S = a.stages;
  const int seg = a.hidden_pad;
  const int nslots = seg >> 3;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.ring_bytes);   // slot filled
  uint64_t* empty = bars + kMaxStages;                                  // slot consumed
  float* s_red = reinterpret_cast<float*>(empty + kMaxStages);
  int* s_flag = reinterpret_cast<int*>(s_red + 2 * VP * 32);
  int32_t* s_ids = s_flag + 4;
  uint8_t* s_bits = reinterpret_cast<uint8_t*>(s_ids + a.id_cap);

  // Programmatic dependent launch: the reduce launch that follows may be
  // scheduled now (it waits for this grid before reading the partial rows).
  // This grid waits for the launches before it before reading x -- and, unless
  // the caller marked the ids ready, before reading the ids too.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!a.ids_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
  // This CTA's share of the id list.
  int n = a.n_ids;
  if (a.n_ids_dev != nullptr) n = min(n, max(0, __ldg(a.n_ids_dev)));
  int first = 0;
  const int64_t rebase = a.id_lo >= 0 ? a.id_lo : 0;
  if (a.id_lo >= 0) {
    // The ids in [id_lo, id_hi) of an ascending list are the run
    // [#ids < id_lo, #ids < id_hi): count both in one coalesced pass (every
    // load in flight at once) and a block reduction.
    unsigned int below_lo = 0, below_hi = 0;
    for (int i = tid; i < n && !producer; i += nthreads) {
      const int64_t id = load_id(a, i);
      below_lo += id < a.id_lo ? 1u : 0u;
      below_hi += id < a.id_hi ? 1u : 0u;
    }
    below_lo = __reduce_add_sync(0xffffffffu, below_lo);
    below_hi = __reduce_add_sync(0xffffffffu, below_hi);
    unsigned int* s_count = reinterpret_cast<unsigned int*>(s_red);  // free until the pipeline starts
    if (lane == 0 && !producer) {
      s_count[2 * warp] = below_lo;
      s_count[2 * warp + 1] = below_hi;
    }
    __syncthreads();
    unsigned int lo = 0, hi = 0;
    for (int w = 0; w < nwarps; ++w) {
      lo += s_count[2 * w];
      hi += s_count[2 * w + 1];
    }
    first = static_cast<int>(lo);
    n = static_cast<int>(hi) - first;
    __syncthreads();  // s_count is s_red, reused by the pipeline
  }
  const int begin = first + static_cast<int>((static_cast<int64_t>(n) * blockIdx.x) / gridDim.x);
  const int end = first + static_cast<int>((static_cast<int64_t>(n) * (blockIdx.x + 1)) / gridDim.x);
  const int cnt = end - begin;

  const uint64_t policy = policy_evict_first();
  int issued = 0;  // meaningful in the producer's lane 0 only
  // Source of the streamed part of record id (read from the kernel parameters
  // at each use, so that no pointer stays live in a register).
  auto part_src = [&](int32_t id) { return a.packed + a.copy_offset + static_cast<int64_t>(id) * a.record_bytes; };

  auto issue = [&](int i, int stage) {  // producer: start the bulk copy of local record i
    const int32_t id = s_ids[i];
    uint64_t* bar = &bars[stage];
    if (id >= 0) {
      const uint32_t bytes = static_cast<uint32_t>(a.copy_bytes);
      mbar_arrive_expect_tx(bar, bytes);
      bulk_load(smem + static_cast<size_t>(stage) * bytes, part_src(id), bytes, bar, policy);
    } else {
      mbar_arrive(bar);  // completes the phase with no data; consumers skip the record
    }
  };
  auto cache_id = [&](int i) {  // id (or -1 when out of range) and token bits of local record i
    const int64_t id = load_id(a, begin + i) - rebase;
    const bool in_range = id >= 0 && id < a.n_records;
    if (!in_range) atomicOr(a.status, QCC_DEV_ID_RANGE);
    s_ids[i] = in_range ? static_cast<int32_t>(id) : -1;
    s_bits[i] = a.token_mask ? static_cast<uint8_t>(__ldg(a.token_mask + begin + i) >> a.mask_shift)
                             : static_cast<uint8_t>(0xFFu);
  };

  float xr[B][VPT][8];
  float yr[B][VPT][8];
  const T* xg = reinterpret_cast<const T*>(a.x);
  auto load_x = [&]() {
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = tid + k * nthreads;
        if (a.x_vec && v < nslots) {
          float f[8];
          widen(load_global_pack8<T>(xg + b * a.ldx + 8 * v), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) xr[b][k][e] = f[e];
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int h = 8 * v + e;
            xr[b][k][e] = (v < nslots && h < a.hidden) ? to_f32<T>(xg[b * a.ldx + h]) : 0.f;
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) yr[b][k][e] = 0.f;
      }
  };

  // Prologue.  Without QCC_IDS_READY every thread first issues its small
  // global loads -- its x slots and its share of the id cache -- so that they
  // are in the memory system before any record copy (loads issued after the
  // copies queue behind ~30 MB of record traffic).  With it, x may only be
  // read after the wait for the preceding launches, so the ids and the first
  // record copies go first and x follows the wait.  The producer fetches the
  // first S ids itself and starts their copies without waiting for the block
  // barrier.
  const int pre = min(S, cnt);
  if (!a.ids_ready && !producer) load_x();
  // The producer's first S ids are loaded into registers together with the
  // cache loads, so one memory latency covers both.
  constexpr int kFirst = MODE == kModeFull ? kMaxStagesFull : kMaxStages;
  int32_t first_ids[kFirst];
  const bool issuer = producer && lane == 0;
  if (issuer) {
#pragma unroll
    for (int i = 0; i < kFirst; ++i) {
      const int64_t id = i < pre ? load_id(a, begin + i) - rebase : -1;
      first_ids[i] = (id >= 0 && id < a.n_records) ? static_cast<int32_t>(id) : -1;
    }
  }
  if (!producer)
    for (int i = tid; i < cnt; i += nthreads) cache_id(i);
  if (issuer) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars[s], 1);
      mbar_init(&empty[s], 1);
    }
    s_flag[0] = 0;  // set by the consumers when they give up
    fence_barrier_init();
#pragma unroll
    for (int i = 0; i < kFirst; ++i) {
      if (i < pre) {
        const int32_t id = first_ids[i];
        uint64_t* bar = &bars[i];
        if (id >= 0) {
          const uint32_t bytes = static_cast<uint32_t>(a.copy_bytes);
          mbar_arrive_expect_tx(bar, bytes);
          bulk_load(smem + static_cast<size_t>(i) * bytes, part_src(id), bytes, bar, policy);
        } else {
          mbar_arrive(bar);
        }
      }
    }
    issued = pre;
  }
  if (a.ids_ready && !producer) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    load_x();
  }
  __syncthreads();

  if (producer) {
    // Refill each slot as soon as the consumers free it (they arrive on
    // empty[slot] after the barrier of the group that used it): record i goes
    // to slot i % S after its (i / S)-th release.  Its copy-issue time (about
    // 0.2 us per two records) is no longer on the compute warps' path.
    if (issuer) {
      for (int i = pre; i < cnt; ++i) {
        const int stage = i % S;
        const uint32_t parity = ((i / S) & 1u) ^ 1u;
        bool ok = mbar_try_wait(&empty[stage], parity);
        if (!ok) {
          const uint64_t start = global_timer_ns();
          while (!(ok = mbar_try_wait(&empty[stage], parity))) {
            if (*reinterpret_cast<volatile int*>(s_flag) != 0 || global_timer_ns() - start > kWaitLimitNs) break;
          }
        }
        if (!ok) break;
        issue(i, stage);
        issued = i + 1;
      }
      // After a give-up (or with every record issued): the copies of the last
      // S issued records have landed before the CTA exits.
      for (int i = max(0, issued - S); i < issued; ++i)
        (void)mbar_wait_bounded(&bars[i % S], (i / S) & 1, kWaitLimitNs);
    }
    return;
  }

  // Software pipeline, one barrier per group of R records:
  //   iteration g: wait for group g, partial dot products -> warp sums ->
  //   s_red[g & 1]; and finish group g-1 (its block sums are complete since
  //   the previous barrier): activation and y += a * down, with group g-1's
  //   down slices already in registers.  After the barrier the group's ring
  //   slots go back to the producer.
  Pack8<T> dn_prev[R][VPT];
  float act_prev[R][B];  // kModeDown: the activations of the previous group (0 where unused)
  int rn_prev = 0;
  int buf = 0;
  int stage0 = 0;    // ring slot of the group's first record
  int stage_prev = 0;  // ring slot of the previous group's first record (DN)
  uint32_t phase0 = 0;
  bool aborted = false;
  for (int g0 = 0;; g0 += R) {
    const int rn = min(R, cnt - g0);
    Pack8<T> dn_cur[R][VPT];
    float act_cur[R][B];
    bool ok = true;
    // Finishing group g-1 needs nothing of group g.  At 1-2 tokens it goes first
    // and runs while group g's records may still be arriving (27.6 against 28.4 us
    // per layer at batch 1); at 3-4 tokens the other order measured slightly faster.
    auto finish_prev = [&]() {
      if (rn_prev > 0) {
        // Block totals of group g-1: value q = lane / kLanesPer summed over warps.
        float t = 0.f;
        if constexpr (MODE != kModeDown) {
          const float* redp = s_red + (buf ^ 1) * VP * 32 + (lane / kLanesPer) * 32;
          for (int w = lane % kLanesPer; w < nwarps; w += kLanesPer) t += redp[w];
  #pragma unroll
          for (int off = kLanesPer / 2; off >= 1; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
        }
  #pragma unroll
        for (int r = 0; r < R; ++r) {
          if (r < rn_prev) {
            const int i = g0 - R + r;
            const int32_t id = s_ids[i];
            const bool valid = id >= 0;
            const unsigned bits = s_bits[i];
  #pragma unroll
            for (int b = 0; b < B; ++b) {
              const bool use = valid && ((bits >> b) & 1u);
              float act;
              if constexpr (MODE == kModeDown) {
                act = act_prev[r][b];
              } else {
                const float g = __shfl_sync(0xffffffffu, t, ((r * B + b) * 2 + 0) * kLanesPer);
                const float u = __shfl_sync(0xffffffffu, t, ((r * B + b) * 2 + 1) * kLanesPer);
                act = use ? __fdividef(g, 1.f + __expf(-g)) * u : 0.f;
              }
              if constexpr (MODE == kModeGateUp) {
                if (use && tid == 0) {
                  a.act_out[b * a.ld_act_out + id] = act;
                  if (a.score_out != nullptr)
                    a.score_out[b * a.ld_score + id] = a.col_w != nullptr ? fabsf(act) * __ldg(a.col_w + id) : fabsf(act);
                }
                continue;
              }
              if (a.a_out != nullptr && tid == 0) store_as(a.a_out, b * a.lda + begin + i, a.a_dtype, act);
              if (use) {
  #pragma unroll
                for (int k = 0; k < VPT; ++k) {
                  const int v = tid + k * nthreads;
                  if (v < nslots) {
                    float df[8];
                    if constexpr (DN) {
                      int st = stage_prev + r;
                      if (st >= S) st -= S;
                      widen(load_pack8(reinterpret_cast<const T*>(smem + static_cast<size_t>(st) * a.copy_bytes) +
                                       2 * seg + 8 * v),
                            df);
                    } else {
                      widen(dn_prev[r][k], df);
                    }
  #pragma unroll
                    for (int e = 0; e < 8; ++e) yr[b][k][e] = fmaf(act, df[e], yr[b][k][e]);
                  }
                }
              }
            }
          }
        }
      }
    };
    auto dot_group = [&]() {
      if (rn > 0) {
        if constexpr (MODE == kModeDown) {
          // The given activations of this group's records, used next iteration.
  #pragma unroll
          for (int r = 0; r < R; ++r) {
            const int i = g0 + r;
            const int32_t id = r < rn ? s_ids[i] : -1;
            const unsigned bits = r < rn ? s_bits[i] : 0u;
  #pragma unroll
            for (int b = 0; b < B; ++b)
              act_cur[r][b] = (id >= 0 && ((bits >> b) & 1u)) ? load_as_f32(a.act_in, b * a.ld_act_in + id,
                                                                             a.act_in_dtype)
                                                              : 0.f;
          }
        }
        float part[VP];
  #pragma unroll
        for (int q = 0; q < VP; ++q) part[q] = 0.f;
  #pragma unroll
        for (int r = 0; r < R; ++r) {
          if (r < rn) {
            int stage = stage0 + r;
            uint32_t phase = phase0;
            if (stage >= S) {
              stage -= S;
              phase ^= 1u;
            }
            ok = ok && mbar_wait_bounded(&bars[stage], phase, kWaitLimitNs);
            const T* rec = reinterpret_cast<const T*>(smem + static_cast<size_t>(stage) * a.copy_bytes);
  #pragma unroll
            for (int k = 0; k < VPT; ++k) {
              const int v = tid + k * nthreads;
              if (v < nslots) {
                if constexpr (MODE == kModeFull && !DN) dn_cur[r][k] = load_pack8(rec + 2 * seg + 8 * v);
                if constexpr (MODE == kModeDown) dn_cur[r][k] = load_pack8(rec + 8 * v);
                if constexpr (MODE == kModeDown) continue;
                const Pack8<T> gr = load_pack8(rec + 8 * v);
                const Pack8<T> ur = load_pack8(rec + seg + 8 * v);
                float gf[8], uf[8];
                widen(gr, gf);
                widen(ur, uf);
  #pragma unroll
                for (int b = 0; b < B; ++b) {
                  float g0a = 0.f, g1a = 0.f, u0a = 0.f, u1a = 0.f;
  #pragma unroll
                  for (int e = 0; e < 8; e += 2) {
                    g0a = fmaf(xr[b][k][e], gf[e], g0a);
                    g1a = fmaf(xr[b][k][e + 1], gf[e + 1], g1a);
                    u0a = fmaf(xr[b][k][e], uf[e], u0a);
                    u1a = fmaf(xr[b][k][e + 1], uf[e + 1], u1a);
                  }
                  part[(r * B + b) * 2 + 0] += g0a + g1a;
                  part[(r * B + b) * 2 + 1] += u0a + u1a;
                }
              }
            }
          }
        }
        if constexpr (MODE != kModeDown) {
          const float wsum = warp_reduce_multi<VP>(part, lane);
          if ((lane % kLanesPer) == 0) s_red[(buf * VP + lane / kLanesPer) * 32 + warp] = wsum;
        }
      }
    };
    if constexpr (B <= 2) {
      finish_prev();
      dot_group();
    } else {
      dot_group();
      finish_prev();
    }
    if (rn <= 0) break;
    if (compute_barrier_or(!ok, nthreads)) {
      aborted = true;
      if (tid == 0) *reinterpret_cast<volatile int*>(s_flag) = 1;  // the producer stops refilling
      break;
    }
    // Every thread has its down slices of this group in registers (of the
    // previous group, with DN: finished above): release those slots to the
    // producer.
    if (tid == 0) {
      const int n_free = DN ? rn_prev : rn;
      const int st0 = DN ? stage_prev : stage0;
      for (int r = 0; r < n_free; ++r) {
        int stage = st0 + r;
        if (stage >= S) stage -= S;
        mbar_arrive(&empty[stage]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) dn_prev[r][k] = dn_cur[r][k];
      if constexpr (MODE == kModeDown) {
#pragma unroll
        for (int b = 0; b < B; ++b) act_prev[r][b] = act_cur[r][b];
      }
    }
    rn_prev = rn;
    buf ^= 1;
    stage_prev = stage0;
    stage0 += R;
    if (stage0 >= S) {
      stage0 -= S;
      phase0 ^= 1u;
    }
  }

  // After a give-up the producer drains the copies in flight (above).
  if (aborted && tid == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
  if constexpr (MODE == kModeGateUp) return;  // activations only: no partial y

  // Every CTA (also one with no records) stores its partial y row.  The row
  // has nvec = B * seg / 4 float4 columns; column c belongs to the slice
  // c / part_per of the reduce launch, and the partials are laid out
  // slice-major -- [slice][cta][slice width] float4, the last slice possibly
  // narrower -- so that each reduce CTA reads its slice of all rows as one
  // contiguous block and the rows take exactly grid * nvec words.
  const int per = a.part_per;
  const int grid = gridDim.x;
  const int nvec = B * seg / 4;
  auto part_index = [&](int c) {
    const int blk = c / per;
    const int width = min(per, nvec - blk * per);
    return static_cast<int64_t>(blk) * grid * per + static_cast<int64_t>(blockIdx.x) * width + (c - blk * per);
  };
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = tid + k * nthreads;
      if (v < nslots) {
        const int c = (b * seg + 8 * v) / 4;
        __stcg(a.partials + part_index(c), make_float4(yr[b][k][0], yr[b][k][1], yr[b][k][2], yr[b][k][3]));
        __stcg(a.partials + part_index(c + 1), make_float4(yr[b][k][4], yr[b][k][5], yr[b][k][6], yr[b][k][7]));
      }
    }
}

// Writes the four outputs of float4 column `col` (element e0 = 4 * col of the
// [B][seg] row) in the output dtype, adding y_in when given.
__device__ __forceinline__ void store_column(const ReduceArgs& a, int col, float4 acc) {
  const int e0 = col * 4;
  const int b = e0 / a.seg;
  const int h0 = e0 - b * a.seg;
  const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (h0 + e < a.hidden)
      store_as(a.y_out, b * a.ldy + h0 + e, a.y_dtype,
               vals[e] + (a.y_in != nullptr ? __ldg(a.y_in + b * a.ld_in + h0 + e) : 0.f));
}

// One CTA per column slice [blockIdx.x * per, + per).  Warp w sums columns
// w, w + nwarps, ... of the slice over all partial rows: lane l adds rows l,
// l + 32, ... (all loads in flight at once), then a shuffle tree -- a fixed
// order, so y does not depend on timing.  With several ranks, lane 0 stores
// the column sum into every rank's exchange buffer, then lane q < world polls
// this rank's buffer for rank q's sum and the warp adds them in rank order.
__global__ void __launch_bounds__(1024) decode_reduce_kernel(const ReduceArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int c0 = blockIdx.x * a.per;
  const int width = max(0, min(a.nvec, c0 + a.per) - c0);
  const float4* blk = a.partials + static_cast<int64_t>(blockIdx.x) * a.rows * a.per;  // [rows][width]
  const bool multi = a.world > 1;
  const unsigned int ep = multi ? *reinterpret_cast<const volatile unsigned int*>(a.epoch) : 0u;
  const int slot = static_cast<int>(ep % kXchgSlots);
  for (int col = warp; col < width; col += nwarps) {
    float4 v[kRowLoads];
#pragma unroll
    for (int u = 0; u < kRowLoads; ++u) {
      const int row = lane + 32 * u;
      v[u] = row < a.rows ? __ldcg(blk + static_cast<int64_t>(row) * width + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 acc = v[0];
#pragma unroll
    for (int u = 1; u < kRowLoads; ++u) {
      acc.x += v[u].x;
      acc.y += v[u].y;
      acc.z += v[u].z;
      acc.w += v[u].w;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
    }
    if (lane == 0) {
      if (!multi) {
        store_column(a, c0 + col, acc);
      } else {
        // -0.0 is the empty mark; the sum it stands for is +0.0.
        const uint4 w = make_uint4(__float_as_uint(acc.x) == kEmptyMark ? 0u : __float_as_uint(acc.x),
                                   __float_as_uint(acc.y) == kEmptyMark ? 0u : __float_as_uint(acc.y),
                                   __float_as_uint(acc.z) == kEmptyMark ? 0u : __float_as_uint(acc.z),
                                   __float_as_uint(acc.w) == kEmptyMark ? 0u : __float_as_uint(acc.w));
        const int64_t at = (static_cast<int64_t>(slot) * a.world + a.rank) * a.slot_words + c0 + col;
        for (int q = 0; q < a.world; ++q) st_relaxed_sys(reinterpret_cast<uint4*>(a.xchg[q]) + at, w);
      }
    }
  }
  if (!multi) return;

  // Sum over ranks in rank order, lane q waiting (bounded) for rank q's words.
  const unsigned long long cfg = *reinterpret_cast<const volatile unsigned long long*>(a.wait_limit);
  const uint64_t limit = cfg != 0ull ? cfg : kWaitLimitNs;
  uint4* mine = reinterpret_cast<uint4*>(a.xchg[a.rank]);
  bool failed = false;  // after one wait ran out, later waits of this warp do not wait again
  for (int col = warp; col < width; col += nwarps) {
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    bool ok = true;
    uint4* src = nullptr;
    if (lane < a.world) {
      src = mine + (static_cast<int64_t>(slot) * a.world + lane) * a.slot_words + c0 + col;
      w = ld_relaxed_sys(src);
      if (has_empty_mark(w)) {
        const uint64_t start = global_timer_ns();
        while (true) {
          w = ld_relaxed_sys(src);
          if (!has_empty_mark(w)) break;
          if (failed || global_timer_ns() - start > limit) {
            ok = false;
            break;
          }
        }
      }
    }
    if (!__all_sync(0xffffffffu, ok)) {
      failed = true;
      if (lane == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
      continue;
    }
    if (lane < a.world) *src = make_uint4(kEmptyMark, kEmptyMark, kEmptyMark, kEmptyMark);  // ready for e + 3
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < a.world; ++q) {
      acc.x += __uint_as_float(__shfl_sync(0xffffffffu, w.x, q));
      acc.y += __uint_as_float(__shfl_sync(0xffffffffu, w.y, q));
      acc.z += __uint_as_float(__shfl_sync(0xffffffffu, w.z, q));
      acc.w += __uint_as_float(__shfl_sync(0xffffffffu, w.w, q));
    }
    if (lane == 0) store_column(a, c0 + col, acc);
  }
  // The last CTA to finish advances the buffer's launch counter (every CTA
  // has read it in this launch) and resets the departure counter.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.depart, 1u) == gridDim.x - 1) {
      *a.depart = 0u;
      *a.epoch += 1u;
    }
  }
}

#include "decode_tc.cuh"

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using KernelFn = void (*)(const DecodeArgs);

// Records per barrier group: two for 16-bit weights (every mode and batch),
// one for fp32, whose records are twice the bytes.
template <typename T>
constexpr int group_records() {
  return sizeof(T) == 2 ? 2 : 1;
}

// Whole records at 3-4 tokens of 16-bit weights read their down slices from
// the ring (DN) instead of holding them in registers, so that two records per
// group fit the register budget.
template <typename T, int B, int MODE>
constexpr bool down_from_ring() {
  return MODE == kModeFull && sizeof(T) == 2 && B >= 3;
}

template <typename T, int B, int VPT, int MODE>
KernelFn kernel_for() {
  return indexed_ffn_decode_kernel<T, B, VPT, group_records<T>(), MODE, down_from_ring<T, B, MODE>()>;
}

// Slots of 8 hidden elements per thread: 1, 2 or 4 (hidden <= 2560, 5120,
// 10240).  Batch per launch: up to 4 tokens with <= 2 slots, 1 with 4.
template <typename T, int MODE>
KernelFn pick_kernel(int batch, int vpt) {
  if (vpt == 1 || vpt == 2) {
    switch (batch) {
      case 1: return vpt == 1 ? kernel_for<T, 1, 1, MODE>() : kernel_for<T, 1, 2, MODE>();
      case 2: return vpt == 1 ? kernel_for<T, 2, 1, MODE>() : kernel_for<T, 2, 2, MODE>();
      case 3: return vpt == 1 ? kernel_for<T, 3, 1, MODE>() : kernel_for<T, 3, 2, MODE>();
      case 4: return vpt == 1 ? kernel_for<T, 4, 1, MODE>() : kernel_for<T, 4, 2, MODE>();
      default: return nullptr;
    }
  }
  if (vpt == 4 && batch == 1) return kernel_for<T, 1, 4, MODE>();
  return nullptr;
}

template <typename T>
KernelFn pick_kernel_mode(int mode, int batch, int vpt) {
  if (mode == kModeGateUp) return pick_kernel<T, kModeGateUp>(batch, vpt);
  if (mode == kModeDown) return pick_kernel<T, kModeDown>(batch, vpt);
  return pick_kernel<T, kModeFull>(batch, vpt);
}

int vpt_for(int hidden_pad_) {
  const int nslots = hidden_pad_ / 8;
  for (int vpt = 1; vpt <= 4; vpt *= 2)
    if (nslots <= vpt * kMaxThreads) return vpt;
  return 0;
}


struct LaunchShape {
  int threads;
  int vpt;
  int stages;
  size_t ring;
  size_t smem;
};

size_t tail_bytes(int id_cap) {
  // mbarriers (filled, consumed), warp partials (at most 2 * 32 values x 32 warps), flag, id cache, token bits
  return 2 * kMaxStages * sizeof(uint64_t) + 2 * 32 * 32 * sizeof(float) + 4 * sizeof(int) +
         static_cast<size_t>(id_cap) * sizeof(int32_t) + (static_cast<size_t>(id_cap) + 15) / 16 * 16;
}

bool plan_launch(int hidden_pad, int64_t record_bytes, int max_smem, int id_cap, int max_stages, LaunchShape* out) {
  const int nslots = hidden_pad / 8;
  const int vpt = vpt_for(hidden_pad);
  if (vpt == 0) return false;
  const int per = (nslots + vpt - 1) / vpt;
  const int threads = std::max(32, (per + 31) / 32 * 32);
  const size_t tail = tail_bytes(id_cap);
  if (record_bytes <= 0 || static_cast<size_t>(max_smem) < tail) return false;
  int stages = static_cast<int>((static_cast<size_t>(max_smem) - tail) / static_cast<size_t>(record_bytes));
  stages = std::min(stages, max_stages);
  if (stages < 2) return false;
  out->threads = threads;
  out->vpt = vpt;
  out->stages = stages;
  out->ring = (static_cast<size_t>(stages) * record_bytes + 15) / 16 * 16;
  out->smem = out->ring + tail;
  return out->smem <= static_cast<size_t>(max_smem);
}

struct OccKey {
  const void* fn;
  int device;
  int threads;
  size_t smem;
  bool operator==(const OccKey& o) const {
    return fn == o.fn && device == o.device && threads == o.threads && smem == o.smem;
  }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return std::hash<const void*>()(k.fn) ^ (static_cast<size_t>(k.device) << 20) ^
           (static_cast<size_t>(k.threads) << 8) ^ (k.smem << 28);
  }
};

// Blocks per SM for a kernel configuration (after raising the kernel's
// dynamic shared-memory limit to the device maximum).  0 on failure.
template <typename Fn>
int blocks_per_sm(Fn fn, int device, int threads, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<OccKey, int, OccHash> cache;
  const OccKey key{reinterpret_cast<const void*>(fn), device, threads, smem};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (!ensure_max_dynamic_smem(reinterpret_cast<const void*>(fn), device)) return 0;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, threads, smem) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = nb;
  return nb;
}

// Both launches are programmatic dependents of what precedes them on the
// stream: the reduce launch is scheduled while the decode CTAs run (it waits
// for them at entry), and the next decode is scheduled while this reduce runs.
template <typename Fn, typename... Args>
bool launch_dependent(Fn fn, unsigned grid, unsigned threads, size_t smem, cudaStream_t stream, const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_ok(cudaLaunchKernelEx(&cfg, fn, args...));
}

}  // namespace

int decode_max_batch(int hidden, int dtype) {
  // The CUDA-core kernel's limit (4 tokens with <= 2 hidden slots per thread,
  // 1 with 4, none beyond), raised to the largest batch <= 8 that the
  // tensor-core kernel plans in every mode (227 KB of shared memory, a typical
  // id share): 8 up to hidden 6144, 6 up to 8192, 4 up to 10240.
  const int hp = hidden_pad(hidden, dtype);
  const int vpt = vpt_for(hp);
  const int cuda_cores = (vpt == 1 || vpt == 2) ? 4 : (vpt == 4 ? 1 : 0);
  if (cuda_cores == 0) return 0;
  for (int b = 8; b > cuda_cores; --b) {
    TcShape s;
    if (tc_plan(kModeFull, b, hp, dtype, 232448, 256, &s) && tc_plan(kModeGateUp, b, hp, dtype, 232448, 256, &s) &&
        tc_plan(kModeDown, b, hp, dtype, 232448, 256, &s))
      return b;
  }
  return cuda_cores;
}

size_t decode_workspace_bytes(int batch, int hidden, int dtype) {
  const int hp = hidden_pad(hidden, dtype);
  const size_t rows = static_cast<size_t>(kMaxGrid) * batch * hp * sizeof(float);
  return kWorkspaceHeader + (rows + 255) / 256 * 256;
}

namespace {

// Everything one call of the decode family needs; the entry points below
// fill the fields their mode uses.
struct DecodeRequest {
  int mode = kModeFull;
  const void* x = nullptr;
  int64_t ldx = 0;
  int batch = 0;
  int hidden = 0;
  const void* packed = nullptr;
  int64_t n_records = 0;
  int dtype = QCC_DTYPE_BF16;
  const void* ids = nullptr;
  int ids_kind = QCC_INDEX_I32;
  int n_ids = 0;
  const int32_t* n_ids_dev = nullptr;
  const uint8_t* token_mask = nullptr;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  void* y_out = nullptr;
  int64_t ldy = 0;
  int y_dtype = QCC_DTYPE_BF16;
  const float* y_in = nullptr;
  int64_t ld_in = 0;
  void* activation_out = nullptr;
  int64_t lda = 0;
  cudaStream_t stream = nullptr;
  void* const* xchg = nullptr;
  size_t xchg_bytes = 0;
  int world = 1;
  int rank = 0;
  int64_t id_lo = -1;
  int64_t id_hi = -1;
  // kModeGateUp
  float* act_out = nullptr;
  int64_t ld_act_out = 0;
  float* score_out = nullptr;
  int64_t ld_score = 0;
  const float* col_w = nullptr;
  // kModeDown
  const void* act_in = nullptr;
  int64_t ld_act_in = 0;
  int act_in_dtype = QCC_DTYPE_F32;
};

int launch_decode(const DecodeRequest& q) {
  const int mode = q.mode;
  if (!valid_dtype(q.dtype) || (mode != kModeGateUp && !valid_dtype(q.y_dtype))) return QCC_ERR_DTYPE;
  if (q.world < 1 || q.world > kMaxRanks || q.rank < 0 || q.rank >= q.world) return QCC_ERR_SHAPE;
  if (q.id_lo >= 0 && q.id_hi < q.id_lo) return QCC_ERR_SHAPE;
  if (mode != kModeGateUp && q.y_dtype != q.dtype && q.y_dtype != QCC_DTYPE_F32) return QCC_ERR_DTYPE;
  if ((q.ids_kind & ~(0xFF | QCC_IDS_READY | QCC_MASK_SHIFT(7))) != 0) return QCC_ERR_DTYPE;
  const int mask_shift = (q.ids_kind >> 12) & 7;
  const int ids_dtype = q.ids_kind & 0xFF;
  if (ids_dtype != QCC_INDEX_I32 && ids_dtype != QCC_INDEX_I64) return QCC_ERR_DTYPE;
  if (mode == kModeDown && !valid_dtype(q.act_in_dtype)) return QCC_ERR_DTYPE;
  if (q.batch < 1 || q.hidden < 1 || q.n_records < 0 || q.n_ids < 0) return QCC_ERR_SHAPE;
  if (mask_shift + q.batch > 8) return QCC_ERR_SHAPE;  // the tokens' bits must lie in the mask byte
  if (q.batch > decode_max_batch(q.hidden, q.dtype)) return QCC_ERR_UNSUPPORTED;
  if (mode != kModeDown && q.ldx < q.hidden) return QCC_ERR_SHAPE;
  if (mode != kModeGateUp && q.ldy < q.hidden) return QCC_ERR_SHAPE;
  if (q.activation_out != nullptr && q.lda < q.n_ids) return QCC_ERR_SHAPE;
  if (q.y_in != nullptr && q.ld_in < q.hidden) return QCC_ERR_SHAPE;
  if (mode == kModeGateUp && (q.ld_act_out < q.n_records || (q.score_out != nullptr && q.ld_score < q.n_records)))
    return QCC_ERR_SHAPE;
  if (mode == kModeDown && q.ld_act_in < q.n_records) return QCC_ERR_SHAPE;
  if (q.workspace == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (mode != kModeDown && q.x == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (mode != kModeGateUp && q.y_out == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (mode == kModeGateUp && q.act_out == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (mode == kModeDown && q.act_in == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  // An empty shard (n_records 0, e.g. an empty slice whose pointer is NULL)
  // reads no record: every id is outside it.
  if (q.n_ids > 0 && ((q.ids == nullptr && mode != kModeGateUp) || (q.packed == nullptr && q.n_records > 0)))
    return QCC_ERR_INVALID_ARGUMENT;
  if (q.workspace_bytes < decode_workspace_bytes(q.batch, q.hidden, q.dtype)) return QCC_ERR_WORKSPACE;
  if (!aligned16(q.packed) || !aligned16(q.workspace)) return QCC_ERR_ALIGNMENT;

  const int hp = hidden_pad(q.hidden, q.dtype);
  const int nvec = q.batch * hp / 4;
  int64_t slot_words = 0;
  if (q.world > 1) {
    if (q.xchg == nullptr) return QCC_ERR_INVALID_ARGUMENT;
    for (int r = 0; r < q.world; ++r)
      if (q.xchg[r] == nullptr || !aligned16(q.xchg[r])) return QCC_ERR_INVALID_ARGUMENT;
    // Slots are spaced by the buffer's capacity (the same on every rank), not
    // by this call's batch, so calls with different batches never overlap.
    if (q.xchg_bytes <= static_cast<size_t>(kXchgHeader)) return QCC_ERR_WORKSPACE;
    slot_words =
        static_cast<int64_t>((q.xchg_bytes - kXchgHeader) / (static_cast<size_t>(kXchgSlots) * q.world * 16));
    if (slot_words < nvec) return QCC_ERR_WORKSPACE;
  }
  const int64_t rec = record_bytes(q.hidden, q.dtype);
  const int64_t part = rec / 3;  // one of the gate / up / down parts (Hp elements)
  const int64_t copy_offset = mode == kModeDown ? 2 * part : 0;
  const int64_t copy_bytes = mode == kModeFull ? rec : (mode == kModeGateUp ? 2 * part : part);
  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const DeviceInfo& info = device_info(device);
  if (info.num_sms <= 0) return QCC_ERR_CUDA;

  // Ids per CTA never exceed ceil(n_ids / min(#SMs, n_ids)): the grid is at
  // least that large whenever it is smaller than n_ids.
  const int n_ids = q.n_ids;
  const int id_cap = std::max(1, (n_ids + std::min(info.num_sms, std::max(1, n_ids)) - 1) /
                                     std::min(info.num_sms, std::max(1, n_ids)));
  // 2-8 tokens of 16-bit records run on the tensor cores; one token, fp32
  // records and hidden sizes that are not a multiple of 128 on the CUDA cores.
  TcShape tc_shape;
  const bool use_tc = tc_plan(mode, q.batch, hp, q.dtype, info.max_smem_optin, id_cap, &tc_shape);
  LaunchShape shape = {};
  KernelFn fn = nullptr;
  TcKernelFn tc_fn = nullptr;
  int block = 0;
  size_t smem = 0;
  if (use_tc) {
    tc_fn = q.dtype == QCC_DTYPE_BF16 ? pick_tc_kernel<__nv_bfloat16>(mode, q.batch) : pick_tc_kernel<__half>(mode, q.batch);
    if (tc_fn == nullptr) return QCC_ERR_UNSUPPORTED;
    block = kTcThreads;
    smem = tc_smem_bytes(tc_shape, id_cap);
    if (blocks_per_sm(tc_fn, device, block, smem) <= 0) return QCC_ERR_CUDA;
  } else {
    if (!plan_launch(hp, copy_bytes, info.max_smem_optin, id_cap, mode == kModeFull ? kMaxStagesFull : kMaxStages,
                     &shape))
      return QCC_ERR_UNSUPPORTED;
    if (q.dtype == QCC_DTYPE_BF16)
      fn = pick_kernel_mode<__nv_bfloat16>(mode, q.batch, shape.vpt);
    else if (q.dtype == QCC_DTYPE_F16)
      fn = pick_kernel_mode<__half>(mode, q.batch, shape.vpt);
    else
      fn = pick_kernel_mode<float>(mode, q.batch, shape.vpt);
    if (fn == nullptr) return QCC_ERR_UNSUPPORTED;
    block = shape.threads + 32;  // compute threads and the producer warp
    smem = shape.smem;
    if (blocks_per_sm(fn, device, block, smem) <= 0) return QCC_ERR_CUDA;
  }
  // At most one CTA per SM (the workspace holds kMaxGrid partial rows); no
  // CTA waits for another, so residency of the whole grid is not required.
  int64_t grid = std::min<int64_t>(info.num_sms, kMaxGrid);
  if (q.n_ids_dev == nullptr && q.id_lo < 0) grid = std::min<int64_t>(grid, std::max(1, n_ids));
  // Reduce launch: one CTA per column slice, about one slice per SM.
  const int slices_wanted = std::max(1, std::min(info.num_sms, nvec));
  const int per = (nvec + slices_wanted - 1) / slices_wanted;
  const int slices = (nvec + per - 1) / per;
  const int reduce_threads = 32 * std::min(per, 32);

  uint8_t* ws = static_cast<uint8_t*>(q.workspace);
  float4* partials = reinterpret_cast<float4*>(ws + kWorkspaceHeader);

  DecodeArgs args;
  args.x = q.x;
  args.ldx = q.ldx;
  args.packed = static_cast<const uint8_t*>(q.packed);
  args.record_bytes = rec;
  args.n_records = q.n_records;
  args.hidden = q.hidden;
  args.hidden_pad = hp;
  args.ids = q.ids;
  args.ids64 = ids_dtype == QCC_INDEX_I64;
  args.ids_ready = (q.ids_kind & QCC_IDS_READY) != 0;
  args.token_mask = q.token_mask;
  args.mask_shift = mask_shift;
  args.n_ids = n_ids;
  args.n_ids_dev = q.n_ids_dev;
  args.status = reinterpret_cast<unsigned int*>(ws);
  args.partials = partials;
  args.part_per = per;
  args.a_out = q.activation_out;
  args.lda = q.lda;
  args.a_dtype = q.dtype;
  args.stages = shape.stages;
  args.id_cap = id_cap;
  args.ring_bytes = static_cast<int64_t>(shape.ring);
  args.x_vec = q.x != nullptr && (q.hidden % 8 == 0) && aligned16(q.x) && ((q.ldx * dtype_bytes(q.dtype)) % 16 == 0);
  args.id_lo = q.id_lo >= 0 ? q.id_lo : -1;
  args.id_hi = q.id_lo >= 0 ? q.id_hi : -1;
  args.copy_offset = copy_offset;
  args.copy_bytes = static_cast<int>(copy_bytes);
  args.act_out = q.act_out;
  args.ld_act_out = q.ld_act_out;
  args.score_out = q.score_out;
  args.ld_score = q.ld_score;
  args.col_w = q.col_w;
  args.act_in = q.act_in;
  args.ld_act_in = q.ld_act_in;
  args.act_in_dtype = q.act_in_dtype;

  clear_stale_error();
  const bool launched = use_tc ? launch_dependent(tc_fn, static_cast<unsigned>(grid), static_cast<unsigned>(block),
                                                  smem, q.stream, args, tc_shape)
                               : launch_dependent(fn, static_cast<unsigned>(grid), static_cast<unsigned>(block), smem,
                                                  q.stream, args);
  if (!launched) return QCC_ERR_CUDA;
  if (mode == kModeGateUp) return QCC_OK;  // no partial rows to reduce

  ReduceArgs red;
  red.partials = partials;
  red.rows = static_cast<int>(grid);
  red.per = per;
  red.nvec = nvec;
  red.seg = hp;
  red.hidden = q.hidden;
  red.y_out = q.y_out;
  red.ldy = q.ldy;
  red.y_dtype = q.y_dtype;
  red.y_in = q.y_in;
  red.ld_in = q.ld_in;
  red.status = reinterpret_cast<unsigned int*>(ws);
  red.depart = reinterpret_cast<unsigned int*>(ws + 8);
  red.world = q.world;
  red.rank = q.rank;
  red.slot_words = slot_words;
  red.epoch = q.world > 1 ? static_cast<unsigned int*>(q.xchg[q.rank]) : nullptr;
  red.wait_limit = q.world > 1 ? reinterpret_cast<const unsigned long long*>(
                                     static_cast<const uint8_t*>(q.xchg[q.rank]) + kXchgLimitOffset)
                               : nullptr;
  for (int r = 0; r < kMaxRanks; ++r)
    red.xchg[r] = r < q.world && q.world > 1 ? static_cast<uint8_t*>(q.xchg[r]) + kXchgHeader : nullptr;
  if (!launch_dependent(decode_reduce_kernel, static_cast<unsigned>(slices), static_cast<unsigned>(reduce_threads), 0,
                        q.stream, red))
    return QCC_ERR_CUDA;
  return QCC_OK;
}

}  // namespace

int indexed_ffn_decode(const void* x, int64_t ldx, int batch, int hidden, const void* packed, int64_t n_records,
                       int dtype, const void* ids, int ids_kind, int n_ids, const int32_t* n_ids_dev,
                       const uint8_t* token_mask, void* workspace, size_t workspace_bytes, void* y_out, int64_t ldy,
                       int y_dtype, const float* y_in, int64_t ld_in, void* activation_out, int64_t lda,
                       cudaStream_t stream, void* const* xchg, size_t xchg_bytes, int world, int rank,
                       int64_t id_lo, int64_t id_hi) {
  DecodeRequest q;
  q.x = x;
  q.ldx = ldx;
  q.batch = batch;
  q.hidden = hidden;
  q.packed = packed;
  q.n_records = n_records;
  q.dtype = dtype;
  q.ids = ids;
  q.ids_kind = ids_kind;
  q.n_ids = n_ids;
  q.n_ids_dev = n_ids_dev;
  q.token_mask = token_mask;
  q.workspace = workspace;
  q.workspace_bytes = workspace_bytes;
  q.y_out = y_out;
  q.ldy = ldy;
  q.y_dtype = y_dtype;
  q.y_in = y_in;
  q.ld_in = ld_in;
  q.activation_out = activation_out;
  q.lda = lda;
  q.stream = stream;
  q.xchg = xchg;
  q.xchg_bytes = xchg_bytes;
  q.world = world;
  q.rank = rank;
  q.id_lo = id_lo;
  q.id_hi = id_hi;
  return launch_decode(q);
}

size_t exchange_bytes(int world, int batch, int hidden, int dtype) {
  if (world < 1 || world > kMaxRanks || batch < 1 || hidden < 1 || !valid_dtype(dtype)) return 0;
  const size_t nvec = static_cast<size_t>(batch) * hidden_pad(hidden, dtype) / 4;
  return kXchgHeader + static_cast<size_t>(kXchgSlots) * world * nvec * 16;
}

}  // namespace qcc

extern "C" int qcc_decode_max_batch(int hidden, int dtype) {
  if (hidden < 1 || !qcc::valid_dtype(dtype)) return 0;
  return qcc::decode_max_batch(hidden, dtype);
}

extern "C" size_t qcc_decode_workspace_bytes(int batch, int hidden, int dtype) {
  if (batch < 1 || hidden < 1 || !qcc::valid_dtype(dtype)) return 0;
  return qcc::decode_workspace_bytes(batch, hidden, dtype);
}

extern "C" int qcc_indexed_ffn_decode(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                      int64_t n_records, int dtype, const void* ids, int ids_dtype, int n_ids,
                                      const int32_t* n_ids_dev, const uint8_t* token_mask, void* workspace,
                                      size_t workspace_bytes, void* y_out, int64_t ldy, int y_dtype,
                                      const float* y_in, int64_t ld_in, void* activation_out, int64_t lda,
                                      cudaStream_t stream) {
  return qcc::indexed_ffn_decode(x, ldx, batch, hidden, packed, n_records, dtype, ids, ids_dtype, n_ids, n_ids_dev,
                                 token_mask, workspace, workspace_bytes, y_out, ldy, y_dtype, y_in, ld_in,
                                 activation_out, lda, stream);
}

extern "C" size_t qcc_exchange_bytes(int world, int batch, int hidden, int dtype) {
  return qcc::exchange_bytes(world, batch, hidden, dtype);
}

extern "C" int qcc_indexed_ffn_decode_allreduce(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                                int64_t n_records, int dtype, const void* ids, int ids_dtype,
                                                int n_ids, const int32_t* n_ids_dev, const uint8_t* token_mask,
                                                void* workspace, size_t workspace_bytes, void* y_out, int64_t ldy,
                                                int y_dtype, const float* y_in, int64_t ld_in, int64_t id_begin,
                                                int64_t id_end, void* const* exchange, size_t exchange_bytes,
                                                int world, int rank, cudaStream_t stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return QCC_ERR_SHAPE;
  if (world > 1 && exchange_bytes < qcc::exchange_bytes(world, batch, hidden, dtype)) return QCC_ERR_WORKSPACE;
  return qcc::indexed_ffn_decode(x, ldx, batch, hidden, packed, n_records, dtype, ids, ids_dtype, n_ids, n_ids_dev,
                                 token_mask, workspace, workspace_bytes, y_out, ldy, y_dtype, y_in, ld_in, nullptr, 0,
                                 stream, exchange, exchange_bytes, world, rank, id_begin, id_end);
}

namespace qcc {
namespace {

int activation_pass(const void* x, int64_t ldx, int batch, int hidden, const void* packed, int64_t n_records,
                    int dtype, const float* col_weights, float* act_out, int64_t ld_act, float* scores_out,
                    int64_t ld_scores, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  DecodeRequest q;
  q.mode = kModeGateUp;
  q.x = x;
  q.ldx = ldx;
  q.batch = batch;
  q.hidden = hidden;
  q.packed = packed;
  q.n_records = n_records;
  q.dtype = dtype;
  q.n_ids = n_records > 0x7fffffff ? -1 : static_cast<int>(n_records);  // every record, in order
  q.workspace = workspace;
  q.workspace_bytes = workspace_bytes;
  q.stream = stream;
  q.act_out = act_out;
  q.ld_act_out = ld_act;
  q.score_out = scores_out;
  q.ld_score = ld_scores;
  q.col_w = col_weights;
  return launch_decode(q);
}

}  // namespace
}  // namespace qcc

extern "C" int qcc_ffn_activations(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                   int64_t n_records, int dtype, const float* col_weights, float* act_out,
                                   int64_t ld_act, float* scores_out, int64_t ld_scores, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
  return qcc::activation_pass(x, ldx, batch, hidden, packed, n_records, dtype, col_weights, act_out, ld_act,
                              scores_out, ld_scores, workspace, workspace_bytes, stream);
}

extern "C" int qcc_indexed_ffn_down(const void* act, int64_t ld_act, int act_dtype, int batch, int hidden,
                                    const void* packed, int64_t n_records, int dtype, const void* ids, int ids_dtype,
                                    int n_ids, const int32_t* n_ids_dev, const uint8_t* token_mask, void* workspace,
                                    size_t workspace_bytes, void* y_out, int64_t ldy, int y_dtype, const float* y_in,
                                    int64_t ld_in, cudaStream_t stream) {
  qcc::DecodeRequest q;
  q.mode = qcc::kModeDown;
  q.batch = batch;
  q.hidden = hidden;
  q.packed = packed;
  q.n_records = n_records;
  q.dtype = dtype;
  q.ids = ids;
  q.ids_kind = ids_dtype;
  q.n_ids = n_ids;
  q.n_ids_dev = n_ids_dev;
  q.token_mask = token_mask;
  q.workspace = workspace;
  q.workspace_bytes = workspace_bytes;
  q.y_out = y_out;
  q.ldy = ldy;
  q.y_dtype = y_dtype;
  q.y_in = y_in;
  q.ld_in = ld_in;
  q.stream = stream;
  q.act_in = act;
  q.ld_act_in = ld_act;
  q.act_in_dtype = act_dtype;
  return qcc::launch_decode(q);
}
