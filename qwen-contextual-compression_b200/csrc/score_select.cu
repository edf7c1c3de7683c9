// Fused score producer + top-K selector (sm_100a).
//
// One cooperative launch replaces the reference's runtime selector path:
// runtime/cuda_selector.py:30-40 (latent_kernel: the encoder GEMV, SiLU,
// residual MLP and LayerNorm in one CTA; head_kernel: one 32-thread CTA per
// neuron) followed by torch.topk(scores, k, sorted=False)
// (runtime/selector.py:24), with the input normalisation folded into the
// encoder as runtime/selector.py:31-38 does.  Per token row:
//   kind 0 (ResidualFactorizedPredictor, predictor/models.py:17-36):
//     r = silu(E x + e); u = silu(F1 r + f1); v = F2 u + f2 + r;
//     z = LayerNorm(v) * g + b
//   kind 1 (FactorizedPredictor, predictor/models.py:6-14): z = E x (+ e)
//   s = W z + w;  ids = the k largest s, ascending, ties to the lower index.
// Everything is computed in fp32; the weights and x are bf16, fp16 or fp32.
//
// The grid holds one group of `cpr` CTAs per row.  A group runs five phases
// separated by four bounded group barriers (a counter per row):
//  1. encoder: (latent output, 512-wide chunk of H) items over the group's
//     warps, each dot product stored to its own slot (no float atomics, so
//     the scores do not depend on timing);
//  2. every CTA sums the slots in a fixed order, runs the latent MLP and the
//     LayerNorm in shared memory (L <= 256), scores its slice of the N
//     neurons into shared memory as order-preserving keys, and adds its
//     12-bit top-digit histogram into the row's global histogram;
//  3. every CTA finds the bin of the k-th largest key and appends its keys of
//     that bin to the row's candidate list;
//  4. every CTA finishes the exact k-th key T over the candidates (two 10-bit
//     digits) and counts its slice's keys above and equal to T;
//  5. every CTA turns the per-CTA counts into its output offset and writes
//     its selected indices, ascending.
// The workspace is left as found (zero counters and histograms) by every
// call that completes.

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <mutex>
#include <string>
#include <unordered_map>

#include "qcc_common.cuh"
#include "qcc_host.h"

namespace qcc {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxLatent = 256;
constexpr int kMaxRows = 32;           // rows per launch (the host loops over more)
constexpr int kMaxCpr = 256;           // CTAs per row
constexpr int kSliceCap = 4096;        // neurons per CTA slice (keys in shared memory)
constexpr int kEncChunk = 512;         // H elements per encoder item (16 per lane)
constexpr int kTop = 4096;             // 12-bit top digit
constexpr int kLow = 1024;             // 10-bit digits
constexpr int kHeader = 512;           // status, depart, barrier counters, candidate counts
constexpr int kBarOffset = 64;         // u32 barrier counter per row
constexpr int kCandCountOffset = kBarOffset + 4 * kMaxRows;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
static_assert(kCandCountOffset + 4 * kMaxRows <= kHeader, "selector workspace header");

struct SelArgs {
  const void* x;
  int64_t ldx;
  int rows;
  int hidden;
  int latent;
  int n;
  int kind;
  const void* enc_w;
  const void* enc_b;
  const void* fc1_w;
  const void* fc1_b;
  const void* fc2_w;
  const void* fc2_b;
  const void* ln_w;
  const void* ln_b;
  float eps;
  const void* out_w;
  const void* out_b;
  int k;
  int32_t* ids;
  int64_t ld_ids;
  float* scores;
  int64_t ld_scores;
  int cpr;
  int nchunk;
  int vec_fc;   // fc1 / fc2 rows load as 16-byte pieces
  int vec_out;  // head rows load as 16-byte pieces
  unsigned int* status;
  unsigned int* depart;
  unsigned int* bar;         // [rows]
  unsigned int* cand_count;  // [rows]
  float* enc_part;           // [rows][latent * nchunk]
  unsigned int* hist;        // [rows][kTop]
  uint2* cand;               // [rows][n] (key, index)
  int2* counts;              // [rows][cpr] (above T, equal to T)
};

template <typename T>
__device__ __forceinline__ float ld_f(const void* p, int64_t i) {
  return to_f32<T>(reinterpret_cast<const T*>(p)[i]);
}

template <typename T>
__device__ __forceinline__ float ld_opt(const void* p, int64_t i, float dflt) {
  return p != nullptr ? to_f32<T>(reinterpret_cast<const T*>(p)[i]) : dflt;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.f + __expf(-v)); }

// Dot product of one weight row (L elements) with a vector in shared memory.
// With vec (L % 8 == 0, 16-byte aligned rows) the row streams in 16-byte
// pieces, eight in flight.
template <typename T>
__device__ __forceinline__ float dot_row(const T* w, const float* z, int L, bool vec) {
  float acc = 0.f;
  if (vec) {
#pragma unroll 8
    for (int j = 0; j < L; j += 8) {
      float f[8];
      widen(load_global_pack8<T>(w + j), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(f[e], z[j + e], acc);
    }
  } else {
#pragma unroll 8
    for (int j = 0; j < L; ++j) acc = fmaf(to_f32<T>(w[j]), z[j], acc);
  }
  return acc;
}

// The same over a row staged in shared memory (16-byte pieces when L % 8 == 0;
// staged rows start on 16-byte boundaries whenever L * sizeof(T) % 16 == 0).
template <typename T>
__device__ __forceinline__ float dot_row_smem(const T* w, const float* z, int L) {
  float acc = 0.f;
  if ((L & 7) == 0) {
#pragma unroll 4
    for (int j = 0; j < L; j += 8) {
      float f[8];
      widen(load_pack8<T>(w + j), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(f[e], z[j + e], acc);
    }
  } else {
    for (int j = 0; j < L; ++j) acc = fmaf(to_f32<T>(w[j]), z[j], acc);
  }
  return acc;
}

// dot_row_smem for rows read one per thread: each thread starts at a
// different 16-byte piece of its row, so that the eight threads of a
// 128-byte shared-memory wavefront hit eight different bank groups (rows of
// 64 bytes would otherwise put sixteen threads of a warp on the same banks).
template <typename T>
__device__ __forceinline__ float dot_row_smem_rot(const T* w, const float* z, int L, int t) {
  if ((L & 7) != 0) return dot_row_smem<T>(w, z, L);
  const int row_bytes = L * static_cast<int>(sizeof(T));
  const int pieces = L / 8;  // 8-element pieces of the row
  const int rot = row_bytes < 128 ? t / (128 / row_bytes) : t;
  float acc = 0.f;
#pragma unroll 4
  for (int c = 0; c < pieces; ++c) {
    int j = c + rot;
    j %= pieces;
    float f[8];
    widen(load_pack8<T>(w + 8 * j), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(f[e], z[8 * j + e], acc);
  }
  return acc;
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Group barrier number `gen` (1-based) of the CTAs of one row: bounded spin on
// the row's counter.  Returns false (and flags QCC_DEV_TIMEOUT) on timeout.
__device__ __forceinline__ bool group_barrier(const SelArgs& a, int row, int gen, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.bar + row, 1u);
    const unsigned int target = static_cast<unsigned int>(gen * a.cpr);
    const uint64_t start = global_timer_ns();
    int ok = 1;
    while (ld_acquire_u32(a.bar + row) < target) {
      if (global_timer_ns() - start > kWaitLimitNs) {
        atomicOr(a.status, QCC_DEV_TIMEOUT);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) score_select_kernel(const SelArgs a) {
  __shared__ float s_r[kMaxLatent];
  __shared__ float s_u[kMaxLatent];
  __shared__ float s_z[kMaxLatent];
  __shared__ uint32_t s_keys[kSliceCap];
  __shared__ int s_hist[kTop];
  __shared__ int s_scan[33];
  __shared__ int s_ok;
  __shared__ int s_bin, s_rem;
  __shared__ float s_stat[2];
  __shared__ int s_base, s_sel_base, s_eq_base;
  __shared__ int2 s_counts[kMaxCpr];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x / a.cpr;
  const int lc = blockIdx.x - row * a.cpr;
  const int L = a.latent;
  const int H = a.hidden;
  const int N = a.n;
  const int n0 = static_cast<int>((static_cast<int64_t>(N) * lc) / a.cpr);
  const int n1 = static_cast<int>((static_cast<int64_t>(N) * (lc + 1)) / a.cpr);
  const int len = n1 - n0;
  const int items = L * a.nchunk;
  float* part = a.enc_part + static_cast<int64_t>(row) * items;
  unsigned int* ghist = a.hist + static_cast<int64_t>(row) * kTop;
  uint2* cand = a.cand + static_cast<int64_t>(row) * N;
  int2* counts = a.counts + static_cast<int64_t>(row) * a.cpr;
  bool ok = true;

  // 1. Encoder dot products, one (output, chunk) item per warp at a time.
  {
    const T* xr = reinterpret_cast<const T*>(a.x) + static_cast<int64_t>(row) * a.ldx;
    for (int item = lc * kWarps + warp; item < items; item += a.cpr * kWarps) {
      const int l = item / a.nchunk;
      const int h0 = (item - l * a.nchunk) * kEncChunk;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < kEncChunk / 32; ++j) {
        const int h = h0 + lane + 32 * j;
        if (h < H) acc = fmaf(to_f32<T>(xr[h]), ld_f<T>(a.enc_w, static_cast<int64_t>(l) * H + h), acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) part[item] = acc;
    }
  }
  ok = group_barrier(a, row, 1, &s_ok);

  // 2. Latent MLP (every CTA of the group, identical order), scores of this
  //    slice, local top-digit histogram into the row's histogram.
  if (ok) {
    for (int b = tid; b < kTop; b += kThreads) s_hist[b] = 0;
    for (int l = tid; l < L; l += kThreads) {
      float pre = ld_opt<T>(a.enc_b, l, 0.f);
      for (int c = 0; c < a.nchunk; ++c) pre += __ldcg(part + l * a.nchunk + c);
      if (a.kind == 0)
        s_r[l] = silu_f(pre);
      else
        s_z[l] = pre;
    }
    __syncthreads();
    if (a.kind == 0) {
      // One thread per output row (L <= blockDim): every row's loads in flight at once.
      for (int l = tid; l < L; l += kThreads) {
        const float acc = dot_row<T>(reinterpret_cast<const T*>(a.fc1_w) + static_cast<int64_t>(l) * L, s_r, L, a.vec_fc);
        s_u[l] = silu_f(acc + ld_opt<T>(a.fc1_b, l, 0.f));
      }
      __syncthreads();
      for (int l = tid; l < L; l += kThreads) {
        const float acc = dot_row<T>(reinterpret_cast<const T*>(a.fc2_w) + static_cast<int64_t>(l) * L, s_u, L, a.vec_fc);
        s_z[l] = acc + ld_opt<T>(a.fc2_b, l, 0.f) + s_r[l];
      }
      __syncthreads();
      if (warp == 0) {
        float sum = 0.f;
        for (int j = lane; j < L; j += 32) sum += s_z[j];
        const float mean = warp_sum(sum) / static_cast<float>(L);
        float sq = 0.f;
        for (int j = lane; j < L; j += 32) {
          const float d = s_z[j] - mean;
          sq = fmaf(d, d, sq);
        }
        const float var = warp_sum(sq) / static_cast<float>(L);
        if (lane == 0) {
          s_stat[0] = mean;
          s_stat[1] = rsqrtf(var + a.eps);
        }
      }
      __syncthreads();
      for (int l = tid; l < L; l += kThreads)
        s_z[l] = (s_z[l] - s_stat[0]) * s_stat[1] * ld_opt<T>(a.ln_w, l, 1.f) + ld_opt<T>(a.ln_b, l, 0.f);
    }
    __syncthreads();
    // Scores of neurons n0 .. n1-1: one thread per neuron.
    for (int i = tid; i < len; i += kThreads) {
      const int n = n0 + i;
      const float s = dot_row<T>(reinterpret_cast<const T*>(a.out_w) + static_cast<int64_t>(n) * L, s_z, L, a.vec_out) +
                      ld_opt<T>(a.out_b, n, 0.f);
      s_keys[i] = score_key(s);
      if (a.scores != nullptr) a.scores[static_cast<int64_t>(row) * a.ld_scores + n] = s;
    }
    __syncthreads();
    for (int i = tid; i < len; i += kThreads) atomicAdd(&s_hist[s_keys[i] >> 20], 1);
    __syncthreads();
    for (int b = tid; b < kTop; b += kThreads)
      if (s_hist[b] != 0) atomicAdd(ghist + b, static_cast<unsigned int>(s_hist[b]));
  }
  ok = group_barrier(a, row, 2, &s_ok) && ok;

  // 3. The top-digit bin of the k-th key; this slice's keys of that bin join
  //    the row's candidate list.
  int bin = 0, rem = 0;
  if (ok) {
    for (int b = tid; b < kTop; b += kThreads) s_hist[b] = static_cast<int>(__ldcg(ghist + b));
    __syncthreads();
    find_bin<kTop / kThreads>(s_hist, a.k, s_scan, &s_bin, &s_rem);
    __syncthreads();
    bin = s_bin;
    rem = s_rem;
    int mine = 0;
    for (int i = tid; i < len; i += kThreads) mine += (s_keys[i] >> 20) == static_cast<uint32_t>(bin) ? 1 : 0;
    int total;
    int pos = block_exclusive_scan(mine, s_scan, &total);
    if (tid == 0) s_base = total > 0 ? static_cast<int>(atomicAdd(a.cand_count + row, static_cast<unsigned>(total))) : 0;
    __syncthreads();
    pos += s_base;
    for (int i = tid; i < len; i += kThreads)
      if ((s_keys[i] >> 20) == static_cast<uint32_t>(bin)) cand[pos++] = make_uint2(s_keys[i], static_cast<uint32_t>(n0 + i));
  }
  ok = group_barrier(a, row, 3, &s_ok) && ok;

  // 4. The exact k-th key over the candidates, then this slice's counts.
  uint32_t thr = 0;
  int need_eq = 0;
  if (ok) {
    const int m = static_cast<int>(ld_acquire_u32(a.cand_count + row));
    for (int b = tid; b < kLow; b += kThreads) s_hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < m; i += kThreads) atomicAdd(&s_hist[(__ldcg(&cand[i].x) >> 10) & (kLow - 1)], 1);
    __syncthreads();
    find_bin<kLow / kThreads>(s_hist, rem, s_scan, &s_bin, &s_rem);
    __syncthreads();
    const int bin_a = s_bin;
    const int rem_a = s_rem;
    __syncthreads();
    for (int b = tid; b < kLow; b += kThreads) s_hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < m; i += kThreads) {
      const uint32_t key = __ldcg(&cand[i].x);
      if (((key >> 10) & (kLow - 1)) == static_cast<uint32_t>(bin_a)) atomicAdd(&s_hist[key & (kLow - 1)], 1);
    }
    __syncthreads();
    find_bin<kLow / kThreads>(s_hist, rem_a, s_scan, &s_bin, &s_rem);
    __syncthreads();
    thr = (static_cast<uint32_t>(bin) << 20) | (static_cast<uint32_t>(bin_a) << 10) | static_cast<uint32_t>(s_bin);
    need_eq = s_rem;
    int gt = 0, eq = 0;
    for (int i = tid; i < len; i += kThreads) {
      gt += s_keys[i] > thr ? 1 : 0;
      eq += s_keys[i] == thr ? 1 : 0;
    }
    int tot_gt, tot_eq;
    (void)block_exclusive_scan(gt, s_scan, &tot_gt);
    (void)block_exclusive_scan(eq, s_scan, &tot_eq);
    if (tid == 0) counts[lc] = make_int2(tot_gt, tot_eq);
    // Every CTA of the row read the histogram before barrier 3: clear this
    // CTA's share of it for the next call.
    const int b0 = (kTop * lc) / a.cpr, b1 = (kTop * (lc + 1)) / a.cpr;
    for (int b = b0 + tid; b < b1; b += kThreads) ghist[b] = 0u;
  }
  ok = group_barrier(a, row, 4, &s_ok) && ok;

  // 5. Output offsets from the per-CTA counts; selected indices ascending.
  if (ok) {
    for (int q = tid; q < a.cpr; q += kThreads) {
      const int2* src = counts + q;
      s_counts[q] = make_int2(__ldcg(&src->x), __ldcg(&src->y));
    }
    __syncthreads();
    if (tid == 0) {
      int sel = 0, eqb = 0;
      for (int q = 0; q < lc; ++q) {
        sel += s_counts[q].x + min(s_counts[q].y, max(0, need_eq - eqb));
        eqb += s_counts[q].y;
      }
      s_sel_base = sel;
      s_eq_base = eqb;
      // Every CTA read the candidate count in phase 4: reset it for the next call.
      if (lc == 0) a.cand_count[row] = 0u;
    }
    __syncthreads();
    const int per = (len + kThreads - 1) / kThreads;
    const int c0 = min(len, tid * per), c1 = min(len, c0 + per);
    int eq = 0;
    for (int i = c0; i < c1; ++i) eq += s_keys[i] == thr ? 1 : 0;
    int tot;
    const int eq_before = s_eq_base + block_exclusive_scan(eq, s_scan, &tot);
    int sel = 0;
    {
      int e = eq_before;
      for (int i = c0; i < c1; ++i) {
        const uint32_t key = s_keys[i];
        if (key > thr) {
          ++sel;
        } else if (key == thr) {
          sel += e < need_eq ? 1 : 0;
          ++e;
        }
      }
    }
    int pos = s_sel_base + block_exclusive_scan(sel, s_scan, &tot);
    int32_t* out = a.ids + static_cast<int64_t>(row) * a.ld_ids;
    int e = eq_before;
    for (int i = c0; i < c1; ++i) {
      const uint32_t key = s_keys[i];
      bool take = key > thr;
      if (key == thr) {
        take = e < need_eq;
        ++e;
      }
      if (take) out[pos++] = n0 + i;
    }
  }

  // The last CTA to leave resets the barrier counters for the next call.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.depart, 1u) == gridDim.x - 1) {
      for (int r = 0; r < a.rows; ++r) a.bar[r] = 0u;
      *a.depart = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// Cluster variant: one thread-block cluster of kCluster CTAs per row.
//
// Used when the row's neurons fit the cluster's shared memory (N <= kCluster *
// kSliceCap).  At launch each CTA starts bulk copies of its slice of the head
// weights (and of fc1 / fc2) into shared memory, so that after the encoder
// every weight the row still needs is on chip.  All exchanges between the
// CTAs of a row go through distributed shared memory, separated by hardware
// cluster barriers (no global atomics, no spin on global counters):
//  encoder items (item i on CTA i % kCluster) -> cluster barrier -> every CTA
//  sums the items in a fixed order, runs the MLP, scores its slice, builds its
//  12-bit histogram -> barrier -> every CTA adds the kCluster histograms bin by
//  bin (DSMEM) and finds the bin of the k-th key; 10-bit histograms of the
//  candidates -> barrier -> sum, bin; last 10 bits -> barrier -> sum, exact
//  key T -> counts above / equal to T -> barrier -> offsets from the counts,
//  ids written -> barrier (no CTA leaves while another may still read its
//  shared memory).
// ---------------------------------------------------------------------------

constexpr int kCluster = 8;
constexpr int kCThreads = 512;
constexpr int kMaxItemsPerCta = 2048;   // encoder items held per CTA
constexpr uint32_t kBulkChunk = 32768;  // bytes per bulk copy

struct ClusterSmem {
  uint64_t bar;
  int ok;
  int bin, rem;
  int sel_base, eq_base;
  float stat[2];
  int scan[33];
  int2 cnt;                           // this CTA's keys above / equal to T (read by the cluster)
  float part[kMaxItemsPerCta];        // this CTA's encoder items
  float r[kMaxLatent], u[kMaxLatent], z[kMaxLatent];
  float vec[5][kMaxLatent];           // enc_b, fc1_b, fc2_b, ln_w, ln_b (staged at launch)
  int2 cnts[kCluster];                // every CTA's counts, gathered
  uint32_t keys[kSliceCap];
  // This CTA's histograms, read by the whole cluster: each digit has fine bins
  // and coarse bins (64 / 32 fine bins each), so that finding a bin reads the
  // cluster's coarse bins and then only the fine bins of one coarse bin.
  int hist[kTop];                     // 12-bit digit
  int c1[kTop / 64];
  int h2[kLow];                       // next 10 bits, candidates of the 12-bit bin
  int c2[kLow / 32];
  int h3[kLow];                       // last 10 bits
  int c3[kLow / 32];
  int gath[kCluster][64];             // bins gathered from the cluster
  int sum[64];
};
// Followed, 128-byte aligned, by the prefetched weights: fc1 | fc2 (when
// prefetched) | head slice (when prefetched).

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

struct ClusterArgs {
  SelArgs a;
  int vec_enc;     // x rows and encoder rows load as 16-byte pieces (hidden % 8 == 0, aligned)
  int fc_smem;     // fc1 / fc2 are prefetched into shared memory
  int head_smem;   // the head slice is prefetched into shared memory
  uint32_t fc_bytes;    // bytes of one of fc1 / fc2
  uint32_t head_off;    // offset of the head slice after the fc weights
};

// Warp 0: the bin (of NB in cnt, visited from the highest) that holds the
// rem-th largest element, and rem minus the elements in higher bins.
template <int NB>
__device__ __forceinline__ void warp_find(const int* cnt, int rem, int* out_bin, int* out_rem) {
  constexpr int PER = NB / 32;
  const int lane = threadIdx.x & 31;
  const int top = NB - 1 - PER * lane;
  int c[PER];
  int s = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    c[j] = cnt[top - j];
    s += c[j];
  }
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  int above = x - s;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (above < rem && above + c[j] >= rem) {
      *out_bin = top - j;
      *out_rem = rem - above;
    }
    above += c[j];
  }
}

// All threads: the bin of the rem-th largest key of a digit whose per-CTA
// histograms (fine[NC * W], coarse[NC]) live in the cluster's CTAs.  Two
// gathers of one remote word per thread: the coarse bins, then the W fine
// bins of the chosen coarse bin.  Returns the fine bin; *rem_out the rank
// left inside it.
template <int NC, int W>
__device__ __forceinline__ int cluster_find(cooperative_groups::cluster_group& cluster, ClusterSmem& sm, int* fine,
                                            int* coarse, int rem, int* rem_out) {
  static_assert(NC <= 64 && W <= 64 && kCluster * 64 <= kCThreads, "gather shape");
  const int tid = threadIdx.x;
  const int q = tid >> 6, j = tid & 63;
  if (j < NC) sm.gath[q][j] = cluster.map_shared_rank(coarse, q)[j];
  __syncthreads();
  if (tid < NC) {
    int t = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) t += sm.gath[r][tid];
    sm.sum[tid] = t;
  }
  __syncthreads();
  if (tid < 32) warp_find<NC>(sm.sum, rem, &sm.bin, &sm.rem);
  __syncthreads();
  const int cb = sm.bin, crem = sm.rem;
  if (j < W) sm.gath[q][j] = cluster.map_shared_rank(fine, q)[cb * W + j];
  __syncthreads();
  if (tid < W) {
    int t = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) t += sm.gath[r][tid];
    sm.sum[tid] = t;
  }
  __syncthreads();
  if (tid < 32) warp_find<W>(sm.sum, crem, &sm.bin, &sm.rem);
  __syncthreads();
  const int fb = cb * W + sm.bin;
  *rem_out = sm.rem;
  __syncthreads();  // sm.bin / sm.rem are written again by the next call
  return fb;
}

template <typename T>
__global__ void __launch_bounds__(kCThreads, 1) score_select_cluster_kernel(const ClusterArgs ca) {
  namespace cg = cooperative_groups;
  const SelArgs& a = ca.a;
  extern __shared__ __align__(128) uint8_t cs_raw[];
  ClusterSmem& sm = *reinterpret_cast<ClusterSmem*>(cs_raw);
  uint8_t* wbuf = cs_raw + (sizeof(ClusterSmem) + 127) / 128 * 128;
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  constexpr int kW = kCThreads / 32;
  const int rank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x / kCluster;
  const int L = a.latent;
  const int H = a.hidden;
  const int N = a.n;
  const int n0 = static_cast<int>((static_cast<int64_t>(N) * rank) / kCluster);
  const int n1 = static_cast<int>((static_cast<int64_t>(N) * (rank + 1)) / kCluster);
  const int len = n1 - n0;
  const int items = L * a.nchunk;
  const T* fc1s = reinterpret_cast<const T*>(wbuf);
  const T* fc2s = reinterpret_cast<const T*>(wbuf + ca.fc_bytes);
  const T* heads = reinterpret_cast<const T*>(wbuf + ca.head_off);

  // Prefetch: one thread starts the bulk copies of the weights this CTA needs
  // after the encoder.
  const uint32_t head_bytes = static_cast<uint32_t>(len) * L * sizeof(T);
  const uint32_t expect = (ca.fc_smem ? 2 * ca.fc_bytes : 0u) + (ca.head_smem ? head_bytes : 0u);
  if (tid == 0 && expect > 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&sm.bar, expect);
    if (ca.fc_smem) {
      bulk_copy(wbuf, a.fc1_w, ca.fc_bytes, &sm.bar);
      bulk_copy(wbuf + ca.fc_bytes, a.fc2_w, ca.fc_bytes, &sm.bar);
    }
    if (ca.head_smem) {
      const uint8_t* src = static_cast<const uint8_t*>(a.out_w) + static_cast<size_t>(n0) * L * sizeof(T);
      for (uint32_t off = 0; off < head_bytes; off += kBulkChunk)
        bulk_copy(wbuf + ca.head_off + off, src + off, min(kBulkChunk, head_bytes - off), &sm.bar);
    }
  }

  // Small vectors and this thread's head biases are loaded now, so that no
  // global round trip sits inside the dependent chain after the encoder.
  for (int l = tid; l < L; l += kCThreads) {
    sm.vec[0][l] = ld_opt<T>(a.enc_b, l, 0.f);
    sm.vec[1][l] = ld_opt<T>(a.fc1_b, l, 0.f);
    sm.vec[2][l] = ld_opt<T>(a.fc2_b, l, 0.f);
    sm.vec[3][l] = ld_opt<T>(a.ln_w, l, 1.f);
    sm.vec[4][l] = ld_opt<T>(a.ln_b, l, 0.f);
  }
  constexpr int kPerThread = kSliceCap / kCThreads;
  float bias[kPerThread];
#pragma unroll
  for (int q = 0; q < kPerThread; ++q) {
    const int i = tid + q * kCThreads;
    bias[q] = i < len ? ld_opt<T>(a.out_b, n0 + i, 0.f) : 0.f;
  }

  // 1. Encoder items i = rank, rank + kCluster, ... over this CTA's warps,
  //    two items per warp at a time (all their loads in flight together).
  {
    const T* xr = reinterpret_cast<const T*>(a.x) + static_cast<int64_t>(row) * a.ldx;
    for (int j = warp; rank + kCluster * j < items; j += 2 * kW) {
      const int j2 = j + kW;
      const bool two = rank + kCluster * j2 < items;
      const int item = rank + kCluster * j, item2 = rank + kCluster * (two ? j2 : j);
      const int l = item / a.nchunk, l2 = item2 / a.nchunk;
      const int h0 = (item - l * a.nchunk) * kEncChunk, h02 = (item2 - l2 * a.nchunk) * kEncChunk;
      float acc = 0.f, acc2 = 0.f;
      if (ca.vec_enc) {
        // Lane owns 16 contiguous elements of the chunk: two 16-byte pieces of
        // x and of each encoder row.
        const T* w1 = reinterpret_cast<const T*>(a.enc_w) + static_cast<int64_t>(l) * H;
        const T* w2 = reinterpret_cast<const T*>(a.enc_w) + static_cast<int64_t>(l2) * H;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = h0 + lane * 16 + e * 8, hb = h02 + lane * 16 + e * 8;
          if (h < H) {
            float fx[8], fw[8];
            widen(load_global_pack8<T>(xr + h), fx);
            widen(load_global_pack8<T>(w1 + h), fw);
#pragma unroll
            for (int q = 0; q < 8; ++q) acc = fmaf(fx[q], fw[q], acc);
          }
          if (hb < H) {
            float fx[8], fw[8];
            widen(load_global_pack8<T>(xr + hb), fx);
            widen(load_global_pack8<T>(w2 + hb), fw);
#pragma unroll
            for (int q = 0; q < 8; ++q) acc2 = fmaf(fx[q], fw[q], acc2);
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < kEncChunk / 32; ++e) {
          const int h = h0 + lane + 32 * e, hb = h02 + lane + 32 * e;
          if (h < H) acc = fmaf(to_f32<T>(xr[h]), ld_f<T>(a.enc_w, static_cast<int64_t>(l) * H + h), acc);
          if (hb < H) acc2 = fmaf(to_f32<T>(xr[hb]), ld_f<T>(a.enc_w, static_cast<int64_t>(l2) * H + hb), acc2);
        }
      }
      acc = warp_sum(acc);
      acc2 = warp_sum(acc2);
      if (lane == 0) {
        sm.part[j] = acc;
        if (two) sm.part[j2] = acc2;
      }
    }
  }
  for (int b = tid; b < kTop; b += kCThreads) sm.hist[b] = 0;
  if (tid < kTop / 64) sm.c1[tid] = 0;
  cluster.sync();

  // 2. Latent MLP (identical in every CTA of the row), this slice's scores.
  for (int l = tid; l < L; l += kCThreads) {
    float pre = sm.vec[0][l];
    for (int c = 0; c < a.nchunk; ++c) {
      const int item = l * a.nchunk + c;
      pre += cluster.map_shared_rank(sm.part, item % kCluster)[item / kCluster];
    }
    if (a.kind == 0)
      sm.r[l] = silu_f(pre);
    else
      sm.z[l] = pre;
  }
  // Every thread observes the copies' completion before reading them.
  const bool have = __syncthreads_and(expect == 0 || mbar_wait_bounded(&sm.bar, 0, kWaitLimitNs)) != 0;
  if (!have && tid == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
  if (a.kind == 0) {
    for (int l = tid; l < L; l += kCThreads) {
      const float acc = ca.fc_smem ? (have ? dot_row_smem<T>(fc1s + static_cast<int64_t>(l) * L, sm.r, L) : 0.f)
                                   : dot_row<T>(reinterpret_cast<const T*>(a.fc1_w) + static_cast<int64_t>(l) * L,
                                                sm.r, L, a.vec_fc);
      sm.u[l] = silu_f(acc + sm.vec[1][l]);
    }
    __syncthreads();
    for (int l = tid; l < L; l += kCThreads) {
      const float acc = ca.fc_smem ? (have ? dot_row_smem<T>(fc2s + static_cast<int64_t>(l) * L, sm.u, L) : 0.f)
                                   : dot_row<T>(reinterpret_cast<const T*>(a.fc2_w) + static_cast<int64_t>(l) * L,
                                                sm.u, L, a.vec_fc);
      sm.z[l] = acc + sm.vec[2][l] + sm.r[l];
    }
    __syncthreads();
    if (warp == 0) {
      float sum = 0.f;
      for (int j = lane; j < L; j += 32) sum += sm.z[j];
      const float mean = warp_sum(sum) / static_cast<float>(L);
      float sq = 0.f;
      for (int j = lane; j < L; j += 32) {
        const float d = sm.z[j] - mean;
        sq = fmaf(d, d, sq);
      }
      const float var = warp_sum(sq) / static_cast<float>(L);
      if (lane == 0) {
        sm.stat[0] = mean;
        sm.stat[1] = rsqrtf(var + a.eps);
      }
    }
    __syncthreads();
    for (int l = tid; l < L; l += kCThreads)
      sm.z[l] = (sm.z[l] - sm.stat[0]) * sm.stat[1] * sm.vec[3][l] + sm.vec[4][l];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < kPerThread; ++q) {
    const int i = tid + q * kCThreads;
    if (i >= len) break;
    const int n = n0 + i;
    float acc;
    if (ca.head_smem)
      acc = have ? dot_row_smem_rot<T>(heads + static_cast<int64_t>(i) * L, sm.z, L, tid) : 0.f;
    else
      acc = dot_row<T>(reinterpret_cast<const T*>(a.out_w) + static_cast<int64_t>(n) * L, sm.z, L, a.vec_out);
    const float sc = acc + bias[q];
    sm.keys[i] = score_key(sc);
    if (a.scores != nullptr) a.scores[static_cast<int64_t>(row) * a.ld_scores + n] = sc;
  }
  __syncthreads();
  // The coarse bins are few and hot, so they are summed from the fine bins
  // rather than counted with atomics of their own.
  for (int i = tid; i < len; i += kCThreads) atomicAdd(&sm.hist[sm.keys[i] >> 20], 1);
  __syncthreads();
  if (tid < kTop / 64) {
    int t = 0;
    for (int b = 0; b < 64; ++b) t += sm.hist[tid * 64 + b];
    sm.c1[tid] = t;
  }
  for (int b = tid; b < kLow; b += kCThreads) {
    sm.h2[b] = 0;
    sm.h3[b] = 0;
  }
  if (tid < kLow / 32) {
    sm.c2[tid] = 0;
    sm.c3[tid] = 0;
  }
  cluster.sync();

  // 3. The bin of the k-th key in the row's 12-bit histogram.
  int rem;
  const uint32_t bin = static_cast<uint32_t>(cluster_find<kTop / 64, 64>(cluster, sm, sm.hist, sm.c1, a.k, &rem));
  for (int i = tid; i < len; i += kCThreads)
    if ((sm.keys[i] >> 20) == bin) {
      atomicAdd(&sm.h2[(sm.keys[i] >> 10) & (kLow - 1)], 1);
      atomicAdd(&sm.c2[(sm.keys[i] >> 15) & 31], 1);
    }
  cluster.sync();

  // 4. Next 10 bits over the cluster's candidates.
  int rem_a;
  const uint32_t prefix =
      (bin << 10) | static_cast<uint32_t>(cluster_find<kLow / 32, 32>(cluster, sm, sm.h2, sm.c2, rem, &rem_a));
  for (int i = tid; i < len; i += kCThreads)
    if ((sm.keys[i] >> 10) == prefix) {
      atomicAdd(&sm.h3[sm.keys[i] & (kLow - 1)], 1);
      atomicAdd(&sm.c3[(sm.keys[i] >> 5) & 31], 1);
    }
  cluster.sync();

  // 5. Last 10 bits: the exact k-th key T and the ties still needed.
  int need_eq;
  const uint32_t thr =
      (prefix << 10) | static_cast<uint32_t>(cluster_find<kLow / 32, 32>(cluster, sm, sm.h3, sm.c3, rem_a, &need_eq));
  // Counts above / equal to T over this thread's contiguous chunk (index
  // order), both prefix-summed by one scan of (above << 16 | equal).
  const int per = (len + kCThreads - 1) / kCThreads;
  const int c0 = min(len, tid * per), c1 = min(len, c0 + per);
  int gt = 0, eqc = 0;
  for (int i = c0; i < c1; ++i) {
    gt += sm.keys[i] > thr ? 1 : 0;
    eqc += sm.keys[i] == thr ? 1 : 0;
  }
  int packed_tot;
  const int packed_before = block_exclusive_scan((gt << 16) | eqc, sm.scan, &packed_tot);
  const int gt_before = packed_before >> 16, eq_before_cta = packed_before & 0xFFFF;
  if (tid == 0) sm.cnt = make_int2(packed_tot >> 16, packed_tot & 0xFFFF);
  cluster.sync();

  // 6. Offsets from the earlier CTAs' counts; selected indices, ascending.
  if (tid < kCluster) sm.cnts[tid] = *cluster.map_shared_rank(&sm.cnt, tid);
  __syncthreads();
  if (tid == 0) {
    int sel = 0, eqb = 0;
    for (int q = 0; q < rank; ++q) {
      const int2 c = sm.cnts[q];
      sel += c.x + min(c.y, max(0, need_eq - eqb));
      eqb += c.y;
    }
    sm.sel_base = sel;
    sm.eq_base = eqb;
  }
  __syncthreads();
  // Ties are taken lowest index first: of this CTA's ties before this
  // thread's chunk, those still needed after the earlier CTAs' ties count.
  const int eq_before = sm.eq_base + eq_before_cta;
  int pos = sm.sel_base + gt_before + min(eq_before_cta, max(0, need_eq - sm.eq_base));
  int32_t* out = a.ids + static_cast<int64_t>(row) * a.ld_ids;
  int e = eq_before;
  for (int i = c0; i < c1; ++i) {
    const uint32_t key = sm.keys[i];
    bool take = key > thr;
    if (key == thr) {
      take = e < need_eq;
      ++e;
    }
    if (take) out[pos++] = n0 + i;
  }
  // No CTA leaves while another may still read its shared memory, nor with
  // its own bulk copies still in flight (after a timed-out wait).
  if (!have && tid == 0) (void)mbar_wait_bounded(&sm.bar, 0, kWaitLimitNs);
  cluster.sync();
}

// Whether a cluster of kCluster CTAs with this much shared memory can be
// scheduled on the device (asked once per kernel, device and size: the
// answer is cached, so later calls -- also under stream capture -- make no
// query).
template <typename Query>
bool cluster_fits(const void* fn, int device, size_t smem, Query query) {
  static std::mutex mu;
  static std::unordered_map<std::string, bool> known;
  std::string key(reinterpret_cast<const char*>(&fn), sizeof(fn));
  key.append(reinterpret_cast<const char*>(&device), sizeof(device));
  key.append(reinterpret_cast<const char*>(&smem), sizeof(smem));
  std::lock_guard<std::mutex> lock(mu);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  int clusters = 0;
  clear_stale_error();
  const bool ok = query(&clusters) == cudaSuccess && clusters > 0;
  clear_stale_error();
  known.emplace(key, ok);
  return ok;
}

struct SelLayout {
  size_t enc, hist, cand, counts, total;
};

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

SelLayout sel_layout(int rows, int hidden, int latent, int n) {
  const size_t nchunk = (static_cast<size_t>(hidden) + kEncChunk - 1) / kEncChunk;
  SelLayout l;
  l.enc = kHeader;
  l.hist = l.enc + align256(static_cast<size_t>(rows) * latent * nchunk * 4);
  l.cand = l.hist + align256(static_cast<size_t>(rows) * kTop * 4);
  l.counts = l.cand + align256(static_cast<size_t>(rows) * n * 8);
  l.total = l.counts + align256(static_cast<size_t>(rows) * kMaxCpr * 8);
  return l;
}

}  // namespace

}  // namespace qcc

extern "C" size_t qcc_selector_workspace_bytes(int batch, int hidden, int latent, int n_out) {
  if (batch < 1 || hidden < 1 || latent < 1 || latent > qcc::kMaxLatent || n_out < 1) return 0;
  return qcc::sel_layout(std::min(batch, qcc::kMaxRows), hidden, latent, n_out).total;
}

extern "C" int qcc_selector_scores_topk(const void* x, int64_t ldx, int batch, int hidden, int latent, int n_out,
                                        int kind, int dtype, const void* enc_w, const void* enc_b, const void* fc1_w,
                                        const void* fc1_b, const void* fc2_w, const void* fc2_b, const void* ln_w,
                                        const void* ln_b, float ln_eps, const void* out_w, const void* out_b, int k,
                                        int32_t* ids, int64_t ld_ids, float* scores, int64_t ld_scores,
                                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace qcc;
  if (!valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (kind != 0 && kind != 1) return QCC_ERR_INVALID_ARGUMENT;
  if (batch < 0 || hidden < 1 || latent < 1 || n_out < 1 || ldx < hidden) return QCC_ERR_SHAPE;
  if (latent > kMaxLatent) return QCC_ERR_UNSUPPORTED;
  if (k < 1 || k > n_out || ld_ids < k || (scores != nullptr && ld_scores < n_out)) return QCC_ERR_SHAPE;
  if (batch == 0) return QCC_OK;
  if (x == nullptr || enc_w == nullptr || out_w == nullptr || ids == nullptr || workspace == nullptr)
    return QCC_ERR_INVALID_ARGUMENT;
  if (kind == 0 && (fc1_w == nullptr || fc2_w == nullptr)) return QCC_ERR_INVALID_ARGUMENT;
  if (!aligned16(workspace)) return QCC_ERR_ALIGNMENT;
  const int rows_max = std::min(batch, kMaxRows);
  const SelLayout lay = sel_layout(rows_max, hidden, latent, n_out);
  if (workspace_bytes < lay.total) return QCC_ERR_WORKSPACE;

  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const DeviceInfo& info = device_info(device);
  if (info.num_sms <= 0) return QCC_ERR_CUDA;

  void (*fn)(const SelArgs) = nullptr;
  if (dtype == QCC_DTYPE_BF16)
    fn = score_select_kernel<__nv_bfloat16>;
  else if (dtype == QCC_DTYPE_F16)
    fn = score_select_kernel<__half>;
  else
    fn = score_select_kernel<float>;
  int per_sm = 0;
  if (!cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, 0)) || per_sm < 1)
    return QCC_ERR_CUDA;
  const int resident = info.num_sms * per_sm;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  SelArgs args;
  args.hidden = hidden;
  args.latent = latent;
  args.n = n_out;
  args.kind = kind;
  args.enc_w = enc_w;
  args.enc_b = enc_b;
  args.fc1_w = fc1_w;
  args.fc1_b = fc1_b;
  args.fc2_w = fc2_w;
  args.fc2_b = fc2_b;
  args.ln_w = ln_w;
  args.ln_b = ln_b;
  args.eps = ln_eps;
  args.out_w = out_w;
  args.out_b = out_b;
  args.k = k;
  args.ld_ids = ld_ids;
  args.ld_scores = ld_scores;
  args.nchunk = (hidden + kEncChunk - 1) / kEncChunk;
  args.vec_fc = latent % 8 == 0 && aligned16(fc1_w) && aligned16(fc2_w);
  args.vec_out = latent % 8 == 0 && aligned16(out_w);
  args.status = reinterpret_cast<unsigned int*>(ws);
  args.depart = reinterpret_cast<unsigned int*>(ws + 4);
  args.bar = reinterpret_cast<unsigned int*>(ws + kBarOffset);
  args.cand_count = reinterpret_cast<unsigned int*>(ws + kCandCountOffset);
  args.enc_part = reinterpret_cast<float*>(ws + lay.enc);
  args.hist = reinterpret_cast<unsigned int*>(ws + lay.hist);
  args.cand = reinterpret_cast<uint2*>(ws + lay.cand);
  args.counts = reinterpret_cast<int2*>(ws + lay.counts);
  const size_t esize = dtype == QCC_DTYPE_F32 ? 4 : 2;

  // Cluster path: the row's neurons fit the cluster's shared memory.
  if (n_out <= kCluster * kSliceCap && (latent * args.nchunk + kCluster - 1) / kCluster <= kMaxItemsPerCta) {
    ClusterArgs ca;
    ca.a = args;
    ca.a.x = x;
    ca.a.ldx = ldx;
    ca.a.rows = batch;
    ca.a.ids = ids;
    ca.a.scores = scores;
    ca.a.cpr = kCluster;
    ca.vec_enc = hidden % 8 == 0 && aligned16(x) && (static_cast<size_t>(ldx) * esize) % 16 == 0 && aligned16(enc_w);
    const size_t base = (sizeof(ClusterSmem) + 127) / 128 * 128;
    const size_t fc_bytes = static_cast<size_t>(latent) * latent * esize;
    const size_t slice_max = static_cast<size_t>((n_out + kCluster - 1) / kCluster) * latent * esize;
    const size_t limit = static_cast<size_t>(info.max_smem_optin);
    ca.fc_smem = kind == 0 && fc_bytes % 16 == 0 && aligned16(fc1_w) && aligned16(fc2_w) &&
                 base + 2 * fc_bytes <= limit;
    ca.fc_bytes = static_cast<uint32_t>(fc_bytes);
    const size_t head_off = ca.fc_smem ? (2 * fc_bytes + 127) / 128 * 128 : 0;
    ca.head_off = static_cast<uint32_t>(head_off);
    ca.head_smem = (static_cast<size_t>(latent) * esize) % 16 == 0 && aligned16(out_w) &&
                   base + head_off + slice_max <= limit;
    const size_t smem = base + head_off + (ca.head_smem ? slice_max : 0);
    void (*cfn)(const ClusterArgs) = nullptr;
    if (dtype == QCC_DTYPE_BF16)
      cfn = score_select_cluster_kernel<__nv_bfloat16>;
    else if (dtype == QCC_DTYPE_F16)
      cfn = score_select_cluster_kernel<__half>;
    else
      cfn = score_select_cluster_kernel<float>;
    if (smem <= limit && ensure_max_dynamic_smem(reinterpret_cast<const void*>(cfn), device)) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(kCluster * batch));
      cfg.blockDim = dim3(kCThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = kCluster;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cluster_fits(reinterpret_cast<const void*>(cfn), device, smem, [&](int* clusters) {
            return cudaOccupancyMaxActiveClusters(clusters, cfn, &cfg);
          })) {
        clear_stale_error();
        if (!cuda_ok(cudaLaunchKernelEx(&cfg, cfn, ca))) return QCC_ERR_CUDA;
        return QCC_OK;
      }
      clear_stale_error();  // no cluster of this size fits: the grid path below
    }
  }

  for (int r0 = 0; r0 < batch; r0 += kMaxRows) {
    const int rows = std::min(kMaxRows, batch - r0);
    // CTAs per row: the SMs shared out, at most one per 64 neurons, at least
    // enough that a slice fits in shared memory.
    int cpr = std::max(1, std::min(info.num_sms / rows, (n_out + 63) / 64));
    cpr = std::max(cpr, (n_out + kSliceCap - 1) / kSliceCap);
    if (cpr > kMaxCpr || static_cast<int64_t>(cpr) * rows > resident) return QCC_ERR_UNSUPPORTED;
    args.x = static_cast<const uint8_t*>(x) + static_cast<size_t>(r0) * ldx * esize;
    args.ldx = ldx;
    args.rows = rows;
    args.ids = ids + static_cast<int64_t>(r0) * ld_ids;
    args.scores = scores != nullptr ? scores + static_cast<int64_t>(r0) * ld_scores : nullptr;
    args.cpr = cpr;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(cpr * rows));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    clear_stale_error();
    if (!cuda_ok(cudaLaunchKernelEx(&cfg, fn, args))) return QCC_ERR_CUDA;
  }
  return QCC_OK;
}
