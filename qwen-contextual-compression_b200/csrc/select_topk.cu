// Deterministic top-K selector and per-token union / shard filter (sm_100a).
//
// qcc_select_topk: one CTA per score row.  Scores are mapped to
// order-preserving 32-bit keys (-0.0 and +0.0 share a key, every NaN maps to
// the largest key) and kept in shared memory.  A radix select finds the exact
// key T of the k-th largest score and how many elements equal to T are still
// needed: a 12-bit top digit, histogrammed while the row is loaded, picks one
// bin; the keys of that bin are compacted into a small candidate list; two
// 10-bit digits over the candidates finish T.  An output pass then emits, in
// ascending index order, every index with key > T plus the lowest-index
// elements with key == T.  The result is
// sort(scores, descending, stable)[:k] sorted ascending, which is one of the
// valid answers of torch.topk(scores, k, sorted=False) as used by
// runtime/selector.py:24 and end_to_end/oracle_sparse_mlp.py:75, with the
// tie order fixed.
//
// qcc_activation_topk: the same selection with the scores made on the fly
// from an activation row a (bf16 / fp16 / fp32) and optional per-column fp32
// weights w: score = |a| (importance "activation", oracle/importance.py:10)
// or |a| * w (the down-column-norm weighting of
// end_to_end/oracle_sparse_mlp.py:75, one fp32 rounding as there), plus an
// optional masked copy of the row (a where selected, 0 elsewhere) -- the
// zeros().scatter_(gather) of the same line -- written in the output pass.
//
// qcc_build_union: one CTA.  Sets per-neuron token bits for all rows in a
// shared byte map over [id_begin, id_end) and compacts the non-zero entries
// with one block-wide scan.

#include <cuda_runtime.h>

#include <algorithm>

#include "qcc_common.cuh"
#include "qcc_host.h"

namespace qcc {

namespace {

constexpr int kSelectThreads = 1024;
constexpr int kUnionThreads = 1024;
constexpr int kUnionLoads = 8;  // id loads in flight per thread in build_union_kernel
constexpr int kDigit1Bins = 1 << 12;                       // key bits 31..20
constexpr int kDigitBins = 1 << 10;                        // key bits 19..10, then 9..0
constexpr int kCandidateCap = kDigit1Bins - kDigitBins;   // candidate keys that fit beside a 10-bit histogram
constexpr int kLoadRound = 8;                              // loads in flight per thread

// How a row element becomes its score.
constexpr int kScoreRaw = 0;       // the fp32 value itself
constexpr int kScoreAbs = 1;       // |a|
constexpr int kScoreAbsScaled = 2;  // |a| * w[i]
constexpr int kScoreBlockSum = 3;   // element i = sum of the scores of block i (the row holds the blocks)

template <int SCORE>
__device__ __forceinline__ float make_score(float v, const float* w, int i) {
  if constexpr (SCORE == kScoreRaw) return v;
  else if constexpr (SCORE == kScoreAbs) return fabsf(v);
  else return fabsf(v) * __ldg(w + i);
}

template <typename T>
__device__ __forceinline__ void widen_any(uint4 raw, float (&f)[16 / sizeof(T)]) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(raw.x);
    f[1] = __uint_as_float(raw.y);
    f[2] = __uint_as_float(raw.z);
    f[3] = __uint_as_float(raw.w);
  } else {
    Pack8<T> p;
    p.w[0] = raw;
    widen(p, f);
  }
}

// n is the length of the row the selection runs over: the scores themselves,
// or with kScoreBlockSum the ceil(n_elems / block) block sums of a score row
// of n_elems entries (zero past its end), summed in fp64 in index order and
// rounded once; sums (optional) receives them.
template <typename T, int SCORE>
__global__ void __launch_bounds__(kSelectThreads, 1)
    select_topk_kernel(const T* __restrict__ scores, int64_t ld_scores, const float* __restrict__ col_w, int n, int k,
                       int32_t* __restrict__ ids, int64_t ld_ids, T* __restrict__ masked, int64_t ld_masked,
                       int block, int n_elems, float* __restrict__ sums, int64_t ld_sums) {
  extern __shared__ __align__(16) uint32_t keys[];
  // Top-digit histogram; after that digit is chosen the same space holds the
  // candidate keys ([0, kCandidateCap)) and the 10-bit histograms after them.
  __shared__ __align__(16) int hist[kDigit1Bins];
  __shared__ int scan_scratch[64];
  __shared__ int warp_gt[32], warp_eq[32];
  __shared__ int s_bin, s_rem, s_count;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const T* src = scores + blockIdx.x * ld_scores;
  int32_t* out = ids + blockIdx.x * ld_ids;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte load

  for (int i = tid; i < kDigit1Bins; i += kSelectThreads) hist[i] = 0;
  if (tid == 0) s_count = 0;
  __syncthreads();

  // 1. Keys into shared memory, fused with the histogram of the top 12 bits.
  //    All loads of a round are issued before any is used (one memory latency
  //    per round); 16-byte loads when the row is 16-byte aligned.
  if constexpr (SCORE == kScoreBlockSum) {
    for (int i = tid; i < n; i += kSelectThreads) {
      const int lo = i * block;
      const int hi = min(n_elems, lo + block);
      double acc = 0.0;
      for (int j = lo; j < hi; ++j) acc += static_cast<double>(to_f32<T>(src[j]));
      const float s = static_cast<float>(acc);
      if (sums != nullptr) sums[blockIdx.x * ld_sums + i] = s;
      const uint32_t key = score_key(s);
      keys[i] = key;
      atomicAdd(&hist[key >> 20], 1);
    }
  }
  const bool vec = SCORE != kScoreBlockSum && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const int n_vec = vec ? n / V : 0;
  for (int base = 0; base < n_vec; base += kLoadRound * kSelectThreads) {
    uint4 v[kLoadRound];
#pragma unroll
    for (int u = 0; u < kLoadRound; ++u) {
      const int i = base + u * kSelectThreads + tid;
      v[u] = i < n_vec ? __ldg(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kLoadRound; ++u) {
      const int i = base + u * kSelectThreads + tid;
      if (i < n_vec) {
        float f[V];
        widen_any<T>(v[u], f);
        uint32_t q[V];
#pragma unroll
        for (int e = 0; e < V; ++e) {
          q[e] = score_key(make_score<SCORE>(f[e], col_w, V * i + e));
          atomicAdd(&hist[q[e] >> 20], 1);
        }
#pragma unroll
        for (int e = 0; e < V; e += 4)
          reinterpret_cast<uint4*>(keys)[(V * i + e) / 4] = make_uint4(q[e], q[e + 1], q[e + 2], q[e + 3]);
      }
    }
  }
  for (int base = SCORE == kScoreBlockSum ? n : V * n_vec; base < n; base += kLoadRound * kSelectThreads) {
    float v[kLoadRound];
#pragma unroll
    for (int u = 0; u < kLoadRound; ++u) {
      const int i = base + u * kSelectThreads + tid;
      v[u] = i < n ? to_f32<T>(src[i]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kLoadRound; ++u) {
      const int i = base + u * kSelectThreads + tid;
      if (i < n) {
        const uint32_t key = score_key(make_score<SCORE>(v[u], col_w, i));
        keys[i] = key;
        atomicAdd(&hist[key >> 20], 1);
      }
    }
  }
  __syncthreads();

  // 2. Top digit of the k-th largest key.
  find_bin<kDigit1Bins / kSelectThreads>(hist, k, scan_scratch, &s_bin, &s_rem);
  __syncthreads();
  uint32_t prefix = static_cast<uint32_t>(s_bin) << 20;
  uint32_t mask = 0xFFF00000u;
  int rem = s_rem;
  const int in_bin = hist[s_bin];
  __syncthreads();  // the histogram space is reused below

  // 3. The keys of that bin become the candidates (warp-aggregated append; the
  //    order does not matter for counting).  A bin larger than the candidate
  //    space (heavily tied inputs) is instead filtered from all keys below.
  uint32_t* cand = reinterpret_cast<uint32_t*>(hist);
  int* hist2 = hist + kCandidateCap;
  const bool compact = in_bin <= kCandidateCap;
  if (compact) {
    const uint32_t bin1 = prefix >> 20;
    for (int base = 0; base < n; base += kSelectThreads) {
      const int i = base + tid;
      const bool take = i < n && (keys[i] >> 20) == bin1;
      const unsigned ballot = __ballot_sync(0xffffffffu, take);
      if (ballot != 0u) {
        const int leader = __ffs(ballot) - 1;
        int pos = 0;
        if (lane == leader) pos = atomicAdd(&s_count, __popc(ballot));
        pos = __shfl_sync(0xffffffffu, pos, leader);
        if (take) cand[pos + __popc(ballot & ((1u << lane) - 1u))] = keys[i];
      }
    }
    __syncthreads();
  }
  const int n_src = compact ? in_bin : n;
  const uint32_t* src_keys = compact ? cand : keys;

  // 4. Two 10-bit digits over the candidates.
  for (int shift = 10; shift >= 0; shift -= 10) {
    for (int i = tid; i < kDigitBins; i += kSelectThreads) hist2[i] = 0;
    __syncthreads();
    for (int i = tid; i < n_src; i += kSelectThreads) {
      const uint32_t key = src_keys[i];
      if ((key & mask) == prefix) atomicAdd(&hist2[(key >> shift) & (kDigitBins - 1)], 1);
    }
    __syncthreads();
    find_bin<kDigitBins / kSelectThreads>(hist2, rem, scan_scratch, &s_bin, &s_rem);
    __syncthreads();
    prefix |= static_cast<uint32_t>(s_bin) << shift;
    mask |= static_cast<uint32_t>(kDigitBins - 1) << shift;
    rem = s_rem;
    __syncthreads();
  }
  const uint32_t thr = prefix;  // key of the k-th largest score
  const int need = rem;         // elements equal to thr to take, lowest index first

  // 5. Output in ascending index order.  Warp w owns a contiguous segment;
  //    lanes read consecutive keys and ballots give each element its rank.
  const int seg = ((n + 31) / 32 + 31) / 32 * 32;
  const int seg_lo = min(n, warp * seg);
  const int seg_hi = min(n, seg_lo + seg);
  int gt = 0, eq = 0;
  for (int base = seg_lo; base < seg_hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < seg_hi ? keys[i] : 0u;
    gt += __popc(__ballot_sync(0xffffffffu, i < seg_hi && key > thr));
    eq += __popc(__ballot_sync(0xffffffffu, i < seg_hi && key == thr));
  }
  if (lane == 0) {
    warp_gt[warp] = gt;
    warp_eq[warp] = eq;
  }
  __syncthreads();
  if (warp == 0) {
    int g = warp_gt[lane], e = warp_eq[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yg = __shfl_up_sync(0xffffffffu, g, o);
      const int ye = __shfl_up_sync(0xffffffffu, e, o);
      if (lane >= o) {
        g += yg;
        e += ye;
      }
    }
    warp_gt[lane] = g - warp_gt[lane];  // exclusive
    warp_eq[lane] = e - warp_eq[lane];
  }
  __syncthreads();
  int run_gt = warp_gt[warp], run_eq = warp_eq[warp];
  const unsigned lt = (1u << lane) - 1u;
  for (int base = seg_lo; base < seg_hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < seg_hi ? keys[i] : 0u;
    const bool is_gt = i < seg_hi && key > thr;
    const bool is_eq = i < seg_hi && key == thr;
    const unsigned b_gt = __ballot_sync(0xffffffffu, is_gt);
    const unsigned b_eq = __ballot_sync(0xffffffffu, is_eq);
    const int gt_before = run_gt + __popc(b_gt & lt);
    const int eq_before = run_eq + __popc(b_eq & lt);
    if (is_gt) out[gt_before + min(eq_before, need)] = i;
    else if (is_eq && eq_before < need) out[gt_before + eq_before] = i;
    if (masked != nullptr && i < seg_hi) {
      const bool chosen = is_gt || (is_eq && eq_before < need);
      masked[blockIdx.x * ld_masked + i] = chosen ? src[i] : T(0.f);
    }
    run_gt += __popc(b_gt);
    run_eq += __popc(b_eq);
  }
}
__global__ void __launch_bounds__(kUnionThreads, 1)
    build_union_kernel(const int32_t* __restrict__ ids, int64_t ld_ids, int batch, int k, int32_t id_begin,
                       int32_t id_end, int32_t* __restrict__ union_ids, uint8_t* __restrict__ token_mask,
                       int32_t* __restrict__ count_out) {
  extern __shared__ __align__(16) uint32_t words[];  // byte map, 4 neurons per word
  __shared__ int scan_scratch[64];
  const int width = id_end - id_begin;
  const int nwords = (width + 3) / 4;
  const int tid = threadIdx.x;
  for (int i = tid; i < nwords; i += blockDim.x) words[i] = 0u;
  __syncthreads();
  // All rows' ids as one range of batch * k elements, kUnionLoads loads in
  // flight per thread before their atomics (row by row, one load at a time,
  // this phase was a chain of ~30 dependent L2 round trips at batch 8).
  const int total_ids = batch * k;
  for (int base = tid; base < total_ids; base += static_cast<int>(blockDim.x) * kUnionLoads) {
    int32_t v[kUnionLoads];
#pragma unroll
    for (int u = 0; u < kUnionLoads; ++u) {
      const int e = base + u * static_cast<int>(blockDim.x);
      v[u] = e < total_ids ? __ldg(ids + static_cast<int64_t>(e / k) * ld_ids + e % k) : 0;
    }
#pragma unroll
    for (int u = 0; u < kUnionLoads; ++u) {
      const int e = base + u * static_cast<int>(blockDim.x);
      if (e < total_ids && v[u] >= id_begin && v[u] < id_end) {
        const int local = v[u] - id_begin;
        atomicOr(&words[local >> 2], (1u << (e / k)) << (8 * (local & 3)));
      }
    }
  }
  __syncthreads();
  const uint8_t* bytes = reinterpret_cast<const uint8_t*>(words);
  const int chunk = (width + blockDim.x - 1) / blockDim.x;
  const int lo = min(width, tid * chunk);
  const int hi = min(width, lo + chunk);
  int c = 0;
  for (int i = lo; i < hi; ++i) c += bytes[i] != 0;
  int total;
  int pos = block_exclusive_scan(c, scan_scratch, &total);
  for (int i = lo; i < hi; ++i) {
    const uint8_t m = bytes[i];
    if (m != 0) {
      union_ids[pos] = i;
      token_mask[pos] = m;
      ++pos;
    }
  }
  if (tid == 0) *count_out = total;
}

// One CTA: per tile of tile_rows consecutive rows, the union of the rows'
// block ids as an ascending list, appended at the running offset.  A bitmap
// of the n_blocks blocks in shared memory, one compaction scan per tile.
__global__ void __launch_bounds__(kUnionThreads, 1)
    tile_block_union_kernel(const int32_t* __restrict__ block_ids, int64_t ld_ids, int rows, int kb, int tile_rows,
                            int n_blocks, int32_t* __restrict__ tile_blocks, int32_t* __restrict__ tile_offsets,
                            int32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint32_t bits[];
  __shared__ int scan_scratch[64];
  const int tid = threadIdx.x;
  const int nwords = (n_blocks + 31) / 32;
  const int n_tiles = (rows + tile_rows - 1) / tile_rows;
  int written = 0;
  if (tid == 0) tile_offsets[0] = 0;
  for (int t = 0; t < n_tiles; ++t) {
    for (int i = tid; i < nwords; i += blockDim.x) bits[i] = 0u;
    __syncthreads();
    const int r0 = t * tile_rows;
    const int r1 = min(rows, r0 + tile_rows);
    for (int e = tid; e < (r1 - r0) * kb; e += blockDim.x) {
      const int r = r0 + e / kb;
      const int32_t b = __ldg(block_ids + r * ld_ids + e % kb);
      if (b >= 0 && b < n_blocks) atomicOr(&bits[b >> 5], 1u << (b & 31));
      else if (status != nullptr) atomicOr(reinterpret_cast<unsigned int*>(status), QCC_DEV_ID_RANGE);
    }
    __syncthreads();
    // Thread i owns word i (32 blocks in order); one exclusive scan of popcounts.
    const uint32_t w = tid < nwords ? bits[tid] : 0u;
    int total;
    int pos = written + block_exclusive_scan(__popc(w), scan_scratch, &total);
    if (tid < nwords) {
      uint32_t m = w;
      while (m != 0u) {
        const int bit = __ffs(m) - 1;
        tile_blocks[pos++] = tid * 32 + bit;
        m &= m - 1u;
      }
    }
    written += total;
    if (tid == 0) tile_offsets[t + 1] = written;
    __syncthreads();
  }
}

}  // namespace

}  // namespace qcc

extern "C" int qcc_block_topk(const float* scores, int64_t ld_scores, int rows, int n, int block, int k,
                              int32_t* block_ids, int64_t ld_ids, float* block_sums, int64_t ld_sums,
                              cudaStream_t stream) {
  if (rows < 0 || n < 0 || block < 1 || k < 1 || ld_scores < n) return QCC_ERR_SHAPE;
  const int n_blocks = (n + block - 1) / block;
  const int kb = std::max(1, std::min(n_blocks, (k + block - 1) / block));
  if (ld_ids < kb || (block_sums != nullptr && ld_sums < n_blocks)) return QCC_ERR_SHAPE;
  if (rows == 0 || n == 0) return QCC_OK;
  if (scores == nullptr || block_ids == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const qcc::DeviceInfo& info = qcc::device_info(device);
  const size_t smem = static_cast<size_t>(n_blocks) * sizeof(uint32_t);
  if (info.max_smem_optin <= 0 || smem + 20 * 1024 > static_cast<size_t>(info.max_smem_optin)) return QCC_ERR_UNSUPPORTED;
  auto fn = qcc::select_topk_kernel<float, qcc::kScoreBlockSum>;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(fn), device)) return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  fn<<<rows, qcc::kSelectThreads, smem, stream>>>(scores, ld_scores, nullptr, n_blocks, kb, block_ids, ld_ids, nullptr,
                                                  0, block, n, block_sums, ld_sums);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_tile_block_union(const int32_t* block_ids, int64_t ld_ids, int rows, int kb, int tile_rows,
                                    int n_blocks, int32_t* tile_blocks, int32_t* tile_offsets, int32_t* status,
                                    cudaStream_t stream) {
  if (rows < 0 || kb < 0 || ld_ids < kb || tile_rows < 1 || n_blocks < 1) return QCC_ERR_SHAPE;
  if (n_blocks > 32 * qcc::kUnionThreads) return QCC_ERR_UNSUPPORTED;
  if (tile_offsets == nullptr || (rows > 0 && kb > 0 && (block_ids == nullptr || tile_blocks == nullptr)))
    return QCC_ERR_INVALID_ARGUMENT;
  const size_t smem = (static_cast<size_t>(n_blocks) + 31) / 32 * 4;
  qcc::clear_stale_error();
  qcc::tile_block_union_kernel<<<1, qcc::kUnionThreads, smem, stream>>>(block_ids, ld_ids, rows, kb, tile_rows,
                                                                        n_blocks, tile_blocks, tile_offsets, status);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_select_topk(const float* scores, int64_t ld_scores, int batch, int n, int k, int32_t* ids_out,
                               int64_t ld_ids, cudaStream_t stream) {
  if (batch < 0 || n < 0 || k < 0 || k > n || ld_scores < n || ld_ids < k) return QCC_ERR_SHAPE;
  if (batch == 0 || k == 0) return QCC_OK;
  if (scores == nullptr || ids_out == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const qcc::DeviceInfo& info = qcc::device_info(device);
  const size_t smem = static_cast<size_t>(n) * sizeof(uint32_t);
  const size_t static_smem = 20 * 1024;  // per-warp histograms, bins, scan scratch
  if (info.max_smem_optin <= 0 || smem + static_smem > static_cast<size_t>(info.max_smem_optin))
    return QCC_ERR_UNSUPPORTED;
  auto fn = qcc::select_topk_kernel<float, qcc::kScoreRaw>;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(fn), device)) return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  fn<<<batch, qcc::kSelectThreads, smem, stream>>>(scores, ld_scores, nullptr, n, k, ids_out, ld_ids, nullptr, 0, 0, 0,
                                                   nullptr, 0);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

namespace {

template <typename T>
int activation_topk(const T* act, int64_t ld_act, int rows, int n, const float* col_weights, int k, int32_t* ids_out,
                    int64_t ld_ids, T* masked, int64_t ld_masked, cudaStream_t stream) {
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const qcc::DeviceInfo& info = qcc::device_info(device);
  const size_t smem = static_cast<size_t>(n) * sizeof(uint32_t);
  const size_t static_smem = 20 * 1024;
  if (info.max_smem_optin <= 0 || smem + static_smem > static_cast<size_t>(info.max_smem_optin))
    return QCC_ERR_UNSUPPORTED;
  auto fn = col_weights != nullptr ? qcc::select_topk_kernel<T, qcc::kScoreAbsScaled>
                                   : qcc::select_topk_kernel<T, qcc::kScoreAbs>;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(fn), device)) return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  fn<<<rows, qcc::kSelectThreads, smem, stream>>>(act, ld_act, col_weights, n, k, ids_out, ld_ids, masked, ld_masked,
                                                  0, 0, nullptr, 0);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

}  // namespace

extern "C" int qcc_activation_topk(const void* act, int64_t ld_act, int dtype, int rows, int n, const float* col_weights,
                                   int k, int32_t* ids_out, int64_t ld_ids, void* masked_out, int64_t ld_masked,
                                   cudaStream_t stream) {
  if (!qcc::valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (rows < 0 || n < 0 || k < 0 || k > n || ld_act < n || ld_ids < k) return QCC_ERR_SHAPE;
  if (masked_out != nullptr && ld_masked < n) return QCC_ERR_SHAPE;
  if (rows == 0 || n == 0) return QCC_OK;
  if (act == nullptr || ids_out == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (dtype == QCC_DTYPE_BF16)
    return activation_topk(static_cast<const __nv_bfloat16*>(act), ld_act, rows, n, col_weights, k, ids_out, ld_ids,
                           static_cast<__nv_bfloat16*>(masked_out), ld_masked, stream);
  if (dtype == QCC_DTYPE_F16)
    return activation_topk(static_cast<const __half*>(act), ld_act, rows, n, col_weights, k, ids_out, ld_ids,
                           static_cast<__half*>(masked_out), ld_masked, stream);
  return activation_topk(static_cast<const float*>(act), ld_act, rows, n, col_weights, k, ids_out, ld_ids,
                         static_cast<float*>(masked_out), ld_masked, stream);
}

extern "C" int qcc_build_union(const int32_t* ids, int64_t ld_ids, int batch, int k, int32_t id_begin,
                               int32_t id_end, int32_t* union_ids, uint8_t* token_mask, int32_t* count_out,
                               cudaStream_t stream) {
  if (batch < 1 || batch > 8 || k < 0 || ld_ids < k || id_end < id_begin) return QCC_ERR_SHAPE;
  if (count_out == nullptr || (k > 0 && ids == nullptr)) return QCC_ERR_INVALID_ARGUMENT;
  if (id_end > id_begin && (union_ids == nullptr || token_mask == nullptr)) return QCC_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const qcc::DeviceInfo& info = qcc::device_info(device);
  const int width = id_end - id_begin;
  const size_t smem = (static_cast<size_t>(width) + 3) / 4 * 4;
  if (info.max_smem_optin <= 0 || smem + 1024 > static_cast<size_t>(info.max_smem_optin)) return QCC_ERR_UNSUPPORTED;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(qcc::build_union_kernel), device))
    return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  qcc::build_union_kernel<<<1, qcc::kUnionThreads, smem, stream>>>(ids, ld_ids, batch, k, id_begin, id_end, union_ids,
                                                                   token_mask, count_out);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}
