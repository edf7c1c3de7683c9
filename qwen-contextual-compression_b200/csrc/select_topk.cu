// Deterministic top-K selector and per-token union / shard filter (sm_100a).
//
// qcc_select_topk: one CTA per score row.  Scores are mapped to
// order-preserving 32-bit keys (-0.0 and +0.0 share a key, every NaN maps to
// the largest key), kept in shared memory, and a 4-pass radix select
// (8 bits per pass, 256-bin shared histogram) finds the exact key T of the
// k-th largest score and how many elements equal to T are still needed.  A
// single block-wide scan then emits, in ascending index order, every index
// with key > T plus the lowest-index elements with key == T.  The result is
// sort(scores, descending, stable)[:k] sorted ascending, which is one of the
// valid answers of torch.topk(scores, k, sorted=False) as used by
// runtime/selector.py:24 and end_to_end/oracle_sparse_mlp.py:75, with the
// tie order fixed.
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

__device__ __forceinline__ uint32_t score_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0xFFFFFFFFu;          // NaN ranks largest
  if ((u & 0x7FFFFFFFu) == 0u) u = 0u;     // -0.0 == +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block scan of one int per thread; returns the prefix, *total
// receives the block sum.  `scratch` holds >= 33 ints.
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nwarps) scratch[lane] = w;  // inclusive warp totals
    if (lane == 31) scratch[32] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? scratch[warp - 1] : 0) + x - v;
  *total = scratch[32];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kSelectThreads, 1)
    select_topk_kernel(const float* __restrict__ scores, int64_t ld_scores, int n, int k, int32_t* __restrict__ ids,
                       int64_t ld_ids) {
  extern __shared__ __align__(16) uint32_t keys[];
  // Per-warp histograms, two 16-bit bin counters per word (a warp sees at most
  // n / 32 <= 1632 keys per pass, so a counter never overflows).
  __shared__ uint32_t whist[kSelectThreads / 32][128];
  __shared__ int hist[256];
  __shared__ int suffix[257];
  __shared__ int scan_scratch[64];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;

  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const float* src = scores + row * ld_scores;
  int32_t* out = ids + row * ld_ids;

  for (int i = tid; i < n; i += blockDim.x) keys[i] = score_key(__ldg(src + i));
  if (tid == 0) {
    s_prefix = 0u;
    s_remaining = k;
  }
  __syncthreads();

  uint32_t mask = 0u;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < nwarps * 128; i += blockDim.x) (&whist[0][0])[i] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    // Lanes of a warp that fall into the same bin are counted by one atomic
    // (score distributions crowd the high-order bins).
    for (int base = 0; base < n; base += blockDim.x) {
      const int i = base + tid;
      const uint32_t key = i < n ? keys[i] : 0u;
      const bool hit = i < n && (key & mask) == prefix;
      const uint32_t bin = (key >> shift) & 0xFFu;
      const unsigned peers = __match_any_sync(0xffffffffu, hit ? bin : 0x100u);
      if (hit && lane == __ffs(peers) - 1)
        atomicAdd(&whist[warp][bin >> 1], static_cast<uint32_t>(__popc(peers)) << (16 * (bin & 1u)));
    }
    __syncthreads();
    if (tid < 256) {
      int c = 0;
      for (int w = 0; w < nwarps; ++w) c += (whist[w][tid >> 1] >> (16 * (tid & 1))) & 0xFFFFu;
      hist[tid] = c;
    }
    __syncthreads();
    // Inclusive suffix sums over the 256 bins (warps 0..7, one bin per thread).
    if (tid < 256) {
      const int w = tid >> 5;
      // Reverse order so that a prefix scan gives suffix sums.
      int x = hist[255 - tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) scan_scratch[w] = x;
      suffix[255 - tid] = x;  // partial: within-warp
    }
    __syncthreads();
    if (tid < 256) {
      const int w = tid >> 5;
      int add = 0;
      for (int q = 0; q < w; ++q) add += scan_scratch[q];
      suffix[255 - tid] += add;  // suffix[b] = sum of hist[b..255]
    }
    if (tid == 0) suffix[256] = 0;
    __syncthreads();
    const int remaining = s_remaining;
    if (tid < 256) {
      const int above = suffix[tid + 1];
      if (suffix[tid] >= remaining && above < remaining) {
        s_prefix = prefix | (static_cast<uint32_t>(tid) << shift);
        s_remaining = remaining - above;
      }
    }
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const int need = s_remaining;  // elements equal to thr to take, lowest index first

  // Contiguous chunk per thread, one scan for (> thr) and one for (== thr).
  const int chunk = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, tid * chunk);
  const int hi = min(n, lo + chunk);
  int gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    gt += key > thr;
    eq += key == thr;
  }
  int total;
  int gt_before = block_exclusive_scan(gt, scan_scratch, &total);
  int eq_before = block_exclusive_scan(eq, scan_scratch, &total);
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    if (key > thr) {
      out[gt_before + min(eq_before, need)] = i;
      ++gt_before;
    } else if (key == thr) {
      if (eq_before < need) out[gt_before + eq_before] = i;
      ++eq_before;
    }
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
  for (int b = 0; b < batch; ++b) {
    const int32_t* row = ids + b * ld_ids;
    for (int j = tid; j < k; j += blockDim.x) {
      const int32_t id = __ldg(row + j);
      if (id >= id_begin && id < id_end) {
        const int local = id - id_begin;
        atomicOr(&words[local >> 2], (1u << b) << (8 * (local & 3)));
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

}  // namespace

}  // namespace qcc

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
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(qcc::select_topk_kernel), device))
    return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  qcc::select_topk_kernel<<<batch, qcc::kSelectThreads, smem, stream>>>(scores, ld_scores, n, k, ids_out, ld_ids);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
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
