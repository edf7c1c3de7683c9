// Host-offload stager: device-side neuron cache policy and host->HBM record
// gather (sm_100a).
//
// A layer's packed records live in two places: an HBM "resident" array of
// n_hot always-resident records followed by `capacity` cache slots, and a
// pinned host store of the remaining (cold) records.  Per decode step:
//
//   qcc_cache_resolve (one CTA) splits the step's sorted ids into resident
//   ones (hot records and cache hits: their resident-array slots) and misses;
//   each miss takes the least recently used cache slot that the step does not
//   use (empty slots first; among equal last use the record with the lower id
//   goes first -- the eviction order of the reference's OrderedDict LRU,
//   runtime/temporal.py:57-75), and the slot table is updated in place.
//
//   qcc_gather_records copies the missed records from the pinned host store
//   (read in place over PCIe through the unified address space) into their
//   cache slots, on a side stream, while the fused decode runs over the
//   resident records; a second decode over the missed slots adds onto that
//   partial result.
//
// Everything stays on the device: no id list crosses back to the host.

#include <cuda_runtime.h>

#include <algorithm>

#include "qcc_common.cuh"
#include "qcc_host.h"

namespace qcc {
namespace {

constexpr int kResolveThreads = 1024;
constexpr int kMaxCapacity = 8192;
constexpr unsigned long long kActiveKey = ~0ull;

// counts_out: [0] resident, [1] misses served, [2] cache hits, [3] evicted,
//             [4] hot hits, [5] 1 if misses exceeded the free slots
__global__ void __launch_bounds__(kResolveThreads, 1)
    cache_resolve_kernel(const int32_t* __restrict__ ids, int k, const int32_t* __restrict__ k_dev,
                         int32_t* __restrict__ slot_of, int n_records, int n_hot, int32_t* __restrict__ owner,
                         int32_t* __restrict__ last_use, int capacity, int sort_n, const int32_t* __restrict__ cold_index,
                         int step, int32_t* __restrict__ resident_out, int32_t* __restrict__ miss_slot_out,
                         int32_t* __restrict__ miss_src_out, int32_t* __restrict__ counts_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);    // [sort_n]
  int32_t* miss_ids = reinterpret_cast<int32_t*>(keys + sort_n);                 // [capacity]
  uint8_t* active = reinterpret_cast<uint8_t*>(miss_ids + capacity);            // [capacity]
  __shared__ int scratch[64];
  __shared__ int s_cnt[4];  // cache hits, hot hits, evicted

  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  int n = k;
  if (k_dev != nullptr) n = min(n, max(0, __ldg(k_dev)));

  for (int c = tid; c < capacity; c += nthreads) active[c] = 0;
  if (tid < 4) s_cnt[tid] = 0;
  __syncthreads();

  // 1. Classify in id order: resident (hot or cache hit) or miss.
  const int chunk = (n + nthreads - 1) / nthreads;
  const int lo = min(n, tid * chunk);
  const int hi = min(n, lo + chunk);
  int n_res = 0, n_miss = 0, hits = 0, hot = 0;
  for (int i = lo; i < hi; ++i) {
    const int32_t id = ids[i];
    const int32_t s = (id >= 0 && id < n_records) ? slot_of[id] : -2;
    if (s >= 0) {
      ++n_res;
      if (s < n_hot) {
        ++hot;
      } else {
        ++hits;
        active[s - n_hot] = 1;
      }
    } else if (s == -1) {
      ++n_miss;
    }
  }
  if (hits) atomicAdd(&s_cnt[0], hits);
  if (hot) atomicAdd(&s_cnt[1], hot);
  int total_res, total_miss;
  int res_pos = block_exclusive_scan(n_res, scratch, &total_res);
  int miss_pos = block_exclusive_scan(n_miss, scratch, &total_miss);
  for (int i = lo; i < hi; ++i) {
    const int32_t id = ids[i];
    const int32_t s = (id >= 0 && id < n_records) ? slot_of[id] : -2;
    if (s >= 0) {
      resident_out[res_pos++] = s;
      if (s >= n_hot) last_use[s - n_hot] = step;
    } else if (s == -1) {
      if (miss_pos < capacity) miss_ids[miss_pos] = id;
      ++miss_pos;
    }
  }
  __syncthreads();

  // 2. Eviction order of the slots this step does not use: empty slots first,
  //    then by last use, then by the held record's id.
  for (int c = tid; c < sort_n; c += nthreads) {
    unsigned long long key = kActiveKey;
    if (c < capacity && !active[c])
      key = (static_cast<unsigned long long>(last_use[c] + 1) << 40) |
            (static_cast<unsigned long long>(owner[c] + 1) << 16) | static_cast<unsigned long long>(c);
    keys[c] = key;
  }
  __syncthreads();
  for (int size = 2; size <= sort_n; size <<= 1) {  // bitonic sort, ascending
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < sort_n / 2; i += nthreads) {
        const int a = 2 * stride * (i / stride) + (i % stride);
        const int b = a + stride;
        const bool up = ((a & size) == 0);
        const unsigned long long ka = keys[a], kb = keys[b];
        if ((ka > kb) == up) {
          keys[a] = kb;
          keys[b] = ka;
        }
      }
      __syncthreads();
    }
  }

  // 3. Miss i takes the i-th slot of that order.
  const int served = min(total_miss, capacity);
  int evicted = 0;
  for (int i = tid; i < served; i += nthreads) {
    const unsigned long long key = keys[i];
    if (key == kActiveKey) continue;  // more misses than free slots: left unserved
    const int c = static_cast<int>(key & 0xFFFFull);
    const int32_t old = owner[c];
    if (old >= 0) {
      slot_of[old] = -1;
      ++evicted;
    }
    const int32_t id = miss_ids[i];
    owner[c] = id;
    last_use[c] = step;
    slot_of[id] = n_hot + c;
    miss_slot_out[i] = n_hot + c;
    miss_src_out[i] = cold_index[id];
  }
  if (evicted) atomicAdd(&s_cnt[2], evicted);
  __syncthreads();
  if (tid == 0) {
    int ok_misses = served;
    while (ok_misses > 0 && keys[ok_misses - 1] == kActiveKey) --ok_misses;
    counts_out[0] = total_res;
    counts_out[1] = ok_misses;
    counts_out[2] = s_cnt[0];
    counts_out[3] = s_cnt[2];
    counts_out[4] = s_cnt[1];
    counts_out[5] = ok_misses < total_miss ? 1 : 0;
  }
}

// Copies count records from a host-resident store (device-accessible pointer)
// into the resident array: grid-stride over 16-byte pieces with four
// independent loads in flight per thread (PCIe latency hiding).
__global__ void __launch_bounds__(512)
    gather_records_kernel(const uint4* __restrict__ host_store, int64_t record_vec, const int32_t* __restrict__ src,
                          const int32_t* __restrict__ dst, const int32_t* __restrict__ count_dev, int max_count,
                          uint4* __restrict__ packed) {
  const int count = count_dev != nullptr ? min(max_count, max(0, __ldg(count_dev))) : max_count;
  const int64_t total = static_cast<int64_t>(count) * record_vec;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; base < total; base += 4 * stride) {
    uint4 v[4];
    int64_t d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t w = base + u * stride;
      d[u] = -1;
      if (w < total) {
        const int64_t r = w / record_vec;
        const int64_t off = w - r * record_vec;
        const int32_t s = src[r];
        const int32_t t = dst[r];
        if (s >= 0 && t >= 0) {
          v[u] = host_store[static_cast<int64_t>(s) * record_vec + off];
          d[u] = static_cast<int64_t>(t) * record_vec + off;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] >= 0) packed[d[u]] = v[u];
  }
}

int pow2_at_least(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace
}  // namespace qcc

extern "C" int qcc_cache_resolve(const int32_t* ids, int k, const int32_t* k_dev, int32_t* slot_of, int n_records,
                                 int n_hot, int32_t* cache_owner, int32_t* cache_last_use, int capacity,
                                 const int32_t* cold_index, int step, int32_t* resident_out, int32_t* miss_slot_out,
                                 int32_t* miss_src_out, int32_t* counts_out, cudaStream_t stream) {
  if (k < 0 || n_records < 0 || n_hot < 0 || capacity < 1 || capacity > qcc::kMaxCapacity) return QCC_ERR_SHAPE;
  if (n_records >= (1 << 24) - 1 || step < 0 || step >= (1 << 24) - 1) return QCC_ERR_UNSUPPORTED;
  if (slot_of == nullptr || cache_owner == nullptr || cache_last_use == nullptr || cold_index == nullptr ||
      counts_out == nullptr ||
      (k > 0 && (ids == nullptr || resident_out == nullptr || miss_slot_out == nullptr || miss_src_out == nullptr)))
    return QCC_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const int sort_n = qcc::pow2_at_least(capacity);
  const size_t smem = static_cast<size_t>(sort_n) * 8 + static_cast<size_t>(capacity) * 5 + 16;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(qcc::cache_resolve_kernel), device))
    return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  qcc::cache_resolve_kernel<<<1, qcc::kResolveThreads, smem, stream>>>(
      ids, k, k_dev, slot_of, n_records, n_hot, cache_owner, cache_last_use, capacity, sort_n, cold_index, step,
      resident_out, miss_slot_out, miss_src_out, counts_out);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_gather_records(const void* host_store, int64_t record_bytes, const int32_t* src_index,
                                  const int32_t* dst_slot, const int32_t* count_dev, int max_count, void* packed,
                                  cudaStream_t stream) {
  if (record_bytes <= 0 || record_bytes % 16 != 0 || max_count < 0) return QCC_ERR_SHAPE;
  if (max_count == 0) return QCC_OK;
  if (host_store == nullptr || src_index == nullptr || dst_slot == nullptr || packed == nullptr)
    return QCC_ERR_INVALID_ARGUMENT;
  if (!qcc::aligned16(host_store) || !qcc::aligned16(packed)) return QCC_ERR_ALIGNMENT;
  // The store must be device-accessible: pinned (page-locked) host memory is
  // read through its device mapping; pageable host memory is refused rather
  // than dereferenced.
  cudaPointerAttributes attr;
  if (!qcc::cuda_ok(cudaPointerGetAttributes(&attr, host_store))) return QCC_ERR_INVALID_ARGUMENT;
  const void* store = host_store;
  if (attr.type == cudaMemoryTypeHost) {
    if (attr.devicePointer == nullptr) return QCC_ERR_INVALID_ARGUMENT;
    store = attr.devicePointer;
  } else if (attr.type == cudaMemoryTypeUnregistered) {
    return QCC_ERR_INVALID_ARGUMENT;
  }
  if (!qcc::aligned16(store)) return QCC_ERR_ALIGNMENT;
  qcc::clear_stale_error();
  qcc::gather_records_kernel<<<32, 512, 0, stream>>>(static_cast<const uint4*>(store), record_bytes / 16,
                                                     src_index, dst_slot, count_dev, max_count,
                                                     static_cast<uint4*>(packed));
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}
