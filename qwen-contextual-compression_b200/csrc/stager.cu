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
//   use (empty slots first; among slots last used by the same step the record
//   with the lower id goes first -- the eviction order of the reference's
//   OrderedDict LRU, runtime/temporal.py:57-75), keeping the slots in an LRU
//   list on the device, and the slot table is updated in place.
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
constexpr int kMaxIds = 16384;

// counts_out: [0] resident, [1] misses served, [2] cache hits, [3] evicted,
//             [4] hot hits, [5] 1 if misses exceeded the free slots
//
// The cache slots are kept in an LRU list, lru[0] least recently used.  One
// step: classify the ids (hot / hit / miss) in id order; stable-partition the
// list into the slots this step does not use and the ones it hits; the
// misses take the first unused slots (evicting their records); the new list
// is the remaining unused slots followed by every slot the step used, in id
// order.  This is the order the reference's OrderedDict reaches by moving
// hits and appending misses id by id (runtime/temporal.py:63-73): empty
// slots never used stay at the front in slot order.
__global__ void __launch_bounds__(kResolveThreads, 1)
    cache_resolve_kernel(const int32_t* __restrict__ ids, int k, const int32_t* __restrict__ k_dev,
                         int32_t* __restrict__ slot_of, int n_records, int n_hot, int32_t* __restrict__ owner,
                         int32_t* __restrict__ last_use, int32_t* __restrict__ lru, int capacity,
                         const int32_t* __restrict__ cold_index, int step, int32_t* __restrict__ resident_out,
                         int32_t* __restrict__ miss_slot_out, int32_t* __restrict__ miss_src_out,
                         int32_t* __restrict__ counts_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* ring = reinterpret_cast<int32_t*>(smem_raw);   // [capacity] LRU order at the start of the step
  int32_t* unused = ring + capacity;                       // [capacity] slots the step does not use, in order
  int32_t* miss_ids = unused + capacity;                   // [capacity] missed ids, in id order
  int32_t* cls = miss_ids + capacity;                      // [kMaxIds] per id: slot >= 0, -1 miss, -2 invalid
  uint8_t* active = reinterpret_cast<uint8_t*>(cls + kMaxIds);  // [capacity]
  __shared__ int scratch[64];
  __shared__ int s_cnt[3];  // cache hits, hot hits, evicted

  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  int n = k;
  if (k_dev != nullptr) n = min(n, max(0, __ldg(k_dev)));
  n = min(n, kMaxIds);

  for (int c = tid; c < capacity; c += nthreads) {
    active[c] = 0;
    ring[c] = lru[c];
  }
  if (tid < 3) s_cnt[tid] = 0;
  __syncthreads();

  // 1. Classify in id order.  Contiguous chunk of ids per thread.
  const int chunk = (n + nthreads - 1) / nthreads;
  const int lo = min(n, tid * chunk);
  const int hi = min(n, lo + chunk);
  int n_res = 0, n_miss = 0, hits = 0, hot = 0;
  for (int i = lo; i < hi; ++i) {
    const int32_t id = ids[i];
    const int32_t s = (id >= 0 && id < n_records) ? slot_of[id] : -2;
    cls[i] = s;
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
  const int miss_base = block_exclusive_scan(n_miss, scratch, &total_miss);
  int miss_pos = miss_base;
  for (int i = lo; i < hi; ++i) {
    const int32_t s = cls[i];
    if (s >= 0) {
      resident_out[res_pos++] = s;
      if (s >= n_hot) last_use[s - n_hot] = step;
    } else if (s == -1) {
      if (miss_pos < capacity) miss_ids[miss_pos] = ids[i];
      ++miss_pos;
    }
  }
  __syncthreads();  // active[] complete

  // 2. Slots the step does not use, in LRU order.
  const int cchunk = (capacity + nthreads - 1) / nthreads;
  const int clo = min(capacity, tid * cchunk);
  const int chi = min(capacity, clo + cchunk);
  int n_unused = 0;
  for (int p = clo; p < chi; ++p) n_unused += !active[ring[p]];
  int total_unused;
  int up = block_exclusive_scan(n_unused, scratch, &total_unused);
  for (int p = clo; p < chi; ++p) {
    const int c = ring[p];
    if (!active[c]) unused[up++] = c;
  }
  __syncthreads();

  // 3. Miss i takes the i-th unused slot.
  const int served = min(total_miss, total_unused);
  int evicted = 0;
  for (int i = tid; i < served; i += nthreads) {
    const int c = unused[i];
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

  // 4. New order: the unused slots not taken, then the slots this step used in id order.
  const int keep = total_unused - served;
  for (int i = served + tid; i < total_unused; i += nthreads) lru[i - served] = unused[i];
  int n_used = 0;
  int mp = miss_base;
  for (int i = lo; i < hi; ++i) {
    const int32_t s = cls[i];
    if (s >= n_hot) {
      ++n_used;
    } else if (s == -1) {
      n_used += mp < served;
      ++mp;
    }
  }
  int total_used;
  int pos = block_exclusive_scan(n_used, scratch, &total_used);
  mp = miss_base;
  for (int i = lo; i < hi; ++i) {
    const int32_t s = cls[i];
    if (s >= n_hot) {
      lru[keep + pos++] = s - n_hot;
    } else if (s == -1) {
      if (mp < served) lru[keep + pos++] = unused[mp];
      ++mp;
    }
  }
  __syncthreads();
  if (tid == 0) {
    counts_out[0] = total_res;
    counts_out[1] = served;
    counts_out[2] = s_cnt[0];
    counts_out[3] = s_cnt[2];
    counts_out[4] = s_cnt[1];
    counts_out[5] = served < total_miss ? 1 : 0;
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

}  // namespace
}  // namespace qcc

extern "C" int qcc_cache_resolve(const int32_t* ids, int k, const int32_t* k_dev, int32_t* slot_of, int n_records,
                                 int n_hot, int32_t* cache_owner, int32_t* cache_last_use, int32_t* lru_order,
                                 int capacity, const int32_t* cold_index, int step, int32_t* resident_out,
                                 int32_t* miss_slot_out, int32_t* miss_src_out, int32_t* counts_out,
                                 cudaStream_t stream) {
  if (k < 0 || k > qcc::kMaxIds || n_records < 0 || n_hot < 0 || capacity < 1 || capacity > qcc::kMaxCapacity)
    return QCC_ERR_SHAPE;
  if (n_records >= (1 << 24) - 1 || step < 0 || step >= (1 << 24) - 1) return QCC_ERR_UNSUPPORTED;
  if (slot_of == nullptr || cache_owner == nullptr || cache_last_use == nullptr || lru_order == nullptr ||
      cold_index == nullptr || counts_out == nullptr ||
      (k > 0 && (ids == nullptr || resident_out == nullptr || miss_slot_out == nullptr || miss_src_out == nullptr)))
    return QCC_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const size_t smem = static_cast<size_t>(capacity) * 13 + static_cast<size_t>(qcc::kMaxIds) * 4 + 16;
  if (!qcc::ensure_max_dynamic_smem(reinterpret_cast<const void*>(qcc::cache_resolve_kernel), device))
    return QCC_ERR_CUDA;
  qcc::clear_stale_error();
  qcc::cache_resolve_kernel<<<1, qcc::kResolveThreads, smem, stream>>>(
      ids, k, k_dev, slot_of, n_records, n_hot, cache_owner, cache_last_use, lru_order, capacity, cold_index, step,
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
