// Shared device helpers for the qcc_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qcc_b200.h"

namespace qcc {

// ---------------------------------------------------------------------------
// Shared-memory addressing, mbarriers and 1-D bulk (TMA) copies.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for a barrier phase. Returns false if `limit_ns` elapsed first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > limit_ns) return false;
  }
}

// Cache policy for data that later reads of the same kernel should find in L2.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Cache policy for streamed weights: read once, do not keep in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// One non-multicast bulk copy global -> this CTA's shared memory; completion
// is signalled on `bar` as transaction bytes.  dst, src and bytes must be
// multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Vector reduction of 4 fp32 values into global memory (performed at L2).
__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// ---------------------------------------------------------------------------
// 8-element vectors: raw shared-memory words and widening to fp32.
// ---------------------------------------------------------------------------

template <typename T>
struct Pack8 {
  static constexpr int kWords = sizeof(T) * 8 / 16;  // 16-byte words
  uint4 w[kWords];
};

template <typename T>
__device__ __forceinline__ Pack8<T> load_pack8(const T* p) {
  Pack8<T> r;
#pragma unroll
  for (int i = 0; i < Pack8<T>::kWords; ++i) r.w[i] = reinterpret_cast<const uint4*>(p)[i];
  return r;
}

// Same 8 elements from global memory through the read-only path (16-byte aligned).
template <typename T>
__device__ __forceinline__ Pack8<T> load_global_pack8(const T* p) {
  Pack8<T> r;
#pragma unroll
  for (int i = 0; i < Pack8<T>::kWords; ++i) r.w[i] = __ldg(reinterpret_cast<const uint4*>(p) + i);
  return r;
}

__device__ __forceinline__ void bf16x2_to_f32(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
}

__device__ __forceinline__ void widen(const Pack8<__nv_bfloat16>& r, float (&f)[8]) {
  bf16x2_to_f32(r.w[0].x, f[0], f[1]);
  bf16x2_to_f32(r.w[0].y, f[2], f[3]);
  bf16x2_to_f32(r.w[0].z, f[4], f[5]);
  bf16x2_to_f32(r.w[0].w, f[6], f[7]);
}

__device__ __forceinline__ void half2_to_f32(uint32_t w, float& lo, float& hi) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 v = __half22float2(h);
  lo = v.x;
  hi = v.y;
}

__device__ __forceinline__ void widen(const Pack8<__half>& r, float (&f)[8]) {
  half2_to_f32(r.w[0].x, f[0], f[1]);
  half2_to_f32(r.w[0].y, f[2], f[3]);
  half2_to_f32(r.w[0].z, f[4], f[5]);
  half2_to_f32(r.w[0].w, f[6], f[7]);
}

__device__ __forceinline__ void widen(const Pack8<float>& r, float (&f)[8]) {
  f[0] = __uint_as_float(r.w[0].x);
  f[1] = __uint_as_float(r.w[0].y);
  f[2] = __uint_as_float(r.w[0].z);
  f[3] = __uint_as_float(r.w[0].w);
  f[4] = __uint_as_float(r.w[1].x);
  f[5] = __uint_as_float(r.w[1].y);
  f[6] = __uint_as_float(r.w[1].z);
  f[7] = __uint_as_float(r.w[1].w);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

// Store one fp32 value as the element type given at run time.
__device__ __forceinline__ void store_as(void* base, int64_t idx, int dtype, float v) {
  if (dtype == QCC_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else if (dtype == QCC_DTYPE_F16)
    reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(base)[idx] = v;
}

// Exclusive block-wide scan of one int per thread (blockDim.x a multiple of
// 32, at most 1024).  Returns this thread's prefix; *total receives the block
// sum.  `scratch` holds >= 33 ints.  Contains __syncthreads: call from every
// thread of the block.
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

// Order-preserving 32-bit key of a score: larger score, larger key.  -0.0
// and +0.0 share a key; every NaN maps to the largest key (it ranks first,
// as in torch.topk).
__device__ __forceinline__ uint32_t score_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0xFFFFFFFFu;
  if ((u & 0x7FFFFFFFu) == 0u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Finds the bin holding the rem-th largest element of a histogram whose bins
// are visited from the highest down.  Thread t holds PER consecutive bins, its
// highest one first, so an exclusive scan in thread order counts the elements
// in all higher bins.  Writes the bin and rem minus the elements above it.
// Requires 1 <= rem <= total count and nbins == PER * blockDim.x.  Contains
// __syncthreads (block_exclusive_scan).
template <int PER>
__device__ __forceinline__ void find_bin(const int* hist, int rem, int* scratch, int* out_bin, int* out_rem) {
  const int top = PER * static_cast<int>(blockDim.x) - 1 - PER * static_cast<int>(threadIdx.x);
  int c[PER];
  int s = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    c[j] = hist[top - j];
    s += c[j];
  }
  int total;
  int above = block_exclusive_scan(s, scratch, &total);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (above < rem && above + c[j] >= rem) {
      *out_bin = top - j;
      *out_rem = rem - above;
    }
    above += c[j];
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace qcc
