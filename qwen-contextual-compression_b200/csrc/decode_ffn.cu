// Fused indexed gated FFN for decode / small batches (sm_100a).
//
// One persistent launch replaces the reference's two kernels
// (runtime/cuda_indexed.py:23-26 gate_up_* then down_*): each CTA owns a
// contiguous run of the selected-id list, streams the selected neurons'
// packed records [gate_row | up_row | down_col] from HBM into a shared-memory
// ring with one non-multicast bulk copy per record (mbarrier completion),
// computes g = G_j.x, u = U_j.x with fp32 accumulation, a_j = silu(g) * u,
// and accumulates a_j * D_j into a per-thread fp32 slice of y held in
// registers.  At the end each CTA adds its partial y into an fp32 workspace
// with vector reductions at L2; the last CTA to finish converts the sum to
// the output dtype and re-zeroes the workspace for the next call.
//
// Thread t of a CTA owns the 8-element hidden slots v = t + k * blockDim.x
// (k < VPT): it holds x[b, 8v:8v+8] and the partial y[b, 8v:8v+8] in
// registers, reads the matching 16-byte pieces of every staged record, and
// all partial dot products meet in one warp-shuffle + shared-atomic
// reduction per group of R records (one __syncthreads per group).

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "qcc_common.cuh"
#include "qcc_host.h"

namespace qcc {

namespace {

constexpr int kWorkspaceHeader = 256;  // status word, counter, padding
constexpr int kMaxStages = 8;
constexpr int kMaxThreads = 640;  // 5120 hidden / 8 per thread; caps registers at 96 per thread
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any barrier wait

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
  const uint8_t* token_mask;
  int n_ids;
  const int32_t* n_ids_dev;
  unsigned int* status;
  unsigned int* counter;
  float* y_acc;
  void* y_out;
  int64_t ldy;
  int y_dtype;
  void* a_out;
  int64_t lda;
  int a_dtype;
  int stages;
};

__device__ __forceinline__ int64_t load_id(const DecodeArgs& a, int j) {
  return a.ids64 ? __ldg(reinterpret_cast<const long long*>(a.ids) + j)
                 : static_cast<int64_t>(__ldg(reinterpret_cast<const int32_t*>(a.ids) + j));
}

template <typename T, int B, int VPT, int R>
__global__ void __launch_bounds__(kMaxThreads, 1) indexed_ffn_decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int nthreads = blockDim.x;
  const int S = a.stages;
  const int seg = a.hidden_pad;
  const int nslots = seg >> 3;
  constexpr int kVals = 2 * R * B;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * a.record_bytes);
  float* s_tot = reinterpret_cast<float*>(bars + kMaxStages);  // [3][kVals]
  int* s_flag = reinterpret_cast<int*>(s_tot + 3 * kVals);

  // This CTA's share of the id list.
  int n = a.n_ids;
  if (a.n_ids_dev != nullptr) n = min(n, max(0, __ldg(a.n_ids_dev)));
  const int begin = static_cast<int>((static_cast<int64_t>(n) * blockIdx.x) / gridDim.x);
  const int end = static_cast<int>((static_cast<int64_t>(n) * (blockIdx.x + 1)) / gridDim.x);
  const int cnt = end - begin;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  for (int i = tid; i < 3 * kVals; i += nthreads) s_tot[i] = 0.f;

  // x and the partial y live in registers (fp32).
  float xr[B][VPT][8];
  float yr[B][VPT][8];
  const T* xg = reinterpret_cast<const T*>(a.x);
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = tid + k * nthreads;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int h = 8 * v + e;
        xr[b][k][e] = (v < nslots && h < a.hidden) ? to_f32<T>(xg[b * a.ldx + h]) : 0.f;
        yr[b][k][e] = 0.f;
      }
    }
  __syncthreads();

  const uint64_t policy = policy_evict_first();
  const uint32_t rec_bytes = static_cast<uint32_t>(a.record_bytes);
  int issued = 0;  // meaningful in thread 0 only

  auto issue = [&](int i) {  // thread 0: start the bulk copy of local record i
    const int64_t id = load_id(a, begin + i);
    uint64_t* bar = &bars[i % S];
    if (id >= 0 && id < a.n_records) {
      mbar_arrive_expect_tx(bar, rec_bytes);
      bulk_load(smem + static_cast<size_t>(i % S) * a.record_bytes, a.packed + id * a.record_bytes, rec_bytes, bar,
                policy);
    } else {
      atomicOr(a.status, QCC_DEV_ID_RANGE);
      mbar_arrive(bar);  // completes the phase with no data; consumers skip it
    }
  };

  if (tid == 0) {
    const int pre = min(S, cnt);
    for (int i = 0; i < pre; ++i) issue(i);
    issued = pre;
  }

  int group = 0;
  int consumed = 0;
  bool aborted = false;
  for (int g0 = 0; g0 < cnt; g0 += R, ++group) {
    const int rn = min(R, cnt - g0);
    float pg[R][B], pu[R][B];
    Pack8<T> dn[R][VPT];
    bool ok = true;
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int b = 0; b < B; ++b) pg[r][b] = pu[r][b] = 0.f;
      if (r < rn) {
        const int i = g0 + r;
        ok = ok && mbar_wait_bounded(&bars[i % S], (i / S) & 1, kWaitLimitNs);
        const T* rec = reinterpret_cast<const T*>(smem + static_cast<size_t>(i % S) * a.record_bytes);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int v = tid + k * nthreads;
          if (v < nslots) {
            const Pack8<T> gr = load_pack8(rec + 8 * v);
            const Pack8<T> ur = load_pack8(rec + seg + 8 * v);
            dn[r][k] = load_pack8(rec + 2 * seg + 8 * v);
            float gf[8], uf[8];
            widen(gr, gf);
            widen(ur, uf);
#pragma unroll
            for (int b = 0; b < B; ++b)
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                pg[r][b] = fmaf(xr[b][k][e], gf[e], pg[r][b]);
                pu[r][b] = fmaf(xr[b][k][e], uf[e], pu[r][b]);
              }
          }
        }
      }
    }
    // Block-wide sums of the 2*R*B partial dot products.
    float* tot = s_tot + (group % 3) * kVals;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float sg = warp_sum(pg[r][b]);
        const float su = warp_sum(pu[r][b]);
        if (lane == 0 && r < rn) {
          atomicAdd(&tot[(r * B + b) * 2 + 0], sg);
          atomicAdd(&tot[(r * B + b) * 2 + 1], su);
        }
      }
    if (tid == 0) {
      float* nxt = s_tot + ((group + 1) % 3) * kVals;
      for (int q = 0; q < kVals; ++q) nxt[q] = 0.f;
    }
    if (__syncthreads_or(!ok)) {
      aborted = true;
      consumed = g0;
      break;
    }
    // Every thread has read the staged records of this group: refill them.
    if (tid == 0) {
      for (int r = 0; r < rn; ++r) {
        const int i = g0 + r + S;
        if (i < cnt) {
          issue(i);
          issued = i + 1;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < rn) {
        const int j = begin + g0 + r;
        const int64_t id = load_id(a, j);
        const bool valid = id >= 0 && id < a.n_records;
        const unsigned bits = a.token_mask ? __ldg(a.token_mask + j) : 0xFFu;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const float g = tot[(r * B + b) * 2 + 0];
          const float u = tot[(r * B + b) * 2 + 1];
          const bool use = valid && ((bits >> b) & 1u);
          const float act = use ? (g / (1.f + expf(-g))) * u : 0.f;
          if (a.a_out != nullptr && tid == 0) store_as(a.a_out, b * a.lda + j, a.a_dtype, act);
          if (use) {
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
              const int v = tid + k * nthreads;
              if (v < nslots) {
                float df[8];
                widen(dn[r][k], df);
#pragma unroll
                for (int e = 0; e < 8; ++e) yr[b][k][e] = fmaf(act, df[e], yr[b][k][e]);
              }
            }
          }
        }
      }
    }
  }

  if (aborted) {
    // Drain this CTA's bulk copies still in flight (bounded) before leaving.
    if (tid == 0) {
      atomicOr(a.status, QCC_DEV_TIMEOUT);
      for (int i = consumed; i < issued; ++i) (void)mbar_wait_bounded(&bars[i % S], (i / S) & 1, kWaitLimitNs);
    }
  } else {
    // Partial y -> fp32 workspace (vector reductions at L2).
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = tid + k * nthreads;
        if (v < nslots && cnt > 0) {
          float* dst = a.y_acc + static_cast<int64_t>(b) * seg + 8 * v;
          red_add_v4(dst, yr[b][k][0], yr[b][k][1], yr[b][k][2], yr[b][k][3]);
          red_add_v4(dst + 4, yr[b][k][4], yr[b][k][5], yr[b][k][6], yr[b][k][7]);
        }
      }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) *s_flag = (atomicAdd(a.counter, 1u) == gridDim.x - 1);
  __syncthreads();
  if (*s_flag) {
    // Last CTA: every partial is in; emit y and leave the workspace zeroed.
    __threadfence();
    for (int idx = tid; idx < B * nslots; idx += nthreads) {
      const int b = idx / nslots;
      const int v = idx - b * nslots;
      float* src = a.y_acc + static_cast<int64_t>(b) * seg + 8 * v;
      const float4 lo = __ldcg(reinterpret_cast<const float4*>(src));
      const float4 hi = __ldcg(reinterpret_cast<const float4*>(src + 4));
      const float vals[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int h = 8 * v + e;
        if (h < a.hidden) store_as(a.y_out, b * a.ldy + h, a.y_dtype, vals[e]);
      }
      __stcg(reinterpret_cast<float4*>(src), make_float4(0.f, 0.f, 0.f, 0.f));
      __stcg(reinterpret_cast<float4*>(src + 4), make_float4(0.f, 0.f, 0.f, 0.f));
    }
    if (tid == 0) *a.counter = 0u;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using KernelFn = void (*)(const DecodeArgs);

// One hidden slot per thread (hidden <= 5120): batch 1..4.  Two slots per
// thread (hidden <= 10240): batch 1..2, which keeps x and y in registers.
template <typename T, int R>
KernelFn pick_kernel(int batch, int vpt) {
  if (vpt == 1) {
    switch (batch) {
      case 1: return indexed_ffn_decode_kernel<T, 1, 1, R>;
      case 2: return indexed_ffn_decode_kernel<T, 2, 1, R>;
      case 3: return indexed_ffn_decode_kernel<T, 3, 1, R>;
      case 4: return indexed_ffn_decode_kernel<T, 4, 1, R>;
      default: return nullptr;
    }
  }
  switch (batch) {
    case 1: return indexed_ffn_decode_kernel<T, 1, 2, R>;
    case 2: return indexed_ffn_decode_kernel<T, 2, 2, R>;
    default: return nullptr;
  }
}

int vpt_for(int hidden_pad_) {
  const int nslots = hidden_pad_ / 8;
  if (nslots <= kMaxThreads) return 1;
  if (nslots <= 2 * kMaxThreads) return 2;
  return 0;
}

constexpr int records_per_group(int dtype) { return dtype == QCC_DTYPE_F32 ? 1 : 2; }

struct LaunchShape {
  int threads;
  int vpt;
  int stages;
  size_t smem;
};

size_t tail_bytes(int batch, int group) {
  return kMaxStages * sizeof(uint64_t) + 3 * 2 * group * batch * sizeof(float) + 16;
}

bool plan_launch(int batch, int hidden_pad, int64_t record_bytes, int dtype, int max_smem, LaunchShape* out) {
  const int nslots = hidden_pad / 8;
  int vpt = 1;
  if (nslots > kMaxThreads) vpt = 2;
  if (nslots > 2 * kMaxThreads) return false;
  const int per = (nslots + vpt - 1) / vpt;
  const int threads = std::max(32, (per + 31) / 32 * 32);
  const int group = records_per_group(dtype);
  const size_t tail = tail_bytes(batch, group);
  if (record_bytes <= 0 || static_cast<size_t>(max_smem) < tail) return false;
  int stages = static_cast<int>((static_cast<size_t>(max_smem) - tail) / static_cast<size_t>(record_bytes));
  stages = std::min(stages, kMaxStages);
  if (stages < 2) return false;
  out->threads = threads;
  out->vpt = vpt;
  out->stages = stages;
  out->smem = static_cast<size_t>(stages) * record_bytes + tail;
  return true;
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

// Blocks per SM for a kernel configuration (also raises the kernel's dynamic
// shared-memory limit once per device).  0 on failure.
int blocks_per_sm(KernelFn fn, int device, int threads, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<OccKey, int, OccHash> cache;
  const OccKey key{reinterpret_cast<const void*>(fn), device, threads, smem};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return 0;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, threads, smem) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = nb;
  return nb;
}

}  // namespace

int decode_max_batch(int hidden, int dtype) {
  const int vpt = vpt_for(hidden_pad(hidden, dtype));
  return vpt == 1 ? 4 : (vpt == 2 ? 2 : 0);
}

size_t decode_workspace_bytes(int batch, int hidden, int dtype) {
  const int hp = hidden_pad(hidden, dtype);
  const size_t y = static_cast<size_t>(batch) * hp * sizeof(float);
  return kWorkspaceHeader + (y + 255) / 256 * 256;
}

int indexed_ffn_decode(const void* x, int64_t ldx, int batch, int hidden, const void* packed, int64_t n_records,
                       int dtype, const void* ids, int ids_dtype, int n_ids, const int32_t* n_ids_dev,
                       const uint8_t* token_mask, void* workspace, size_t workspace_bytes, void* y_out, int64_t ldy,
                       int y_dtype, void* activation_out, int64_t lda, cudaStream_t stream) {
  if (!valid_dtype(dtype) || !valid_dtype(y_dtype)) return QCC_ERR_DTYPE;
  if (y_dtype != dtype && y_dtype != QCC_DTYPE_F32) return QCC_ERR_DTYPE;
  if (ids_dtype != QCC_INDEX_I32 && ids_dtype != QCC_INDEX_I64) return QCC_ERR_DTYPE;
  if (batch < 1 || hidden < 1 || n_records < 0 || n_ids < 0) return QCC_ERR_SHAPE;
  if (batch > decode_max_batch(hidden, dtype)) return QCC_ERR_UNSUPPORTED;
  if (ldx < hidden || ldy < hidden || (activation_out != nullptr && lda < n_ids)) return QCC_ERR_SHAPE;
  if (x == nullptr || y_out == nullptr || workspace == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (n_ids > 0 && (ids == nullptr || packed == nullptr)) return QCC_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < decode_workspace_bytes(batch, hidden, dtype)) return QCC_ERR_WORKSPACE;
  if (!aligned16(packed) || !aligned16(workspace)) return QCC_ERR_ALIGNMENT;

  const int hp = hidden_pad(hidden, dtype);
  const int64_t rec = record_bytes(hidden, dtype);
  int device = 0;
  if (!cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  const DeviceInfo& info = device_info(device);
  if (info.num_sms <= 0) return QCC_ERR_CUDA;

  LaunchShape shape;
  if (!plan_launch(batch, hp, rec, dtype, info.max_smem_optin, &shape)) return QCC_ERR_UNSUPPORTED;

  KernelFn fn = nullptr;
  if (dtype == QCC_DTYPE_BF16)
    fn = pick_kernel<__nv_bfloat16, records_per_group(QCC_DTYPE_BF16)>(batch, shape.vpt);
  else if (dtype == QCC_DTYPE_F16)
    fn = pick_kernel<__half, records_per_group(QCC_DTYPE_F16)>(batch, shape.vpt);
  else
    fn = pick_kernel<float, records_per_group(QCC_DTYPE_F32)>(batch, shape.vpt);
  if (fn == nullptr) return QCC_ERR_UNSUPPORTED;

  const int nb = blocks_per_sm(fn, device, shape.threads, shape.smem);
  if (nb <= 0) {
    record_cuda_error(cudaGetLastError());
    return QCC_ERR_CUDA;
  }
  int64_t grid = static_cast<int64_t>(info.num_sms) * nb;
  if (n_ids_dev == nullptr) grid = std::min<int64_t>(grid, std::max(1, n_ids));

  DecodeArgs args;
  args.x = x;
  args.ldx = ldx;
  args.packed = static_cast<const uint8_t*>(packed);
  args.record_bytes = rec;
  args.n_records = n_records;
  args.hidden = hidden;
  args.hidden_pad = hp;
  args.ids = ids;
  args.ids64 = ids_dtype == QCC_INDEX_I64;
  args.token_mask = token_mask;
  args.n_ids = n_ids;
  args.n_ids_dev = n_ids_dev;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  args.status = reinterpret_cast<unsigned int*>(ws);
  args.counter = reinterpret_cast<unsigned int*>(ws + 4);
  args.y_acc = reinterpret_cast<float*>(ws + kWorkspaceHeader);
  args.y_out = y_out;
  args.ldy = ldy;
  args.y_dtype = y_dtype;
  args.a_out = activation_out;
  args.lda = lda;
  args.a_dtype = dtype;
  args.stages = shape.stages;

  fn<<<static_cast<unsigned>(grid), shape.threads, shape.smem, stream>>>(args);
  if (!cuda_ok(cudaGetLastError())) return QCC_ERR_CUDA;
  return QCC_OK;
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
                                      void* activation_out, int64_t lda, cudaStream_t stream) {
  return qcc::indexed_ffn_decode(x, ldx, batch, hidden, packed, n_records, dtype, ids, ids_dtype, n_ids, n_ids_dev,
                                 token_mask, workspace, workspace_bytes, y_out, ldy, y_dtype, activation_out, lda,
                                 stream);
}
