// Library-wide C entry points: version, status text, workspace set-up, the
// neuron-major packer and the fp32 cast used after a cross-rank sum.

#include <cuda_runtime.h>

#include <cstring>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "qcc_common.cuh"
#include "qcc_host.h"

namespace qcc {

namespace {
thread_local cudaError_t g_last_error = cudaSuccess;

// record n = [gate[n, :Hp] | up[n, :Hp] | down[:Hp, n]], zero padded.
// Grid-stride over (record, element) pairs: consecutive threads of a warp
// write 32 consecutive elements of one record.  Down element (h, n) is read
// at h * sh + n * sn (row-major [hidden, n_records] or the transposed copy).
// Packing runs once per layer, so the strided down reads are not tuned.
template <typename T>
__global__ void pack_records_kernel(const T* __restrict__ gate, const T* __restrict__ up, int64_t ld_gu,
                                    const T* __restrict__ down, int64_t sh, int64_t sn, int64_t n_records,
                                    int hidden, int hp, T* __restrict__ packed) {
  const int64_t per = 3ll * hp;
  const int64_t total = n_records * per;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / per;
    const int64_t r = i - n * per;
    const int part = static_cast<int>(r / hp);
    const int h = static_cast<int>(r - static_cast<int64_t>(part) * hp);
    T v = T(0.f);
    if (h < hidden) {
      if (part == 0)
        v = gate[n * ld_gu + h];
      else if (part == 1)
        v = up[n * ld_gu + h];
      else
        v = down[static_cast<int64_t>(h) * sh + n * sn];
    }
    packed[i] = v;
  }
}

// ||W[:, c]||_2 for the columns of a row-major [rows, cols] matrix: thread c
// walks its column down the rows (consecutive threads read consecutive
// columns, so every row read is coalesced), accumulating squares in fp64, and
// rounds the square root once to fp32.  The 8 rows of an unrolled step are
// loaded before any is added, so eight loads per thread are in flight.
template <typename T>
__global__ void column_norms_kernel(const T* __restrict__ w, int64_t ld, int64_t rows, int64_t cols,
                                    float* __restrict__ out) {
  const int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (c >= cols) return;
  double acc = 0.0;
  int64_t r = 0;
  for (; r + 8 <= rows; r += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = to_f32<T>(w[(r + u) * ld + c]);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc += static_cast<double>(v[u]) * static_cast<double>(v[u]);
  }
  for (; r < rows; ++r) {
    const double v = to_f32<T>(w[r * ld + c]);
    acc += v * v;
  }
  out[c] = static_cast<float>(sqrt(acc));
}

__global__ void cast_f32_kernel(const float* __restrict__ src, void* dst, int64_t n, int dtype) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_as(dst, i, dtype, src[i]);
}

}  // namespace

void record_cuda_error(cudaError_t err) {
  if (err != cudaSuccess) g_last_error = err;
}

bool cuda_ok(cudaError_t err) {
  if (err == cudaSuccess) return true;
  record_cuda_error(err);
  (void)cudaGetLastError();  // do not leave a non-sticky error for the next caller to find
  return false;
}

bool launch_ok() {
  const cudaError_t err = cudaGetLastError();
  return cuda_ok(err);
}

void clear_stale_error() { (void)cudaGetLastError(); }

const DeviceInfo& device_info(int device) {
  static std::mutex mu;
  static DeviceInfo infos[64];
  static bool ready[64] = {};
  static DeviceInfo none;
  if (device < 0 || device >= 64) return none;
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[device]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess)
      return none;
    infos[device] = d;
    ready[device] = true;
  }
  return infos[device];
}

bool ensure_max_dynamic_smem(const void* kernel, int device) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(kernel, device);
  if (done.count(key)) return true;
  const DeviceInfo& info = device_info(device);
  if (info.max_smem_optin <= 0) return false;
  cudaFuncAttributes attr;
  if (!cuda_ok(cudaFuncGetAttributes(&attr, kernel))) return false;
  const int dynamic_max = info.max_smem_optin - static_cast<int>(attr.sharedSizeBytes);
  if (!cuda_ok(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dynamic_max)))
    return false;
  done.insert(key);
  return true;
}

}  // namespace qcc

extern "C" int qcc_version(void) { return QCC_ABI_VERSION; }

extern "C" const char* qcc_status_string(int status) {
  switch (status) {
    case QCC_OK:
      return "ok";
    case QCC_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, negative size or unknown enum)";
    case QCC_ERR_SHAPE:
      return "inconsistent shape or stride";
    case QCC_ERR_DTYPE:
      return "unsupported dtype";
    case QCC_ERR_ALIGNMENT:
      return "pointer or stride is not 16-byte aligned";
    case QCC_ERR_UNSUPPORTED:
      return "size beyond what the kernels support";
    case QCC_ERR_WORKSPACE:
      return "workspace missing or too small";
    case QCC_ERR_CUDA:
      return "CUDA runtime error";
    default:
      return "unknown status";
  }
}

extern "C" const char* qcc_last_cuda_error_string(void) { return cudaGetErrorString(qcc::g_last_error); }

extern "C" int qcc_hidden_pad(int hidden, int dtype) { return qcc::hidden_pad(hidden, dtype); }

extern "C" int64_t qcc_record_bytes(int hidden, int dtype) {
  if (!qcc::valid_dtype(dtype) || hidden < 1) return 0;
  return qcc::record_bytes(hidden, dtype);
}

extern "C" size_t qcc_workspace_status_offset(void) { return 0; }

extern "C" int qcc_workspace_init(void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (workspace == nullptr || workspace_bytes == 0) return QCC_ERR_WORKSPACE;
  if (!qcc::cuda_ok(cudaMemsetAsync(workspace, 0, workspace_bytes, stream))) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_pack_records(const void* gate, const void* up, int64_t ld_gu, const void* down,
                                int64_t down_stride_h, int64_t down_stride_n, int64_t n_records, int hidden,
                                int dtype, void* packed, cudaStream_t stream) {
  if (!qcc::valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (n_records < 0 || hidden < 1 || ld_gu < hidden || down_stride_h < 1 || down_stride_n < 1) return QCC_ERR_SHAPE;
  if (n_records == 0) return QCC_OK;
  if (gate == nullptr || up == nullptr || down == nullptr || packed == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  if (!qcc::aligned16(packed)) return QCC_ERR_ALIGNMENT;
  const int hp = qcc::hidden_pad(hidden, dtype);
  const int64_t total = n_records * 3ll * hp;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148ll * 16);
#define QCC_PACK(T)                                                                                              \
  qcc::pack_records_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(                            \
      static_cast<const T*>(gate), static_cast<const T*>(up), ld_gu, static_cast<const T*>(down), down_stride_h, \
      down_stride_n, n_records, hidden, hp, static_cast<T*>(packed))
  qcc::clear_stale_error();
  if (dtype == QCC_DTYPE_BF16)
    QCC_PACK(__nv_bfloat16);
  else if (dtype == QCC_DTYPE_F16)
    QCC_PACK(__half);
  else
    QCC_PACK(float);
#undef QCC_PACK
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_column_norms(const void* w, int64_t ld, int64_t rows, int64_t cols, int dtype, float* out,
                                cudaStream_t stream) {
  if (!qcc::valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (rows < 0 || cols < 0 || ld < cols) return QCC_ERR_SHAPE;
  if (cols == 0) return QCC_OK;
  if (w == nullptr || out == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  const int threads = 128;
  const int64_t blocks = (cols + threads - 1) / threads;
  qcc::clear_stale_error();
  if (dtype == QCC_DTYPE_BF16)
    qcc::column_norms_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(w), ld, rows, cols, out);
  else if (dtype == QCC_DTYPE_F16)
    qcc::column_norms_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(static_cast<const __half*>(w), ld,
                                                                                   rows, cols, out);
  else
    qcc::column_norms_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(static_cast<const float*>(w), ld,
                                                                                   rows, cols, out);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_cast_f32(const float* src, void* dst, int64_t n, int dtype, cudaStream_t stream) {
  if (!qcc::valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (n < 0) return QCC_ERR_SHAPE;
  if (n == 0) return QCC_OK;
  if (src == nullptr || dst == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 148ll * 8);
  qcc::clear_stale_error();
  qcc::cast_f32_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(src, dst, n, dtype);
  if (!qcc::launch_ok()) return QCC_ERR_CUDA;
  return QCC_OK;
}

// ---------------------------------------------------------------------------
// Cross-rank exchange buffers (setup time: these allocate and map memory).
// ---------------------------------------------------------------------------

namespace {
__global__ void fill_u32_kernel(uint32_t* p, size_t n, uint32_t v) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}
}  // namespace

// The 256-byte header (launch counter, wait bound) starts at zero, the
// column-sum words after it as the empty mark (the bits of -0.0f).
extern "C" int qcc_exchange_init(void* ptr, size_t bytes) {
  if (ptr == nullptr || bytes <= 256 || bytes % 16 != 0) return QCC_ERR_INVALID_ARGUMENT;
  qcc::clear_stale_error();
  fill_u32_kernel<<<64, 256>>>(static_cast<uint32_t*>(ptr) + 64, (bytes - 256) / 4, 0x80000000u);
  if (!qcc::launch_ok() || !qcc::cuda_ok(cudaMemset(ptr, 0, 256)) || !qcc::cuda_ok(cudaDeviceSynchronize()))
    return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_exchange_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes <= 256 || bytes % 16 != 0) return QCC_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (!qcc::cuda_ok(cudaMalloc(&p, bytes))) return QCC_ERR_CUDA;
  const int status = qcc_exchange_init(p, bytes);
  if (status != QCC_OK) {
    cudaFree(p);
    return status;
  }
  *ptr = p;
  return QCC_OK;
}

extern "C" int qcc_exchange_set_wait_limit(void* ptr, uint64_t limit_ns) {
  if (ptr == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  // u64 at byte 8 of the header; the decode reduce launch reads it there.
  if (!qcc::cuda_ok(cudaMemcpy(static_cast<uint8_t*>(ptr) + 8, &limit_ns, sizeof(limit_ns), cudaMemcpyHostToDevice)))
    return QCC_ERR_CUDA;
  return QCC_OK;
}

extern "C" int qcc_exchange_free(void* ptr) {
  if (ptr == nullptr) return QCC_OK;
  return qcc::cuda_ok(cudaFree(ptr)) ? QCC_OK : QCC_ERR_CUDA;
}

extern "C" int qcc_ipc_handle(void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  static_assert(sizeof(cudaIpcMemHandle_t) == QCC_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (!qcc::cuda_ok(cudaIpcGetMemHandle(&h, ptr))) return QCC_ERR_CUDA;
  std::memcpy(handle, &h, sizeof(h));
  return QCC_OK;
}

extern "C" int qcc_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return QCC_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (!qcc::cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))) return QCC_ERR_CUDA;
  *ptr = p;
  return QCC_OK;
}

extern "C" int qcc_ipc_close(void* ptr) {
  if (ptr == nullptr) return QCC_OK;
  return qcc::cuda_ok(cudaIpcCloseMemHandle(ptr)) ? QCC_OK : QCC_ERR_CUDA;
}
