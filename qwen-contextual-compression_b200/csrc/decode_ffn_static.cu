// qcc_indexed_ffn_decode_static: the fused decode entry point without a
// caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run the
// layer: code running inside another framework's memory pool or allocator
// callback, plugin hosts that hand out only the input and output buffers, or
// real-time loops that forbid cudaMalloc/cudaFree (both can synchronise the
// device).  For them this entry point keeps its scratch in a fixed array that
// is part of the library image, so a call allocates nothing.
//
// The scratch is kStaticScratchBytes (4 MiB) of device memory that every GPU
// holds from the time the library's module is loaded on it until the process
// exits.  It is large enough for one token at hidden sizes up to 6552 (the
// status / counter header plus one fp32 partial row of the hidden size per
// CTA, for up to 160 CTAs); larger requests are rejected.
//
// All calls on one device share the array.  The first call on each device
// looks up the array's device address with cudaGetSymbolAddress (this may
// load the module on that device), so make that first call before any stream
// capture.  The address is kept for the life of the process: after a
// cudaDeviceReset (or any other teardown of the device's primary context) it
// no longer names the reloaded array, and this entry point must not be used
// on that device again.  Nothing in the array needs clearing between calls:
// the single-device decode reads no counter from its scratch, only writes the
// status word (which this entry point cannot report) and the partial rows it
// reads back in the same call.  Calls that can overlap on the GPU (different
// streams without ordering, or several host threads) race on the array and
// must be serialised by the caller.

#include <cuda_runtime.h>

#include <mutex>

#include "qcc_host.h"

namespace qcc {
namespace {

constexpr size_t kStaticScratchBytes = QCC_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Zero-initialised when the module is loaded; only device code and the
// address returned by cudaGetSymbolAddress may touch it (in host code the name
// is a host-side stand-in, not a device address).
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on `device` (the current device), looked
// up once per device.  Null when the lookup fails.
void* scratch_for_device(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (!cuda_ok(cudaGetSymbolAddress(&ptr, g_decode_scratch))) return nullptr;
    g_scratch_ptr[device] = ptr;
  }
  return g_scratch_ptr[device];
}

}  // namespace
}  // namespace qcc

extern "C" int qcc_indexed_ffn_decode_static(const void* x, int64_t ldx, int batch, int hidden, const void* packed,
                                             int64_t n_records, int dtype, const void* ids, int ids_dtype, int n_ids,
                                             const int32_t* n_ids_dev, const uint8_t* token_mask, void* y_out,
                                             int64_t ldy, int y_dtype, void* activation_out, int64_t lda,
                                             cudaStream_t stream) {
  if (!qcc::valid_dtype(dtype)) return QCC_ERR_DTYPE;
  if (batch < 1 || hidden < 1) return QCC_ERR_SHAPE;
  const size_t needed = qcc::decode_workspace_bytes(batch, hidden, dtype);
  if (needed > qcc::kStaticScratchBytes) return QCC_ERR_WORKSPACE;  // beyond the built-in scratch
  int device = 0;
  if (!qcc::cuda_ok(cudaGetDevice(&device))) return QCC_ERR_CUDA;
  void* scratch = qcc::scratch_for_device(device);
  if (scratch == nullptr) return QCC_ERR_CUDA;
  return qcc::indexed_ffn_decode(x, ldx, batch, hidden, packed, n_records, dtype, ids, ids_dtype, n_ids, n_ids_dev,
                                 token_mask, scratch, qcc::kStaticScratchBytes, y_out, ldy, y_dtype, nullptr, 0,
                                 activation_out, lda, stream);
}
