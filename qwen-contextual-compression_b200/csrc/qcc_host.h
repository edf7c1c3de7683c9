// Host-side helpers shared by the qcc_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "qcc_b200.h"

namespace qcc {

struct DeviceInfo {
  int num_sms = 0;
  int max_smem_optin = 0;  // bytes of dynamic shared memory one block may opt into
};

// Cached per-device properties (thread-safe).
const DeviceInfo& device_info(int device);

// Raises a kernel's dynamic shared-memory limit to the device maximum, once
// per (kernel, device) for the whole process (thread-safe).  Raising it to
// the maximum, rather than to the size of one launch, keeps every later
// launch of that kernel valid whatever its size.
bool ensure_max_dynamic_smem(const void* kernel, int device);

inline bool valid_dtype(int dtype) {
  return dtype == QCC_DTYPE_BF16 || dtype == QCC_DTYPE_F16 || dtype == QCC_DTYPE_F32;
}

inline int dtype_bytes(int dtype) { return dtype == QCC_DTYPE_F32 ? 4 : 2; }

inline int hidden_pad(int hidden, int /*dtype*/) { return (hidden + 7) / 8 * 8; }

inline int64_t record_bytes(int hidden, int dtype) {
  return 3ll * hidden_pad(hidden, dtype) * dtype_bytes(dtype);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Remembers the error text for qcc_last_cuda_error_string(); true on success.
bool cuda_ok(cudaError_t err);
void record_cuda_error(cudaError_t err);
// Clears a pending error left by earlier runtime calls (so a launch check
// reports only this library's launch), and checks the launch just made.
void clear_stale_error();
bool launch_ok();

int decode_max_batch(int hidden, int dtype);
size_t decode_workspace_bytes(int batch, int hidden, int dtype);

int indexed_ffn_decode(const void* x, int64_t ldx, int batch, int hidden, const void* packed, int64_t n_records,
                       int dtype, const void* ids, int ids_kind, int n_ids, const int32_t* n_ids_dev,
                       const uint8_t* token_mask, void* workspace, size_t workspace_bytes, void* y_out, int64_t ldy,
                       int y_dtype, const float* y_in, int64_t ld_in, void* activation_out, int64_t lda,
                       cudaStream_t stream, void* const* xchg = nullptr, size_t xchg_bytes = 0, int world = 1,
                       int rank = 0, int64_t id_lo = -1, int64_t id_hi = -1);

// Bytes of one rank's cross-rank exchange buffer for this world / batch / hidden.
size_t exchange_bytes(int world, int batch, int hidden, int dtype);

}  // namespace qcc
