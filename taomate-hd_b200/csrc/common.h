// Internal host-side helpers shared by the translation units of
// libtaomate_w8a8.so: status plumbing, per-device properties and the TMA
// descriptor encoder (resolved from the driver at run time, so the library
// links only the CUDA runtime).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/taomate_w8a8.h"

namespace tmw {

// Device address of this device's status word (see tm_device_status).
// Resolved once per device; returns nullptr when CUDA fails.
int* device_status_ptr(int device);

// Number of SMs of `device` (cached).
int sm_count(int device);

// Current device of the calling thread, or -1.
int current_device();

// Encode a 2-D tensor map over a row-major byte matrix [rows, cols] with row
// stride `row_stride_bytes`, box [box_rows, box_cols], 128-byte swizzle.
// Returns false when the driver rejects the request.
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                    uint64_t cols, uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols,
                    uint32_t box_rows, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int check_launch() {
  return cudaGetLastError() == cudaSuccess ? TM_OK : TM_ERR_CUDA;
}

// Launch with programmatic dependent launch allowed (the kernel calls
// griddep_wait before reading global data): `attrs` are the launch's other
// attributes.  Should the driver refuse the combination, the launch is
// repeated without it (the kernel's griddep_wait is then a no-op).
template <typename... KArgs, typename... Args>
cudaError_t launch_with_pdl(cudaLaunchConfig_t cfg, const cudaLaunchAttribute* attrs, int nattrs,
                            void (*kernel)(KArgs...), Args&&... args) {
  cudaLaunchAttribute all[4];
  int n = 0;
  for (int i = 0; i < nattrs && n < 3; ++i) all[n++] = attrs[i];
  all[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  all[n].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = all;
  cfg.numAttrs = static_cast<unsigned>(n + 1);
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (err != cudaSuccess) {
    cudaGetLastError();
    cfg.numAttrs = static_cast<unsigned>(n);
    err = cudaLaunchKernelEx(&cfg, kernel, args...);
  }
  return err;
}

}  // namespace tmw
