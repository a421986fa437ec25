// Library-wide runtime pieces: the per-device status word, cached device
// properties, the TMA descriptor encoder and the status/version entry points.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.h"

namespace tmw {

// One status word per device that loads the library.  Kernels record wait
// timeouts here; the host reads it with tm_device_status().
__device__ int g_device_status = 0;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int* device_status_ptr(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_ptr[device] == nullptr) {
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return nullptr;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return nullptr;
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_device_status);
    if (prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return nullptr;
    g_status_ptr[device] = static_cast<int*>(p);
  }
  return g_status_ptr[device];
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_sm_count[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    g_sm_count[device] = n;
  }
  return g_sm_count[device];
}

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t cols,
                    uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                    CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr)
        return false;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box,
                              elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tmw

extern "C" {

const char* tm_status_string(int status) {
  switch (status) {
    case TM_OK: return "ok";
    case TM_ERR_NULL_POINTER: return "a required pointer is NULL";
    case TM_ERR_SHAPE: return "invalid or inconsistent sizes/strides";
    case TM_ERR_ALIGNMENT: return "pointer or stride alignment requirement not met";
    case TM_ERR_DTYPE: return "unsupported dtype";
    case TM_ERR_UNSUPPORTED: return "unsupported request";
    case TM_ERR_CUDA: return "CUDA runtime error";
    case TM_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
    case TM_ERR_TOO_LARGE: return "size exceeds the documented maximum";
    default: return "unknown status";
  }
}

int tm_version(void) { return 100; }

int tm_device_status(int device, int* code, int clear) {
  if (code == nullptr) return TM_ERR_NULL_POINTER;
  int* p = tmw::device_status_ptr(device);
  if (p == nullptr) return TM_ERR_CUDA;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return TM_ERR_CUDA;
  if (prev != device && cudaSetDevice(device) != cudaSuccess) return TM_ERR_CUDA;
  int value = 0;
  cudaError_t err = cudaMemcpy(&value, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (err == cudaSuccess && clear) {
    const int zero = 0;
    err = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  if (prev != device) cudaSetDevice(prev);
  if (err != cudaSuccess) return TM_ERR_CUDA;
  *code = value;
  return TM_OK;
}

}  // extern "C"
