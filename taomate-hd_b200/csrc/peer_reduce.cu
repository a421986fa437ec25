// Row-parallel reduction over NVLink peer memory (sm_100a).
//
// The fused reduce-scatter of a row-parallel W8A8 linear works in two steps
// on every rank:
//   1. the scaled-GEMM epilogue (gemm_i8.cu, scatter mode) stores each bf16
//      partial tile of rows owned by rank j directly into rank j's receive
//      buffer, slot [source rank], over NVLink, then publishes a per-tile
//      flag in rank j's flag array (system-scope release);
//   2. rs_reduce_kernel on each owner waits (bounded) for the tile's flags
//      from every source, sums the slots in fixed rank order in fp32, adds
//      the bias once and writes the owner's output rows.
// The transfers overlap the GEMM's remaining tiles; the reduction reads only
// local HBM.  No NVLS / multimem: plain peer stores and loads.
//
// Buffers are plain cudaMalloc allocations shared with CUDA IPC handles
// (tm_peer_alloc / tm_peer_open); they are allocated once per layer shape,
// never per call.
#include <cuda_bf16.h>

#include <cstring>

#include "common.h"
#include "ptx.cuh"
#include "peer_reduce.h"

namespace tmw {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Flag values are call epochs; "reached" is a wrap-safe epoch comparison.
__device__ __forceinline__ bool epoch_reached(uint32_t flag, uint32_t epoch) {
  return static_cast<int32_t>(flag - epoch) >= 0;
}

__global__ void __launch_bounds__(256) rs_reduce_kernel(const RsReduceArgs a) {
  __shared__ int abort_tile;
  const int tile = blockIdx.x;
  const int lrb = tile / a.num_n;  // 128-row block inside this owner's rows
  const int nb = tile - lrb * a.num_n;
  const int rbpo = a.rows_per_owner / 128;
  if (threadIdx.x == 0) abort_tile = 0;
  __syncthreads();
  if (threadIdx.x < a.world) {
    // One thread per source rank polls that source's flag for this tile.
    const uint32_t* f = a.flags + (static_cast<int64_t>(threadIdx.x) * rbpo + lrb) * a.num_n + nb;
    bool ok = epoch_reached(ld_acquire_sys(f), a.epoch);
    if (!ok) {
      const uint64_t t0 = globaltimer_ns();
      while (!(ok = epoch_reached(ld_acquire_sys(f), a.epoch))) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        __nanosleep(64);
      }
    }
    if (!ok) {
      abort_tile = 1;
      if (a.status) atomicExch(a.status, kDevWaitTimeout);
    }
  }
  __syncthreads();
  if (abort_tile) return;

  const int col0 = nb * a.tile_n;
  const int cols = min(a.tile_n, a.n - col0);  // multiple of 16
  const int vec_per_row = cols / 8;
  const int total = 128 * vec_per_row;
  const int64_t slot_elems = static_cast<int64_t>(a.rows_per_owner) * a.n;
  for (int v = threadIdx.x; v < total; v += blockDim.x) {
    const int r = v / vec_per_row;
    const int c = col0 + (v - r * vec_per_row) * 8;
    const int64_t row = static_cast<int64_t>(lrb) * 128 + r;
    const int64_t off = row * a.n + c;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int s = 0; s < a.world; ++s) {
      const uint4 raw = ld_cg16(a.recv + s * slot_elems + off);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
        acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
      }
    }
    if (a.bias != nullptr) {
      const uint4 braw = __ldg(reinterpret_cast<const uint4*>(a.bias + c));
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&braw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
        acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
      }
    }
    uint4 o;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) op[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(a.out + row * a.ldo + c) = o;
  }
}

}  // namespace

int launch_rs_reduce(const RsReduceArgs& args, cudaStream_t stream) {
  const int tiles = (args.rows_per_owner / 128) * args.num_n;
  if (tiles <= 0) return TM_OK;
  rs_reduce_kernel<<<tiles, 256, 0, stream>>>(args);
  return check_launch();
}

}  // namespace tmw

extern "C" {

int tm_peer_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int tm_peer_alloc(uint64_t bytes, void** ptr, void* handle_out) {
  if (ptr == nullptr || handle_out == nullptr) return TM_ERR_NULL_POINTER;
  if (bytes == 0) return TM_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TM_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return TM_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return TM_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return TM_OK;
}

int tm_peer_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return TM_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return TM_ERR_CUDA;
  *ptr = p;
  return TM_OK;
}

int tm_peer_close(void* ptr) {
  if (ptr == nullptr) return TM_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? TM_OK : TM_ERR_CUDA;
}

int tm_peer_free(void* ptr) {
  if (ptr == nullptr) return TM_ERR_NULL_POINTER;
  return cudaFree(ptr) == cudaSuccess ? TM_OK : TM_ERR_CUDA;
}

}  // extern "C"
