// Shared declarations of the fused row-parallel reduce-scatter: the owner-side
// reduction launched after the scatter-mode GEMM (peer_reduce.cu).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tmw {

constexpr int kMaxPeers = 8;

struct RsReduceArgs {
  const __nv_bfloat16* recv;   // this owner's receive slots [world][rows_per_owner][n]
  const uint32_t* flags;       // this owner's flags [world][rows_per_owner / 128][num_n]
  const __nv_bfloat16* bias;   // [n] or null (added once, after the sum)
  __nv_bfloat16* out;          // [rows_per_owner][ldo]
  int64_t ldo;
  int world;
  int rows_per_owner;          // multiple of 256
  int n;                       // multiple of 16
  int tile_n;                  // N width of the GEMM tile that produced the flags
  int num_n;                   // ceil(n / tile_n)
  uint32_t epoch;              // value the sources publish for this call
  int* status;
};

int launch_rs_reduce(const RsReduceArgs& args, cudaStream_t stream);

}  // namespace tmw
