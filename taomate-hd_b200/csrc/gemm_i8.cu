// Scaled int8 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   out[m, n] = cvt(scale_a[m] * (scale_b[n] * float(sum_k a[m,k] * b[n,k])) (+ bias[n]))
//
// Replaces vLLM's cutlass_scaled_mm as called by the reference
// (src/taomate_hd/inference/w8a8.py:72 and :142-144).
//
// Kernel structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: per k-block, one 128 x 128 A tile and one
//               BN x 128 B tile (int8, K-major, 128-byte swizzle) into a
//               STAGES-deep shared-memory ring; completion by transaction
//               bytes on the stage's `full` mbarrier.
//   warp 1      TMEM owner + MMA issuer: allocates 2 x BN TMEM columns (two
//               int32 accumulators of 128 lanes x BN), one thread issues
//               tcgen05.mma.kind::i8 (M=128, N=BN, K=32) four times per
//               k-block and commits to the stage's `empty` barrier; after the
//               last k-block it commits to the accumulator's `tmem_full`.
//   warps 2..5  epilogue: wait `tmem_full`, tcgen05.ld 32 columns at a time
//               (warp w reads TMEM lanes 32*(w%4)..+31 = tile rows), apply
//               the fp32 dequant / bias / activation, store bf16/fp16, then
//               release the accumulator via `tmem_empty`.  With two
//               accumulators the epilogue of tile i overlaps the main loop of
//               tile i+1.
// Tiles are visited in groups of 16 M-blocks so that concurrently resident
// CTAs share A and B panels in L2.  M, N and K tails are handled by TMA
// zero fill (loads) and predicated stores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"
#include "ptx.cuh"

namespace tmw {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes == int8 elements per k-block (one swizzle row)
constexpr int kThreads = 192;
constexpr int kGroupM = 16;

struct GemmArgs {
  const float* sa;
  const float* sb;
  int sa_per_row;
  int sb_per_col;
  const void* bias;
  void* out;
  int64_t ldo;
  int32_t* acc_debug;
  int M, N, K;
  int num_m, num_n, kblocks;
  uint32_t epilogue;
  int* status;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  static constexpr int kTotal = kBarOffset + kBarBytes + 1024;  // + alignment slack
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int group_size = kGroupM * num_n;
  const int group = tile / group_size;
  const int first_m = group * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int local = tile - group * group_size;
  mb = first_m + local % gm;
  nb = local / gm;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
  const float k_beta = 0.7978845608028654f;
  const float k_kappa = 0.044715f;
  const float inner = k_beta * (x + k_kappa * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

template <typename OutT>
__device__ __forceinline__ float out_to_f32(OutT v);
template <>
__device__ __forceinline__ float out_to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float out_to_f32<__half>(__half v) {
  return __half2float(v);
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename OutT>
__device__ __forceinline__ float round_out(float v);
template <>
__device__ __forceinline__ float round_out<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <>
__device__ __forceinline__ float round_out<__half>(float v) {
  return __half2float(__float2half_rn(v));
}

// Epilogue for 16 consecutive columns held in r[0..15] of one row.
template <typename OutT>
__device__ __forceinline__ void epilogue16(const GemmArgs& g, const uint32_t* r, float sa,
                                           int64_t row, int col) {
  float sb[16];
  if (g.sb_per_col) {
    const float4* p = reinterpret_cast<const float4*>(g.sb + col);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = __ldg(p + j);
      sb[4 * j] = v.x;
      sb[4 * j + 1] = v.y;
      sb[4 * j + 2] = v.z;
      sb[4 * j + 3] = v.w;
    }
  } else {
    const float s = __ldg(g.sb);
#pragma unroll
    for (int j = 0; j < 16; ++j) sb[j] = s;
  }
  // y = sa * (sb * float(acc)) (+ bias): the evaluation order of vLLM's
  // ScaledEpilogue / ScaledEpilogueBias (multiply, then multiply-add).
  float y[16];
  if (g.bias != nullptr) {
    const uint4* bp = reinterpret_cast<const uint4*>(static_cast<const OutT*>(g.bias) + col);
    const uint4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
    const OutT* be0 = reinterpret_cast<const OutT*>(&b0);
    const OutT* be1 = reinterpret_cast<const OutT*>(&b1);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float b = out_to_f32<OutT>(j < 8 ? be0[j] : be1[j - 8]);
      y[j] = __fmaf_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))), b);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      y[j] = __fmul_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))));
  }
  if (g.epilogue & TM_EPI_GELU_TANH) {
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = gelu_tanh(round_out<OutT>(y[j]));
  }
  uint4 o0, o1;
  o0.x = pack2<OutT>(y[0], y[1]);
  o0.y = pack2<OutT>(y[2], y[3]);
  o0.z = pack2<OutT>(y[4], y[5]);
  o0.w = pack2<OutT>(y[6], y[7]);
  o1.x = pack2<OutT>(y[8], y[9]);
  o1.y = pack2<OutT>(y[10], y[11]);
  o1.z = pack2<OutT>(y[12], y[13]);
  o1.w = pack2<OutT>(y[14], y[15]);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<OutT*>(g.out) + row * g.ldo + col);
  dst[0] = o0;
  dst[1] = o1;
  if (g.acc_debug != nullptr) {
    uint4* d = reinterpret_cast<uint4*>(g.acc_debug + row * static_cast<int64_t>(g.N) + col);
    d[0] = make_uint4(r[0], r[1], r[2], r[3]);
    d[1] = make_uint4(r[4], r[5], r[6], r[7]);
    d[2] = make_uint4(r[8], r[9], r[10], r[11]);
    d[3] = make_uint4(r[12], r[13], r[14], r[15]);
  }
}

template <int BN, int STAGES, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemmArgs g) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = g.num_m * g.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;    // stages with a load in flight
      uint32_t issued_parity = 0;  // parity of that load's full phase
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, g.num_m, g.num_n, mb, nb);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, g.status)) {
            ok = false;
            break;
          }
          issued_mask &= ~(1u << stage);  // the previous load on this stage was consumed
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(&tm_a, &full[stage], s_a + stage * L::kABytes, kb * kBK, mb * kBM);
          tma_load_2d(&tm_b, &full[stage], s_b + stage * L::kBBytes, kb * kBK, nb * BN);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: every copy this thread started must land before exit.
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) mbar_wait_drain(&full[s], (issued_parity >> s) & 1u, g.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = make_idesc_i8(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, g.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, g.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(s_a + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(s_b + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            umma_i8(d_tmem, make_desc_kmajor_sw128(a_addr + k * 32),
                    make_desc_kmajor_sw128(b_addr + k * 32), kIdesc,
                    (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Every issued batch of MMAs was followed by a commit to its stage's
        // `empty` barrier, so the phase of the last such commit completing
        // means the tensor pipe has drained and TMEM may be released.
        const int last = (stage + STAGES - 1) % STAGES;
        const uint32_t last_phase = (stage == 0) ? (phase ^ 1u) : phase;
        mbar_wait_drain(&empty[last], last_phase, g.status);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, g.num_m, g.num_n, mb, nb);
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, g.status)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(mb) * kBM + q * 32 + lane;
      const bool row_ok = row < g.M;
      const float sa = row_ok ? (g.sa_per_row ? __ldg(g.sa + row) : __ldg(g.sa)) : 0.f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
        tmem_ld_wait();
        const int col0 = nb * BN + c * 32;
        if (row_ok) {
          if (col0 < g.N) epilogue16<OutT>(g, r, sa, row, col0);
          if (col0 + 16 < g.N) epilogue16<OutT>(g, r + 16, sa, row, col0 + 16);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------------------------ host
template <int BN, int STAGES, typename OutT>
int launch_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const GemmArgs& args,
                cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kTotal <= 227 * 1024, "shared memory budget");
  CUtensorMap ta, tb;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, args.K, args.M, lda, kBK, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  if (!encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, args.K, args.N, ldb, kBK, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  auto kernel = gemm_i8_kernel<BN, STAGES, OutT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
      cudaSuccess)
    return TM_ERR_CUDA;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return TM_ERR_CUDA;
  const int tiles = args.num_m * args.num_n;
  const int grid = tiles < sms ? tiles : sms;
  kernel<<<grid, kThreads, L::kTotal, stream>>>(ta, tb, args);
  return check_launch();
}

// Choose the N tile: the one that minimises (waves x per-tile cost), where a
// tile's main loop costs ~BN and each tile pays a fixed overhead.
int pick_bn(int num_m, int n, int sms) {
  int best_bn = 256;
  long best = -1;
  for (int bn : {256, 128, 64}) {
    const long tiles = static_cast<long>(num_m) * ((n + bn - 1) / bn);
    const long waves = (tiles + sms - 1) / sms;
    const long cost = waves * (bn + 32);
    if (best < 0 || cost < best) {
      best = cost;
      best_bn = bn;
    }
  }
  return best_bn;
}

template <typename OutT>
int dispatch_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, GemmArgs args,
                  int bn, cudaStream_t stream) {
  args.num_n = (args.N + bn - 1) / bn;
  switch (bn) {
    case 256: return launch_gemm<256, 4, OutT>(a, lda, b, ldb, args, stream);
    case 128: return launch_gemm<128, 6, OutT>(a, lda, b, ldb, args, stream);
    case 64: return launch_gemm<64, 8, OutT>(a, lda, b, ldb, args, stream);
    default: return TM_ERR_UNSUPPORTED;
  }
}

int scaled_mm_impl(void* out, int out_dtype, const int8_t* a, const int8_t* b, const float* sa,
                   int64_t sa_numel, const float* sb, int64_t sb_numel, const void* bias,
                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldo,
                   uint32_t epilogue, int32_t* acc_debug, int force_bn, cudaStream_t stream) {
  if (out_dtype != TM_DTYPE_BF16 && out_dtype != TM_DTYPE_FP16) return TM_ERR_DTYPE;
  if (m < 0 || n <= 0 || k <= 0) return TM_ERR_SHAPE;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  if (k % 16 != 0 || n % 16 != 0) return TM_ERR_SHAPE;
  if (lda < k || ldb < k || ldo < n) return TM_ERR_SHAPE;
  if (lda % 16 != 0 || ldb % 16 != 0 || ldo % 8 != 0) return TM_ERR_ALIGNMENT;
  if (sa_numel != 1 && sa_numel != m) return TM_ERR_SHAPE;
  if (sb_numel != 1 && sb_numel != n) return TM_ERR_SHAPE;
  if (epilogue & ~TM_EPI_GELU_TANH) return TM_ERR_UNSUPPORTED;
  if (m == 0) return TM_OK;
  if (!out || !a || !b || !sa || !sb) return TM_ERR_NULL_POINTER;
  if (!aligned16(a) || !aligned16(b) || !aligned16(out) || (bias && !aligned16(bias)) ||
      (sb_numel != 1 && !aligned16(sb)) || (acc_debug && !aligned16(acc_debug)))
    return TM_ERR_ALIGNMENT;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return TM_ERR_CUDA;
  GemmArgs args{};
  args.sa = sa;
  args.sb = sb;
  args.sa_per_row = sa_numel != 1 || m == 1;
  args.sb_per_col = sb_numel != 1 || n == 1;
  args.bias = bias;
  args.out = out;
  args.ldo = ldo;
  args.acc_debug = acc_debug;
  args.M = static_cast<int>(m);
  args.N = static_cast<int>(n);
  args.K = static_cast<int>(k);
  args.num_m = static_cast<int>((m + kBM - 1) / kBM);
  args.kblocks = static_cast<int>((k + kBK - 1) / kBK);
  args.epilogue = epilogue;
  args.status = device_status_ptr(dev);
  if (args.status == nullptr) return TM_ERR_CUDA;
  const int bn = force_bn ? force_bn : pick_bn(args.num_m, args.N, sms);
  if (out_dtype == TM_DTYPE_BF16)
    return dispatch_gemm<__nv_bfloat16>(a, lda, b, ldb, args, bn, stream);
  return dispatch_gemm<__half>(a, lda, b, ldb, args, bn, stream);
}

}  // namespace
}  // namespace tmw

extern "C" {

int tm_cutlass_scaled_mm(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldo, void* stream) {
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                            bias, m, n, k, lda, ldb, ldo, 0u, nullptr, 0, tmw::as_stream(stream));
}

int tm_scaled_mm_i8_ex(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                       const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                       int64_t scale_b_numel, const void* bias, int64_t m, int64_t n, int64_t k,
                       int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                       int32_t* acc_debug, void* stream) {
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                            bias, m, n, k, lda, ldb, ldo, epilogue, acc_debug, 0,
                            tmw::as_stream(stream));
}

// Same as tm_scaled_mm_i8_ex with a forced N-tile width (256, 128 or 64);
// used by tests to cover every kernel instantiation.
int tm_scaled_mm_i8_tile(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                         int32_t* acc_debug, int tile_n, void* stream) {
  if (tile_n != 256 && tile_n != 128 && tile_n != 64) return TM_ERR_UNSUPPORTED;
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                            bias, m, n, k, lda, ldb, ldo, epilogue, acc_debug, tile_n,
                            tmw::as_stream(stream));
}

}  // extern "C"
