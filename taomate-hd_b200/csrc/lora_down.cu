// LoRA down-projection T = x A^T on the tensor cores (sm_100a).
//
// The reference's LoRA wrapper (src/taomate_hd/inference/lora_checkpoint.py:
// 135-136 and 146-147, the inner torch.nn.functional.linear(inputs,
// lora_a)) multiplies the bf16 activations x [M, K] by the adapter's
// A [r, K] before the up-projection.  r is small (64 in the DiT adapters), so
// the product is a skinny bf16 GEMM whose cost is reading x once: about 2 r
// flops per byte, beyond CUDA-core rates at HBM speed but light for the
// tensor cores.
//
// One CTA per 128-row tile of x, two CTAs per SM: warp 0 streams 64-column
// boxes of x (16 KiB) and of A (r x 128 bytes, L2-resident) by TMA into a
// 4-stage ring; warp 1 issues tcgen05 kind::f16 MMAs (M = 128, N = r,
// K = 16) into an fp32 TMEM accumulator; warps 2-5 read it back (one row per
// lane), round to bf16 and store the row's r values.  fp32 accumulation of
// exact bf16 products, one rounding at the end: the reference's bf16 linear
// (fp32 accumulate, bf16 out) up to the order of the fp32 additions.
#include <cuda_bf16.h>

#include "common.h"
#include "ptx.cuh"

namespace tmw {
namespace {

constexpr int kDpRows = 128;       // rows of x per CTA (MMA M)
constexpr int kDpKb = 64;          // bf16 elements per TMA box: one 128-byte swizzle row
constexpr int kDpThreads = 192;    // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kDpXBytes = kDpRows * kDpKb * 2;       // 16 KiB per box
constexpr int kDpABytes = 64 * kDpKb * 2;            // room for r <= 64 rows of A per box

// A stage holds BOXES consecutive 64-column boxes of x and of A (each row of
// x is then fetched BOXES x 128 contiguous bytes at a time); STAGES stages.
template <int BOXES, int STAGES>
struct DpLayout {
  static constexpr int kStageBytes = BOXES * (kDpXBytes + kDpABytes);
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kSmem = kBarOffset + 128 + 1024;  // barriers + 1 KiB alignment slack
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};
static_assert(kDpXBytes % 1024 == 0 && kDpABytes % 1024 == 0, "1 KiB swizzle atoms");

struct DownArgs {
  __nv_bfloat16* t;
  int64_t ldt;
  int64_t m;
  int rank;        // r: multiple of 8, <= 64 (the MMA's N is r rounded up to 16)
  int kblocks;     // 64-column boxes along K
  uint32_t idesc;  // kind::f16, M = 128, N = r
  uint32_t tmem_cols;
  int* status;
};

template <int BOXES, int STAGES>
__global__ void __launch_bounds__(kDpThreads, 2)
    lora_down_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_a, const DownArgs g) {
  using L = DpLayout<BOXES, STAGES>;
  constexpr int kDpStages = STAGES;
  constexpr int kDpStageBytes = L::kStageBytes;
  constexpr int kDpBarOffset = L::kBarOffset;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDpBarOffset);
  uint64_t* empty = full + kDpStages;
  uint64_t* tmem_full = empty + kDpStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = static_cast<int>(blockIdx.x) * kDpRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_a);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, g.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // x may come from the kernel before this one on the stream
  griddep_launch_dependents();

  // stage j holds boxes [j * BOXES, j * BOXES + BOXES) (the last one may be
  // partial): BOXES x-boxes, then BOXES A-boxes
  const int groups = (g.kblocks + BOXES - 1) / BOXES;
  const uint32_t box_bytes = static_cast<uint32_t>(kDpXBytes + g.rank * kDpKb * 2);
  if (warp == 0) {
    if (lane == 0) {
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int kg = 0; kg < groups; ++kg) {
        const int s = kg % kDpStages;
        const uint32_t phase = static_cast<uint32_t>(kg / kDpStages) & 1u;
        if (!mbar_wait(&empty[s], phase ^ 1u, abort_flag, g.status)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kDpStageBytes;
        const int nbox = min(BOXES, g.kblocks - kg * BOXES);
        mbar_arrive_expect_tx(&full[s], box_bytes * static_cast<uint32_t>(nbox));
        for (int b = 0; b < nbox; ++b)
          tma_load_2d(&tm_x, &full[s], st + b * kDpXBytes, (kg * BOXES + b) * kDpKb, row0);
        for (int b = 0; b < nbox; ++b)
          tma_load_2d(&tm_a, &full[s], st + BOXES * kDpXBytes + b * kDpABytes,
                      (kg * BOXES + b) * kDpKb, 0);
        issued_mask |= 1u << s;
        issued_parity = (issued_parity & ~(1u << s)) | (phase << s);
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        for (int s = 0; s < kDpStages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait_drain(&full[s], (issued_parity >> s) & 1u, g.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true, issued_any = false;
      int kg = 0;
      for (; kg < groups; ++kg) {
        const int s = kg % kDpStages;
        const uint32_t phase = static_cast<uint32_t>(kg / kDpStages) & 1u;
        if (!mbar_wait(&full[s], phase, abort_flag, g.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * kDpStageBytes);
        const int nbox = min(BOXES, g.kblocks - kg * BOXES);
        for (int b = 0; b < nbox; ++b) {
          const uint32_t x_addr = st + b * kDpXBytes;
          const uint32_t a_addr = st + BOXES * kDpXBytes + b * kDpABytes;
#pragma unroll
          for (int k = 0; k < kDpKb / 16; ++k)  // K = 16 bf16 (32 bytes) per MMA
            umma_bf16(tmem_base, make_desc_kmajor_sw128(x_addr + k * 32),
                      make_desc_kmajor_sw128(a_addr + k * 32), g.idesc,
                      (kg | b | k) != 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&empty[s]);
      }
      if (ok) {
        umma_commit(tmem_full);
      } else if (issued_any) {  // the last MMAs must finish before TMEM is freed
        const int last = (kg - 1) % kDpStages;
        mbar_wait_drain(&empty[last], static_cast<uint32_t>((kg - 1) / kDpStages) & 1u, g.status);
      }
    }
    __syncwarp();
  } else {
    // warps 2-5: TMEM lane quarter warp % 4, one row per lane
    const int q = warp & 3;
    const int64_t row = static_cast<int64_t>(row0) + q * 32 + lane;
    if (mbar_wait(tmem_full, 0u, abort_flag, g.status)) {
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < g.rank; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c), r);
        tmem_ld_wait();
        if (row < g.m) {
          uint4* dst = reinterpret_cast<uint4*>(g.t + row * g.ldt + c);
          const int vecs = min(32, g.rank - c) / 8;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (v < vecs) {
              uint4 o;
              uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                __nv_bfloat162 p = __floats2bfloat162_rn(__uint_as_float(r[8 * v + 2 * j]),
                                                         __uint_as_float(r[8 * v + 2 * j + 1]));
                w[j] = *reinterpret_cast<uint32_t*>(&p);
              }
              dst[v] = o;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, g.tmem_cols);
  }
}

template <int BOXES, int STAGES>
int launch_down(const CUtensorMap& tx, const CUtensorMap& ta, const DownArgs& g, int64_t m,
                cudaStream_t stream) {
  using L = DpLayout<BOXES, STAGES>;
  auto kernel = lora_down_kernel<BOXES, STAGES>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) !=
      cudaSuccess)
    return TM_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((m + kDpRows - 1) / kDpRows));
  cfg.blockDim = dim3(kDpThreads);
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = stream;
  if (launch_with_pdl(cfg, nullptr, 0, kernel, tx, ta, g) != cudaSuccess) return TM_ERR_CUDA;
  return check_launch();
}

}  // namespace
}  // namespace tmw

extern "C" {

int tm_lora_down_proj(void* t, int64_t ldt, const void* x, int64_t ldx, const void* a,
                      int64_t lda, int rank, int64_t m, int64_t k, void* stream) {
  using namespace tmw;
  if (m < 0 || k <= 0) return TM_ERR_SHAPE;
  if (rank < 8 || rank > 64 || rank % 8 != 0) return TM_ERR_UNSUPPORTED;
  if (m == 0) return TM_OK;
  if (t == nullptr || x == nullptr || a == nullptr) return TM_ERR_NULL_POINTER;
  if (m > 0x7fffffffLL - kDpRows || k > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  if (ldx < k || lda < k || ldt < rank) return TM_ERR_SHAPE;
  // TMA: 16-byte aligned bases and row strides; T rows are written 16 bytes
  // at a time
  if (!aligned16(t) || !aligned16(x) || !aligned16(a) || (ldx * 2) % 16 != 0 ||
      (lda * 2) % 16 != 0 || (ldt * 2) % 16 != 0)
    return TM_ERR_ALIGNMENT;
  const int dev = current_device();
  if (dev < 0) return TM_ERR_CUDA;
  CUtensorMap tx, ta;
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, static_cast<uint64_t>(k),
                      static_cast<uint64_t>(m), static_cast<uint64_t>(ldx) * 2, kDpKb, kDpRows,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, static_cast<uint64_t>(k),
                      static_cast<uint64_t>(rank), static_cast<uint64_t>(lda) * 2, kDpKb,
                      static_cast<uint32_t>(rank), CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  DownArgs g;
  g.t = static_cast<__nv_bfloat16*>(t);
  g.ldt = ldt;
  g.m = m;
  g.rank = rank;
  g.kblocks = static_cast<int>((k + kDpKb - 1) / kDpKb);
  // N = r rounded up to 16: for r = 8, 24, ... the MMA also multiplies the
  // stale rows after A's r rows in shared memory into columns that are
  // never stored
  const int mma_n = (rank + 15) / 16 * 16;
  g.idesc = make_idesc_bf16(kDpRows, mma_n);
  g.tmem_cols = mma_n <= 32 ? 32u : 64u;
  g.status = device_status_ptr(dev);
  // One 64-column box per stage, four stages: 97 KiB, two CTAs per SM.  On
  // B200 this beat two boxes per stage (256 contiguous bytes per row) and the
  // deeper one-CTA-per-SM rings (6 stages, 2 x 3, 2 x 4, 4 x 2): with
  // 160 row tiles at M = 20480 those leave a second wave of 12 CTAs.
  return launch_down<1, 4>(tx, ta, g, m, as_stream(stream));
}

}  // extern "C"
