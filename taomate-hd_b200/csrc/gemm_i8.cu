// Scaled int8 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   out[m, n] = cvt(scale_a[m] * (scale_b[n] * float(sum_k a[m,k] * b[n,k])) (+ bias[n]))
//
// Replaces vLLM's cutlass_scaled_mm as called by the reference
// (src/taomate_hd/inference/w8a8.py:72 and :142-144).
//
// Three persistent, warp-specialised kernels share one epilogue:
//
//   gemm_i8_pair_kernel  CTA pairs (clusters of 2).  A pair owns a 256 x BN
//     output tile: each CTA fetches its 128 rows of A and BN/2 rows of B into
//     its own shared memory; the leader CTA issues tcgen05.mma.cta_group::2
//     (M=256, N=BN, K=32), which reads both CTAs' operands and writes each
//     CTA's 128 x BN accumulator into that CTA's TMEM.  Per SM this moves
//     2/3 of the operand bytes of a 128 x 256 one-CTA tile for the same MMA
//     work, which is what lets the tensor pipe run near its rate from L2.
//   gemm_i8_kernel       one CTA per tile of 128 x BN (small or ragged shapes).
//   gemm_i8_pair_lora_kernel  the 256 x 256 pair tile with the bf16 LoRA delta
//     added on the tensor cores between two epilogue passes.
//
// Warp roles (320 threads per CTA):
//   warp 0      TMA producer: a STAGES-deep ring of (A, B) k-blocks of 128
//               bytes of K, 128-byte swizzled, completion by transaction bytes.
//   warp 1      TMEM owner (2 x BN int32 columns = two accumulators) and MMA
//               issuer (one thread; in the pair kernel only on the leader).
//   warps 2..9  epilogue: warp w reads TMEM lane quarter w % 4 (tile rows
//               32*(w%4)..+31) and column half (w-2)/4; fp32 dequant
//               sa * (sb * acc) (+ bias) (+ GELU-tanh) -> bf16/fp16 stores.
// With two accumulators the epilogue of one tile overlaps the main loop of
// the next.  Tiles are visited in groups of 16 M-blocks for L2 reuse (or in
// N-fastest groups when K is long); tails use TMA zero fill and predicated
// stores.  Outputs go to local memory by TMA stores, or, as 128-byte row
// segments over NVLink, to the rows' owners (the fused reduce-scatter /
// all-reduce, followed by the owner-side reduction in the same launch) or to
// the heads' ranks (the Ulysses exchange).  Non-cooperative launches use
// programmatic dependent launch.  Every wait is bounded (ptx.cuh).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.h"
#include "ptx.cuh"

namespace tmw {
namespace {

constexpr int kBM = 128;  // rows of A per CTA
constexpr int kBK = 128;  // bytes == int8 elements of K per k-block (one swizzle row)
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kGroupM = 16;
constexpr int kMaxPeers = 8;

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
  int num_m, num_n, kblocks;  // tile grid (in units of the kernel's tile)
  uint32_t epilogue;
  int* status;
  // Local output written by TMA stores of the staged blocks (the kernel's
  // tm_out map) instead of per-lane stores; set only without split-K or
  // scatter.
  int tma_store;
  // Ulysses send layout (ul_world > 0; merged QKV projection, n = 3 x heads
  // x head_dim): the output is the all-to-all send buffer
  // [ul_world][3][M][ul_local x head_dim], ul_local = ceil(heads / ul_world)
  // (the reference's _merged_qkv_send_layout, distributed/ulysses.py:153-193,
  // with its zero-padded head shards) instead of [M][N]; see ulysses_coords.
  int ul_world, ul_heads, ul_head_dim, ul_local;
  // Ulysses exchange over NVLink (ul_peer != 0): instead of a local send
  // buffer, each 64-column pass goes straight into destination rank w's
  // receive buffer peer_part[w] ([ul_world][3][M][ul_local x head_dim], this
  // rank's slot ul_rank); element counts per destination are added to
  // peer_count[w][ul_rank], and the launch ends once this rank's counters
  // show every source's rows (ul_uses x the source's element count).
  int ul_peer, ul_rank, ul_uses;
  // Split-K (one-CTA kernel): each tile's K range is cut into `splits`
  // slices of kb_per_split k-blocks; every (tile, slice) unit stores its exact
  // int32 partial in ws[slice][M][N] and bumps tile_counters[tile]; the unit
  // that arrives last sums the slices, runs the epilogue and resets the
  // counter to 0.  splits == 1 disables it.
  int splits, kb_per_split;
  int32_t* ws;
  unsigned int* tile_counters;
  // Row-parallel fused reduce-scatter; world == 0 disables it.  Rank j owns
  // rows [j * rows_per_owner, +rows_per_owner).  The epilogue stores each
  // bf16 partial 128-row block of owner j's rows into peer_part[j], slot
  // `rank` ([world][rows_per_owner][N], an NVLink peer store unless
  // j == rank).  When a CTA has stored all its blocks it drains its stores
  // once and adds the number of elements it sent to owner j to
  // peer_count[j][rank] (a 64-bit counter that only grows).  CTAs that run
  // out of GEMM tiles then wait until every source's counter reaches
  // `uses` x rows_per_owner x N, and reduce this rank's rows from its own
  // slots (local HBM reads): sum in rank order, add red_bias, store to red_out.
  int world, rank, rows_per_owner;
  // Owner-interleaved tile order (scatter and all-reduce modes, m_owners =
  // world, else 0): raster M-block v is M-block v / m_owners of owner
  // v % m_owners, so every wave of concurrent tiles covers all owners and
  // each rank's NVLink egress stays busy through the whole GEMM.  In plain
  // raster order the ranks would all push to the same few owners at once
  // (sharing their ingress), and each rank would alternate between local
  // writes and pushes.
  int m_owners, mb_per_owner;
  // Raster for long K (group_n > 0): tiles in groups of group_n N-blocks
  // spanning every M-block, N fastest; see tile_coords.  0 = groups of
  // kGroupM M-blocks, M fastest.
  int group_n;
  uint32_t uses;  // 1-based count of calls made with this buffer set
  const __nv_bfloat16* red_bias;
  __nv_bfloat16* red_out;
  int64_t red_ldo;
  __nv_bfloat16* peer_part[kMaxPeers];
  unsigned long long* peer_count[kMaxPeers];
  // Fused all-reduce (peer_out[0] != nullptr): every rank's full [M][N]
  // output (ld N).  After reducing a block the owner stores it into all
  // ranks' outputs at its global rows and, once its blocks are drained, adds
  // the element count to peer_count[j][world + rank] (the gather counters);
  // the kernel ends when this rank's gather counters show every owner's
  // rows have arrived.
  __nv_bfloat16* peer_out[kMaxPeers];
};

// Raster order of output tiles.  Concurrent tiles should share operand
// panels in L2.  Default: groups of kGroupM M-blocks, M fastest -- a wave
// shares kGroupM A panels and a few B panels.  With group_n > 0 (long K,
// where kGroupM A panels of K bytes per row would not stay in L2 beside B):
// groups of group_n N-blocks over all M-blocks, N fastest -- a wave shares
// a few A panels, each read from DRAM once, while the group's B panels stay
// resident for every M-block.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb,
                                            int m_owners, int mb_per_owner, int group_n = 0) {
  if (group_n > 0) {
    const int group_size = group_n * num_m;
    const int group = tile / group_size;
    const int first_n = group * group_n;
    const int gn = min(num_n - first_n, group_n);
    const int local = tile - group * group_size;
    nb = first_n + local % gn;
    mb = local / gn;
  } else {
    const int group_size = kGroupM * num_n;
    const int group = tile / group_size;
    const int first_m = group * kGroupM;
    const int gm = min(num_m - first_m, kGroupM);
    const int local = tile - group * group_size;
    mb = first_m + local % gm;
    nb = local / gm;
  }
  if (m_owners > 1) {  // num_m == m_owners x mb_per_owner
    const int owner = mb % m_owners;
    mb = owner * mb_per_owner + mb / m_owners;
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), every operation explicit
  // (no contraction left to the compiler), so each epilogue path that
  // inlines it computes the same bits
  // inner = x (beta + beta kappa x^2); result = 0.5 x + 0.5 x tanh(inner)
  const float k_beta = 0.7978845608028654f;          // sqrt(2 / pi)
  const float k_beta_kappa = 0.035677408136300125f;  // sqrt(2 / pi) * 0.044715
  const float inner = __fmul_rn(x, __fmaf_rn(k_beta_kappa, __fmul_rn(x, x), k_beta));
  const float h = __fmul_rn(0.5f, x);
  return __fmaf_rn(h, tanh_approx(inner), h);
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

// Round two values to OutT and back with one paired conversion (the same
// bits as two round_out calls; the conversion unit, which bounds the
// epilogue's arithmetic, does half the work for bf16).
template <typename OutT>
__device__ __forceinline__ void round2_out(float& a, float& b);
template <>
__device__ __forceinline__ void round2_out<__nv_bfloat16>(float& a, float& b) {
  const uint32_t p = pack2<__nv_bfloat16>(a, b);  // a in the low half, b in the high half
  a = __uint_as_float(p << 16);
  b = __uint_as_float(p & 0xffff0000u);
}
template <>
__device__ __forceinline__ void round2_out<__half>(float& a, float& b) {
  a = round_out<__half>(a);
  b = round_out<__half>(b);
}

// Dequantise 16 consecutive columns held in r[0..15] of one row and pack
// them into two 16-byte words of OutT.  Columns past N are never stored.
template <typename OutT>
__device__ __forceinline__ void epilogue16(const GemmArgs& g, const uint32_t* r, float sa,
                                           int col, uint4& o0, uint4& o1) {
  if (col >= g.N) {
    o0 = o1 = make_uint4(0, 0, 0, 0);
    return;
  }
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
    for (int j = 0; j < 16; ++j) y[j] = __fmul_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))));
  }
  if (g.epilogue & TM_EPI_GELU_TANH) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) round2_out<OutT>(y[j], y[j + 1]);
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = gelu_tanh(y[j]);
  }
  o0.x = pack2<OutT>(y[0], y[1]);
  o0.y = pack2<OutT>(y[2], y[3]);
  o0.z = pack2<OutT>(y[4], y[5]);
  o0.w = pack2<OutT>(y[6], y[7]);
  o1.x = pack2<OutT>(y[8], y[9]);
  o1.y = pack2<OutT>(y[10], y[11]);
  o1.z = pack2<OutT>(y[12], y[13]);
  o1.w = pack2<OutT>(y[14], y[15]);
}

// Output row pointer: the row itself, or (scatter mode) its owner's slot.
template <typename OutT>
__device__ __forceinline__ OutT* out_row_ptr(const GemmArgs& g, int64_t row) {
  if (g.world > 0) {
    const int owner = static_cast<int>(row / g.rows_per_owner);
    const int64_t local = row - static_cast<int64_t>(owner) * g.rows_per_owner;
    return reinterpret_cast<OutT*>(g.peer_part[owner]) +
           (static_cast<int64_t>(g.rank) * g.rows_per_owner + local) * g.N;
  }
  return static_cast<OutT*>(g.out) + row * g.ldo;
}

// Ulysses send layout: output column `col` (a multiple of 32, never crossing
// a head) of row `row` goes to the send buffer viewed as
// [ul_world * 3 * M rows][ul_local * head_dim columns]: row
// (w * 3 + qkv) * M + row, column (head % ul_local) * head_dim + d, with
// qkv = col / (heads * head_dim), head = that part / head_dim and
// w = head / ul_local.  Padded head slots (w * ul_local + h >= heads) are
// never written here; the host zeroes them before the launch.
__device__ __forceinline__ void ulysses_coords(const GemmArgs& g, int col, int64_t row, int& x,
                                               int64_t& y) {
  const int width = g.ul_heads * g.ul_head_dim;
  const int qkv = col / width;
  const int within = col - qkv * width;
  const int head = within / g.ul_head_dim;
  const int w = head / g.ul_local;
  x = within - w * g.ul_local * g.ul_head_dim;
  y = static_cast<int64_t>(w * 3 + qkv) * g.M + row;
}

// Ulysses exchange over NVLink: the destination rank of output column `col`
// (a multiple of 64 inside one head) and the address of row 0 of that
// column in the destination's receive buffer (row stride ul_local x
// head_dim).
__device__ __forceinline__ int ul_peer_dest(const GemmArgs& g, int col) {
  const int width = g.ul_heads * g.ul_head_dim;
  const int within = col - (col / width) * width;
  return (within / g.ul_head_dim) / g.ul_local;
}

template <typename OutT>
__device__ __forceinline__ OutT* ul_peer_base(const GemmArgs& g, int col) {
  int x;
  int64_t y;
  ulysses_coords(g, col, 0, x, y);  // y = (w * 3 + qkv) * M for row 0
  const int w = ul_peer_dest(g, col);
  const int64_t qkv_rows = y - static_cast<int64_t>(w) * 3 * g.M;  // qkv * M
  const int64_t ld = static_cast<int64_t>(g.ul_local) * g.ul_head_dim;
  return reinterpret_cast<OutT*>(g.peer_part[w]) +
         (static_cast<int64_t>(g.ul_rank) * 3 * g.M + qkv_rows) * ld + x;
}

// Per-warp staging tile: 32 rows x 128 bytes, 16-byte chunks XOR-swizzled by
// row so that both the row-per-lane writes and the row-segment reads are
// free of bank conflicts.
constexpr int kStageRowBytes = 128;
constexpr int kEpiStageBytes = 32 * kStageRowBytes;  // per epilogue warp

__device__ __forceinline__ uint4* stage_slot(uint8_t* stage, int row, int chunk) {
  return reinterpret_cast<uint4*>(stage + row * kStageRowBytes + ((chunk ^ (row & 7)) << 4));
}

// One epilogue warp's share of a 128 x BN accumulator held in this CTA's
// TMEM at column `acc_col`: lane quarter warp % 4, column half (warp-2)/4.
// Each group of 64 columns is dequantised (lane = row), staged in shared
// memory, and written back as 128-byte row segments (8 lanes per row), so
// global and NVLink peer stores are full-line writes.
template <int BN, typename OutT>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, uint32_t tmem_base,
                                              uint32_t acc_col, int64_t row0, int col0,
                                              int warp, int lane, uint8_t* stage) {
  constexpr int kHalf = BN / 2;
  constexpr int kColsPerPass = kStageRowBytes / sizeof(OutT);  // 64
  const int q = warp & 3;
  const int h = (warp - 2) >> 2;
  const int64_t row_base = row0 + q * 32;
  const int64_t row = row_base + lane;
  const bool row_ok = row < g.M;
  const float sa = row_ok ? (g.sa_per_row ? __ldg(g.sa + row) : __ldg(g.sa)) : 0.f;
  int32_t* dbg_row = (g.acc_debug != nullptr && row_ok)
                         ? g.acc_debug + row * static_cast<int64_t>(g.N) : nullptr;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc_col +
                         static_cast<uint32_t>(h * kHalf);
#pragma unroll 1
  for (int pass = 0; pass * kColsPerPass < kHalf; ++pass) {
    const int pass_cols = min(kColsPerPass, kHalf - pass * kColsPerPass);  // 64 or 32
    const int pass_col0 = col0 + h * kHalf + pass * kColsPerPass;
#pragma unroll 1
    for (int c = 0; c < pass_cols / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(pass * kColsPerPass + c * 32), r);
      tmem_ld_wait();
      const int col = pass_col0 + c * 32;
      uint4 o[4];
      epilogue16<OutT>(g, r, sa, col, o[0], o[1]);
      epilogue16<OutT>(g, r + 16, sa, col + 16, o[2], o[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) *stage_slot(stage, lane, c * 4 + j) = o[j];
      if (dbg_row != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (col + j < g.N)
            *reinterpret_cast<uint4*>(dbg_row + col + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
      }
    }
    __syncwarp();
    const int chunks = pass_cols * static_cast<int>(sizeof(OutT)) / 16;  // 8 or 4 per row
    const int rows_per_store = 32 / chunks;
    const int chunk = lane % chunks;
    // Ulysses exchange: the whole pass lies in one head of one destination
    OutT* ul_base = (g.ul_peer && pass_col0 < g.N) ? ul_peer_base<OutT>(g, pass_col0) : nullptr;
    const int64_t ul_ld = static_cast<int64_t>(g.ul_local) * g.ul_head_dim;
#pragma unroll 1
    for (int rr = lane / chunks; rr < 32; rr += rows_per_store) {
      const int64_t out_r = row_base + rr;
      const int col = pass_col0 + chunk * (16 / static_cast<int>(sizeof(OutT)));
      if (out_r < g.M && col < g.N) {
        OutT* dst = ul_base != nullptr ? ul_base + out_r * ul_ld + (col - pass_col0)
                                       : out_row_ptr<OutT>(g, out_r) + col;
        *reinterpret_cast<uint4*>(dst) = *stage_slot(stage, rr, chunk);
      }
    }
    __syncwarp();
  }
}

__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ------------------------------------------------- TMA-store epilogue (local)
// For local outputs each epilogue warp's 4 KiB shared region holds a 2 KiB
// staging tile (32 rows x 64 bytes in the 64-byte swizzle layout a TMA
// store reads) and a column cache: the per-column weight scales and bias of
// the warp's kHalf columns.  The cache for tile t is filled from registers
// that were loaded while tile t-1 was being processed, so the scale/bias
// loads never sit between the accumulator and the math.
constexpr int kStage64Bytes = 32 * 64;
constexpr int kColCacheOffset = kStage64Bytes;            // kHalf <= 128 floats
constexpr int kBiasCacheOffset = kColCacheOffset + 512;  // kHalf <= 128 x 16-bit
static_assert(kBiasCacheOffset + 256 <= kEpiStageBytes, "epilogue warp region");

__device__ __forceinline__ uint4* stage64_slot(uint8_t* stage, int row, int chunk) {
  return reinterpret_cast<uint4*>(stage + row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

// One lane's share of a tile's column constants: 4 scales, 4 bias values,
// and the per-token scale of its row.
struct ColPrefetch {
  float4 sb;
  uint2 bias;
  float sa;
};

template <typename OutT>
__device__ __forceinline__ ColPrefetch col_prefetch(const GemmArgs& g, int col_base, int cols,
                                                    int64_t row, int lane) {
  ColPrefetch p;
  p.sb = make_float4(0.f, 0.f, 0.f, 0.f);
  p.bias = make_uint2(0u, 0u);
  const int c = col_base + 4 * lane;
  if (4 * lane < cols && c < g.N) {  // N % 16 == 0: 4 columns are all in or all out
    if (g.sb_per_col) {
      p.sb = __ldg(reinterpret_cast<const float4*>(g.sb + c));
    } else {
      const float v = __ldg(g.sb);
      p.sb = make_float4(v, v, v, v);
    }
    if (g.bias != nullptr) p.bias = __ldg(reinterpret_cast<const uint2*>(static_cast<const OutT*>(g.bias) + c));
  }
  p.sa = row < g.M ? (g.sa_per_row ? __ldg(g.sa + row) : __ldg(g.sa)) : 0.f;
  return p;
}

__device__ __forceinline__ void col_cache_store(uint8_t* region, const ColPrefetch& p, int cols,
                                                int lane) {
  if (4 * lane < cols) {
    *reinterpret_cast<float4*>(region + kColCacheOffset + 16 * lane) = p.sb;
    *reinterpret_cast<uint2*>(region + kBiasCacheOffset + 8 * lane) = p.bias;
  }
}

// Dequantise 16 columns with their constants from the column cache (all
// lanes read the same words: shared-memory broadcasts).  Same arithmetic as
// epilogue16.
template <typename OutT>
__device__ __forceinline__ void dequant16_cached(const GemmArgs& g, const uint32_t* r, float sa,
                                                 const float* sb_s, const OutT* bias_s,
                                                 uint4& o0, uint4& o1) {
  float sb[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 v = reinterpret_cast<const float4*>(sb_s)[j];
    sb[4 * j] = v.x;
    sb[4 * j + 1] = v.y;
    sb[4 * j + 2] = v.z;
    sb[4 * j + 3] = v.w;
  }
  float y[16];
  if (g.bias != nullptr) {
    const uint4 b0 = reinterpret_cast<const uint4*>(bias_s)[0];
    const uint4 b1 = reinterpret_cast<const uint4*>(bias_s)[1];
    const OutT* be0 = reinterpret_cast<const OutT*>(&b0);
    const OutT* be1 = reinterpret_cast<const OutT*>(&b1);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float b = out_to_f32<OutT>(j < 8 ? be0[j] : be1[j - 8]);
      y[j] = __fmaf_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))), b);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = __fmul_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))));
  }
  if (g.epilogue & TM_EPI_GELU_TANH) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) round2_out<OutT>(y[j], y[j + 1]);
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = gelu_tanh(y[j]);
  }
  o0.x = pack2<OutT>(y[0], y[1]);
  o0.y = pack2<OutT>(y[2], y[3]);
  o0.z = pack2<OutT>(y[4], y[5]);
  o0.w = pack2<OutT>(y[6], y[7]);
  o1.x = pack2<OutT>(y[8], y[9]);
  o1.y = pack2<OutT>(y[10], y[11]);
  o1.z = pack2<OutT>(y[12], y[13]);
  o1.w = pack2<OutT>(y[14], y[15]);
}

// One epilogue warp's share of a 128 x BN accumulator (lane quarter
// warp % 4, column half (warp-2)/4), stored by TMA: per 32-column pass, one
// TMEM load, dequantise from the column cache, stage, and one lane issues
// a 32 x 32 bulk tensor store.  `release` (the accumulator-empty arrival)
// runs as soon as the last TMEM load of the tile has landed, so the tensor
// cores start the next tile while this one is converted and stored.  Rows
// and columns past M/N are clipped by the TMA unit.  The column cache must
// hold this tile's constants (col_cache_store) and `sa` this lane's row.
template <int BN, typename OutT, typename Release>
__device__ __forceinline__ void epilogue_tile_tma(const GemmArgs& g, const CUtensorMap* tm_out,
                                                  uint32_t tmem_base, uint32_t acc_col,
                                                  int64_t row0, int col0, int warp, int lane,
                                                  uint8_t* region, float sa, Release release) {
  constexpr int kHalf = BN / 2;
  constexpr int kPasses = kHalf / 32;
  static_assert(kHalf % 32 == 0 && kHalf <= 128, "32-column passes, cache of 128 columns");
  const int q = warp & 3;
  const int h = (warp - 2) >> 2;
  const int64_t row_base = row0 + q * 32;
  const int64_t row = row_base + lane;
  int32_t* dbg_row = (g.acc_debug != nullptr && row < g.M)
                         ? g.acc_debug + row * static_cast<int64_t>(g.N) : nullptr;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc_col +
                         static_cast<uint32_t>(h * kHalf);
  const float* sb_s = reinterpret_cast<const float*>(region + kColCacheOffset);
  const OutT* bias_s = reinterpret_cast<const OutT*>(region + kBiasCacheOffset);
#pragma unroll 1
  for (int pass = 0; pass < kPasses; ++pass) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(pass * 32), r);
    tmem_ld_wait();
    if (pass == kPasses - 1) release();
    const int col = col0 + h * kHalf + pass * 32;
    uint4 o[4];
    dequant16_cached<OutT>(g, r, sa, sb_s + pass * 32, bias_s + pass * 32, o[0], o[1]);
    dequant16_cached<OutT>(g, r + 16, sa, sb_s + pass * 32 + 16, bias_s + pass * 32 + 16, o[2],
                           o[3]);
    if (dbg_row != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        if (col + j < g.N)
          *reinterpret_cast<uint4*>(dbg_row + col + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    }
    if (lane == 0) bulk_wait_read_all();  // the previous pass's store has left the tile
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) *stage64_slot(region, lane, j) = o[j];
    fence_async_shared();
    __syncwarp();
    if (lane == 0 && row_base < g.M && col < g.N) {
      int x = col;
      int64_t y = row_base;
      if (g.ul_world > 0) ulysses_coords(g, col, row_base, x, y);
      tma_store_2d(tm_out, region, x, static_cast<int>(y));
      bulk_commit();
    }
  }
}

// SwiGLU epilogue (TM_EPI_SWIGLU, the reference's fused_swiglu after the
// merged fc1, fused_kernels.py:298-309 and model/layers.py:525-533).  The
// weight rows arrive interleaved in blocks of 16 -- gate rows j..j+15, then
// the matching up rows -- so every 32 accumulator columns hold 16 (gate, up)
// pairs.  Per 64-column pass: dequantise both halves to the rounded linear
// output (as the unfused linear would store them), then
// out = round(round(g * sigmoid(g)) * u) for 32 output columns, staged and
// TMA-stored at output column (acc column) / 2.  `release` as in
// epilogue_tile_tma.
__device__ __forceinline__ float sigmoid_f32(float x) {
  return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-x)));
}

template <int BN, typename OutT, typename Release>
__device__ __forceinline__ void epilogue_tile_swiglu(const GemmArgs& g, const CUtensorMap* tm_out,
                                                     uint32_t tmem_base, uint32_t acc_col,
                                                     int64_t row0, int col0, int warp, int lane,
                                                     uint8_t* region, float sa, Release release) {
  constexpr int kHalf = BN / 2;
  constexpr int kPasses = kHalf / 64;
  static_assert(kHalf % 64 == 0 && kHalf <= 128, "64-column passes, cache of 128 columns");
  const int q = warp & 3;
  const int h = (warp - 2) >> 2;
  const int64_t row_base = row0 + q * 32;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc_col +
                         static_cast<uint32_t>(h * kHalf);
  const float* sb_s = reinterpret_cast<const float*>(region + kColCacheOffset);
  const OutT* bias_s = reinterpret_cast<const OutT*>(region + kBiasCacheOffset);
#pragma unroll 1
  for (int pass = 0; pass < kPasses; ++pass) {
    uint32_t r[2][32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(pass * 64), r[0]);
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(pass * 64 + 32), r[1]);
    tmem_ld_wait();
    if (pass == kPasses - 1) release();
    float out[32];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int cc = pass * 64 + k * 32;  // cache column of this 32-column chunk
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float y[2];
#pragma unroll
        for (int part = 0; part < 2; ++part) {  // 0: gate column, 1: up column
          const int c = cc + part * 16 + j;
          const float x = __fmul_rn(sb_s[c], __int2float_rn(static_cast<int>(r[k][part * 16 + j])));
          const float v = g.bias != nullptr ? __fmaf_rn(sa, x, out_to_f32<OutT>(bias_s[c]))
                                            : __fmul_rn(sa, x);
          y[part] = round_out<OutT>(v);
        }
        const float act = round_out<OutT>(__fmul_rn(y[0], sigmoid_f32(y[0])));
        out[k * 16 + j] = __fmul_rn(act, y[1]);
      }
    }
    uint4 o[4];
#pragma unroll
    for (int qd = 0; qd < 4; ++qd)
      o[qd] = make_uint4(pack2<OutT>(out[8 * qd], out[8 * qd + 1]),
                         pack2<OutT>(out[8 * qd + 2], out[8 * qd + 3]),
                         pack2<OutT>(out[8 * qd + 4], out[8 * qd + 5]),
                         pack2<OutT>(out[8 * qd + 6], out[8 * qd + 7]));
    const int out_col = (col0 + h * kHalf + pass * 64) / 2;
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) *stage64_slot(region, lane, qd) = o[qd];
    fence_async_shared();
    __syncwarp();
    if (lane == 0 && row_base < g.M && 2 * out_col < g.N) {
      tma_store_2d(tm_out, region, out_col, static_cast<int>(row_base));
      bulk_commit();
    }
  }
}

// Fused reduce-scatter: after a CTA's epilogue warps have issued the stores
// of all their blocks, one thread drains them (the named barrier orders
// every warp's stores before that thread's system-scope fence; fences are
// cumulative) and adds the per-owner element counts to the owners' counters.
// One drain per CTA instead of one per block keeps the NVLink stores
// streaming while the GEMM runs.
__device__ __forceinline__ void publish_counts(const GemmArgs& g, const long long* sent, int warp,
                                               int lane) {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
  if (warp == 2 && lane == 0) {
    __threadfence_system();
    for (int j = 0; j < g.world; ++j)
      if (sent[j] > 0)
        asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(g.peer_count[j] + g.rank),
                     "l"(static_cast<unsigned long long>(sent[j]))
                     : "memory");
  }
}

// Ulysses exchange: as publish_counts, to destination w's counter of this
// source (peer_count[w][ul_rank]).
__device__ __forceinline__ void publish_ul_counts(const GemmArgs& g, const long long* sent,
                                                  int warp, int lane) {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
  if (warp == 2 && lane == 0) {
    __threadfence_system();
    for (int w = 0; w < g.ul_world; ++w)
      if (sent[w] > 0)
        asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(g.peer_count[w] + g.ul_rank),
                     "l"(static_cast<unsigned long long>(sent[w]))
                     : "memory");
  }
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The owner-side reduction works in strips of kRedRows rows x one column
// tile: at TP = 8 an owner's 1024 x 3072 block is then 384 work items for
// the 148 CTAs instead of 96 128-row blocks of 512 KiB each.
constexpr int kRedRows = 32;

// Sum one strip's partials from `world` (<= W) source slots, V vectors of 8
// columns per thread per round: all V x world 16-byte loads of a round are
// issued before any is consumed, keeping ~32 registers of NVLink loads in
// flight per thread (3-5 MB across the GPU, enough to keep NVLink busy).
template <int V, int W>
__device__ __forceinline__ void reduce_block(const GemmArgs& g, int lrb, int col0,
                                             int vec_per_row) {
  const int total = kRedRows * vec_per_row;
  for (int v0 = threadIdx.x; v0 < total; v0 += V * blockDim.x) {
    uint4 raw[V][W];
    int64_t off[V];
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const int v = v0 + u * static_cast<int>(blockDim.x);
      const int vv = v < total ? v : v0;
      const int r = vv / vec_per_row;
      off[u] = (static_cast<int64_t>(lrb) * kRedRows + r) * g.N + col0 + (vv - r * vec_per_row) * 8;
    }
    const __nv_bfloat16* slots = g.peer_part[g.rank];
    const int64_t slot_elems = static_cast<int64_t>(g.rows_per_owner) * g.N;
#pragma unroll
    for (int src = 0; src < W; ++src)
      if (src < g.world) {
#pragma unroll
        for (int u = 0; u < V; ++u) raw[u][src] = ld_cg16(slots + src * slot_elems + off[u]);
      }
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const int v = v0 + u * static_cast<int>(blockDim.x);
      if (v >= total) continue;
      const int r = v / vec_per_row;
      const int c = col0 + (v - r * vec_per_row) * 8;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int src = 0; src < W; ++src)
        if (src < g.world) {
          const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&raw[u][src]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(hp[j]);
            acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
            acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
          }
        }
      if (g.red_bias != nullptr) {
        const uint4 braw = __ldg(reinterpret_cast<const uint4*>(g.red_bias + c));
        const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&braw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(bp[j]);
          acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
          acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
        }
      }
      uint4 o;
      __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) op[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      if (g.peer_out[0] == nullptr) {
        *reinterpret_cast<uint4*>(g.red_out + (static_cast<int64_t>(lrb) * kRedRows + r) * g.red_ldo +
                                  c) = o;
      } else {
        // all-gather by push: this owner's rows into every rank's output,
        // starting with the next rank so that the ranks' stores spread
        // over the destinations
        const int64_t go = (static_cast<int64_t>(g.rank) * g.rows_per_owner +
                            static_cast<int64_t>(lrb) * kRedRows + r) * g.N + c;
#pragma unroll
        for (int d = 1; d <= W; ++d)
          if (d <= g.world) {
            int j = g.rank + d;
            j = j >= g.world ? j - g.world : j;
            *reinterpret_cast<uint4*>(g.peer_out[j] + go) = o;
          }
      }
    }
  }
}

// After a bounded wait ran out, overwrite with NaN this CTA's share (the
// tiles cta, cta + ctas, ... of a rows_per_owner x N block, the reduction's
// own tiling) of an owner block that could not be produced, so that a
// consumer reads NaN instead of stale or partial sums.  Local memory only:
// nothing is written to a peer that may be gone.
__device__ void poison_owner_block(const GemmArgs& g, __nv_bfloat16* block, int64_t ld, int bn,
                                   int cta, int ctas) {
  const int tiles = (g.rows_per_owner / kRedRows) * g.num_n;
  const uint4 nan8 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
  for (int t = cta; t < tiles; t += ctas) {
    const int lrb = t / g.num_n;
    const int col0 = (t - lrb * g.num_n) * bn;
    const int vec_per_row = min(bn, g.N - col0) / 8;
    for (int v = threadIdx.x; v < kRedRows * vec_per_row; v += blockDim.x) {
      const int r = v / vec_per_row;
      const int c = col0 + (v - r * vec_per_row) * 8;
      *reinterpret_cast<uint4*>(block + (static_cast<int64_t>(lrb) * kRedRows + r) * ld + c) = nan8;
    }
  }
}

// Fused reduce-scatter, owner side, run by every thread of a CTA that has no
// GEMM tiles left (all CTAs of the cooperative persistent grid are resident,
// and peers run concurrently on their own GPUs, so every wait here is on work
// that is already executing).  Wait until every source's counter shows all
// of this rank's blocks have landed, then for each (row block, column tile)
// read the bf16 partials the sources pushed into this rank's slots (local
// HBM), sum in rank order in fp32, add the bias, store.  The wait is
// bounded; a timeout records the device status and skips the reduction.
__device__ void reduce_phase(const GemmArgs& g, int bn, int cta, int ctas) {
  const int rbpo = g.rows_per_owner / kRedRows;
  const int tiles = rbpo * g.num_n;
  if (cta >= tiles) return;
  // Every source sends each element of this rank's rows_per_owner x N block
  // once per call; its counter reaches uses x rows_per_owner x N once all of
  // them have landed (independent of the tile configuration).
  const unsigned long long target = static_cast<unsigned long long>(g.uses) *
                                    static_cast<unsigned long long>(g.rows_per_owner) *
                                    static_cast<unsigned long long>(g.N);
  int ok = 1;
  if (threadIdx.x < static_cast<unsigned>(g.world)) {
    const unsigned long long* c = g.peer_count[g.rank] + threadIdx.x;
    bool seen = ld_acquire_sys_u64(c) >= target;
    if (!seen) {
      const uint64_t t0 = globaltimer_ns();
      while (!(seen = ld_acquire_sys_u64(c) >= target)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        __nanosleep(64);
      }
    }
    if (!seen) {
      ok = 0;
      if (g.status) atomicExch(g.status, kDevWaitTimeout);
    }
  }
  const bool have_all = __syncthreads_and(ok) != 0;
  unsigned long long reduced = 0;
  if (!have_all) {
    // a source never reported: this rank's rows cannot be summed.  In
    // all-reduce mode nothing is published either, so every rank's gather
    // wait below runs out for this owner and poisons its copy of the rows.
    poison_owner_block(g, g.red_out, g.red_ldo, bn, cta, ctas);
  }
  for (int t = cta; have_all && t < tiles; t += ctas) {
    const int lrb = t / g.num_n;
    const int nb = t - lrb * g.num_n;
    const int col0 = nb * bn;
    const int vec_per_row = min(bn, g.N - col0) / 8;
    reduced += static_cast<unsigned long long>(kRedRows) * vec_per_row * 8;
    if (g.world <= 2)
      reduce_block<4, 2>(g, lrb, col0, vec_per_row);
    else if (g.world <= 4)
      reduce_block<2, 4>(g, lrb, col0, vec_per_row);
    else
      reduce_block<1, 8>(g, lrb, col0, vec_per_row);
  }
  if (g.peer_out[0] == nullptr) return;
  // All-reduce: drain this CTA's gather stores once, publish the element
  // count to every rank, then wait until every owner's rows are here.
  __syncthreads();
  if (have_all && threadIdx.x == 0) {
    __threadfence_system();
    for (int j = 0; j < g.world; ++j)
      asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(g.peer_count[j] + g.world +
                                                                     g.rank),
                   "l"(reduced)
                   : "memory");
  }
  __shared__ unsigned int missing;  // owners whose reduced rows never arrived
  if (threadIdx.x == 0) missing = 0u;
  __syncthreads();
  if (threadIdx.x < static_cast<unsigned>(g.world)) {
    const unsigned long long* c = g.peer_count[g.rank] + g.world + threadIdx.x;
    bool seen = ld_acquire_sys_u64(c) >= target;
    if (!seen) {
      const uint64_t t0 = globaltimer_ns();
      while (!(seen = ld_acquire_sys_u64(c) >= target)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        __nanosleep(64);
      }
    }
    if (!seen) {
      if (g.status) atomicExch(g.status, kDevWaitTimeout);
      atomicOr(&missing, 1u << threadIdx.x);
    }
  }
  __syncthreads();
  const unsigned int lost = missing;
  for (int j = 0; j < g.world; ++j)
    if (lost & (1u << j))
      poison_owner_block(g, g.peer_out[g.rank] + static_cast<int64_t>(j) * g.rows_per_owner * g.N,
                         g.N, bn, cta, ctas);
  __syncthreads();
}

// Ulysses exchange, receiving side, run by one CTA after its tiles: wait
// (bounded) until every source's counter shows its rows of the heads this
// rank holds (3 x M x real heads x head_dim elements per call), so that the
// launch ends with the receive buffer complete.  A source that never reports
// leaves its slot overwritten with NaN and the device status set.
__device__ void ulysses_wait_phase(const GemmArgs& g) {
  const int real = max(0, min(g.ul_local, g.ul_heads - g.ul_rank * g.ul_local));
  const unsigned long long target = static_cast<unsigned long long>(g.ul_uses) * 3ull *
                                    static_cast<unsigned long long>(g.M) *
                                    static_cast<unsigned long long>(real) *
                                    static_cast<unsigned long long>(g.ul_head_dim);
  __shared__ unsigned int ul_missing;
  if (threadIdx.x == 0) ul_missing = 0u;
  __syncthreads();
  if (threadIdx.x < static_cast<unsigned>(g.ul_world)) {
    const unsigned long long* c = g.peer_count[g.ul_rank] + threadIdx.x;
    bool seen = ld_acquire_sys_u64(c) >= target;
    if (!seen) {
      const uint64_t t0 = globaltimer_ns();
      while (!(seen = ld_acquire_sys_u64(c) >= target)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        __nanosleep(64);
      }
    }
    if (!seen) {
      if (g.status) atomicExch(g.status, kDevWaitTimeout);
      atomicOr(&ul_missing, 1u << threadIdx.x);
    }
  }
  __syncthreads();
  const unsigned int lost = ul_missing;
  if (lost == 0u) return;
  const int64_t slot = 3ll * g.M * g.ul_local * g.ul_head_dim;  // elements per source slot
  const uint4 nan8 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
  for (int s = 0; s < g.ul_world; ++s) {
    if (!(lost & (1u << s))) continue;
    uint4* dst = reinterpret_cast<uint4*>(g.peer_part[g.ul_rank] + s * slot);
    for (int64_t v = threadIdx.x; v < slot / 8; v += blockDim.x) dst[v] = nan8;
  }
}

// Write a staged 32-row x (chunks x 16 bytes) block back as row segments:
// `chunks` lanes cover one row, 32 / chunks rows per store instruction.
template <typename OutT>
__device__ __forceinline__ void write_staged(const GemmArgs& g, uint8_t* stage, int64_t row_base,
                                             int col0, int chunks, int lane) {
  const int rows_per_store = 32 / chunks;
  const int chunk = lane % chunks;
  const int col = col0 + chunk * (16 / static_cast<int>(sizeof(OutT)));
#pragma unroll 1
  for (int rr = lane / chunks; rr < 32; rr += rows_per_store) {
    const int64_t out_r = row_base + rr;
    if (out_r < g.M && col < g.N)
      *reinterpret_cast<uint4*>(out_row_ptr<OutT>(g, out_r) + col) = *stage_slot(stage, rr, chunk);
  }
}

// Split-K epilogue of one epilogue warp for one (tile, slice) unit:
//  1. store this slice's int32 partial (lane quarter warp % 4, column half
//     (warp-2)/4) to ws[slice] as 128-byte row segments;
//  2. count the unit on the tile; the unit that arrives last
//  3. sums every slice's partial (exact int32) and runs the usual
//     dequant / bias / GELU epilogue on the sum.
template <int BN, typename OutT>
__device__ __forceinline__ void splitk_epilogue(const GemmArgs& g, uint32_t tmem_base,
                                                uint32_t acc_col, int64_t row0, int col0,
                                                int tile, int slice, int warp, int lane,
                                                uint8_t* stage, volatile int* last_flag) {
  constexpr int kHalf = BN / 2;
  const int q = warp & 3;
  const int h = (warp - 2) >> 2;
  const int64_t row_base = row0 + q * 32;
  const int64_t row = row_base + lane;
  const int64_t slice_elems = static_cast<int64_t>(g.M) * g.N;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc_col +
                         static_cast<uint32_t>(h * kHalf);
#pragma unroll 1
  for (int c = 0; c < kHalf / 32; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *stage_slot(stage, lane, j) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    __syncwarp();
    const int col_c = col0 + h * kHalf + c * 32;
    const int chunk = lane % 8;
    const int col = col_c + chunk * 4;
#pragma unroll 1
    for (int rr = lane / 8; rr < 32; rr += 4) {
      const int64_t out_r = row_base + rr;
      if (out_r < g.M && col < g.N)
        *reinterpret_cast<uint4*>(g.ws + slice * slice_elems + out_r * g.N + col) =
            *stage_slot(stage, rr, chunk);
    }
    __syncwarp();
  }
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
  if (warp == 2 && lane == 0) {
    const unsigned int prior = atomicAdd(g.tile_counters + tile, 1u);
    const int last = prior == static_cast<unsigned int>(g.splits - 1);
    if (last) g.tile_counters[tile] = 0u;  // every slice has arrived: reset for the next call
    *last_flag = last;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
  if (!*last_flag) return;
  __threadfence();
  const bool row_ok = row < g.M;
  const float sa = row_ok ? (g.sa_per_row ? __ldg(g.sa + row) : __ldg(g.sa)) : 0.f;
  int32_t* dbg_row = (g.acc_debug != nullptr && row_ok)
                         ? g.acc_debug + row * static_cast<int64_t>(g.N) : nullptr;
#pragma unroll 1
  for (int c = 0; c < kHalf / 32; ++c) {
    const int col = col0 + h * kHalf + c * 32;
    uint32_t sum[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) sum[j] = 0u;
    if (row_ok) {
      for (int sl = 0; sl < g.splits; ++sl) {
        const int32_t* src = g.ws + sl * slice_elems + row * g.N + col;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (col + 4 * j < g.N) {
            const uint4 v = ld_cg16(src + 4 * j);
            sum[4 * j] += v.x;
            sum[4 * j + 1] += v.y;
            sum[4 * j + 2] += v.z;
            sum[4 * j + 3] += v.w;
          }
        }
      }
    }
    uint4 o[4];
    epilogue16<OutT>(g, sum, sa, col, o[0], o[1]);
    epilogue16<OutT>(g, sum + 16, sa, col + 16, o[2], o[3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) *stage_slot(stage, lane, j) = o[j];
    if (dbg_row != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        if (col + j < g.N)
          *reinterpret_cast<uint4*>(dbg_row + col + j) =
              make_uint4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
    }
    __syncwarp();
    write_staged<OutT>(g, stage, row_base, col, 32 * static_cast<int>(sizeof(OutT)) / 16, lane);
    __syncwarp();
  }
}

template <int BN_CTA, int STAGES>
struct Smem {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN_CTA * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  // 1 KiB aligned: the staging tiles are read by TMA in the 128-byte swizzle
  static constexpr int kEpiOffset = (kBarOffset + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int kTotal = kEpiOffset + kEpiWarps * kEpiStageBytes + 1024;  // + align slack
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

struct Barriers {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tmem_full;
  uint64_t* tmem_empty;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  volatile int* split_last;  // split-K: "this CTA completes the tile"
};

template <int STAGES>
__device__ __forceinline__ Barriers carve_barriers(uint8_t* base) {
  Barriers b;
  b.full = reinterpret_cast<uint64_t*>(base);
  b.empty = b.full + STAGES;
  b.tmem_full = b.empty + STAGES;
  b.tmem_empty = b.tmem_full + 2;
  b.tmem_slot = reinterpret_cast<uint32_t*>(b.tmem_empty + 2);
  b.abort_flag = reinterpret_cast<volatile int*>(b.tmem_slot + 1);
  b.split_last = reinterpret_cast<volatile int*>(b.tmem_slot + 2);
  return b;
}

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                    ~static_cast<uintptr_t>(1023));
}

// Before a kernel waits for its predecessor on the stream (programmatic
// dependent launch), its producer pulls the weight rows of its first tile
// towards L2: weights are never written by the kernel before, so the reads
// can overlap that kernel's tail.  With few M tiles (skinny token counts, a
// weight-bound GEMM) the whole K range is requested; otherwise only the
// k-blocks the pipeline fills first, since many CTAs share each panel.
template <int STAGES>
__device__ __forceinline__ void prefetch_weight_panel(const CUtensorMap* tm_b, const GemmArgs& g,
                                                      int kb0, int kb1, int b_row) {
  const int count = g.num_m <= 2 ? kb1 - kb0 : min(kb1 - kb0, STAGES);
  for (int i = 0; i < count; ++i) tma_prefetch_l2_2d(tm_b, (kb0 + i) * kBK, b_row);
}

// ====================================================================== one CTA
template <int BN, int STAGES, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_out, const GemmArgs g) {
  using L = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * L::kABytes;
  const Barriers bar = carve_barriers<STAGES>(smem + L::kBarOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = g.num_m * g.num_n * g.splits;  // (tile, K slice) work units

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar.full[s], 1);
      mbar_init(&bar.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar.tmem_full[b], 1);
      mbar_init(&bar.tmem_empty[b], kEpiWarps);
    }
    *bar.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (g.tma_store) tma_prefetch_desc(&tm_out);
    if (static_cast<int>(blockIdx.x) < units) {
      const int tile = blockIdx.x / g.splits;
      const int kb0 = (blockIdx.x - tile * g.splits) * g.kb_per_split;
      const int kb1 = min(kb0 + g.kb_per_split, g.kblocks);
      int mb, nb;
      tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      prefetch_weight_panel<STAGES>(&tm_b, g, kb0, kb1, nb * BN);
    }
  }
  if (warp == 1) {
    tmem_alloc(bar.tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *bar.tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
        const int tile = unit / g.splits;
        const int kb0 = (unit - tile * g.splits) * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kblocks);
        int mb, nb;
        tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bar.empty[stage], phase ^ 1u, bar.abort_flag, g.status)) {
            ok = false;
            break;
          }
          issued_mask &= ~(1u << stage);
          mbar_arrive_expect_tx(&bar.full[stage], L::kStageBytes);
          tma_load_2d(&tm_a, &bar.full[stage], s_a + stage * L::kABytes, kb * kBK, mb * kBM);
          tma_load_2d(&tm_b, &bar.full[stage], s_b + stage * L::kBBytes, kb * kBK, nb * BN);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            mbar_wait_drain(&bar.full[s], (issued_parity >> s) & 1u, g.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = make_idesc_i8(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued_any = false;
      for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
        const int tile = unit / g.splits;
        const int kb0 = (unit - tile * g.splits) * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kblocks);
        if (!mbar_wait(&bar.tmem_empty[acc], acc_phase ^ 1u, bar.abort_flag, g.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bar.full[stage], phase, bar.abort_flag, g.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(s_a + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(s_b + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            umma_i8(d_tmem, make_desc_kmajor_sw128(a_addr + k * 32),
                    make_desc_kmajor_sw128(b_addr + k * 32), kIdesc,
                    ((kb - kb0) | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit(&bar.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&bar.tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Every batch of MMAs was followed by a commit to its stage's `empty`
        // barrier: once the last one completes the tensor pipe has drained.
        const int last = (stage + STAGES - 1) % STAGES;
        mbar_wait_drain(&bar.empty[last], stage == 0 ? (phase ^ 1u) : phase, g.status);
      }
    }
    __syncwarp();
  } else {
    int acc = 0;
    uint32_t acc_phase = 0;
    long long sent[kMaxPeers] = {};
    uint8_t* stage = smem + L::kEpiOffset + (warp - 2) * kEpiStageBytes;
    // TMA-store epilogue: column constants of this warp's kHalf columns
    // and its row's token scale, one tile ahead
    constexpr int kHalf = BN / 2;
    const int epi_h = (warp - 2) >> 2;
    const int epi_row = (warp & 3) * 32 + lane;
    ColPrefetch pf{};
    if (g.tma_store && static_cast<int>(blockIdx.x) < units) {
      int mb0, nb0;
      tile_coords(static_cast<int>(blockIdx.x), g.num_m, g.num_n, mb0, nb0, g.m_owners, g.mb_per_owner, g.group_n);
      pf = col_prefetch<OutT>(g, nb0 * BN + epi_h * kHalf, kHalf,
                              static_cast<int64_t>(mb0) * kBM + epi_row, lane);
    }
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
      const int tile = unit / g.splits;
      int mb, nb;
      tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      float sa_tile = 0.f;
      if (g.tma_store) {
        col_cache_store(stage, pf, kHalf, lane);
        sa_tile = pf.sa;
        __syncwarp();
        const int next = unit + static_cast<int>(gridDim.x);
        if (next < units) {
          int mb1, nb1;
          tile_coords(next, g.num_m, g.num_n, mb1, nb1, g.m_owners, g.mb_per_owner, g.group_n);
          pf = col_prefetch<OutT>(g, nb1 * BN + epi_h * kHalf, kHalf,
                                  static_cast<int64_t>(mb1) * kBM + epi_row, lane);
        }
      }
      if (!mbar_wait(&bar.tmem_full[acc], acc_phase, bar.abort_flag, g.status)) break;
      tc_fence_after();
      if (g.splits > 1)
        splitk_epilogue<BN, OutT>(g, tmem_base, static_cast<uint32_t>(acc * BN),
                                  static_cast<int64_t>(mb) * kBM, nb * BN, tile,
                                  unit - tile * g.splits, warp, lane, stage, bar.split_last);
      const auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar.tmem_empty[acc]);
      };
      if (g.splits > 1) {
        release();
      } else if (g.tma_store) {
        bool done = false;
        if constexpr ((BN / 2) % 64 == 0) {
          if (g.epilogue & TM_EPI_SWIGLU) {
            epilogue_tile_swiglu<BN, OutT>(g, &tm_out, tmem_base, static_cast<uint32_t>(acc * BN),
                                           static_cast<int64_t>(mb) * kBM, nb * BN, warp, lane,
                                           stage, sa_tile, release);
            done = true;
          }
        }
        if (!done)
          epilogue_tile_tma<BN, OutT>(g, &tm_out, tmem_base, static_cast<uint32_t>(acc * BN),
                                      static_cast<int64_t>(mb) * kBM, nb * BN, warp, lane, stage,
                                      sa_tile, release);
      } else {
        epilogue_tile<BN, OutT>(g, tmem_base, static_cast<uint32_t>(acc * BN),
                                static_cast<int64_t>(mb) * kBM, nb * BN, warp, lane, stage);
        release();
      }
      if (g.world > 0 && static_cast<int64_t>(mb) * kBM < g.M)
        sent[static_cast<int>(static_cast<int64_t>(mb) * kBM / g.rows_per_owner)] +=
            kBM * min(BN, g.N - nb * BN);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (g.tma_store && lane == 0) bulk_wait_all();  // stores done before the CTA ends
    if (g.world > 0) publish_counts(g, sent, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
  if (g.world > 0) reduce_phase(g, BN, blockIdx.x, gridDim.x);
}

// ====================================================================== CTA pair
// BN is the pair's N tile; each CTA holds BN/2 rows of B and 128 rows of A.
template <int BN>
struct PairTmem {
  static constexpr uint32_t kCols = BN <= 128 ? 256u : 512u;  // power of two >= 2*BN
};

template <int BN, int STAGES, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                        const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_out, const GemmArgs g) {
  constexpr int kBNHalf = BN / 2;
  using L = Smem<kBNHalf, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * L::kABytes;
  const Barriers bar = carve_barriers<STAGES>(smem + L::kBarOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader (issues the MMAs)
  const bool leader = rank == 0;
  const int tiles = g.num_m * g.num_n;  // pair tiles of 256 x BN
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar.full[s], 1);
      mbar_init(&bar.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar.tmem_full[b], 1);
      mbar_init(&bar.tmem_empty[b], 2 * kEpiWarps);  // both CTAs' epilogue warps
    }
    *bar.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (g.tma_store) tma_prefetch_desc(&tm_out);
    if (pair < tiles) {
      int mb, nb;
      tile_coords(pair, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      prefetch_weight_panel<STAGES>(&tm_b, g, 0, g.kblocks,
                                    nb * BN + static_cast<int>(rank) * kBNHalf);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(bar.tmem_slot, PairTmem<BN>::kCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *bar.tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        int mb, nb;
        tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
        const int a_row = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int b_row = nb * BN + static_cast<int>(rank) * kBNHalf;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&bar.empty[stage], phase ^ 1u, bar.abort_flag, g.status)) {
            ok = false;
            break;
          }
          issued_mask &= ~(1u << stage);
          // The leader's `full` barrier counts the bytes landing in both CTAs.
          if (leader) mbar_arrive_expect_tx(&bar.full[stage], 2 * L::kStageBytes);
          const uint32_t full_leader = map_to_cta(smem_u32(&bar.full[stage]), 0);
          tma_load_2d_pair(&tm_a, full_leader, s_a + stage * L::kABytes, kb * kBK, a_row);
          tma_load_2d_pair(&tm_b, full_leader, s_b + stage * L::kBBytes, kb * kBK, b_row);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        if (leader) {
          for (int s = 0; s < STAGES; ++s)
            if (issued_mask & (1u << s))
              mbar_wait_drain(&bar.full[s], (issued_parity >> s) & 1u, g.status);
        } else {
          // The peer's copies complete on the leader's barriers, which this
          // CTA cannot poll; give any in-flight copy ample time to land.
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(1000);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t kIdesc = make_idesc_i8(2 * kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued_any = false;
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        if (!mbar_wait(&bar.tmem_empty[acc], acc_phase ^ 1u, bar.abort_flag, g.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&bar.full[stage], phase, bar.abort_flag, g.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(s_a + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(s_b + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            umma_i8_pair(d_tmem, make_desc_kmajor_sw128(a_addr + k * 32),
                         make_desc_kmajor_sw128(b_addr + k * 32), kIdesc,
                         (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit_pair(&bar.empty[stage], 0x3);  // frees the stage in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&bar.tmem_full[acc], 0x3);  // both CTAs' accumulators ready
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        const int last = (stage + STAGES - 1) % STAGES;
        mbar_wait_drain(&bar.empty[last], stage == 0 ? (phase ^ 1u) : phase, g.status);
      }
    }
    __syncwarp();
  } else {
    const uint32_t empty_leader0 = map_to_cta(smem_u32(&bar.tmem_empty[0]), 0);
    const uint32_t empty_leader1 = map_to_cta(smem_u32(&bar.tmem_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    long long sent[kMaxPeers] = {};
    uint8_t* stage = smem + L::kEpiOffset + (warp - 2) * kEpiStageBytes;
    // TMA-store epilogue: column constants of this warp's kHalf columns
    // and its row's token scale, one tile ahead
    constexpr int kHalf = BN / 2;
    const int epi_h = (warp - 2) >> 2;
    const int epi_row = static_cast<int>(rank) * kBM + (warp & 3) * 32 + lane;
    ColPrefetch pf{};
    if (g.tma_store && pair < tiles) {
      int mb0, nb0;
      tile_coords(pair, g.num_m, g.num_n, mb0, nb0, g.m_owners, g.mb_per_owner, g.group_n);
      pf = col_prefetch<OutT>(g, nb0 * BN + epi_h * kHalf, kHalf,
                              static_cast<int64_t>(mb0) * 2 * kBM + epi_row, lane);
    }
    for (int tile = pair; tile < tiles; tile += pairs) {
      int mb, nb;
      tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      float sa_tile = 0.f;
      if (g.tma_store) {
        col_cache_store(stage, pf, kHalf, lane);
        sa_tile = pf.sa;
        __syncwarp();
        if (tile + pairs < tiles) {
          int mb1, nb1;
          tile_coords(tile + pairs, g.num_m, g.num_n, mb1, nb1, g.m_owners, g.mb_per_owner, g.group_n);
          pf = col_prefetch<OutT>(g, nb1 * BN + epi_h * kHalf, kHalf,
                                  static_cast<int64_t>(mb1) * 2 * kBM + epi_row, lane);
        }
      }
      if (!mbar_wait(&bar.tmem_full[acc], acc_phase, bar.abort_flag, g.status)) break;
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(mb) * 2 * kBM + rank * kBM;
      const auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc == 0 ? empty_leader0 : empty_leader1);
      };
      if (g.tma_store) {
        bool done = false;
        if constexpr ((BN / 2) % 64 == 0) {
          if (g.epilogue & TM_EPI_SWIGLU) {
            epilogue_tile_swiglu<BN, OutT>(g, &tm_out, tmem_base, static_cast<uint32_t>(acc * BN),
                                           row0, nb * BN, warp, lane, stage, sa_tile, release);
            done = true;
          }
        }
        if (!done)
          epilogue_tile_tma<BN, OutT>(g, &tm_out, tmem_base, static_cast<uint32_t>(acc * BN),
                                      row0, nb * BN, warp, lane, stage, sa_tile, release);
      } else {
        epilogue_tile<BN, OutT>(g, tmem_base, static_cast<uint32_t>(acc * BN), row0, nb * BN, warp,
                                lane, stage);
        release();
      }
      if (g.world > 0 && row0 < g.M)
        sent[static_cast<int>(row0 / g.rows_per_owner)] += kBM * min(BN, g.N - nb * BN);
      if (g.ul_peer && row0 < g.M) {  // elements this tile sent to each destination
        const long long rows = min(static_cast<int64_t>(kBM), g.M - row0);
        for (int c = nb * BN; c < min((nb + 1) * BN, g.N); c += 64) sent[ul_peer_dest(g, c)] += rows * 64;
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (g.tma_store && lane == 0) bulk_wait_all();  // stores done before the CTA ends
    if (g.world > 0) publish_counts(g, sent, warp, lane);
    if (g.ul_peer) publish_ul_counts(g, sent, warp, lane);
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, PairTmem<BN>::kCols);
  }
  if (g.world > 0) reduce_phase(g, BN, blockIdx.x, gridDim.x);
  if (g.ul_peer && blockIdx.x == 0) ulysses_wait_phase(g);
}

// ====================================================================== CTA pair + LoRA
// The BF16 LoRA delta in the epilogue (the reference's
// H3InferenceParallelLinearLoRA.forward, lora_checkpoint.py:126-154:
// output + bf16(bf16(x A^T) B^T) * scale).  T = x A^T ([M, r] bf16, r <= 64)
// is computed by the caller; B_lora ([N, r] bf16) carries the adapter scale.
// Per 256 x 256 pair tile, after the int8 main loop:
//   1. every epilogue warp dequantises its accumulator columns to the
//      rounded output value y (OutT-rounded, held as fp32) and writes them
//      back into the same TMEM columns, then signals the leader (conv);
//   2. the leader's MMA thread adds T_tile * B_lora_tile^T onto them with
//      four kind::f16 MMAs (K = 64) and commits lora_done to both CTAs;
//   3. the epilogue reads y + T B^T (fp32), applies GELU if asked, rounds
//      once and TMA-stores the tile.
// The accumulator stays 2 x 256 TMEM columns (the 256-wide tile keeps its
// operand efficiency); T and B_lora tiles use one 32 KiB shared buffer, so
// the ring has one stage fewer.  The update is added in fp32 and rounded once
// with y (the reference rounds T B^T to bf16 first): within one bf16 step.
template <int STAGES>
struct LoraSmem {
  static constexpr int kABytes = kBM * kBK;             // 16 KiB
  static constexpr int kBBytes = 128 * kBK;             // 16 KiB (half of N = 256)
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kLoraOffset = STAGES * kStageBytes;
  static constexpr int kLoraBytes = 2 * 128 * 128;      // T rows + B_lora rows, 128 B each
  static constexpr int kBarOffset = kLoraOffset + kLoraBytes;
  static constexpr int kBarBytes = (2 * STAGES + 10) * 8 + 16;
  static constexpr int kEpiOffset = (kBarOffset + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int kTotal = kEpiOffset + kEpiWarps * kEpiStageBytes + 1024;
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

// Phase 1 of the LoRA epilogue: one warp's 128 columns of int32 accumulator
// -> rounded output value (fp32 bits) in place.  Constants from the column
// cache; same arithmetic as dequant16_cached without GELU.
template <typename OutT>
__device__ __forceinline__ void lora_convert_in_place(const GemmArgs& g, uint32_t t_row, float sa,
                                                      const uint8_t* region) {
  const float* sb_s = reinterpret_cast<const float*>(region + kColCacheOffset);
  const OutT* bias_s = reinterpret_cast<const OutT*>(region + kBiasCacheOffset);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
    float sb[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 v = reinterpret_cast<const float4*>(sb_s + c * 32)[j];
      sb[4 * j] = v.x;
      sb[4 * j + 1] = v.y;
      sb[4 * j + 2] = v.z;
      sb[4 * j + 3] = v.w;
    }
    tmem_ld_wait();
    if (g.bias != nullptr) {
      uint4 braw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) braw[j] = reinterpret_cast<const uint4*>(bias_s + c * 32)[j];
      const OutT* be = reinterpret_cast<const OutT*>(braw);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float y0 = __fmaf_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))), out_to_f32<OutT>(be[j]));
        float y1 = __fmaf_rn(sa, __fmul_rn(sb[j + 1], __int2float_rn(static_cast<int>(r[j + 1]))),
                             out_to_f32<OutT>(be[j + 1]));
        round2_out<OutT>(y0, y1);
        r[j] = __float_as_uint(y0);
        r[j + 1] = __float_as_uint(y1);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float y0 = __fmul_rn(sa, __fmul_rn(sb[j], __int2float_rn(static_cast<int>(r[j]))));
        float y1 = __fmul_rn(sa, __fmul_rn(sb[j + 1], __int2float_rn(static_cast<int>(r[j + 1]))));
        round2_out<OutT>(y0, y1);
        r[j] = __float_as_uint(y0);
        r[j + 1] = __float_as_uint(y1);
      }
    }
    tmem_st_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
  }
  tmem_st_wait();
}

// Phase 3: read y + T B^T, GELU if asked, round, stage, TMA store.
template <typename OutT, typename Release>
__device__ __forceinline__ void lora_store_tile(const GemmArgs& g, const CUtensorMap* tm_out,
                                                uint32_t t_row, int64_t row_base, int col_base,
                                                int lane, uint8_t* region, Release release) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
    tmem_ld_wait();
    if (c == 3) release();
    float y[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(r[j]);
    if (g.epilogue & TM_EPI_GELU_TANH) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) round2_out<OutT>(y[j], y[j + 1]);
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = gelu_tanh(y[j]);
    }
    uint4 o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = make_uint4(pack2<OutT>(y[8 * q], y[8 * q + 1]), pack2<OutT>(y[8 * q + 2], y[8 * q + 3]),
                        pack2<OutT>(y[8 * q + 4], y[8 * q + 5]),
                        pack2<OutT>(y[8 * q + 6], y[8 * q + 7]));
    const int col = col_base + c * 32;
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) *stage64_slot(region, lane, q) = o[q];
    fence_async_shared();
    __syncwarp();
    if (lane == 0 && row_base < g.M && col < g.N) {
      tma_store_2d(tm_out, region, col, static_cast<int>(row_base));
      bulk_commit();
    }
  }
}

// Phase 3 for scatter outputs (the row-parallel reduce-scatter / all-reduce
// modes, which allow no activation): read y + T B^T, round, and store each
// 64-column half through the row-per-lane staging tile as 128-byte row
// segments to the rows' owners (out_row_ptr), like epilogue_tile.  The
// column cache in the same region is dead by now (phase 1 used it).
template <typename OutT, typename Release>
__device__ __forceinline__ void lora_store_tile_scatter(const GemmArgs& g, uint32_t t_row,
                                                        int64_t row_base, int col_base, int lane,
                                                        uint8_t* region, Release release) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
    tmem_ld_wait();
    if (c == 3) release();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *stage_slot(region, lane, (c & 1) * 4 + q) = make_uint4(
          pack2<OutT>(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1])),
          pack2<OutT>(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
          pack2<OutT>(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
          pack2<OutT>(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
    if (c & 1) {
      __syncwarp();
      write_staged<OutT>(g, region, row_base, col_base + (c - 1) * 32,
                         64 * static_cast<int>(sizeof(OutT)) / 16, lane);
      __syncwarp();
    }
  }
}

template <int STAGES, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_pair_lora_kernel(const __grid_constant__ CUtensorMap tm_a,
                             const __grid_constant__ CUtensorMap tm_b,
                             const __grid_constant__ CUtensorMap tm_out,
                             const __grid_constant__ CUtensorMap tm_lt,
                             const __grid_constant__ CUtensorMap tm_lb, const GemmArgs g) {
  constexpr int BN = 256;
  constexpr int kBNHalf = BN / 2;
  using L = LoraSmem<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * L::kABytes;
  uint8_t* s_lt = smem + L::kLoraOffset;
  uint8_t* s_lb = s_lt + 128 * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* conv = tmem_empty + 2;       // at the leader: both CTAs' epilogue warps
  uint64_t* lora_done = conv + 2;        // LoRA MMAs of the accumulator complete
  uint64_t* lora_full = lora_done + 2;   // T / B_lora tiles landed (leader)
  uint64_t* lora_empty = lora_full + 1;  // LoRA buffer consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lora_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int tiles = g.num_m * g.num_n;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 2 * kEpiWarps);
      mbar_init(&conv[b], 2 * kEpiWarps);
      mbar_init(&lora_done[b], 1);
    }
    mbar_init(lora_full, 1);
    mbar_init(lora_empty, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_out);
    tma_prefetch_desc(&tm_lt);
    tma_prefetch_desc(&tm_lb);
    if (pair < tiles) {
      int mb, nb;
      tile_coords(pair, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      prefetch_weight_panel<STAGES>(&tm_b, g, 0, g.kblocks,
                                    nb * BN + static_cast<int>(rank) * kBNHalf);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, lora_phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true, lora_inflight = false;
      const uint32_t lora_full_leader = map_to_cta(smem_u32(lora_full), 0);
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        int mb, nb;
        tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
        const int a_row = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int b_row = nb * BN + static_cast<int>(rank) * kBNHalf;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, g.status)) {
            ok = false;
            break;
          }
          issued_mask &= ~(1u << stage);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t full_leader = map_to_cta(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(&tm_a, full_leader, s_a + stage * L::kABytes, kb * kBK, a_row);
          tma_load_2d_pair(&tm_b, full_leader, s_b + stage * L::kBBytes, kb * kBK, b_row);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // this tile's LoRA operands, once the previous tile's LoRA MMAs are done
        if (!mbar_wait(lora_empty, lora_phase ^ 1u, abort_flag, g.status)) {
          ok = false;
          break;
        }
        lora_inflight = false;
        if (leader) mbar_arrive_expect_tx(lora_full, 2 * L::kLoraBytes);
        tma_load_2d_pair(&tm_lt, lora_full_leader, s_lt, 0, a_row);
        tma_load_2d_pair(&tm_lb, lora_full_leader, s_lb, 0, b_row);
        lora_inflight = true;
        lora_phase ^= 1u;
      }
      if (!ok) {
        if (leader) {
          for (int s = 0; s < STAGES; ++s)
            if (issued_mask & (1u << s))
              mbar_wait_drain(&full[s], (issued_parity >> s) & 1u, g.status);
          if (lora_inflight) mbar_wait_drain(lora_full, lora_phase ^ 1u, g.status);
        } else {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(1000);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t kIdesc = make_idesc_i8(2 * kBM, BN);
      constexpr uint32_t kIdescL = make_idesc_bf16(2 * kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t conv_phase[2] = {0u, 0u};
      uint32_t lora_phase = 0;
      int pending = 0;      // tiles whose LoRA MMAs are not issued yet (<= 2)
      int oldest_acc = 0;   // accumulator of the oldest such tile
      bool ok = true, issued_any = false;
      // The LoRA MMAs of the oldest pending tile: wait for its converted
      // accumulator (both CTAs) and its operand tiles, add T B^T, release.
      const auto service = [&](bool block) -> bool {
        const int a = oldest_acc;
        if (!block && !mbar_test(&conv[a], conv_phase[a])) return true;
        if (block && !mbar_wait(&conv[a], conv_phase[a], abort_flag, g.status)) return false;
        if (!mbar_wait(lora_full, lora_phase, abort_flag, g.status)) return false;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(a * BN);
        const uint32_t lt_addr = smem_u32(s_lt);
        const uint32_t lb_addr = smem_u32(s_lb);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // K = 64 bf16 = 4 x 16
          umma_bf16_pair(d_tmem, make_desc_kmajor_sw128(lt_addr + k * 32),
                         make_desc_kmajor_sw128(lb_addr + k * 32), kIdescL, 1u);
        umma_commit_pair(&lora_done[a], 0x3);
        umma_commit_pair(lora_empty, 0x3);
        conv_phase[a] ^= 1u;
        lora_phase ^= 1u;
        oldest_acc ^= 1;
        --pending;
        return true;
      };
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        // the accumulator's previous tile must get its LoRA update before
        // the epilogue can hand the accumulator back
        if (pending == 2 && !service(true)) {
          ok = false;
          break;
        }
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
          for (int k = 0; k < kBK / 32; ++k)
            umma_i8_pair(d_tmem, make_desc_kmajor_sw128(a_addr + k * 32),
                         make_desc_kmajor_sw128(b_addr + k * 32), kIdesc,
                         (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (pending > 0 && !service(false)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tmem_full[acc], 0x3);
        ++pending;
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      while (ok && pending > 0)
        if (!service(true)) ok = false;
      if (!ok && issued_any) {
        const int last = (stage + STAGES - 1) % STAGES;
        mbar_wait_drain(&empty[last], stage == 0 ? (phase ^ 1u) : phase, g.status);
      }
    }
    __syncwarp();
  } else {
    const uint32_t empty_leader[2] = {map_to_cta(smem_u32(&tmem_empty[0]), 0),
                                      map_to_cta(smem_u32(&tmem_empty[1]), 0)};
    const uint32_t conv_leader[2] = {map_to_cta(smem_u32(&conv[0]), 0),
                                     map_to_cta(smem_u32(&conv[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    long long sent[kMaxPeers] = {};
    uint8_t* region = smem + L::kEpiOffset + (warp - 2) * kEpiStageBytes;
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int epi_row = static_cast<int>(rank) * kBM + q * 32 + lane;
    ColPrefetch pf{};
    if (pair < tiles) {
      int mb0, nb0;
      tile_coords(pair, g.num_m, g.num_n, mb0, nb0, g.m_owners, g.mb_per_owner, g.group_n);
      pf = col_prefetch<OutT>(g, nb0 * BN + h * kBNHalf, kBNHalf,
                              static_cast<int64_t>(mb0) * 2 * kBM + epi_row, lane);
    }
    for (int tile = pair; tile < tiles; tile += pairs) {
      int mb, nb;
      tile_coords(tile, g.num_m, g.num_n, mb, nb, g.m_owners, g.mb_per_owner, g.group_n);
      col_cache_store(region, pf, kBNHalf, lane);
      const float sa_tile = pf.sa;
      __syncwarp();
      if (tile + pairs < tiles) {
        int mb1, nb1;
        tile_coords(tile + pairs, g.num_m, g.num_n, mb1, nb1, g.m_owners, g.mb_per_owner, g.group_n);
        pf = col_prefetch<OutT>(g, nb1 * BN + h * kBNHalf, kBNHalf,
                                static_cast<int64_t>(mb1) * 2 * kBM + epi_row, lane);
      }
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, g.status)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + h * kBNHalf);
      lora_convert_in_place<OutT>(g, t_row, sa_tile, region);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(conv_leader[acc]);
      if (!mbar_wait(&lora_done[acc], acc_phase, abort_flag, g.status)) break;
      tc_fence_after();
      const int64_t row_base = static_cast<int64_t>(mb) * 2 * kBM + rank * kBM + q * 32;
      const auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(empty_leader[acc]);
      };
      if (g.tma_store)
        lora_store_tile<OutT>(g, &tm_out, t_row, row_base, nb * BN + h * kBNHalf, lane, region,
                              release);
      else
        lora_store_tile_scatter<OutT>(g, t_row, row_base, nb * BN + h * kBNHalf, lane, region,
                                      release);
      const int64_t tile_row0 = static_cast<int64_t>(mb) * 2 * kBM + rank * kBM;
      if (g.world > 0 && tile_row0 < g.M)
        sent[static_cast<int>(tile_row0 / g.rows_per_owner)] += kBM * min(BN, g.N - nb * BN);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (g.tma_store && lane == 0) bulk_wait_all();
    if (g.world > 0) publish_counts(g, sent, warp, lane);
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
  if (g.world > 0) reduce_phase(g, BN, blockIdx.x, gridDim.x);
}

// ====================================================================== host
struct Operands {
  const int8_t* a;
  int64_t lda;
  const int8_t* b;
  int64_t ldb;
};

// Output map for the TMA-store epilogue (32 x 32 boxes, 64-byte swizzle),
// or switch that epilogue off where it does not apply: split-K and scatter
// outputs.  The map is left zeroed (and never read) when unused.
template <int BN, typename OutT>
bool encode_out_map(CUtensorMap* map, GemmArgs& args) {
  memset(map, 0, sizeof(*map));
  args.tma_store = args.world == 0 && args.splits == 1 && args.ul_peer == 0;
  if (!args.tma_store) return true;
  const CUtensorMapDataType dt = std::is_same<OutT, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (args.ul_world > 0) {  // send buffer as [world * 3 * M][local heads x head_dim]
    const uint64_t cols = static_cast<uint64_t>(args.ul_local) * args.ul_head_dim;
    return encode_tmap_2d(map, dt, args.out, cols, static_cast<uint64_t>(3) * args.ul_world * args.M,
                          cols * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  // SwiGLU writes N / 2 output columns
  const uint64_t out_cols = (args.epilogue & TM_EPI_SWIGLU) ? args.N / 2 : args.N;
  return encode_tmap_2d(map, dt, args.out, out_cols, args.M, static_cast<uint64_t>(args.ldo) * 2,
                        32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

// Raster choice (GemmArgs::group_n).  Once kGroupM A panels (rows_per_mb x K
// bytes each) pass kAGroupBudget they no longer stay in L2 next to the B
// panels a wave reads (the 480p fc2, K = 12288: 16 x 3 MiB of A), so the
// tiles switch to N-fastest groups whose B panels fit kBGroupBudget.
constexpr uint64_t kAGroupBudget = 24ull << 20;
constexpr uint64_t kBGroupBudget = 48ull << 20;

int choose_group_n(int num_n, int rows_per_mb, int bn, int k) {
  const uint64_t a_group = static_cast<uint64_t>(kGroupM) * rows_per_mb * static_cast<uint64_t>(k);
  if (a_group <= kAGroupBudget) return 0;
  const uint64_t b_panel = static_cast<uint64_t>(bn) * static_cast<uint64_t>(k);
  const uint64_t fit = b_panel > 0 ? kBGroupBudget / b_panel : 1;
  return static_cast<int>(fit < 1 ? 1 : (fit > static_cast<uint64_t>(num_n) ? num_n : fit));
}

template <int BN, int STAGES, typename OutT>
int launch_single(const Operands& op, GemmArgs args, int sms, cudaStream_t stream) {
  using L = Smem<BN, STAGES>;
  args.num_m = (args.M + kBM - 1) / kBM;
  args.num_n = (args.N + BN - 1) / BN;
  args.m_owners = args.world;
  args.mb_per_owner = args.world > 0 ? args.rows_per_owner / kBM : 0;
  args.group_n = choose_group_n(args.num_n, kBM, BN, args.K);
  CUtensorMap ta, tb;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.a, args.K, args.M, op.lda, kBK, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.b, args.K, args.N, op.ldb, kBK, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  CUtensorMap to;
  if (!encode_out_map<BN, OutT>(&to, args)) return TM_ERR_CUDA;
  auto kernel = gemm_i8_kernel<BN, STAGES, OutT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
      cudaSuccess)
    return TM_ERR_CUDA;
  const int units = args.num_m * args.num_n * args.splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(units < sms ? units : sms));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  // The fused reduce-scatter waits on blocks produced by other CTAs of the
  // same launch: require them all to be resident at once.
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = args.world > 0 ? 1 : 0;
  const cudaError_t err = args.world > 0 ? cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, args)
                                         : launch_with_pdl(cfg, attr, 0, kernel, ta, tb, to, args);
  if (err != cudaSuccess) return TM_ERR_CUDA;
  return check_launch();
}

template <int BN, int STAGES, typename OutT>
int launch_pair(const Operands& op, GemmArgs args, int max_pairs, cudaStream_t stream) {
  using L = Smem<BN / 2, STAGES>;
  args.num_m = (args.M + 2 * kBM - 1) / (2 * kBM);
  args.num_n = (args.N + BN - 1) / BN;
  args.m_owners = args.world;
  args.mb_per_owner = args.world > 0 ? args.rows_per_owner / (2 * kBM) : 0;
  args.group_n = choose_group_n(args.num_n, 2 * kBM, BN, args.K);
  CUtensorMap ta, tb;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.a, args.K, args.M, op.lda, kBK, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.b, args.K, args.N, op.ldb, kBK,
                      BN / 2, CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  CUtensorMap to;
  if (!encode_out_map<BN, OutT>(&to, args)) return TM_ERR_CUDA;
  auto kernel = gemm_i8_pair_kernel<BN, STAGES, OutT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
      cudaSuccess)
    return TM_ERR_CUDA;
  const int tiles = args.num_m * args.num_n;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // The fused reduce-scatter waits on blocks produced by other CTAs of the
  // same launch: require them all to be resident at once.
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  const bool coop = args.world > 0 || args.ul_peer;
  cfg.numAttrs = coop ? 2 : 1;
  const cudaError_t err = coop ? cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, args)
                                         : launch_with_pdl(cfg, attr, 1, kernel, ta, tb, to, args);
  if (err != cudaSuccess) return TM_ERR_CUDA;
  return check_launch();
}

// LoRA operands: T = x A^T [M, r] and B_lora [N, r], bf16, r <= 64.
struct LoraSpec {
  const void* t;
  int64_t ldt;
  const void* b;
  int64_t ldb;
  int rank;
};

template <typename OutT>
int launch_pair_lora(const Operands& op, GemmArgs args, const LoraSpec& lora, int max_pairs,
                     cudaStream_t stream) {
  constexpr int kStages = 5;
  using L = LoraSmem<kStages>;
  args.num_m = (args.M + 2 * kBM - 1) / (2 * kBM);
  args.num_n = (args.N + 255) / 256;
  args.m_owners = args.world;
  args.mb_per_owner = args.world > 0 ? args.rows_per_owner / (2 * kBM) : 0;
  args.group_n = choose_group_n(args.num_n, 2 * kBM, 256, args.K);
  args.tma_store = args.world == 0;  // scatter outputs go to peers as row segments
  const CUtensorMapDataType dt = std::is_same<OutT, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb, to, tlt, tlb;
  memset(&to, 0, sizeof(to));  // never read without the TMA-store epilogue
  // T and B_lora: r columns, boxes of 64 columns (128 bytes; columns past r
  // read as zero) x 128 rows
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.a, args.K, args.M, op.lda, kBK, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, op.b, args.K, args.N, op.ldb, kBK, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      (args.tma_store &&
       !encode_tmap_2d(&to, dt, args.out, args.N, args.M, static_cast<uint64_t>(args.ldo) * 2,
                       32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) ||
      !encode_tmap_2d(&tlt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lora.t, lora.rank, args.M,
                      static_cast<uint64_t>(lora.ldt) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tlb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lora.b, lora.rank, args.N,
                      static_cast<uint64_t>(lora.ldb) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return TM_ERR_CUDA;
  auto kernel = gemm_i8_pair_lora_kernel<kStages, OutT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
      cudaSuccess)
    return TM_ERR_CUDA;
  const int tiles = args.num_m * args.num_n;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // The fused reduction waits on blocks produced by other CTAs of the same
  // launch: require them all to be resident at once.
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = args.world > 0
                              ? cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, tlt, tlb, args)
                              : launch_with_pdl(cfg, attr, 1, kernel, ta, tb, to, tlt, tlb, args);
  if (err != cudaSuccess) return TM_ERR_CUDA;
  return check_launch();
}

// Tile configurations: 0 = heuristic; 64/128/256 = one-CTA kernel with that
// N tile; kPairFlag + {128, 192, 256} = CTA-pair kernel with that N tile.
constexpr int kPairFlag = 1000;

template <typename OutT>
int dispatch(const Operands& op, const GemmArgs& args, int cfg, int sms, int max_pairs,
             cudaStream_t stream) {
  switch (cfg) {
    case 256: return launch_single<256, 4, OutT>(op, args, sms, stream);
    case 128: return launch_single<128, 6, OutT>(op, args, sms, stream);
    case 64: return launch_single<64, 8, OutT>(op, args, sms, stream);
    case kPairFlag + 256: return launch_pair<256, 6, OutT>(op, args, max_pairs, stream);
    case kPairFlag + 192: return launch_pair<192, 6, OutT>(op, args, max_pairs, stream);
    case kPairFlag + 128: return launch_pair<128, 8, OutT>(op, args, max_pairs, stream);
    default: return TM_ERR_UNSUPPORTED;
  }
}

// Relative time of an unsplit configuration: waves of tiles over the
// resident CTAs (or pairs) times the per-SM length of one tile -- its
// k-blocks (plus ~2 for filling the pipeline) times its N width, divided by
// that configuration's sustained efficiency.  The efficiencies are B200
// measurements at M=20480, N=9216, K=3072 (normalised to the 256-wide pair
// tile): narrower tiles need more operand bytes per MMA.
double estimate(int cfg, int m, int n, int kblocks, int sms, int max_pairs) {
  const bool pair = cfg > kPairFlag;
  const int bn = pair ? cfg - kPairFlag : cfg;
  double eff;
  switch (cfg) {
    case kPairFlag + 256: eff = 1.00; break;
    case kPairFlag + 192: eff = 0.77; break;
    case kPairFlag + 128: eff = 0.52; break;
    case 256: eff = 0.91; break;
    case 128: eff = 0.60; break;
    default: eff = 0.30; break;
  }
  const double rows = pair ? 2.0 * kBM : kBM;
  const double tiles = std::ceil(m / rows) * std::ceil(static_cast<double>(n) / bn);
  const double slots = pair ? max_pairs : sms;
  return std::ceil(tiles / slots) * (kblocks + 2.0) * bn / eff;
}

struct Choice {
  int cfg;
  int splits;
};

// Best (configuration, K slices).  Split-K (one-CTA kernel, 64-wide tiles)
// pays only when K is long and the tile grid leaves most SMs idle: on B200 a
// (tile, slice) unit has a fixed cost of several microseconds (pipeline fill,
// the int32 partial round trip through L2), so at K = 3072 splitting never
// won, while at K = 12288 and M <= 256 it cut the time by 1.4-2x (3-6
// slices).  Rule: K >= 48 k-blocks and at most half the SMs covered by the
// unsplit 64-wide grid; slices = as many as keep one wave of units and at
// least 16 k-blocks per slice, up to 8.
Choice pick_choice(int m, int n, int kblocks, int sms, int max_pairs, bool allow_split) {
  if (allow_split && kblocks >= 48) {
    const int tiles64 = ((m + kBM - 1) / kBM) * ((n + 63) / 64);
    if (2 * tiles64 <= sms) {
      int splits = sms / tiles64;
      splits = min(splits, kblocks / 16);
      splits = min(splits, 8);
      if (splits >= 2) return Choice{64, splits};
    }
  }
  static const int kConfigs[] = {kPairFlag + 256, kPairFlag + 192, kPairFlag + 128, 256, 128, 64};
  Choice best{256, 1};
  double best_t = -1.0;
  for (int cfg : kConfigs) {
    if (cfg > kPairFlag && max_pairs <= 0) continue;
    const double t = estimate(cfg, m, n, kblocks, sms, max_pairs);
    if (best_t < 0 || t < best_t) {
      best_t = t;
      best = Choice{cfg, 1};
    }
  }
  return best;
}

// Effective slice count (no empty slice) and workspace bytes of a split-K
// run: per-tile counters (256-byte aligned) followed by `splits` int32 [M, N].
// Split-K workspaces start with a fixed counter region: the counters reset
// themselves to zero at the end of every call, and the int32 partials always
// start after the region, so a call's partials can never land on the
// counters of a later call with more tiles (a workspace is zeroed once and
// reused).
constexpr uint64_t kCounterRegion = 64 * 1024;

struct SplitPlan {
  int splits;
  int kb_per_split;
  uint64_t counter_bytes;
  uint64_t bytes;
};

SplitPlan plan_split(int cfg, int splits, int64_t m, int64_t n, int kblocks) {
  SplitPlan p{1, kblocks, 0, 0};
  if (splits <= 1 || cfg > kPairFlag) return p;
  const int64_t bn = cfg;
  p.kb_per_split = (kblocks + splits - 1) / splits;
  p.splits = (kblocks + p.kb_per_split - 1) / p.kb_per_split;
  if (p.splits <= 1) {
    p.splits = 1;
    p.kb_per_split = kblocks;
    return p;
  }
  // 64-bit tile arithmetic: m and n may be anything up to 2^31 - 1 here
  const uint64_t tiles = static_cast<uint64_t>((m + kBM - 1) / kBM) *
                         static_cast<uint64_t>((n + bn - 1) / bn);
  p.counter_bytes = kCounterRegion;
  if (tiles * 4 > kCounterRegion) {  // more tiles than counters: no workspace can hold it
    p.bytes = ~0ull;
    return p;
  }
  // tiles <= 16384 bounds m * n below 2^46, so the product cannot wrap
  p.bytes = p.counter_bytes + static_cast<uint64_t>(p.splits) * static_cast<uint64_t>(m) *
                                  static_cast<uint64_t>(n) * 4u;
  return p;
}

// Resident CTA pairs of the pair kernel on a device (cached per device).
int max_resident_pairs(int device, int sms) {
  static int cache[64] = {};
  if (device < 0 || device >= 64) return 0;
  if (cache[device] == 0) {
    using L = Smem<128, 6>;
    auto kernel = gemm_i8_pair_kernel<256, 6, __nv_bfloat16>;
    int clusters = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = L::kTotal;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();  // a failed query must not poison later launches
    cache[device] = clusters > 0 ? clusters : -1;
  }
  return cache[device] > 0 ? cache[device] : 0;
}

// Fused reduce-scatter request (row-parallel linears); see
// tm_scaled_mm_i8_reduce_scatter.
struct ScatterSpec {
  void* const* peer_part;
  void* const* peer_flags;
  int world;
  int rank;
  uint32_t epoch;
  void* const* peer_out = nullptr;  // all-reduce: every rank's [M][N] output
};

// Ulysses send layout of a merged QKV projection.
struct UlyssesSpec {
  int heads, head_dim, world;
  // exchange over NVLink (peer_recv != nullptr): every rank's receive
  // buffer and counters, this rank, and the call's use count
  void* const* peer_recv = nullptr;
  void* const* peer_flags = nullptr;
  int rank = 0;
  uint32_t epoch = 0;
};

// Optional split-K workspace (zeroed by the caller before its first use; the
// kernel leaves its counters at zero again after every complete call).
struct Workspace {
  void* ptr;
  uint64_t bytes;
  int force_splits;  // 0 = heuristic
};

// Host-side argument checks of every scaled-GEMM entry point: shapes,
// strides, dtypes, epilogue flags, pointers and alignment.  Touches neither
// the device nor the stream.  `ldo` may be adjusted (Ulysses layout).
int validate_scaled_mm(const void* out, int out_dtype, const int8_t* a, const int8_t* b,
                       const float* sa, int64_t sa_numel, const float* sb, int64_t sb_numel,
                       const void* bias, int64_t m, int64_t n, int64_t k, int64_t lda,
                       int64_t ldb, int64_t& ldo, uint32_t epilogue, const int32_t* acc_debug,
                       const ScatterSpec* scatter, const LoraSpec* lora,
                       const UlyssesSpec* ul) {
  if (out_dtype != TM_DTYPE_BF16 && out_dtype != TM_DTYPE_FP16) return TM_ERR_DTYPE;
  if (m < 0 || n <= 0 || k <= 0) return TM_ERR_SHAPE;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  if (k % 16 != 0 || n % 16 != 0) return TM_ERR_SHAPE;
  const bool swiglu = (epilogue & TM_EPI_SWIGLU) != 0;
  if (ul != nullptr) {
    if (ul->world < 1 || ul->heads < 1) return TM_ERR_SHAPE;
    if (ul->head_dim % 32 != 0 || n != 3LL * ul->heads * ul->head_dim) return TM_ERR_SHAPE;
    if (m % 32 != 0) return TM_ERR_SHAPE;  // a 32-row store box never crosses a group
    if (3LL * ul->world * m > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
    if (swiglu || scatter != nullptr || lora != nullptr) return TM_ERR_UNSUPPORTED;
    ldo = n;  // the row-stride checks below see a [m, n] output; the layout is the send buffer
    if (ul->peer_recv != nullptr) {  // exchange over NVLink
      // a 64-column epilogue pass must stay inside one head (one destination)
      if (ul->head_dim % 64 != 0) return TM_ERR_SHAPE;
      if (ul->world > kMaxPeers) return TM_ERR_TOO_LARGE;
      if (ul->rank < 0 || ul->rank >= ul->world) return TM_ERR_SHAPE;
      if (out_dtype != TM_DTYPE_BF16 || epilogue != 0) return TM_ERR_UNSUPPORTED;
      if (ul->peer_flags == nullptr) return TM_ERR_NULL_POINTER;
      for (int j = 0; j < ul->world; ++j) {
        if (!ul->peer_recv[j] || !ul->peer_flags[j]) return TM_ERR_NULL_POINTER;
        if (!aligned16(ul->peer_recv[j]) || !aligned16(ul->peer_flags[j]))
          return TM_ERR_ALIGNMENT;
      }
    }
  }
  // SwiGLU: n interleaved (gate, up) columns in, n / 2 columns out
  if (lda < k || ldb < k || ldo < (swiglu ? n / 2 : n)) return TM_ERR_SHAPE;
  if (lda % 16 != 0 || ldb % 16 != 0 || ldo % 8 != 0) return TM_ERR_ALIGNMENT;
  if (sa_numel != 1 && sa_numel != m) return TM_ERR_SHAPE;
  if (sb_numel != 1 && sb_numel != n) return TM_ERR_SHAPE;
  if (epilogue & ~(TM_EPI_GELU_TANH | TM_EPI_SWIGLU)) return TM_ERR_UNSUPPORTED;
  if (swiglu) {
    if (epilogue & TM_EPI_GELU_TANH) return TM_ERR_UNSUPPORTED;
    if (n % 64 != 0) return TM_ERR_SHAPE;
    if (scatter != nullptr || lora != nullptr) return TM_ERR_UNSUPPORTED;
  }
  if (scatter != nullptr) {
    if (scatter->world < 1 || scatter->world > kMaxPeers) return TM_ERR_TOO_LARGE;
    if (scatter->rank < 0 || scatter->rank >= scatter->world) return TM_ERR_SHAPE;
    if (m % (static_cast<int64_t>(scatter->world) * 2 * kBM) != 0) return TM_ERR_SHAPE;
    if (out_dtype != TM_DTYPE_BF16 || epilogue != 0) return TM_ERR_UNSUPPORTED;
    if (!scatter->peer_part || !scatter->peer_flags) return TM_ERR_NULL_POINTER;
    for (int j = 0; j < scatter->world; ++j) {
      if (!scatter->peer_part[j] || !scatter->peer_flags[j]) return TM_ERR_NULL_POINTER;
      if (!aligned16(scatter->peer_part[j]) || !aligned16(scatter->peer_flags[j]))
        return TM_ERR_ALIGNMENT;
      if (scatter->peer_out != nullptr) {
        if (!scatter->peer_out[j]) return TM_ERR_NULL_POINTER;
        if (!aligned16(scatter->peer_out[j])) return TM_ERR_ALIGNMENT;
      }
    }
  }
  if (m == 0) return TM_OK;
  if (!out || !a || !b || !sa || !sb) return TM_ERR_NULL_POINTER;
  if (!aligned16(a) || !aligned16(b) || !aligned16(out) || (bias && !aligned16(bias)) ||
      (sb_numel != 1 && !aligned16(sb)) || (acc_debug && !aligned16(acc_debug)))
    return TM_ERR_ALIGNMENT;
  return TM_OK;
}

int scaled_mm_impl(void* out, int out_dtype, const int8_t* a, const int8_t* b, const float* sa,
                   int64_t sa_numel, const float* sb, int64_t sb_numel, const void* bias,
                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldo,
                   uint32_t epilogue, int32_t* acc_debug, int force_cfg, cudaStream_t stream,
                   const ScatterSpec* scatter = nullptr, const Workspace* ws = nullptr,
                   const LoraSpec* lora = nullptr, const UlyssesSpec* ul = nullptr) {
  const int rc = validate_scaled_mm(out, out_dtype, a, b, sa, sa_numel, sb, sb_numel, bias, m, n,
                                    k, lda, ldb, ldo, epilogue, acc_debug, scatter, lora, ul);
  if (rc != TM_OK || m == 0) return rc;
  const bool swiglu = (epilogue & TM_EPI_SWIGLU) != 0;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return TM_ERR_CUDA;
  GemmArgs args{};
  args.sa = sa;
  args.sb = sb;
  args.sa_per_row = sa_numel != 1 || m == 1;
  args.sb_per_col = sb_numel != 1 || n == 1;
  args.bias = scatter ? nullptr : bias;  // scatter mode: the owner adds the bias after the sum
  args.out = out;
  args.ldo = ldo;
  args.acc_debug = acc_debug;
  args.M = static_cast<int>(m);
  args.N = static_cast<int>(n);
  args.K = static_cast<int>(k);
  args.kblocks = static_cast<int>((k + kBK - 1) / kBK);
  args.epilogue = epilogue;
  args.status = device_status_ptr(dev);
  if (args.status == nullptr) return TM_ERR_CUDA;
  if (ul != nullptr) {
    args.ul_world = ul->world;
    args.ul_heads = ul->heads;
    args.ul_head_dim = ul->head_dim;
    args.ul_local = (ul->heads + ul->world - 1) / ul->world;
    if (ul->peer_recv != nullptr) {
      args.ul_peer = 1;
      args.ul_rank = ul->rank;
      args.ul_uses = static_cast<int>(ul->epoch);
      for (int j = 0; j < ul->world; ++j) {
        args.peer_part[j] = static_cast<__nv_bfloat16*>(ul->peer_recv[j]);
        args.peer_count[j] = static_cast<unsigned long long*>(ul->peer_flags[j]);
      }
    }
  }
  if (scatter != nullptr) {
    args.world = scatter->world;
    args.rank = scatter->rank;
    args.rows_per_owner = static_cast<int>(m / scatter->world);
    args.uses = scatter->epoch;
    args.red_bias = static_cast<const __nv_bfloat16*>(bias);
    args.red_out = static_cast<__nv_bfloat16*>(out);
    args.red_ldo = ldo;
    for (int j = 0; j < scatter->world; ++j) {
      args.peer_part[j] = static_cast<__nv_bfloat16*>(scatter->peer_part[j]);
      args.peer_count[j] = static_cast<unsigned long long*>(scatter->peer_flags[j]);
      if (scatter->peer_out != nullptr)
        args.peer_out[j] = static_cast<__nv_bfloat16*>(scatter->peer_out[j]);
    }
  }
  const int max_pairs = max_resident_pairs(dev, sms);
  const bool can_split =
      ws != nullptr && ws->ptr != nullptr && scatter == nullptr && !swiglu && ul == nullptr;
  Choice choice = pick_choice(args.M, args.N, args.kblocks, sms, max_pairs, can_split);
  if (force_cfg) choice = Choice{force_cfg, 1};
  // the exchange's generic-store epilogue and its counts run in the 256-wide
  // pair kernel
  if (args.ul_peer) choice = Choice{kPairFlag + 256, 1};
  if (can_split && ws->force_splits > 0) choice.splits = ws->force_splits;
  if (swiglu) {
    // the SwiGLU epilogue works in 64-column passes of each warp's half tile
    if (choice.cfg == 64) choice.cfg = 128;
    if (choice.cfg == kPairFlag + 192) choice.cfg = kPairFlag + 256;
    choice.splits = 1;
  }
  const int cfg = choice.cfg;
  if (cfg > kPairFlag && max_pairs <= 0) return TM_ERR_UNSUPPORTED;
  args.splits = 1;
  args.kb_per_split = args.kblocks;
  if (can_split && choice.splits > 1 && cfg < kPairFlag) {
    const SplitPlan plan = plan_split(cfg, choice.splits, args.M, args.N, args.kblocks);
    if (plan.splits > 1) {
      if (plan.bytes > ws->bytes) {
        if (ws->force_splits > 0) return TM_ERR_TOO_LARGE;  // forced split needs the space
      } else if (!aligned16(ws->ptr)) {
        return TM_ERR_ALIGNMENT;
      } else {
        args.splits = plan.splits;
        args.kb_per_split = plan.kb_per_split;
        args.tile_counters = static_cast<unsigned int*>(ws->ptr);
        args.ws = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws->ptr) + plan.counter_bytes);
      }
    }
  }
  const Operands op{a, lda, b, ldb};
  if (lora != nullptr) {
    if (max_pairs <= 0) return TM_ERR_UNSUPPORTED;
    args.splits = 1;
    args.kb_per_split = args.kblocks;
    if (out_dtype == TM_DTYPE_BF16)
      return launch_pair_lora<__nv_bfloat16>(op, args, *lora, max_pairs, stream);
    return launch_pair_lora<__half>(op, args, *lora, max_pairs, stream);
  }
  if (out_dtype == TM_DTYPE_BF16)
    return dispatch<__nv_bfloat16>(op, args, cfg, sms, max_pairs, stream);
  return dispatch<__half>(op, args, cfg, sms, max_pairs, stream);
}

}  // namespace

// Host checks of the LoRA operands shared by the LoRA entry points.
int check_lora(const void* lora_t, int64_t ldt, const void* lora_b, int64_t ldlb, int lora_rank,
               int64_t m) {
  if (lora_rank < 8 || lora_rank > 64 || lora_rank % 8 != 0) return TM_ERR_UNSUPPORTED;
  if (ldt < lora_rank || ldlb < lora_rank) return TM_ERR_SHAPE;
  if (ldt % 8 != 0 || ldlb % 8 != 0) return TM_ERR_ALIGNMENT;
  if (m > 0 && (lora_t == nullptr || lora_b == nullptr)) return TM_ERR_NULL_POINTER;
  if ((lora_t && !aligned16(lora_t)) || (lora_b && !aligned16(lora_b))) return TM_ERR_ALIGNMENT;
  return TM_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free split-K (tm_scaled_mm_i8_splitk_noalloc).
//
// Scratch for callers that must not allocate device memory: a fixed array in
// the library's own device image, present on every GPU that loads the
// library until the process exits.  Host code may not use the array's name as
// a pointer (on the host it is only a stand-in for the symbol); its device
// address is looked up once per device with cudaGetSymbolAddress while that
// device is current.
constexpr uint64_t kNoAllocScratchBytes = TM_SPLITK_NOALLOC_MAX_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of this device's scratch array (resolved on first use).
void* noalloc_scratch(int device) {
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_noalloc_ptr[device] = p;
  }
  return g_noalloc_ptr[device];
}

}  // namespace
}  // namespace tmw

extern "C" {

int tm_scaled_mm_i8_splitk_noalloc(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                                   const float* scale_a, int64_t scale_a_numel,
                                   const float* scale_b, int64_t scale_b_numel, const void* bias,
                                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                   int64_t ldo, uint32_t epilogue, int tile_n, int splits,
                                   void* stream) {
  if (tile_n != 256 && tile_n != 128 && tile_n != 64) return TM_ERR_UNSUPPORTED;
  if (splits < 1 || splits > 64) return TM_ERR_UNSUPPORTED;
  // every argument check runs before anything is enqueued on `stream`
  int rc = tmw::validate_scaled_mm(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b,
                                   scale_b_numel, bias, m, n, k, lda, ldb, ldo, epilogue, nullptr,
                                   nullptr, nullptr, nullptr);
  if (rc != TM_OK || m == 0) return rc;
  // the SwiGLU epilogue has no split-K form
  if (splits > 1 && (epilogue & TM_EPI_SWIGLU)) return TM_ERR_UNSUPPORTED;
  const int kblocks = static_cast<int>((k + tmw::kBK - 1) / tmw::kBK);
  const tmw::SplitPlan plan = tmw::plan_split(tile_n, splits, m, n, kblocks);
  // m * n fits 64 bits; bound it before trusting splits * m * n * 4
  const uint64_t mn = static_cast<uint64_t>(m) * static_cast<uint64_t>(n);
  if (plan.splits > 1 &&
      (mn > tmw::kNoAllocScratchBytes / 4 || plan.bytes > tmw::kNoAllocScratchBytes))
    return TM_ERR_TOO_LARGE;
  const int dev = tmw::current_device();
  void* scratch = tmw::noalloc_scratch(dev);
  if (scratch == nullptr) return TM_ERR_CUDA;
  // The array keeps the previous call's contents: the per-tile counters must
  // start at zero (the partial slices are fully rewritten by every call).
  if (plan.splits > 1 &&
      cudaMemsetAsync(scratch, 0, plan.counter_bytes, tmw::as_stream(stream)) != cudaSuccess)
    return TM_ERR_CUDA;
  const tmw::Workspace ws{scratch, tmw::kNoAllocScratchBytes, splits};
  rc = tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                           bias, m, n, k, lda, ldb, ldo, epilogue, nullptr, tile_n,
                           tmw::as_stream(stream), nullptr, &ws);
  return rc;
}


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

int tm_scaled_mm_i8_reduce_scatter(void* out, const int8_t* a, const int8_t* b,
                                   const float* scale_a, int64_t scale_a_numel,
                                   const float* scale_b, int64_t scale_b_numel, const void* bias,
                                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                   int64_t ldo, void* const* peer_part, void* const* peer_flags,
                                   int world, int rank, uint32_t epoch, int tile_n, void* stream) {
  const tmw::ScatterSpec spec{peer_part, peer_flags, world, rank, epoch};
  return tmw::scaled_mm_impl(out, TM_DTYPE_BF16, a, b, scale_a, scale_a_numel, scale_b,
                             scale_b_numel, bias, m, n, k, lda, ldb, ldo, 0u, nullptr, tile_n,
                             tmw::as_stream(stream), &spec);
}

int tm_scaled_mm_i8_all_reduce(const int8_t* a, const int8_t* b, const float* scale_a,
                               int64_t scale_a_numel, const float* scale_b, int64_t scale_b_numel,
                               const void* bias, int64_t m, int64_t n, int64_t k, int64_t lda,
                               int64_t ldb, void* const* peer_part, void* const* peer_flags,
                               void* const* peer_out, int world, int rank, uint32_t epoch,
                               int tile_n, void* stream) {
  if (peer_out == nullptr) return TM_ERR_NULL_POINTER;
  if (world < 1 || world > tmw::kMaxPeers) return TM_ERR_TOO_LARGE;
  if (rank < 0 || rank >= world) return TM_ERR_SHAPE;
  if (peer_out[rank] == nullptr) return TM_ERR_NULL_POINTER;
  const tmw::ScatterSpec spec{peer_part, peer_flags, world, rank, epoch, peer_out};
  // the owner's reduced rows land in its own output at their global offset
  void* own_rows = static_cast<__nv_bfloat16*>(peer_out[rank]) + rank * (m / world) * n;
  return tmw::scaled_mm_impl(own_rows, TM_DTYPE_BF16, a, b, scale_a, scale_a_numel, scale_b,
                             scale_b_numel, bias, m, n, k, lda, ldb, n, 0u, nullptr, tile_n,
                             tmw::as_stream(stream), &spec);
}

int tm_scaled_mm_i8_lora(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, const void* lora_t,
                         int64_t ldt, const void* lora_b, int64_t ldlb, int lora_rank, int64_t m,
                         int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldo,
                         uint32_t epilogue, void* stream) {
  const int rc = tmw::check_lora(lora_t, ldt, lora_b, ldlb, lora_rank, m);
  if (rc != TM_OK) return rc;
  const tmw::LoraSpec spec{lora_t, ldt, lora_b, ldlb, lora_rank};
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                             bias, m, n, k, lda, ldb, ldo, epilogue, nullptr, 0,
                             tmw::as_stream(stream), nullptr, nullptr, &spec);
}

int tm_scaled_mm_i8_lora_reduce_scatter(void* out, const int8_t* a, const int8_t* b,
                                        const float* scale_a, int64_t scale_a_numel,
                                        const float* scale_b, int64_t scale_b_numel,
                                        const void* bias, const void* lora_t, int64_t ldt,
                                        const void* lora_b, int64_t ldlb, int lora_rank,
                                        int64_t m, int64_t n, int64_t k, int64_t lda,
                                        int64_t ldb, int64_t ldo, void* const* peer_part,
                                        void* const* peer_flags, int world, int rank,
                                        uint32_t epoch, void* stream) {
  const int rc = tmw::check_lora(lora_t, ldt, lora_b, ldlb, lora_rank, m);
  if (rc != TM_OK) return rc;
  const tmw::LoraSpec lora{lora_t, ldt, lora_b, ldlb, lora_rank};
  const tmw::ScatterSpec spec{peer_part, peer_flags, world, rank, epoch};
  return tmw::scaled_mm_impl(out, TM_DTYPE_BF16, a, b, scale_a, scale_a_numel, scale_b,
                             scale_b_numel, bias, m, n, k, lda, ldb, ldo, 0u, nullptr, 0,
                             tmw::as_stream(stream), &spec, nullptr, &lora);
}

int tm_scaled_mm_i8_lora_all_reduce(const int8_t* a, const int8_t* b, const float* scale_a,
                                    int64_t scale_a_numel, const float* scale_b,
                                    int64_t scale_b_numel, const void* bias, const void* lora_t,
                                    int64_t ldt, const void* lora_b, int64_t ldlb, int lora_rank,
                                    int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                    void* const* peer_part, void* const* peer_flags,
                                    void* const* peer_out, int world, int rank, uint32_t epoch,
                                    void* stream) {
  const int rc = tmw::check_lora(lora_t, ldt, lora_b, ldlb, lora_rank, m);
  if (rc != TM_OK) return rc;
  if (peer_out == nullptr) return TM_ERR_NULL_POINTER;
  if (world < 1 || world > tmw::kMaxPeers) return TM_ERR_TOO_LARGE;
  if (rank < 0 || rank >= world) return TM_ERR_SHAPE;
  if (peer_out[rank] == nullptr) return TM_ERR_NULL_POINTER;
  const tmw::LoraSpec lora{lora_t, ldt, lora_b, ldlb, lora_rank};
  const tmw::ScatterSpec spec{peer_part, peer_flags, world, rank, epoch, peer_out};
  void* own_rows = static_cast<__nv_bfloat16*>(peer_out[rank]) + rank * (m / world) * n;
  return tmw::scaled_mm_impl(own_rows, TM_DTYPE_BF16, a, b, scale_a, scale_a_numel, scale_b,
                             scale_b_numel, bias, m, n, k, lda, ldb, n, 0u, nullptr, 0,
                             tmw::as_stream(stream), &spec, nullptr, &lora);
}

int tm_scaled_mm_i8_ulysses_send(void* send, int out_dtype, const int8_t* a, const int8_t* b,
                                 const float* scale_a, int64_t scale_a_numel,
                                 const float* scale_b, int64_t scale_b_numel, const void* bias,
                                 int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                 int num_heads, int head_dim, int world, void* stream) {
  const tmw::UlyssesSpec spec{num_heads, head_dim, world};
  const int rc = tmw::scaled_mm_impl(send, out_dtype, a, b, scale_a, scale_a_numel, scale_b,
                                     scale_b_numel, bias, m, n, k, lda, ldb, n, 0u, nullptr, 0,
                                     tmw::as_stream(stream), nullptr, nullptr, nullptr, &spec);
  if (rc != TM_OK || m == 0) return rc;
  // Zero-padded head shards (the reference pads num_heads up to a multiple of
  // world with zero heads, distributed/ulysses.py:188-193): the padded slots
  // h >= heads - w * local of each rank chunk w are never written by the
  // GEMM; clear them, stream-ordered with it.
  const int local = (num_heads + world - 1) / world;
  const size_t row_bytes = static_cast<size_t>(local) * head_dim * 2;
  for (int w = 0; w < world; ++w) {
    const int real = num_heads - w * local;  // real heads in chunk w (may be <= 0)
    const int first_pad = real < 0 ? 0 : (real > local ? local : real);
    if (first_pad == local) continue;
    for (int qkv = 0; qkv < 3; ++qkv) {
      uint8_t* base = static_cast<uint8_t*>(send) +
                      (static_cast<size_t>(w) * 3 + qkv) * static_cast<size_t>(m) * row_bytes +
                      static_cast<size_t>(first_pad) * head_dim * 2;
      if (cudaMemset2DAsync(base, row_bytes, 0, static_cast<size_t>(local - first_pad) * head_dim * 2,
                            static_cast<size_t>(m), tmw::as_stream(stream)) != cudaSuccess)
        return TM_ERR_CUDA;
    }
  }
  return TM_OK;
}

int tm_scaled_mm_i8_ulysses_exchange(const int8_t* a, const int8_t* b, const float* scale_a,
                                     int64_t scale_a_numel, const float* scale_b,
                                     int64_t scale_b_numel, const void* bias, int64_t m,
                                     int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                     int num_heads, int head_dim, void* const* peer_recv,
                                     void* const* peer_flags, int world, int rank,
                                     uint32_t epoch, void* stream) {
  if (peer_recv == nullptr || peer_flags == nullptr) return TM_ERR_NULL_POINTER;
  if (world < 1 || world > tmw::kMaxPeers) return TM_ERR_TOO_LARGE;
  if (rank < 0 || rank >= world) return TM_ERR_SHAPE;
  if (peer_recv[rank] == nullptr) return TM_ERR_NULL_POINTER;
  tmw::UlyssesSpec spec{num_heads, head_dim, world};
  spec.peer_recv = peer_recv;
  spec.peer_flags = peer_flags;
  spec.rank = rank;
  spec.epoch = epoch;
  // `out` only has to pass the pointer checks: every store goes to a receive
  // buffer through peer_recv
  return tmw::scaled_mm_impl(peer_recv[rank], TM_DTYPE_BF16, a, b, scale_a, scale_a_numel,
                             scale_b, scale_b_numel, bias, m, n, k, lda, ldb, n, 0u, nullptr, 0,
                             tmw::as_stream(stream), nullptr, nullptr, nullptr, &spec);
}

int tm_scaled_mm_i8_workspace_size(int64_t m, int64_t n, int64_t k, uint64_t* bytes) {
  if (bytes == nullptr) return TM_ERR_NULL_POINTER;
  *bytes = 0;
  if (m < 0 || n <= 0 || k <= 0) return TM_ERR_SHAPE;
  if (m == 0) return TM_OK;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  const int dev = tmw::current_device();
  const int sms = tmw::sm_count(dev);
  if (sms <= 0) return TM_ERR_CUDA;
  const int kblocks = static_cast<int>((k + tmw::kBK - 1) / tmw::kBK);
  const int max_pairs = tmw::max_resident_pairs(dev, sms);
  const tmw::Choice c = tmw::pick_choice(static_cast<int>(m), static_cast<int>(n), kblocks, sms,
                                         max_pairs, true);
  *bytes = tmw::plan_split(c.cfg, c.splits, m, n, kblocks).bytes;
  return TM_OK;
}

int tm_scaled_mm_i8_ws(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                       const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                       int64_t scale_b_numel, const void* bias, int64_t m, int64_t n, int64_t k,
                       int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                       int32_t* acc_debug, void* workspace, uint64_t workspace_bytes,
                       void* stream) {
  const tmw::Workspace ws{workspace, workspace_bytes, 0};
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                             bias, m, n, k, lda, ldb, ldo, epilogue, acc_debug, 0,
                             tmw::as_stream(stream), nullptr, &ws);
}

int tm_scaled_mm_i8_splitk(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                           const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                           int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                           int64_t k, int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                           int32_t* acc_debug, int tile_n, int splits, void* workspace,
                           uint64_t workspace_bytes, void* stream) {
  if (tile_n != 256 && tile_n != 128 && tile_n != 64) return TM_ERR_UNSUPPORTED;
  if (splits < 1 || splits > 64) return TM_ERR_UNSUPPORTED;
  if (workspace == nullptr) return TM_ERR_NULL_POINTER;
  const tmw::Workspace ws{workspace, workspace_bytes, splits};
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                             bias, m, n, k, lda, ldb, ldo, epilogue, acc_debug, tile_n,
                             tmw::as_stream(stream), nullptr, &ws);
}

int tm_scaled_mm_i8_splitk_workspace_size(int64_t m, int64_t n, int64_t k, int tile_n,
                                          int splits, uint64_t* bytes) {
  if (bytes == nullptr) return TM_ERR_NULL_POINTER;
  if (tile_n != 256 && tile_n != 128 && tile_n != 64) return TM_ERR_UNSUPPORTED;
  if (m <= 0 || n <= 0 || k <= 0) return TM_ERR_SHAPE;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  const int kblocks = static_cast<int>((k + tmw::kBK - 1) / tmw::kBK);
  *bytes = tmw::plan_split(tile_n, splits, m, n, kblocks).bytes;
  return TM_OK;
}

int tm_scaled_mm_i8_tile(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                         int32_t* acc_debug, int tile_n, void* stream) {
  switch (tile_n) {
    case 256:
    case 128:
    case 64:
    case tmw::kPairFlag + 256:
    case tmw::kPairFlag + 192:
    case tmw::kPairFlag + 128:
      break;
    default:
      return TM_ERR_UNSUPPORTED;
  }
  return tmw::scaled_mm_impl(out, out_dtype, a, b, scale_a, scale_a_numel, scale_b, scale_b_numel,
                             bias, m, n, k, lda, ldb, ldo, epilogue, acc_debug, tile_n,
                             tmw::as_stream(stream));
}

}  // extern "C"
