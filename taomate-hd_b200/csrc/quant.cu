// Row-wise int8 quantisation kernels (sm_100a).
//
//   * dynamic per-token symmetric quant   -> vLLM dynamic_scaled_int8_quant
//   * static per-tensor symmetric quant   -> vLLM static_scaled_int8_quant
//   * per-output-channel weight quant     -> w8a8.py:175-179
//   * adaLN modulate + quant              -> fused_kernels.py:220-236 feeding w8a8.py:71
//   * RMSNorm + modulate + quant          -> fused_kernels.py:322-347 feeding w8a8.py:71
//
// Design: a "row group" of TPR threads (32..256, a power of two) owns one
// row.  Each thread issues all of its 16-byte loads up front (VPT vectors,
// strided by TPR so each warp-wide load is one contiguous 512-byte span),
// keeps the values in registers, reduces |x| max with warp shuffles (plus a
// shared-memory step when the group spans several warps) and writes int8 +
// the fp32 scale: one HBM read of the activations, one write of int8.
// Rows whose width is not a multiple of the vector or whose base is not
// 16-byte aligned take a two-pass scalar kernel (one block per row).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.h"
#include "ptx.cuh"

namespace tmw {
namespace {

enum QuantMode : int {
  kDynamic = 0,    // per-row amax/127
  kStatic = 1,     // given per-tensor scale, q = x / s
  kWeight = 2,     // per-row amax/127 clamped at 1e-12, q = clamp(x / s, +-127)
  kModulate = 3,   // adaLN modulate, then dynamic
  kRmsModulate = 4,  // RMSNorm, adaLN modulate, then dynamic
  kResGateRmsModulate = 5,  // gated residual add, then as kRmsModulate
  kModulateRows = 6  // kModulate with one table row per row (no index): tables loaded with x
};

// adaLN modulate without RMSNorm (indexed or per-row tables)
__host__ __device__ constexpr bool modulate_only(int mode) {
  return mode == kModulate || mode == kModulateRows;
}

struct QuantParams {
  const void* x;
  int64_t ldx;
  int8_t* q;          // [rows, cols], row stride cols
  float* scales;      // [rows]
  const float* static_scale;
  __nv_bfloat16* hidden_out;  // optional [rows, cols] bf16 (modulate modes)
  const __nv_bfloat16* shift;
  const __nv_bfloat16* mod_scale;
  const int64_t* index;
  int64_t table_stride;
  const __nv_bfloat16* norm_w;
  float eps;
  double inv_cols;  // 1 / cols, correctly rounded (RMSNorm modes)
  // kResGateRmsModulate: x is the residual stream; branch [rows, cols] and
  // the gate table (row stride table_stride) update it, and the updated
  // residual is written to residual_out [rows, cols]
  const __nv_bfloat16* branch;
  const __nv_bfloat16* gate;
  __nv_bfloat16* residual_out;
  int64_t rows;
  int64_t cols;
  int tpr_log2;
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

// Round-to-nearest-even through bf16 and back (identical to the reference's
// _round_bf16 for finite values, fused_kernels.py:57-61).
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Saturating round-half-even float -> int8 (NaN -> 0).
__device__ __forceinline__ int f2i8_rn_sat(float x) {
  int r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// The same value as f2i8_rn_sat for x in [-127.5, 127.5] or NaN, on the FP32
// pipe: NaN becomes 0, then adding 1.5 * 2^23 makes the addition's
// round-to-nearest-even leave round(x) in the low mantissa bits; the low byte
// of the result is the two's-complement int8 (the bits of 1.5 * 2^23 are
// 0x4B400000).
__device__ __forceinline__ uint32_t f2i8_rn_fast(float x) {
  return __float_as_uint(__fadd_rn(x == x ? x : 0.0f, 12582912.0f));
}

// Pack the low bytes of four words into one.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t b0, uint32_t b1, uint32_t b2,
                                                   uint32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

template <typename T>
struct VecTraits {
  static constexpr int kElems = 16 / sizeof(T);
};

// Unpack one 16-byte vector into floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float (&out)[VecTraits<T>::kElems]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < VecTraits<T>::kElems; ++j) out[j] = to_f32<T>(e[j]);
}

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Read-only 16-byte load the compiler may schedule freely (not volatile):
// the adaLN tables and the gated branch are never written by the kernel, so
// an unrolled loop's loads can all be issued ahead of its stores instead of
// one L2 round trip per iteration.
__device__ __forceinline__ uint4 ld_nc16(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_cached16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Max / sum over the TPR threads of a row group.  Groups of <= 32 threads
// live inside one warp; wider groups combine per-warp partials through
// shared memory (every thread of the block reaches the __syncthreads).
template <bool kMax>
__device__ __forceinline__ float group_reduce(float v, int tpr, float* red) {
  const int lane_span = tpr < 32 ? tpr : 32;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (off < lane_span) {
      const float o = __shfl_xor_sync(0xffffffffu, v, off);
      v = kMax ? fmaxf(v, o) : v + o;
    }
  }
  if (tpr > 32) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    __syncthreads();  // protect `red` from the previous use
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int wpr = tpr >> 5;
    const int first = (warp / wpr) * wpr;
    float acc = red[first];
    for (int w = 1; w < wpr; ++w) acc = kMax ? fmaxf(acc, red[first + w]) : acc + red[first + w];
    v = acc;
  }
  return v;
}

// Sum of one double per thread over the row group (the RMSNorm sum of
// squares).  `red` must hold 8 doubles.
__device__ __forceinline__ double group_sum_f64(double v, int tpr, double* red) {
  const int lane_span = tpr < 32 ? tpr : 32;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (off < lane_span) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  }
  if (tpr > 32) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    __syncthreads();  // protect `red` from the previous use
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int wpr = tpr >> 5;
    const int first = (warp / wpr) * wpr;
    double acc = red[first];
    for (int w = 1; w < wpr; ++w) acc = __dadd_rn(acc, red[first + w]);
    v = acc;
  }
  return v;
}

// Quantise a thread's VPT vectors of E values and store them.  kFast: the
// FP32-pipe rounding (dynamic modes, rows where it equals the conversion);
// chosen per row outside the loop so each path is straight-line code.
template <int MODE, bool kFast, int VPT, int E>
__device__ __forceinline__ void store_q(const float (&v)[VPT][E], int8_t* qr, int t, int tpr,
                                        int64_t nvec, float inv, float static_s) {
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = t + static_cast<int64_t>(i) * tpr;
    if (vi < nvec) {
      uint32_t packed[E / 4];
#pragma unroll
      for (int w = 0; w < E / 4; ++w) {
        uint32_t bytes[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const float xv = v[i][4 * w + b];
          if constexpr (MODE == kStatic) {
            bytes[b] = static_cast<uint32_t>(f2i8_rn_sat(__fdiv_rn(xv, static_s)));
          } else if constexpr (MODE == kWeight) {
            const int qi = f2i8_rn_sat(__fdiv_rn(xv, inv));
            bytes[b] = static_cast<uint32_t>(qi < -127 ? -127 : qi);
          } else if constexpr (kFast) {
            bytes[b] = f2i8_rn_fast(__fmul_rn(xv, inv));
          } else {
            bytes[b] = static_cast<uint32_t>(f2i8_rn_sat(__fmul_rn(xv, inv)));
          }
        }
        packed[w] = pack_low_bytes(bytes[0], bytes[1], bytes[2], bytes[3]);
      }
      if constexpr (E == 8) {
        *reinterpret_cast<uint2*>(qr + vi * E) = make_uint2(packed[0], packed[1]);
      } else {
        *reinterpret_cast<uint32_t*>(qr + vi * E) = packed[0];
      }
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// Correctly rounded fp32 square root and reciprocal without the library's
// division / square-root subroutines (whose slow-path calls make the caller
// save its live registers: the producers hold a whole row in registers).
// Method: a hardware approximation (rsqrt.approx / rcp.approx, about 2^-22
// relative), one Newton-Raphson step in fp64, rounding to fp32, then an exact
// rounding test against the two neighbouring midpoints (Tuckerman's test):
// a midpoint has at most 25 significant bits, so its square or its product
// with a 24-bit value is exact in fp64 and the comparisons decide the
// rounding exactly.  Exact midpoint ties cannot occur for either operation.
__device__ __forceinline__ float f32_next_up(float v) {
  return __uint_as_float(__float_as_uint(v) + 1u);  // v positive and finite
}
__device__ __forceinline__ float f32_next_down(float v) {
  return __uint_as_float(__float_as_uint(v) - 1u);  // v positive
}

// fp32(sqrt(v)) for v positive, finite and normal.
__device__ __forceinline__ float sqrt_rn_normal(float v) {
  float y0;
  asm("rsqrt.approx.f32 %0, %1;" : "=f"(y0) : "f"(v));
  const double vd = static_cast<double>(v);
  double y = static_cast<double>(y0);
  // y <- y (3 - v y^2) / 2: Newton-Raphson for 1 / sqrt(v)
  y = __dmul_rn(y, __fma_rn(-0.5 * vd, __dmul_rn(y, y), 1.5));
  float s = __double2float_rn(__dmul_rn(vd, y));
  const double hi = 0.5 * (static_cast<double>(s) + static_cast<double>(f32_next_up(s)));
  const double lo = 0.5 * (static_cast<double>(s) + static_cast<double>(f32_next_down(s)));
  if (vd >= __dmul_rn(hi, hi)) {
    s = f32_next_up(s);
  } else if (vd < __dmul_rn(lo, lo)) {
    s = f32_next_down(s);
  }
  return s;
}

// fp32(1 / fp32(sqrt(v))), IEEE semantics for v >= 0 (and NaN).
__device__ __forceinline__ float rsqrt_two_step_rn(float v) {
  if (!(v > 0.0f)) return v == 0.0f ? __int_as_float(0x7f800000) : v;  // +inf / NaN
  if (v == __int_as_float(0x7f800000)) return 0.0f;
  float s;
  if (v < 1.17549435e-38f) {  // subnormal: sqrt(v * 2^32) = sqrt(v) * 2^16, exactly
    s = __fmul_rn(sqrt_rn_normal(__fmul_rn(v, 4294967296.0f)), 1.52587890625e-05f);
  } else {
    s = sqrt_rn_normal(v);
  }
  // s is normal here (s >= sqrt of the smallest subnormal), and so is 1 / s
  float r0;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r0) : "f"(s));
  const double sd = static_cast<double>(s);
  double r = static_cast<double>(r0);
  r = __fma_rn(r, __fma_rn(-sd, r, 1.0), r);  // r <- r (2 - s r)
  float q = __double2float_rn(r);
  const double hi = 0.5 * (static_cast<double>(q) + static_cast<double>(f32_next_up(q)));
  const double lo = 0.5 * (static_cast<double>(q) + static_cast<double>(f32_next_down(q)));
  if (__dmul_rn(sd, hi) <= 1.0) {  // 1 / s >= hi
    q = f32_next_up(q);
  } else if (__dmul_rn(sd, lo) > 1.0) {  // 1 / s < lo
    q = f32_next_down(q);
  }
  return q;
}

// adaLN producers on a row held as packed bf16 (8 values per uint4; every
// intermediate below is rounded to bf16, so the packed form loses nothing):
//   kResGateRmsModulate: x = bf16(x + bf16(gate[t] * branch)) -> residual_out
//   kRmsModulate (and the above): x = bf16(x * rsqrt(mean(x^2) + eps) * w)
//   all three:          h = bf16(bf16(x * bf16(1 + scale[t])) + shift[t])
// h replaces the row in `raw` (and goes to hidden_out when requested); the
// caller quantises it as a plain bf16 row.  Table loads are plain read-only
// loads the compiler can issue ahead of the stores.
template <int VPT, int MODE>
__device__ __forceinline__ void adaln_rows(const QuantParams& p, uint4 (&raw)[VPT],
                                           const uint4 (&pre_sc)[VPT],
                                           const uint4 (&pre_sh)[VPT], int64_t row,
                                           int t, int tpr, int64_t nvec, bool active,
                                           double* red) {
  constexpr int E = 8;
  const int64_t trow = active ? (p.index ? p.index[row] : row) : 0;
  if constexpr (MODE == kResGateRmsModulate) {
    const __nv_bfloat16* gate_row = p.gate + trow * p.table_stride;
    const __nv_bfloat16* branch_row = p.branch + row * p.cols;
    uint4 gr[VPT], br[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t vi = t + static_cast<int64_t>(i) * tpr;
      if (active && vi < nvec) {
        gr[i] = ld_cached16(gate_row + vi * E);
        br[i] = ld_nc16(branch_row + vi * E);
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t vi = t + static_cast<int64_t>(i) * tpr;
      if (active && vi < nvec) {
        uint32_t* xw = reinterpret_cast<uint32_t*>(&raw[i]);
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gr[i]);
        const uint32_t* bw = reinterpret_cast<const uint32_t*>(&br[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = unpack_bf16x2(xw[j]), g = unpack_bf16x2(gw[j]),
                       b = unpack_bf16x2(bw[j]);
          xw[j] = pack_bf16x2(round_bf16(__fadd_rn(x.x, round_bf16(__fmul_rn(g.x, b.x)))),
                              round_bf16(__fadd_rn(x.y, round_bf16(__fmul_rn(g.y, b.y)))));
        }
        *reinterpret_cast<uint4*>(p.residual_out + row * p.cols + vi * E) = raw[i];
      }
    }
  }
  float rinv = 0.f;
  if constexpr (MODE == kRmsModulate || MODE == kResGateRmsModulate) {
    // rinv = fp32(1 / fp32(sqrt(fp32(mean(x^2)) + eps))) with every step
    // correctly rounded, as the reference kernel's arithmetic is restated by
    // its oracle (a float64 mean, then IEEE fp32 add, sqrt and division; no
    // approximate rsqrt).  The square of a bf16 value is exact in fp32; each
    // thread sums its squares in four compensated fp32 chains (TwoSum: the
    // rounding error of every add is kept in a second word), so s + c carries
    // the sum to about 2^-40 relative; the pairs are then added in fp64.
    float cs[4] = {0.f, 0.f, 0.f, 0.f}, cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack_bf16x2(xw[j]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = e ? x.y : x.x;
          const float sq = __fmul_rn(v, v);
          const float t = __fadd_rn(cs[j], sq);
          const float z = __fsub_rn(t, cs[j]);
          cc[j] = __fadd_rn(cc[j], __fadd_rn(__fsub_rn(cs[j], __fsub_rn(t, z)), __fsub_rn(sq, z)));
          cs[j] = t;
        }
      }
    }
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      ss = __dadd_rn(ss, __dadd_rn(static_cast<double>(cs[j]), static_cast<double>(cc[j])));
    ss = group_sum_f64(ss, tpr, red);
    const float variance = __double2float_rn(__dmul_rn(ss, p.inv_cols));
    rinv = rsqrt_two_step_rn(__fadd_rn(variance, p.eps));
  }
  const __nv_bfloat16* sc_row = p.mod_scale + trow * p.table_stride;
  const __nv_bfloat16* sh_row = p.shift + trow * p.table_stride;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = t + static_cast<int64_t>(i) * tpr;
    if (active && vi < nvec) {
      uint4 wr = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (!modulate_only(MODE)) wr = ld_cached16(p.norm_w + vi * E);
      // per-row tables were loaded together with x
      const uint4 scr = MODE == kModulateRows ? pre_sc[i] : ld_cached16(sc_row + vi * E);
      const uint4 shr = MODE == kModulateRows ? pre_sh[i] : ld_cached16(sh_row + vi * E);
      uint32_t* xw = reinterpret_cast<uint32_t*>(&raw[i]);
      const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wr);
      const uint32_t* cw = reinterpret_cast<const uint32_t*>(&scr);
      const uint32_t* hw = reinterpret_cast<const uint32_t*>(&shr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 x = unpack_bf16x2(xw[j]);
        if constexpr (!modulate_only(MODE)) {
          const float2 w = unpack_bf16x2(ww[j]);
          x.x = round_bf16(__fmul_rn(__fmul_rn(x.x, rinv), w.x));
          x.y = round_bf16(__fmul_rn(__fmul_rn(x.y, rinv), w.y));
        }
        const float2 c = unpack_bf16x2(cw[j]), sh = unpack_bf16x2(hw[j]);
        const float m0 = round_bf16(__fmul_rn(x.x, round_bf16(__fadd_rn(1.0f, c.x))));
        const float m1 = round_bf16(__fmul_rn(x.y, round_bf16(__fadd_rn(1.0f, c.y))));
        xw[j] = pack_bf16x2(__fadd_rn(m0, sh.x), __fadd_rn(m1, sh.y));
      }
      if (p.hidden_out != nullptr)
        *reinterpret_cast<uint4*>(p.hidden_out + row * p.cols + vi * E) = raw[i];
    }
  }
}

// The RMSNorm adaLN modes with one warp per row (VPT >= 8) keep two blocks
// resident: 16 independent rows per SM, the registers capped at 128.
template <int MODE, int VPT>
constexpr int quant_min_blocks() {
  return (MODE == kRmsModulate || MODE == kResGateRmsModulate) && VPT >= 8 ? 2 : 1;
}

template <typename T, int VPT, int MODE>
__global__ void __launch_bounds__(256, (quant_min_blocks<MODE, VPT>())) quant_rows_kernel(
    const QuantParams p) {
  constexpr int E = VecTraits<T>::kElems;
  griddep_wait();  // the rows may come from the previous kernel on the stream
  griddep_launch_dependents();
  __shared__ double red_f64[8];  // the RMSNorm sum; also 8 floats for the maxima
  float* red = reinterpret_cast<float*>(red_f64);
  const int tpr = 1 << p.tpr_log2;
  const int local_row = threadIdx.x >> p.tpr_log2;
  const int t = threadIdx.x & (tpr - 1);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> p.tpr_log2) + local_row;
  const bool active = row < p.rows;
  const int64_t nvec = p.cols / E;
  const T* xr = reinterpret_cast<const T*>(p.x) + (active ? row : 0) * p.ldx;

  constexpr bool kAdaLN = modulate_only(MODE) || MODE == kRmsModulate ||
                          MODE == kResGateRmsModulate;
  static_assert(!kAdaLN || std::is_same<T, __nv_bfloat16>::value, "adaLN modes are bf16");
  if constexpr ((MODE == kDynamic || kAdaLN) && std::is_same<T, __nv_bfloat16>::value) {
    // Plain dynamic quant of bf16: the row maximum from packed bf16 pairs
    // (|x| and max are exact in bf16, and equal the fp32 maximum of the
    // converted values; NaN elements are left out as by fmaxf), a second
    // NaN-propagating packed maximum flags rows with NaN, and only the
    // multiply-and-round runs per element in fp32.  Rows with NaN, inf or a
    // subnormal maximum take the conversion instruction.
    // adaLN modes first turn the row into the modulated bf16 row h.
    uint4 raw[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t vi = t + static_cast<int64_t>(i) * tpr;
      raw[i] = (active && vi < nvec) ? ld_stream16(xr + vi * E) : make_uint4(0u, 0u, 0u, 0u);
    }
    // Modulate with per-row tables (the per-token adaLN of the BASELINE
    // configuration): the row's shift / scale rows come from HBM like x, so
    // they are loaded in the same burst and a row costs one memory round
    // trip instead of two (768p, 20480 x 3072: 121 -> 107 us).  Indexed
    // tables stay cache-resident and keep the lighter register set (loading
    // them early measured 74 -> 86 us); the RMSNorm modes need the row's
    // reduction first.
    uint4 pre_sc[VPT], pre_sh[VPT];
    if constexpr (MODE == kModulateRows) {
      const int64_t trow = active ? row : 0;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t vi = t + static_cast<int64_t>(i) * tpr;
        const bool in = active && vi < nvec;
        pre_sc[i] = in ? ld_cached16(p.mod_scale + trow * p.table_stride + vi * E)
                       : make_uint4(0u, 0u, 0u, 0u);
        pre_sh[i] = in ? ld_cached16(p.shift + trow * p.table_stride + vi * E)
                       : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if constexpr (kAdaLN)
      adaln_rows<VPT, MODE>(p, raw, pre_sc, pre_sh, row, t, tpr, nvec, active, red_f64);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f), n2 = m2;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 a = __habs2(h[j]);
        m2 = __hmax2(m2, a);
        n2 = __hmax2_nan(n2, a);
      }
    }
    float amax = fmaxf(__bfloat162float(m2.x), __bfloat162float(m2.y));
    float has_nan = (__hisnan(n2.x) || __hisnan(n2.y)) ? 1.0f : 0.0f;
    amax = group_reduce<true>(amax, tpr, red);
    has_nan = group_reduce<true>(has_nan, tpr, red);
    if (!active) return;
    if (t == 0) p.scales[row] = __fdiv_rn(amax, 127.0f);
    const float inv = amax == 0.f ? 0.f : __fdiv_rn(127.0f, amax);
    const bool fast = has_nan == 0.0f && isfinite(amax) && isfinite(inv);
    int8_t* qr = p.q + row * p.cols;
    // one straight-line store loop per rounding path, chosen once per row
    const auto store_row = [&](auto fast_tag) {
      constexpr bool kFast = decltype(fast_tag)::value;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t vi = t + static_cast<int64_t>(i) * tpr;
        if (vi < nvec) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
          uint32_t bytes[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            const float y0 = __fmul_rn(f.x, inv), y1 = __fmul_rn(f.y, inv);
            if constexpr (kFast) {  // no NaN / inf here: |y| rounds into [-127, 127]
              bytes[2 * j] = __float_as_uint(__fadd_rn(y0, 12582912.0f));
              bytes[2 * j + 1] = __float_as_uint(__fadd_rn(y1, 12582912.0f));
            } else {
              bytes[2 * j] = static_cast<uint32_t>(f2i8_rn_sat(y0));
              bytes[2 * j + 1] = static_cast<uint32_t>(f2i8_rn_sat(y1));
            }
          }
          *reinterpret_cast<uint2*>(qr + vi * E) =
              make_uint2(pack_low_bytes(bytes[0], bytes[1], bytes[2], bytes[3]),
                         pack_low_bytes(bytes[4], bytes[5], bytes[6], bytes[7]));
        }
      }
    };
    if (fast)
      store_row(std::true_type{});
    else
      store_row(std::false_type{});
    return;
  }

  float v[VPT][E];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = t + static_cast<int64_t>(i) * tpr;
    if (active && vi < nvec) {
      unpack16<T>(ld_stream16(xr + vi * E), v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[i][j] = 0.f;
    }
  }

  float inv;
  // dynamic modes: with a finite row maximum (NaN elements do not enter it)
  // and a finite 127 / amax every x * inv of a finite x rounds into
  // [-127, 127] (|x| <= amax), and NaN elements give NaN, so the FP32-pipe
  // rounding gives the conversion's result; other rows (an infinite element,
  // or a subnormal maximum) keep the conversion instruction
  bool fast = false;
  if constexpr (MODE == kStatic) {
    inv = 0.f;  // unused: static mode divides by the given scale
  } else {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < E; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    amax = group_reduce<true>(amax, tpr, red);
    if constexpr (MODE == kWeight) {
      const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
      if (active && t == 0) p.scales[row] = s;
      inv = s;  // weight mode divides by the clamped scale
    } else {
      if (active && t == 0) p.scales[row] = __fdiv_rn(amax, 127.0f);
      inv = amax == 0.f ? 0.f : __fdiv_rn(127.0f, amax);
      fast = isfinite(amax) && isfinite(inv);
    }
  }
  const float static_s = MODE == kStatic ? *p.static_scale : 0.f;

  if (!active) return;
  int8_t* qr = p.q + row * p.cols;
  if constexpr (MODE == kStatic || MODE == kWeight) {
    store_q<MODE, false>(v, qr, t, tpr, nvec, inv, static_s);
  } else if (fast) {
    store_q<MODE, true>(v, qr, t, tpr, nvec, inv, static_s);
  } else {
    store_q<MODE, false>(v, qr, t, tpr, nvec, inv, static_s);
  }
}

// Two-pass scalar fallback: any width, any alignment.  One block per row.
template <typename T, int MODE>
__global__ void __launch_bounds__(256) quant_rows_scalar_kernel(const QuantParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  if (row >= p.rows) return;
  const T* xr = reinterpret_cast<const T*>(p.x) + row * p.ldx;
  float inv = 0.f;
  float s_use = 0.f;
  if constexpr (MODE == kStatic) {
    s_use = *p.static_scale;
  } else {
    float amax = 0.f;
    for (int64_t c = threadIdx.x; c < p.cols; c += blockDim.x) amax = fmaxf(amax, fabsf(to_f32<T>(xr[c])));
    amax = group_reduce<true>(amax, 256, red);
    if constexpr (MODE == kWeight) {
      s_use = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
      if (threadIdx.x == 0) p.scales[row] = s_use;
    } else {
      if (threadIdx.x == 0) p.scales[row] = __fdiv_rn(amax, 127.0f);
      inv = amax == 0.f ? 0.f : __fdiv_rn(127.0f, amax);
    }
  }
  int8_t* qr = p.q + row * p.cols;
  for (int64_t c = threadIdx.x; c < p.cols; c += blockDim.x) {
    const float xv = to_f32<T>(xr[c]);
    int qi;
    if constexpr (MODE == kStatic) {
      qi = f2i8_rn_sat(__fdiv_rn(xv, s_use));
    } else if constexpr (MODE == kWeight) {
      qi = f2i8_rn_sat(__fdiv_rn(xv, s_use));
      qi = qi < -127 ? -127 : qi;
    } else {
      qi = f2i8_rn_sat(__fmul_rn(xv, inv));
    }
    qr[c] = static_cast<int8_t>(qi);
  }
}

// ------------------------------------------------------------------ host
constexpr int kMaxVpt = 16;

// Pick threads-per-row (power of two, 32..256) and vectors-per-thread.
bool pick_layout(int64_t nvec, int* tpr_log2, int* vpt) {
  for (int l = 5; l <= 8; ++l) {
    const int64_t v = (nvec + (1 << l) - 1) >> l;
    if (v <= 8 || (l == 8 && v <= kMaxVpt)) {
      *tpr_log2 = l;
      *vpt = static_cast<int>(v);
      return true;
    }
  }
  return false;
}

// Round vpt up to an instantiated value.
int round_vpt(int v) {
  static const int kSet[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int s : kSet)
    if (v <= s) return s;
  return -1;
}

template <typename T, int MODE>
int launch_vec(const QuantParams& base, int tpr_log2, int vpt, cudaStream_t stream) {
  QuantParams p = base;
  p.tpr_log2 = tpr_log2;
  const int rpb = 256 >> tpr_log2;
  const int64_t grid = (p.rows + rpb - 1) / rpb;
  if (grid > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaError_t err;
  switch (round_vpt(vpt)) {
    case 1: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 1, MODE>, p); break;
    case 2: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 2, MODE>, p); break;
    case 3: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 3, MODE>, p); break;
    case 4: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 4, MODE>, p); break;
    case 6: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 6, MODE>, p); break;
    case 8: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 8, MODE>, p); break;
    case 12: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 12, MODE>, p); break;
    case 16: err = launch_with_pdl(cfg, nullptr, 0, quant_rows_kernel<T, 16, MODE>, p); break;
    default: return TM_ERR_UNSUPPORTED;
  }
  return err == cudaSuccess ? check_launch() : TM_ERR_CUDA;
}

template <typename T, int MODE>
int launch_quant_typed(const QuantParams& p, cudaStream_t stream) {
  constexpr int E = VecTraits<T>::kElems;
  int tpr_log2 = 0, vpt = 0;
  const bool vec_ok = (p.cols % E == 0) && (p.ldx % E == 0) && aligned16(p.x) &&
                      aligned16(p.q) && pick_layout(p.cols / E, &tpr_log2, &vpt);
  if (vec_ok) return launch_vec<T, MODE>(p, tpr_log2, vpt, stream);
  if (p.rows > 0x7fffffffLL) return TM_ERR_TOO_LARGE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  if (launch_with_pdl(cfg, nullptr, 0, quant_rows_scalar_kernel<T, MODE>, p) != cudaSuccess)
    return TM_ERR_CUDA;
  return check_launch();
}

template <int MODE>
int launch_quant(const QuantParams& p, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case TM_DTYPE_BF16: return launch_quant_typed<__nv_bfloat16, MODE>(p, stream);
    case TM_DTYPE_FP16: return launch_quant_typed<__half, MODE>(p, stream);
    case TM_DTYPE_FP32: return launch_quant_typed<float, MODE>(p, stream);
    default: return TM_ERR_DTYPE;
  }
}

int check_rows_cols(int64_t rows, int64_t cols, int64_t ld) {
  if (rows < 0 || cols <= 0) return TM_ERR_SHAPE;
  if (ld < cols) return TM_ERR_SHAPE;
  return TM_OK;
}

template <int MODE>
int launch_modulate(QuantParams p, cudaStream_t stream) {
  // Modulate modes need the vector layout (bf16, width % 8, aligned rows).
  if (p.cols % 8 != 0 || p.table_stride % 8 != 0 || !aligned16(p.x) || !aligned16(p.q) ||
      !aligned16(p.shift) || !aligned16(p.mod_scale) ||
      (p.hidden_out != nullptr && !aligned16(p.hidden_out)) ||
      (!modulate_only(MODE) && !aligned16(p.norm_w)) ||
      (MODE == kResGateRmsModulate &&
       (!aligned16(p.branch) || !aligned16(p.gate) || !aligned16(p.residual_out))))
    return TM_ERR_ALIGNMENT;
  // RMSNorm modes: one warp per row where it fits in 12 vectors per thread
  // (widths up to 3072): the row's two reductions are warp shuffles, with no
  // block-wide barrier tying the block's rows together, so each row's
  // load / reduce / load chain overlaps the others' (768p, 20480 x 3072:
  // 102 -> 95 us with RMSNorm, 191 -> 156 us with the gated residual).  The
  // modulate-only mode, with a single reduction, is faster on the shared
  // layout (59 against 65 us).
  int tpr_log2 = 0, vpt = 0;
  const int64_t nvec = p.cols / 8;
  if (!modulate_only(MODE) && nvec <= 32 * 12) {
    tpr_log2 = 5;
    vpt = static_cast<int>((nvec + 31) / 32);
  } else if (!pick_layout(nvec, &tpr_log2, &vpt)) {
    return TM_ERR_TOO_LARGE;
  }
  return launch_vec<__nv_bfloat16, MODE>(p, tpr_log2, vpt, stream);
}

}  // namespace
}  // namespace tmw

extern "C" {

int tm_dynamic_scaled_int8_quant(int8_t* out, const void* input, int input_dtype, float* scales,
                                 int32_t* azp, int64_t rows, int64_t cols,
                                 int64_t input_row_stride, void* stream) {
  if (azp != nullptr) return TM_ERR_UNSUPPORTED;
  if (int s = tmw::check_rows_cols(rows, cols, input_row_stride)) return s;
  if (rows == 0) return TM_OK;
  if (!out || !input || !scales) return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = input;
  p.ldx = input_row_stride;
  p.q = out;
  p.scales = scales;
  p.rows = rows;
  p.cols = cols;
  return tmw::launch_quant<tmw::kDynamic>(p, input_dtype, tmw::as_stream(stream));
}

int tm_static_scaled_int8_quant(int8_t* out, const void* input, int input_dtype,
                                const float* scale, int32_t* azp, int64_t rows, int64_t cols,
                                int64_t input_row_stride, void* stream) {
  if (azp != nullptr) return TM_ERR_UNSUPPORTED;
  if (int s = tmw::check_rows_cols(rows, cols, input_row_stride)) return s;
  if (rows == 0) return TM_OK;
  if (!out || !input || !scale) return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = input;
  p.ldx = input_row_stride;
  p.q = out;
  p.static_scale = scale;
  p.rows = rows;
  p.cols = cols;
  return tmw::launch_quant<tmw::kStatic>(p, input_dtype, tmw::as_stream(stream));
}

int tm_quantize_weight_int8(int8_t* q, float* scales, const void* w, int w_dtype, int64_t n,
                            int64_t k, void* stream) {
  if (int s = tmw::check_rows_cols(n, k, k)) return s;
  if (n == 0) return TM_OK;
  if (!q || !scales || !w) return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = w;
  p.ldx = k;
  p.q = q;
  p.scales = scales;
  p.rows = n;
  p.cols = k;
  return tmw::launch_quant<tmw::kWeight>(p, w_dtype, tmw::as_stream(stream));
}

int tm_modulate_int8_quant(int8_t* out, float* scales, void* hidden_out, const void* x,
                           const void* shift, const void* scale, const int64_t* index,
                           int64_t table_stride, int64_t rows, int64_t cols, void* stream) {
  if (int s = tmw::check_rows_cols(rows, cols, cols)) return s;
  if (table_stride < cols) return TM_ERR_SHAPE;
  if (rows == 0) return TM_OK;
  if (!out || !scales || !x || !shift || !scale) return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = x;
  p.ldx = cols;
  p.q = out;
  p.scales = scales;
  p.hidden_out = static_cast<__nv_bfloat16*>(hidden_out);
  p.shift = static_cast<const __nv_bfloat16*>(shift);
  p.mod_scale = static_cast<const __nv_bfloat16*>(scale);
  p.index = index;
  p.table_stride = table_stride;
  p.rows = rows;
  p.cols = cols;
  return index == nullptr ? tmw::launch_modulate<tmw::kModulateRows>(p, tmw::as_stream(stream))
                          : tmw::launch_modulate<tmw::kModulate>(p, tmw::as_stream(stream));
}

int tm_rms_norm_modulate_int8_quant(int8_t* out, float* scales, void* hidden_out,
                                    const void* x, const void* norm_weight, float eps,
                                    const void* shift, const void* scale, const int64_t* index,
                                    int64_t table_stride, int64_t rows, int64_t cols,
                                    void* stream) {
  if (int s = tmw::check_rows_cols(rows, cols, cols)) return s;
  if (table_stride < cols) return TM_ERR_SHAPE;
  if (rows == 0) return TM_OK;
  if (!out || !scales || !x || !norm_weight || !shift || !scale) return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = x;
  p.ldx = cols;
  p.q = out;
  p.scales = scales;
  p.hidden_out = static_cast<__nv_bfloat16*>(hidden_out);
  p.shift = static_cast<const __nv_bfloat16*>(shift);
  p.mod_scale = static_cast<const __nv_bfloat16*>(scale);
  p.index = index;
  p.table_stride = table_stride;
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  p.eps = eps;
  p.inv_cols = 1.0 / static_cast<double>(cols);
  p.rows = rows;
  p.cols = cols;
  return tmw::launch_modulate<tmw::kRmsModulate>(p, tmw::as_stream(stream));
}

int tm_residual_gate_rms_norm_modulate_int8_quant(
    int8_t* out, float* scales, void* residual_out, void* hidden_out, const void* residual,
    const void* branch, const void* gate, const void* norm_weight, float eps, const void* shift,
    const void* scale, const int64_t* index, int64_t table_stride, int64_t rows, int64_t cols,
    void* stream) {
  if (int s = tmw::check_rows_cols(rows, cols, cols)) return s;
  if (table_stride < cols) return TM_ERR_SHAPE;
  if (rows == 0) return TM_OK;
  if (!out || !scales || !residual_out || !residual || !branch || !gate || !norm_weight ||
      !shift || !scale)
    return TM_ERR_NULL_POINTER;
  tmw::QuantParams p{};
  p.x = residual;
  p.ldx = cols;
  p.q = out;
  p.scales = scales;
  p.hidden_out = static_cast<__nv_bfloat16*>(hidden_out);
  p.shift = static_cast<const __nv_bfloat16*>(shift);
  p.mod_scale = static_cast<const __nv_bfloat16*>(scale);
  p.index = index;
  p.table_stride = table_stride;
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  p.eps = eps;
  p.inv_cols = 1.0 / static_cast<double>(cols);
  p.branch = static_cast<const __nv_bfloat16*>(branch);
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.residual_out = static_cast<__nv_bfloat16*>(residual_out);
  p.rows = rows;
  p.cols = cols;
  return tmw::launch_modulate<tmw::kResGateRmsModulate>(p, tmw::as_stream(stream));
}

}  // extern "C"
