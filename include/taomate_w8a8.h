/*
 * taomate_w8a8.h -- C ABI of the B200 (sm_100a) selective-W8A8 linear path.
 *
 * Plain pointers, sizes and a CUDA stream passed as `void*` (a cudaStream_t;
 * NULL means the legacy default stream).  All pointers are device pointers
 * unless stated otherwise.  Nothing here allocates device memory, retains a
 * pointer after returning, or synchronises the stream.  Every function
 * returns a tm_status code; argument errors are detected on the host before
 * any launch.  Wait timeouts inside kernels are recorded in a per-device
 * status word read with tm_device_status().
 *
 * The reference (TaoMate-HD) reaches this path through two vLLM operators:
 *   torch.ops._C.dynamic_scaled_int8_quant(out, input, scales, azp)
 *       src/taomate_hd/inference/w8a8.py:71   (workspace path)
 *       src/taomate_hd/inference/w8a8.py:141  (vllm._custom_ops.scaled_int8_quant)
 *   torch.ops._C.cutlass_scaled_mm(out, a, b, scale_a, scale_b, bias)
 *       src/taomate_hd/inference/w8a8.py:72   (workspace path)
 *       src/taomate_hd/inference/w8a8.py:142  (vllm._custom_ops.cutlass_scaled_mm)
 * Weight conversion is src/taomate_hd/inference/w8a8.py:175-179 and the
 * adaLN producers are src/taomate_hd/inference/fused_kernels.py:220-236 and
 * :322-347.
 */
#ifndef TAOMATE_W8A8_H
#define TAOMATE_W8A8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define TM_OK 0
#define TM_ERR_NULL_POINTER 1     /* a required pointer is NULL */
#define TM_ERR_SHAPE 2            /* negative / inconsistent sizes or strides */
#define TM_ERR_ALIGNMENT 3        /* pointer or stride alignment not met */
#define TM_ERR_DTYPE 4            /* unsupported dtype code */
#define TM_ERR_UNSUPPORTED 5      /* valid request this build does not implement */
#define TM_ERR_CUDA 6             /* a CUDA runtime call failed */
#define TM_ERR_DEVICE_TIMEOUT 7   /* a kernel wait gave up (tm_device_status) */
#define TM_ERR_TOO_LARGE 8        /* size exceeds a documented maximum */

/* ---- dtype codes ------------------------------------------------------- */
#define TM_DTYPE_BF16 0
#define TM_DTYPE_FP16 1
#define TM_DTYPE_FP32 2

/* ---- GEMM epilogue flags (tm_scaled_mm_i8_ex) -------------------------- */
/* gelu_tanh applied to the rounded output: y = round(gelu(round(x)))      */
#define TM_EPI_GELU_TANH 0x1u
/*
 * SwiGLU after a merged gate/up projection (the reference's fused_swiglu,
 * src/taomate_hd/inference/fused_kernels.py:298-309, after the merged fc1,
 * model/layers.py:525-533): the weight's n rows (and scales, bias) come
 * interleaved in blocks of 16 -- 16 gate rows, then the 16 matching up rows
 * -- and the output has n / 2 columns, out = round(round(g * sigmoid(g)) * u)
 * with g, u the rounded linear outputs.  n % 64 == 0; not combined with
 * GELU, the fused reductions or LoRA.
 */
#define TM_EPI_SWIGLU 0x2u

/* Human-readable text for a status code (static storage). */
const char* tm_status_string(int status);

/* Library version, major * 10000 + minor * 100 + patch. */
int tm_version(void);

/*
 * Read (and optionally clear) the device status word of `device`: 0 when no
 * kernel of this library has recorded an error since the last clear,
 * otherwise a device status (1 = wait timeout, 2 = drain timeout).
 * Synchronises the device.  The word's address is looked up once per device
 * and kept: do not use the library across a cudaDeviceReset.
 */
int tm_device_status(int device, int* code, int clear);

/*
 * Dynamic per-token symmetric int8 quantisation.
 * Replaces torch.ops._C.dynamic_scaled_int8_quant(out, input, scales, azp)
 * (src/taomate_hd/inference/w8a8.py:71) and the dynamic branch of
 * vllm._custom_ops.scaled_int8_quant (src/taomate_hd/inference/w8a8.py:141).
 * For each row r of input[rows, cols] (row stride `input_row_stride`
 * elements):
 *   amax      = max_k |x[r,k]|                 (fp32)
 *   scales[r] = amax / 127                      (fp32, IEEE division)
 *   inv       = amax == 0 ? 0 : 127 / amax      (fp32, IEEE division)
 *   out[r,k]  = sat_int8(round_half_even(x[r,k] * inv))
 * out is [rows, cols] contiguous int8; scales is [rows] fp32.
 * azp must be NULL (asymmetric quantisation is not used by the reference).
 */
int tm_dynamic_scaled_int8_quant(int8_t* out, const void* input, int input_dtype,
                                 float* scales, int32_t* azp, int64_t rows, int64_t cols,
                                 int64_t input_row_stride, void* stream);

/*
 * Static per-tensor symmetric int8 quantisation with a device-resident fp32
 * scale[0]: out = sat_int8(round_half_even(x / scale)).
 * Replaces torch.ops._C.static_scaled_int8_quant, the static branch of
 * vllm._custom_ops.scaled_int8_quant (the reference calls it only with
 * scale=None, src/taomate_hd/inference/w8a8.py:141).
 */
int tm_static_scaled_int8_quant(int8_t* out, const void* input, int input_dtype,
                                const float* scale, int32_t* azp, int64_t rows, int64_t cols,
                                int64_t input_row_stride, void* stream);

/*
 * Scaled int8 GEMM with bf16/fp16 output.
 * Replaces torch.ops._C.cutlass_scaled_mm(out, a, b, scale_a, scale_b, bias)
 * (src/taomate_hd/inference/w8a8.py:72, :142-144).
 *   out[m,n] = cvt(scale_a[m] * (scale_b[n] * float(sum_k a[m,k] * b[k,n])) (+ bias[n]))
 * a: int8 [m, k] row-major, row stride lda (elements, multiple of 16).
 * b: int8 [k, n] column-major, i.e. the [n, k] row-major weight storage,
 *    column stride ldb (multiple of 16) -- the `weight.t()` view.
 * scale_a: fp32, numel 1 (per-tensor) or m (per-token).
 * scale_b: fp32, numel 1 (per-tensor) or n (per-channel).
 * bias: NULL or [n] in out_dtype.  out: [m, n] row-major, row stride ldo.
 * Requires k % 16 == 0 and n % 16 == 0 (the same contract as vLLM's CUTLASS
 * path), 16-byte aligned a/b/out.
 */
int tm_cutlass_scaled_mm(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                         int64_t k, int64_t lda, int64_t ldb, int64_t ldo, void* stream);

/*
 * tm_cutlass_scaled_mm plus fused epilogue options (TM_EPI_* flags) and an
 * optional raw int32 accumulator output acc_debug[m, n] (row stride n), which
 * exposes the exact int32 sums for bit-exact checking.
 * Replaces cutlass_scaled_mm (src/taomate_hd/inference/w8a8.py:72) followed by
 * the activation: TM_EPI_SWIGLU is the merged fc1 and fused_swiglu
 * (src/taomate_hd/inference/fused_kernels.py:298-309, called at
 * src/taomate_hd/model/layers.py:525-533); TM_EPI_GELU_TANH is the BASELINE
 * configuration's fc1 (bias + GELU-tanh), which has no reference call site.
 */
int tm_scaled_mm_i8_ex(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                       const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                       int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                       int64_t k, int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                       int32_t* acc_debug, void* stream);

/*
 * tm_scaled_mm_i8_ex with a forced tile configuration instead of the size
 * heuristic; lets tests and benchmarks cover every kernel instantiation.
 * tile_n: 256, 128, 64 = one-CTA kernel with a 128 x tile_n tile;
 * 1256, 1192, 1128 = CTA-pair kernel with a 256 x (tile_n - 1000) tile.
 * Same reference counterpart as tm_cutlass_scaled_mm.
 */
int tm_scaled_mm_i8_tile(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                         int64_t k, int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                         int32_t* acc_debug, int tile_n, void* stream);

/*
 * Split-K for skinny M.  tm_scaled_mm_i8_ws is tm_scaled_mm_i8_ex plus a
 * caller-provided workspace; when the shape leaves most SMs idle (small M)
 * it cuts K into slices computed by separate CTAs, which store exact int32
 * partials in the workspace; the last slice of each tile to finish sums them
 * and runs the epilogue (results are identical to the unsplit GEMM).  The workspace (a 64 KiB counter region,
 * then the partials) must be 16-byte aligned and zeroed before its first use;
 * every complete call leaves its counters at zero again.  Calls that share a
 * workspace must not overlap on the GPU.  With workspace_bytes smaller than
 * tm_scaled_mm_i8_workspace_size(m, n, k) the call runs unsplit.
 * tm_scaled_mm_i8_splitk forces a one-CTA tile width (256/128/64) and a
 * slice count (for tests); tm_scaled_mm_i8_splitk_workspace_size gives its
 * workspace bytes.  Same reference counterpart as tm_cutlass_scaled_mm.
 */
int tm_scaled_mm_i8_workspace_size(int64_t m, int64_t n, int64_t k, uint64_t* bytes);
int tm_scaled_mm_i8_ws(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                       const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                       int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                       int64_t k, int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                       int32_t* acc_debug, void* workspace, uint64_t workspace_bytes,
                       void* stream);
int tm_scaled_mm_i8_splitk(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                           const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                           int64_t scale_b_numel, const void* bias, int64_t m, int64_t n,
                           int64_t k, int64_t lda, int64_t ldb, int64_t ldo, uint32_t epilogue,
                           int32_t* acc_debug, int tile_n, int splits, void* workspace,
                           uint64_t workspace_bytes, void* stream);
int tm_scaled_mm_i8_splitk_workspace_size(int64_t m, int64_t n, int64_t k, int tile_n,
                                          int splits, uint64_t* bytes);

/*
 * Scaled GEMM with the BF16 LoRA delta added in the epilogue (the reference's
 * H3InferenceParallelLinearLoRA.forward, src/taomate_hd/inference/
 * lora_checkpoint.py:126-154: output + bf16(bf16(x A^T) B^T) * scale).
 * out = epi(dequant(a b^T) (+bias) + lora_t lora_b^T), where lora_t = x A^T
 * (bf16 [m, r], row stride ldt) and lora_b = scale * B (bf16 [n, r], row
 * stride ldlb); r = lora_rank in {8, 16, ..., 64}, ldt and ldlb multiples of
 * 8, both pointers 16-byte aligned.  The update is accumulated in fp32 on the
 * tensor cores onto the rounded base output and rounded once with it; GELU
 * (TM_EPI_GELU_TANH) applies to the sum.  Other arguments as
 * tm_cutlass_scaled_mm.  Runs the 256 x 256 CTA-pair kernel.
 */
int tm_scaled_mm_i8_lora(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                         const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                         int64_t scale_b_numel, const void* bias, const void* lora_t,
                         int64_t ldt, const void* lora_b, int64_t ldlb, int lora_rank, int64_t m,
                         int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldo,
                         uint32_t epilogue, void* stream);

/*
 * The merged QKV projection with the Ulysses all-to-all done by its epilogue
 * over NVLink (the reference's merged_qkv_sequence_to_heads,
 * src/taomate_hd/distributed/ulysses.py:166-212: the linear, the send
 * layout, then all_to_all_single): each 64-column pass of the output is
 * stored straight into the receive buffer of the rank that holds its head,
 * in this rank's slot, so that every rank's peer_recv[j] ends up as the
 * reference's all-to-all output [world][3][m][ceil(heads / world)][head_dim]
 * (slot s from rank s; padded head slots are never written and stay as the
 * buffer was zeroed at allocation).  Each CTA drains its stores once and
 * adds its per-destination element counts to peer_flags[w][rank]; the launch
 * returns when this rank's `world` counters show every source's rows
 * (epoch x 3 x m x its real heads x head_dim), so the buffer is complete for
 * the work that follows on `stream`.  peer_recv[j] / peer_flags[j]: rank j's
 * receive buffer and `world` uint64 counters (zeroed at allocation, never
 * reset; alternate two buffer sets by call, epoch = uses of the set).  m
 * tokens per rank (m % 32 == 0), head_dim a multiple of 64, bf16 output, no
 * activation; waits are bounded: a source that never reports leaves NaN in
 * its slot and sets the device status.
 */
int tm_scaled_mm_i8_ulysses_exchange(const int8_t* a, const int8_t* b, const float* scale_a,
                                     int64_t scale_a_numel, const float* scale_b,
                                     int64_t scale_b_numel, const void* bias, int64_t m,
                                     int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                     int num_heads, int head_dim, void* const* peer_recv,
                                     void* const* peer_flags, int world, int rank,
                                     uint32_t epoch, void* stream);

/*
 * The row-parallel LoRA linears with their reduction fused into the kernel
 * (the reference's fused-row-reduce LoRA forward,
 * src/taomate_hd/inference/lora_checkpoint.py:127-143: each rank adds its
 * update_partial * scale to base_partial, the sum is reduced over the TP
 * group, then the bias is added): the LoRA epilogue of tm_scaled_mm_i8_lora
 * with no activation, whose bf16 partial goes to the rows' owners as in
 * tm_scaled_mm_i8_reduce_scatter / tm_scaled_mm_i8_all_reduce (same peer
 * buffers, counters, epochs and rules).  Each rank's partial is
 * round(round(dequant(a b^T)) + lora_t lora_b^T) (fp32 add, one rounding);
 * the owner sums the partials in rank order in fp32, adds the bias once and
 * rounds.  bf16 output only.
 */
int tm_scaled_mm_i8_lora_reduce_scatter(void* out, const int8_t* a, const int8_t* b,
                                        const float* scale_a, int64_t scale_a_numel,
                                        const float* scale_b, int64_t scale_b_numel,
                                        const void* bias, const void* lora_t, int64_t ldt,
                                        const void* lora_b, int64_t ldlb, int lora_rank,
                                        int64_t m, int64_t n, int64_t k, int64_t lda,
                                        int64_t ldb, int64_t ldo, void* const* peer_part,
                                        void* const* peer_flags, int world, int rank,
                                        uint32_t epoch, void* stream);
int tm_scaled_mm_i8_lora_all_reduce(const int8_t* a, const int8_t* b, const float* scale_a,
                                    int64_t scale_a_numel, const float* scale_b,
                                    int64_t scale_b_numel, const void* bias, const void* lora_t,
                                    int64_t ldt, const void* lora_b, int64_t ldlb, int lora_rank,
                                    int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                    void* const* peer_part, void* const* peer_flags,
                                    void* const* peer_out, int world, int rank, uint32_t epoch,
                                    void* stream);

/*
 * LoRA down-projection t = x a^T (the inner linear of the reference's LoRA
 * forward, src/taomate_hd/inference/lora_checkpoint.py:135-136 and 146-147,
 * torch.nn.functional.linear(inputs, lora_a)): x bf16 [m, k] (row stride
 * ldx), a bf16 [rank, k] (row stride lda), t bf16 [m, rank] (row stride ldt);
 * rank in {8, 16, ..., 64}.  fp32 accumulation on the tensor cores, one
 * rounding to bf16.  The three pointers 16-byte aligned and the three row
 * strides multiples of 8 elements.  m == 0 is a no-op.  Feeds lora_t of
 * tm_scaled_mm_i8_lora.
 */
int tm_lora_down_proj(void* t, int64_t ldt, const void* x, int64_t ldx, const void* a,
                      int64_t lda, int rank, int64_t m, int64_t k, void* stream);

/*
 * Merged QKV projection written straight into the Ulysses all-to-all send
 * layout (the reference's merged_qkv_sequence_to_heads builds it with a
 * permute copy, src/taomate_hd/distributed/ulysses.py:153-212): the GEMM of
 * tm_cutlass_scaled_mm with n = 3 x num_heads x head_dim, whose epilogue
 * stores row r, column (qkv, head, d) at send[w][qkv][r][(head % lh) *
 * head_dim + d], w = head / lh, lh = ceil(num_heads / world); `send` is a
 * contiguous [world][3][m][lh x head_dim] buffer to pass to the all-to-all.
 * When world does not divide num_heads the slots of the padded heads
 * (w * lh + h >= num_heads) are set to zero, as the reference's zero-padded
 * head shards (ulysses.py:188-193, ulysses_layout.py:9-42).
 * head_dim % 32 == 0, m % 32 == 0.
 */
int tm_scaled_mm_i8_ulysses_send(void* send, int out_dtype, const int8_t* a, const int8_t* b,
                                 const float* scale_a, int64_t scale_a_numel,
                                 const float* scale_b, int64_t scale_b_numel, const void* bias,
                                 int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                 int num_heads, int head_dim, int world, void* stream);

/*
 * Split-K GEMM that allocates nothing, for callers that cannot call
 * cudaMalloc: code running inside a host process whose device memory is
 * owned and budgeted by someone else (an inference server's pre-partitioned
 * pool, a plugin invoked from another runtime's launch path), or a latency-
 * critical path where an allocation's implicit synchronisation is not
 * acceptable.  Same computation and arguments as tm_scaled_mm_i8_splitk
 * without the workspace and acc_debug: the int32 partials live in a
 * TM_SPLITK_NOALLOC_MAX_BYTES (16 MiB) array compiled into the library,
 * which every GPU that loads the library holds until the process exits.
 * Requests whose split needs more than that (a 64 KiB counter region plus
 * splits x m x n x 4 bytes) fail with TM_ERR_TOO_LARGE.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress), so make
 * that first call before any stream capture.  The address is kept for the
 * life of the process: the library must not be used across a
 * cudaDeviceReset (or any other re-creation of the device's primary
 * context).  Every call shares the one array and clears its counters on
 * `stream` before use, after all argument checks have passed (a refused call
 * enqueues nothing): calls that overlap on the GPU (other streams, other
 * host threads) race and must be serialised by the caller.  TM_EPI_SWIGLU
 * with splits > 1 returns TM_ERR_UNSUPPORTED.  Results are identical, bit
 * for bit, to the unsplit GEMM.  No counterpart in the reference.
 */
#define TM_SPLITK_NOALLOC_MAX_BYTES (16ull << 20)
int tm_scaled_mm_i8_splitk_noalloc(void* out, int out_dtype, const int8_t* a, const int8_t* b,
                                   const float* scale_a, int64_t scale_a_numel,
                                   const float* scale_b, int64_t scale_b_numel, const void* bias,
                                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                   int64_t ldo, uint32_t epilogue, int tile_n, int splits,
                                   void* stream);

/*
 * Row-parallel scaled GEMM with the reduce-scatter fused into the kernel
 * (the row-parallel fc2 / out-projection; the reference's
 * RowParallelLinear.forward = forward_local + tp all-reduce + bias,
 * src/taomate_hd/distributed/linear.py:259-289 and collectives.py:19-40).
 * Every rank of a TP group of `world` ranks calls it with its K-shard
 * (a: [m, k] local activations, b: the [n, k] local weight).  Rows are
 * owned in `world` contiguous blocks of m / world (m % (256 * world) == 0).
 * The epilogue stores each bf16 partial 128-row block of owner j's rows into
 * peer_part[j], slot `rank` (NVLink peer stores), while the GEMM runs; each
 * CTA then drains its stores once and adds the number of elements it sent
 * to owner j to peer_flags[j][rank].  CTAs without GEMM work left wait
 * (bounded) until every source's counter shows all of this rank's blocks,
 * sum them in rank order in fp32, add `bias` ([n] bf16 or NULL) once and
 * write out[m / world, n] (row stride ldo).
 * peer_part[j]: device pointer (local or IPC-mapped) to rank j's receive
 *   buffer of world x (m / world) x n bf16; peer_flags[j]: rank j's array of
 *   `world` uint64 counters, zeroed once at allocation and never reset.
 * epoch: 1-based count of calls made with this buffer set, identical on all
 * ranks; consecutive calls must alternate between two buffer sets (a rank may
 * run one call ahead), and every call on a set must use the same m, n and
 * world.  tile_n: 0 = heuristic, or a tm_scaled_mm_i8_tile configuration.
 * Waits that run out record a device status (tm_device_status).
 */
int tm_scaled_mm_i8_reduce_scatter(void* out, const int8_t* a, const int8_t* b,
                                   const float* scale_a, int64_t scale_a_numel,
                                   const float* scale_b, int64_t scale_b_numel, const void* bias,
                                   int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                   int64_t ldo, void* const* peer_part, void* const* peer_flags,
                                   int world, int rank, uint32_t epoch, int tile_n, void* stream);

/*
 * Row-parallel scaled GEMM with the all-reduce fused into the kernel (the
 * reference's row-parallel out-projection: forward_local, then the tp
 * all-reduce, then bias, src/taomate_hd/distributed/linear.py:279-289,
 * collectives.py:19-40).  The reduce-scatter half is the one of
 * tm_scaled_mm_i8_reduce_scatter; then each owner stores its reduced rows
 * (bias added once) into every rank's output peer_out[j] ([m, n] bf16,
 * row stride n) at their global row offset, drains once per CTA and adds
 * the element count to peer_flags[j][world + rank].  The kernel returns
 * when this rank's `world` gather counters show every owner's rows, so
 * peer_out[rank] holds the full sum for the work that follows on `stream`.
 * peer_flags[j]: rank j's 2 x world uint64 counters (reduce-scatter, then
 *   gather), zeroed at allocation and never reset; peer_out[j]: rank j's
 *   output buffer (local or IPC-mapped).  Same epoch / buffer-set /
 *   alignment rules as tm_scaled_mm_i8_reduce_scatter; the output of a call
 *   stays valid until the second call after it on the same buffer set pair.
 */
int tm_scaled_mm_i8_all_reduce(const int8_t* a, const int8_t* b, const float* scale_a,
                               int64_t scale_a_numel, const float* scale_b, int64_t scale_b_numel,
                               const void* bias, int64_t m, int64_t n, int64_t k, int64_t lda,
                               int64_t ldb, void* const* peer_part, void* const* peer_flags,
                               void* const* peer_out, int world, int rank, uint32_t epoch,
                               int tile_n, void* stream);

/*
 * Buffers shared between the ranks of a node for the fused reduction.
 * tm_peer_alloc: cudaMalloc `bytes`, zero them, and write the CUDA IPC
 * handle (tm_peer_handle_size() bytes) to handle_out.  tm_peer_open maps a
 * peer's handle into this process; tm_peer_close unmaps it; tm_peer_free
 * releases an allocation made here.  Called once per layer shape at set-up,
 * never per call.  No reference counterpart (the reference uses NCCL).
 */
int tm_peer_handle_size(void);
int tm_peer_alloc(uint64_t bytes, void** ptr, void* handle_out);
int tm_peer_open(const void* handle, void** ptr);
int tm_peer_close(void* ptr);
int tm_peer_free(void* ptr);

/*
 * Per-output-channel symmetric weight quantisation, bit-exact with
 * _quantize_cutlass_w8a8_weight (src/taomate_hd/inference/w8a8.py:175-179):
 *   scales[n] = max(float(max_k |w[n,k]|) / 127, 1e-12)
 *   q[n,k]    = clamp(round_half_even(float(w[n,k]) / scales[n]), -127, 127)
 * w: [n, k] row-major (row stride k) in w_dtype; q: [n, k]; scales: [n].
 */
int tm_quantize_weight_int8(int8_t* q, float* scales, const void* w, int w_dtype, int64_t n,
                            int64_t k, void* stream);

/*
 * adaLN modulate fused into the dynamic per-token quantisation.
 * Follows _modulate_kernel (src/taomate_hd/inference/fused_kernels.py:220-236):
 *   t    = index ? index[r] : r
 *   h    = bf16(bf16(x[r,c] * bf16(1 + scale[t,c])) + shift[t,c])
 * then h is quantised exactly as tm_dynamic_scaled_int8_quant.  x, shift,
 * scale and hidden_out are bf16; shift/scale rows have stride table_stride.
 * hidden_out (optional, NULL to skip) receives h as [rows, cols] bf16.
 */
int tm_modulate_int8_quant(int8_t* out, float* scales, void* hidden_out, const void* x,
                           const void* shift, const void* scale, const int64_t* index,
                           int64_t table_stride, int64_t rows, int64_t cols, void* stream);

/*
 * RMSNorm + adaLN modulate fused into the dynamic per-token quantisation.
 * Follows _rms_norm_modulate_kernel
 * (src/taomate_hd/inference/fused_kernels.py:322-347):
 *   n = bf16(x * rsqrt(mean(x^2) + eps) * weight)
 *   h = bf16(bf16(n * bf16(1 + scale[t])) + shift[t])
 * then quantised as tm_dynamic_scaled_int8_quant.  All tensors bf16.
 */
int tm_rms_norm_modulate_int8_quant(int8_t* out, float* scales, void* hidden_out,
                                    const void* x, const void* norm_weight, float eps,
                                    const void* shift, const void* scale, const int64_t* index,
                                    int64_t table_stride, int64_t rows, int64_t cols,
                                    void* stream);

/*
 * Gated residual add + RMSNorm + adaLN modulate fused into the dynamic
 * per-token quantisation: the producer of the fc1 input after attention.
 * Follows _residual_gate_rms_norm_modulate_kernel
 * (src/taomate_hd/inference/fused_kernels.py:349-382, wrapper :757-797):
 *   t    = index ? index[r] : r
 *   x    = bf16(residual[r,c] + bf16(gate[t,c] * branch[r,c]))  -> residual_out
 *   n    = bf16(x * rsqrt(mean(x^2) + eps) * norm_weight)
 *   h    = bf16(bf16(n * bf16(1 + scale[t,c])) + shift[t,c])   -> hidden_out
 * then h is quantised as tm_dynamic_scaled_int8_quant.  All tensors bf16;
 * gate, shift and scale rows share table_stride (the reference passes
 * gate.stride(0) for all three).  residual_out is required, hidden_out may
 * be NULL.
 */
int tm_residual_gate_rms_norm_modulate_int8_quant(
    int8_t* out, float* scales, void* residual_out, void* hidden_out, const void* residual,
    const void* branch, const void* gate, const void* norm_weight, float eps, const void* shift,
    const void* scale, const int64_t* index, int64_t table_stride, int64_t rows, int64_t cols,
    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TAOMATE_W8A8_H */
