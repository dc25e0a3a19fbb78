/*
 * kz.h -- C ABI of libkz, the B200 (sm_100a) backend of Kansai's int8
 * quantized-linear path.
 *
 * Plain C: device pointers, sizes, a CUDA stream handle and an int status.
 * No exceptions and no C++ or PyTorch types cross this boundary.  Every entry
 * point returns KZ_OK (0) or an error code; kz_last_error() returns the
 * message of the calling thread's most recent failure.
 *
 * Each entry point names the reference interface it replaces
 * (reference file:line, paths inside the KansaiML checkout).  The reference
 * reaches all of them through its `kansai._core` extension
 * (python/bindings.cpp:17), which gains one thin wrapper per entry point
 * (GIL released, non-zero status raised as RuntimeError).
 *
 * Memory: the library allocates no device memory.  Outputs, and the small
 * `partials` buffers some entry points use to hand an absmax from one kernel
 * to the next, are caller-owned device buffers.
 *
 * Errors found on the device (a NaN/Inf in a tensor being quantized, a wait
 * inside a kernel that ran out) cannot be returned synchronously; kernels
 * record them in a sticky per-device status word read by kz_device_status().
 *
 * Per-device state (the status word's device address, the static scratch of
 * kz_quantize_cols_f32_noalloc) is resolved on the first call on each device
 * and cached for the life of the process.  cudaDeviceReset ends the context
 * that state lives in: do not call libkz on a device after resetting it.
 */
#ifndef KZ_H_
#define KZ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same handle as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* kz_stream_t;

enum kz_status_code {
    KZ_OK = 0,
    KZ_ERR_INVALID_ARGUMENT = 1,  /* bad shape, pointer, stride or alignment */
    KZ_ERR_NONFINITE = 2,         /* NaN/Inf in a tensor being quantized
                                     (quantize.py:69 raises ValueError/OverflowError) */
    KZ_ERR_CUDA = 3,              /* a CUDA runtime/driver call failed */
    KZ_ERR_UNSUPPORTED_DEVICE = 4,/* current device is not sm_100 (B200) */
    KZ_ERR_DEVICE_TIMEOUT = 5     /* a bounded wait inside a kernel ran out */
};

enum kz_activation { KZ_ACT_NONE = 0, KZ_ACT_RELU = 1, KZ_ACT_GELU = 2 };

/* Words in an absmax `partials` buffer (uint32_t[KZ_PARTIALS_WORDS]).
 * Word 0 holds the number of valid partials P (P <= KZ_PARTIALS_WORDS - 3);
 * words 1..P hold the bit patterns of non-negative fp32 partial maxima (|x| as
 * uint32 bits, so unsigned max == float max, and NaN sorts above +Inf).
 * Because the partials are plain maxima, an element-wise integer MAX
 * all-reduce of words 0..P across ranks yields the global absmax (config 5).
 * The second-to-last word is the grid barrier of kz_quantize_tensor_f32's
 * single-launch form and the last word is reserved: ZERO-FILL A BUFFER ONCE
 * BEFORE ITS FIRST USE; every completed single-launch call leaves the low 31
 * bits of the barrier word at zero and flips its bit 31.  One buffer per stream
 * (calls on one stream are ordered; calls on different streams must not share
 * a buffer). */
#define KZ_PARTIALS_WORDS 1024

/* ------------------------------------------------------------------ misc */

const char* kz_last_error(void);
int kz_version(void);
/* 1 when `device` is an sm_100 GPU this library has code for, else 0. */
int kz_device_supported(int device);

/* Replaces Tensor::randn (core/src/Tensor.cpp:85-92): fills n floats on the
 * HOST from std::mt19937(seed) through std::normal_distribution<float>(0, std),
 * the same generator and distribution the reference uses, so weights created
 * with a seed equal the reference's bit for bit.  seed == 0 draws a random seed
 * as the reference does. */
int kz_randn_host(float* out, int64_t n, float stddev, uint64_t seed);

/* Reads the current device's sticky status word (0 or a kz_status_code) after
 * synchronising `stream`; clears it when `clear` != 0. */
int kz_device_status(int* code, int clear, kz_stream_t stream);

/* ------------------------------------------- quantize (quantize.py:50-70) */

/* Per-tensor absmax of x[0..n): writes partial maxima into `partials`.
 * Replaces `max(abs(v) for v in flat)` (quantize.py:67). */
int kz_absmax_f32(const float* x, int64_t n, uint32_t* partials, kz_stream_t stream);

/* Per-tensor quantize given absmax partials (from kz_absmax_f32, the int8
 * GEMM's epilogue, or a MAX all-reduce of either across ranks).
 * Replaces quantize.py:68-69: scale = max_abs / 127 (double; 1.0 when
 * max_abs == 0), q = clamp(round_half_even(x / scale), -127, 127), bit-exact.
 * Writes q[0..n), *scale (double) and *scale_f32 ((float)*scale, may be NULL).
 * A NaN/Inf absmax writes q = 0, *scale = NaN and sets KZ_ERR_NONFINITE in
 * the device status word. */
int kz_quantize_partials_f32(const float* x, int64_t n, const uint32_t* partials, int8_t* q,
                             double* scale, float* scale_f32, kz_stream_t stream);

/* quantize_symmetric (quantize.py:50-70) on the device.  Tensors of 65536
 * elements or more run as ONE cooperative launch (absmax, a bounded grid
 * barrier in the second-to-last word of `partials`, quantize; with x and q
 * 16-byte aligned each block keeps its slice of x in shared memory, so x is
 * read from HBM once); smaller ones as kz_absmax_f32 + kz_quantize_partials_f32.
 * `partials` is caller scratch, zero-filled before its first use (see
 * KZ_PARTIALS_WORDS). */
int kz_quantize_tensor_f32(const float* x, int64_t n, int8_t* q, double* scale, float* scale_f32,
                           uint32_t* partials, kz_stream_t stream);

/* LayerNorm over the last axis of x[M, D] in the reference's operation order
 * (nn.py:323-331): mean = sum(dim) * fl32(1/D), with sum(dim) adding each
 * row's elements one by one in index order (Tensor.cpp:831-880 ->
 * backend/cpu/src/Ops.cpp:157-190); centered = x - mean; var = the same
 * ordered sum of centered * centered times fl32(1/D); y = centered *
 * fl32(1 / sqrt(var + eps)) * gamma + beta (Tensor::div multiplies by the
 * reciprocal, Tensor.cpp:677-679); every step one fp32 operation rounded to
 * nearest, so y equals the reference's LayerNorm bit for bit.  gamma / beta
 * may be NULL: ones / zeros, the reference's initial parameters.  Also writes
 * the absmax partials of y in the KZ_PARTIALS_WORDS format, so
 * kz_quantize_partials_f32 quantizes y per tensor without another pass over
 * it: the prologue of a quantized Linear that follows a LayerNorm (the
 * reference runs LayerNorm and quantize_symmetric separately). */
int kz_layernorm_partials_f32(const float* x, int64_t M, int64_t D, const float* gamma, const float* beta, float eps,
                              float* y, uint32_t* partials, kz_stream_t stream);

/* kz_layernorm_partials_f32 of x + res, with the sum also written to sum_out:
 * a pre-LN block's residual connection (nn.py:476-477, x = x.add(...))
 * folded into the LayerNorm that follows it.  Each element of the sum is one
 * fp32 add, rounded as the reference's Tensor::add rounds it, so sum_out and
 * y equal the unfused x.add(res) followed by kz_layernorm_partials_f32 bit for
 * bit.  sum_out must not alias x, res or y. */
int kz_add_layernorm_partials_f32(const float* x, const float* res, int64_t M, int64_t D, const float* gamma,
                                  const float* beta, float eps, float* sum_out, float* y, uint32_t* partials,
                                  kz_stream_t stream);

/* Scaled dot-product attention, fp32, in the reference's operation order
 * (replaces the Tensor-op composition of MultiHeadAttention.forward,
 * python/kansai/nn.py:410-427, between the projections):
 *   s[i][j] = (sum_t q[i][t] * k[j][t]) * scale     t ascending, no FMA
 *   s[i][j] = s[i][j] + mask[i][j]                   (mask may be NULL)
 *   e = exp(s - max_j s);  w = e * (1 / sum_j e)     j ascending
 *   out[i][t] = sum_j w[i][j] * v[j][t]              j ascending, no FMA
 * every operation an fp32 round-to-nearest step; exp is the correctly rounded
 * fp32 exponential (the host libm's expf, which the reference calls, agrees
 * with it except on rare near-halfway inputs).
 * Layouts (floats): q(b, h, i, t) = q[(b * seq_q + i) * q_row_stride + h * d_k + t],
 * k and v the same with seq_k; out(b, i, h * d_k + t) =
 * out[(b * seq_q + i) * out_row_stride + h * d_k + t] (heads merged);
 * mask(b, h, i, j) = mask[b * mask_batch_stride + h * mask_head_stride +
 * i * mask_row_stride + j] (0 strides broadcast).  causal != 0 (needs
 * seq_q == seq_k) gives keys j > i weight 0 -- causal_mask()'s -1e9 entries --
 * and ignores mask.  d_k in {32, 64, 128}; q, k, v, out 16-byte aligned, row
 * strides multiples of 4; seq_k limited by the on-chip score rows
 * (kz_attention_smem_bytes returns 0 past it).  absmax_partials (may be NULL):
 * partial maxima of |out| in the KZ_PARTIALS_WORDS format. */
int kz_attention_f32(const float* q, const float* k, const float* v, int64_t batch, int64_t heads, int64_t seq_q,
                     int64_t seq_k, int64_t d_k, int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                     const float* mask, int64_t mask_batch_stride, int64_t mask_head_stride, int64_t mask_row_stride,
                     int causal, float scale, float* out, int64_t out_row_stride, uint32_t* absmax_partials,
                     kz_stream_t stream);
/* Dynamic shared memory kz_attention_f32 needs for seq_k keys of d_k, or 0
 * when that exceeds what one CTA can hold. */
int kz_attention_smem_bytes(int64_t seq_k, int64_t d_k);

/* Per-output-channel quantize of a reference-layout weight w[K, N] (row-major,
 * nn.py:74-81: [in_features, out_features]); channel n is column n.  Writes
 * K-major codes qT[N, K], scales[N] (double) and scales_f32[N].  Each column
 * follows quantize.py:66-70 exactly.  `workspace` must hold
 * kz_quantize_cols_workspace_bytes(K, N) bytes. */
size_t kz_quantize_cols_workspace_bytes(int64_t K, int64_t N);
int kz_quantize_cols_f32(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales, float* scales_f32,
                         void* workspace, size_t workspace_bytes, kz_stream_t stream);

/* kz_quantize_cols_f32 for callers that cannot call cudaMalloc (a host
 * runtime that owns the GPU's memory through its own allocator or arena, or
 * must not allocate after start-up): same arguments and results, but no
 * workspace -- its scratch is a static 256 KB device array inside libkz that
 * every GPU loading the library keeps until exit.  No counterpart in the
 * reference (it has no device code).  Limits: N <= 65536 output channels
 * (larger N returns KZ_ERR_INVALID_ARGUMENT).  All calls share the array, so
 * calls that overlap on the GPU race: order them on one stream.  The first
 * call on each device resolves the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture. */
int kz_quantize_cols_f32_noalloc(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales,
                                 float* scales_f32, kz_stream_t stream);

/* Per-row (per-token) quantize of x[M, K]: row m gets its own scale,
 * quantize.py:66-70 applied to each row. */
int kz_quantize_rows_f32(const float* x, int64_t M, int64_t K, int8_t* q, double* scales, float* scales_f32,
                         kz_stream_t stream);

/* ----------------------------------------- dequantize (quantize.py:73-77) */

/* out[i] = (float)((double)q[i] * scale): quantize.py:76 in double, narrowed
 * to fp32 as Tensor::from_flat does (core/src/Tensor.cpp:94-100). */
int kz_dequantize_i8_f32(const int8_t* q, int64_t n, double scale, float* out, kz_stream_t stream);
/* Which exact form kz_dequantize_i8_f32 takes for `scale` (host-only, no
 * device call): 0 the table-free split form (fp32 fma(q, s_hi, q * s_lo),
 * which equals (float)((double)q * scale) for every byte at this scale), 1
 * the shared-memory table of the 256 values (any other scale; rare). */
int kz_dequantize_uses_table(double scale);

/* Inverse of kz_quantize_cols_f32: out[K, N] (reference layout) from qT[N, K]
 * and per-channel double scales (device pointer). */
int kz_dequantize_cols_i8_f32(const int8_t* qT, int64_t K, int64_t N, const double* scales, float* out,
                              kz_stream_t stream);

/* ------------------------------- qlinear, reference semantics (W8A32) */

/* Replaces qlinear (quantize.py:115-122) = Tensor::matmul (core/src/Tensor.cpp:332-362
 * -> backend/cpu/src/Ops.cpp:328-337) on dequantize(q, scale), then
 * Tensor::add bias (Ops.cpp:34-38), then an optional activation (nn.ReLU ->
 * Ops.cpp:197-199, nn.GELU -> Ops.cpp:250-256).
 * out[M, N] = act(x[M, K] @ dequantize(q[K, N], scale) + bias[N]); bias may be NULL.
 * Accumulation runs in k order with every product and sum rounded to fp32
 * separately, as the reference's loop does, so relu/none outputs are
 * bit-identical to the reference. */
int kz_qlinear_w8a32_f32(const float* x, int64_t M, int64_t K, const int8_t* q, double scale,
                         const float* bias, int64_t N, int act, float* out, kz_stream_t stream);

/* ------------------------------------------------- int8 GEMM (W8A8) */

/* acc[m, n] = sum_k A[m, k] * B[n, k]  (int8 x int8 -> int32, exact), on the
 * sm_100a tensor cores (tcgen05.mma kind::i8, TMA-fed, TMEM accumulators).
 * New behaviour: the reference has no int8 GEMM (quantize.py:35-44); this is
 * the contraction inside qlinear (quantize.py:121) once both operands are int8.
 *
 *   A: int8, K-major.  With a_kblock == K it is the plain row-major [M, K].
 *      With a_kblock = K / G it is G blocks [G][M][K/G] (block g holds columns
 *      g*K/G .. of A): the rank-major layout an all-gather of G column shards
 *      produces, consumed without relayout.  a_kblock must divide K and, when
 *      != K, be a multiple of 128.
 *   B: int8 [N, K], K-major (the weight codes kz_quantize_cols_f32 writes).
 *   K must be a multiple of 16 (TMA row pitch); M, N, K > 0 otherwise ragged.
 *
 * Epilogue, fused (each step an fp32 operation, round to nearest):
 *   y = ((float)acc * row_scale[m * rs_stride]) * col_scale[n * cs_stride]
 *   y = y + bias[n]            (bias may be NULL)
 *   y = act(y)
 * rs_stride / cs_stride: 0 broadcasts one scale (per-tensor), 1 indexes it
 * (per-row / per-channel).  Scales may be NULL only when out_f32 is NULL.
 * Outputs (either may be NULL, not both): out_f32[M, ldo] = y and
 * out_i32[M, ldo] = acc.
 * absmax_partials (may be NULL): receives partial maxima of |y| in the
 * KZ_PARTIALS_WORDS format, so the output can be re-quantized per tensor by
 * kz_quantize_partials_f32 without another pass over it. */
int kz_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
               const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
               const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
               uint32_t* absmax_partials, kz_stream_t stream);

/* Caps the SMs that the int8 GEMMs launched on the current device afterwards
 * use (0, the default: every SM), so that a kernel running at the same time on
 * another stream -- an NCCL all-gather overlapped with the GEMM of the chunk
 * before it -- finds SMs free instead of waiting behind a persistent grid.
 * The same knob as cublasSetSmCountTarget.  No reference counterpart. */
int kz_set_sm_count_target(int sms);

/* kz_gemm_i8 with its A operand in the blocked layout [G][M][a_kblock]
 * (G = K / a_kblock <= 32) still being assembled while the kernel runs (no
 * reference counterpart; config 5's all-gather overlapped with the next
 * layer's GEMM).  Block first_block is resident at launch.  The other blocks
 * arrive in row chunks of flag_rows rows (a multiple of 128, or >= M for whole
 * blocks): before a tile's first load from rows chunk c of block g the TMA
 * producer waits until a_ready[g * C + c] (device memory, uint32,
 * C = ceil(M / flag_rows)) equals ready_token -- a bounded wait: after 1 s the
 * kernel records KZ_ERR_DEVICE_TIMEOUT and unwinds.  Every tile walks the K
 * blocks starting at first_block, so the GEMM computes on resident data while
 * the rest arrives (kz_copy_and_flag).  a_kblock must be a multiple of 128. */
int kz_gemm_i8_gated(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
                     const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
                     const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
                     uint32_t* absmax_partials, const uint32_t* a_ready, uint32_t ready_token, int first_block,
                     int64_t flag_rows, kz_stream_t stream);

/* Config 5's all-gather fused into the next layer's GEMM (no reference
 * counterpart).  Rank `rank` of `world` (2..8) holds the full A operand's
 * layout [world][M][K/world] in A (this GPU's memory), of which only block
 * `rank` is filled at launch.  peer_A[h] / peer_flags[h] (h != rank) are rank
 * h's own A buffer and flags array, mapped here with kz_peer_open (entry
 * `rank` ignored).  The launch's first copy_ctas CTAs (even, 2..32) push this
 * rank's block into every peer's A (stores into peer memory over NVLink) in
 * row chunks of
 * flag_rows rows (a multiple of 128 dividing M) and after each chunk write
 * `token` into every peer's flags[rank * (M / flag_rows) + c]; the other CTAs
 * run the GEMM of kz_gemm_i8_gated on the local flags (bounded waits, 1 s),
 * starting every tile at block `rank`.  flags (this rank's, zeroed once)
 * holds 2 * world * (M / flag_rows) words: the ready flags the peers write,
 * then this rank's per-chunk arrival counters, left at zero.  Every rank's
 * previous use of the A buffer must be finished before any rank launches (a
 * barrier).  fp32 output with fused rescale, act none. */
int kz_gemm_i8_allgather(const int8_t* A, int8_t* const* peer_A, uint32_t* const* peer_flags, int world, int rank,
                         const int8_t* B, int64_t M, int64_t N, int64_t K, const float* row_scale, int64_t rs_stride,
                         const float* col_scale, int64_t cs_stride, float* out_f32, int64_t ldo,
                         uint32_t* absmax_partials, uint32_t* flags, uint32_t token, int64_t flag_rows, int copy_ctas,
                         kz_stream_t stream);

/* ------------------------------------------------- peer exchange buffers
 * No reference counterpart (the reference's DTensor moves shards through host
 * lists, python/kansai/distributed.py:157-176).  One process per GPU: a rank
 * allocates device memory it will share (kz_peer_alloc: zero-filled cudaMalloc
 * plus a KZ_IPC_HANDLE_BYTES CUDA IPC handle), sends the handle to the other ranks
 * of the node, which map it (kz_peer_open: peer access over NVLink).  No
 * multicast object is created.  kz_peer_close unmaps a peer's buffer,
 * kz_peer_free releases one's own (after every peer closed it). */
#define KZ_IPC_HANDLE_BYTES 64
int kz_peer_alloc(size_t bytes, void** ptr, void* handle_out);
int kz_peer_open(const void* handle, void** ptr);
int kz_peer_close(void* ptr);
int kz_peer_free(void* ptr);

/* On `stream`: copy `bytes` from src (this GPU's memory or a peer's mapped by
 * kz_peer_open) to dst, then write `token` (< 65536) into *flag (a uint32 in
 * this GPU's memory), ordered after the copy's data.  Neither step uses an SM
 * (the copy runs on a copy engine, the flag is a stream memory write, or a
 * 4-byte copy from a pinned host table where the driver lacks that), so they
 * make progress while a kernel holding every SM waits on the flag -- the
 * producer side of kz_gemm_i8_gated.  bytes == 0 publishes the flag only. */
int kz_copy_and_flag(void* dst, const void* src, size_t bytes, uint32_t* flag, uint32_t token, kz_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KZ_H_ */
