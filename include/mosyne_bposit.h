/* mosyne_bposit.h -- C ABI of libmosyne_bposit.so (B200 / sm_100a build).
 *
 * The first block is the reference's shipped ABI, symbol for symbol
 * (packages/mosyne_bposit/src/mosyne_bposit/_cuda/libmosyne_bposit.cu):
 * same names, argument meaning, layouts (column-major x[M,K], w[K,N],
 * y[M,N]), return codes, and stream semantics (legacy default stream, no
 * synchronisation).  Everything after it is an addition with no counterpart
 * in the reference's C ABI; each cites the reference code whose behaviour it
 * exposes.
 *
 * Return codes: 0 ok; -1 launch error; -2 GEMM launch failure; -10 library
 * not initialised; -11 scratch allocation failed; -20 invalid argument;
 * -30 a device-side wait gave up (see mosyne_bposit_last_error).
 *
 * All pointers are device pointers unless the name says _host.  bf16 and
 * fp16 buffers are passed as 16-bit words (binary compatible with
 * __nv_bfloat16 / __half).
 */
#ifndef MOSYNE_BPOSIT_H
#define MOSYNE_BPOSIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t mosyne_bf16_t;
typedef uint16_t mosyne_fp16_t;
typedef void* mosyne_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* 256-bit two's-complement fixed point, 96 fraction bits, little-endian
 * words (kernels/bposit16_encode.cuh:30). */
typedef struct mosyne_quire256 {
  uint64_t w[4];
} mosyne_quire256;

/* ------------------------------------------------------------------------
 * Reference ABI (libmosyne_bposit.cu)
 * ------------------------------------------------------------------------ */

/* libmosyne_bposit.cu:95 -- idempotent; 0 on success. */
int mosyne_bposit_init(void);

/* libmosyne_bposit.cu:145 -- frees all cached state; safe to repeat. */
void mosyne_bposit_shutdown(void);

/* libmosyne_bposit.cu:183 -- w column-major [K,N] fp32 -> int8 [K,N] and
 * w_scale[N] = 127/max|w[:,n]| (1.0 for an all-zero column).  Does not
 * require init. */
int mosyne_bposit_quantize_weight_per_channel(const float* w_fp32, int K, int N,
                                              int8_t* w_i8_out, float* w_scale_out);

/* libmosyne_bposit.cu:322 -- y[M,N] = (x_q @ w_i8) / (x_scale[m] * w_scale[n]),
 * per-token activation quantisation inside; all column-major. */
int mosyne_bposit_linear_w8a8(const float* d_x_fp32, int M, int K, const int8_t* d_w_i8,
                              const float* d_w_scale, int N, float* d_y_fp32);

/* libmosyne_bposit.cu:354 -- bf16 x, fp32 y. */
int mosyne_bposit_linear_w8a8_bf16(const mosyne_bf16_t* d_x_bf16, int M, int K,
                                   const int8_t* d_w_i8, const float* d_w_scale, int N,
                                   float* d_y_fp32);

/* libmosyne_bposit.cu:383 -- bf16 x, bf16 y. */
int mosyne_bposit_linear_w8a8_bf16_io(const mosyne_bf16_t* d_x_bf16, int M, int K,
                                      const int8_t* d_w_i8, const float* d_w_scale, int N,
                                      mosyne_bf16_t* d_y_bf16);

/* libmosyne_bposit.cu:412 -- fp16 x, fp32 y. */
int mosyne_bposit_linear_w8a8_fp16(const mosyne_fp16_t* d_x_fp16, int M, int K,
                                   const int8_t* d_w_i8, const float* d_w_scale, int N,
                                   float* d_y_fp32);

/* libmosyne_bposit.cu:440 -- fp16 x, fp16 y. */
int mosyne_bposit_linear_w8a8_fp16_io(const mosyne_fp16_t* d_x_fp16, int M, int K,
                                      const int8_t* d_w_i8, const float* d_w_scale, int N,
                                      mosyne_fp16_t* d_y_fp16);

/* libmosyne_bposit.cu:466 -- host round trip: auto-init, upload x and the fp32
 * weight, quantise the weight per call, run, copy y back (synchronous). */
int mosyne_bposit_linear_w8a8_host(const float* host_x, int M, int K, const float* host_w,
                                   int N, float* host_y);

/* ------------------------------------------------------------------------
 * Additions (no counterpart in the reference's C ABI)
 * ------------------------------------------------------------------------ */

/* dtype codes */
#define MOSYNE_DT_F32 0
#define MOSYNE_DT_BF16 1
#define MOSYNE_DT_F16 2
#define MOSYNE_DT_F64 3

/* flags */
#define MOSYNE_RTNE_BP32 0x1     /* bposit32 outputs round to nearest even (default: truncate) */
#define MOSYNE_RTNE_BP16 0x2     /* bposit16 outputs round to nearest even (default: truncate) */
#define MOSYNE_XS_SCALAR 0x4     /* x_scale is one value (per-tensor) */
#define MOSYNE_WS_SCALAR 0x8     /* w_scale is one value (per-tensor) */
#define MOSYNE_OUT_ROW_MAJOR 0x10 /* outputs row-major [M,N] instead of column-major */
#define MOSYNE_X_ROW_MAJOR 0x20  /* linear: x is row-major [M,K] instead of column-major */
#define MOSYNE_X_PER_TENSOR 0x40 /* linear: one activation scale for the whole x */
/* gemm_i8: the bposit outputs encode acc / 2^s (s = 0..31) instead of acc,
 * the scale_shift of kernels/test_int32_to_bposit32.cu:94-126; the bposit8
 * path (int8 operands with 6 fraction bits each) uses s = 12. */
#define MOSYNE_BP_SHIFT(s) ((((unsigned)(s)) & 31u) << 24)

/* Version string of this build. */
const char* mosyne_bposit_version(void);

/* Synchronises the current device and reports (then clears) the device error
 * word: 0 if every device-side wait completed, -30 if one gave up, or a CUDA
 * error as -1. */
int mosyne_bposit_last_error(void);

/* No counterpart in the reference (cuBLASLt's SM-count target plays this role
 * there): the GEMMs of the current device launch on at most `sms` SMs from
 * now on (0 or >= the device's count: all), leaving the others to kernels
 * that run beside them -- e.g. the collectives of a K-split, which then
 * overlap the next chunk's GEMM.  Per device; not thread-safe. */
int mosyne_bposit_set_sm_count_target(int sms);

/* Diagnostic: launches one bounded device-side wait that nothing satisfies;
 * it gives up after limit_ns (capped at 2 s) and sets the device error word,
 * so the next mosyne_bposit_last_error() returns -30.  Exercises the
 * give-up path of every pipeline wait without hanging the GPU. */
int mosyne_bposit_debug_wait_timeout(unsigned long long limit_ns, mosyne_stream_t stream);

/* Fused INT8 GEMM, kernels/test_mera_isometry_imma.cu:277-352 (cuBLASLt GEMM
 * + int32 -> bposit32 epilogue) and libmosyne_bposit.cu:252-319 (IMMA +
 * dequant) in one tcgen05 kernel:
 *   acc[m,n] = sum_k A[m,k] * B[n,k]          (exact INT32)
 *   out_bp32 = bposit32(acc)   == quire256_to_bposit32(acc << 96)
 *   out_bp16 = bposit16(acc)
 *   (acc / 2^s for both with flags MOSYNE_BP_SHIFT(s))
 *   out_f32  = (float)acc / (x_scale[m] * w_scale[n])
 *   out_i32  = acc
 * A is [M,K] with K contiguous; B is [N,K] with K contiguous (= column-major
 * [K,N]).  Any output pointer may be NULL (skipped).  Outputs are
 * column-major [M,N] unless MOSYNE_OUT_ROW_MAJOR.  y_dtype selects the
 * dequant output type (MOSYNE_DT_F32/BF16/F16) written to out_y. */
int mosyne_bposit_gemm_i8(const int8_t* A, const int8_t* B, int M, int N, int K,
                          const float* x_scale, const float* w_scale, uint32_t* out_bp32,
                          uint16_t* out_bp16, void* out_y, int y_dtype, int32_t* out_i32,
                          int flags, mosyne_stream_t stream);

/* A batch of independent GEMMs of the same shape (attention scores Q K^T
 * per head: kernels/test_ffn_layer_* shapes of the C4 QK^T workload):
 * A [batch][M][K], B [batch][N][K] (K contiguous), x_scale [batch][M] and
 * w_scale [batch][N] (or single values with the SCALAR flags), each output
 * [batch] x ([M,N] column- or row-major) contiguous per batch entry.  Same
 * outputs and flags as mosyne_bposit_gemm_i8 for every entry. */
int mosyne_bposit_gemm_i8_batched(const int8_t* A, const int8_t* B, int batch, int M, int N,
                                  int K, const float* x_scale, const float* w_scale,
                                  uint32_t* out_bp32, uint16_t* out_bp16, void* out_y,
                                  int y_dtype, int32_t* out_i32, int flags,
                                  mosyne_stream_t stream);

/* Host-buffer round trip of mosyne_bposit_gemm_i8 (A, B and outputs in host
 * memory; synchronous), the end-to-end form of the GEMM. */
int mosyne_bposit_gemm_i8_host(const int8_t* A, const int8_t* B, int M, int N, int K,
                               uint32_t* out_bp32, int32_t* out_i32, int flags);

/* W8A8 linear with every option: x dtype (MOSYNE_DT_*), x layout
 * (MOSYNE_X_ROW_MAJOR), per-token or per-tensor activation scale
 * (MOSYNE_X_PER_TENSOR), dequant output y (y_dtype; may be NULL), raw
 * dot-product bposit32/bposit16 outputs (may be NULL), stream.  The
 * reference's five device entry points are this call with fixed options. */
int mosyne_bposit_linear_w8a8_ex(const void* x, int x_dtype, int M, int K,
                                 const int8_t* w_i8, const float* w_scale, int N,
                                 void* y, int y_dtype, uint32_t* y_bp32, uint16_t* y_bp16,
                                 int flags, mosyne_stream_t stream);

/* libmosyne_bposit.cu:206-244: per-token quantisation of x [M,K] (column-major,
 * or row-major with MOSYNE_X_ROW_MAJOR) to x_i8 [M,K] with K contiguous and
 * x_scale[M]. */
int mosyne_bposit_quantize_per_token(const void* x, int x_dtype, int M, int K, int8_t* x_i8,
                                     float* x_scale, int flags, mosyne_stream_t stream);

/* Per-tensor quantisation (scale = 127/max|t|, the per-token convention) of a
 * [rows, cols] tensor.  With MOSYNE_X_ROW_MAJOR the input is row-major,
 * otherwise column-major; the output is always row-major [rows, cols]
 * (K contiguous when rows = M, cols = K). */
int mosyne_bposit_quantize_per_tensor(const void* t, int dtype, int rows, int cols,
                                      int8_t* q, float* scale, int flags,
                                      mosyne_stream_t stream);

/* Per-row |max| of x [M,K] (column-major, or row-major with
 * MOSYNE_X_ROW_MAJOR) into row_max[M] -- the first half of the per-token
 * quantiser (libmosyne_bposit.cu:215-233), exposed so a K-split across GPUs
 * can reduce the maxima before quantising (max is exact and order free). */
int mosyne_bposit_row_absmax(const void* x, int x_dtype, int M, int K, float* row_max, int flags,
                             mosyne_stream_t stream);

/* The second half (libmosyne_bposit.cu:234-243) with caller-supplied row
 * maxima: x_scale[m] = 127/row_max[m], x_i8 [M,K] K contiguous. */
int mosyne_bposit_quantize_with_max(const void* x, int x_dtype, int M, int K, const float* row_max,
                                    int8_t* x_i8, float* x_scale, int flags,
                                    mosyne_stream_t stream);

/* libmosyne_bposit.cu:162-193 on a stream, for fp32/bf16/fp16 weights. */
int mosyne_bposit_quantize_weight_per_channel_ex(const void* w, int dtype, int K, int N,
                                                 int8_t* w_i8_out, float* w_scale_out,
                                                 mosyne_stream_t stream);

/* Exact (order independent) sum of n bposit16 codes in quire256
 * (kernels/test_determinism_headline.cu:65-97, shannon_entropy_bposit16.cu:
 * 45-119): writes the quire and its bposit16 / bposit32 encodings (any output
 * may be NULL).  flags: MOSYNE_RTNE_BP16 / MOSYNE_RTNE_BP32. */
int mosyne_bposit_quire_sum_bp16(const uint16_t* x, size_t n, mosyne_quire256* q_out,
                                 uint16_t* bp16_out, uint32_t* bp32_out, int flags,
                                 mosyne_stream_t stream);

/* Shannon entropy H = -sum_i p_i log2(p_i) of n bposit16 probabilities
 * (kernels/shannon_entropy_bposit16.cu:63-119; bposit16_reference.py:813-824):
 * every p is mapped through the term table bposit16(p * log2(p))
 * (build_bposit_luts.py:102-110), the negated terms are summed exactly in
 * quire256 in one grid-wide launch, and the quire is written with its
 * bposit32 / bposit16 encodings (any output may be NULL; truncating unless
 * MOSYNE_RTNE_BP32 / MOSYNE_RTNE_BP16).  Asynchronous on `stream`; n == 0
 * gives H = 0.  Returns 0 or a negative MOSYNE_RC_* code. */
int mosyne_bposit_shannon_entropy_bp16(const uint16_t* p, size_t n, mosyne_quire256* q_out,
                                       uint32_t* bp32_out, uint16_t* bp16_out, int flags,
                                       mosyne_stream_t stream);

/* The reference's entropy entry point, same name, arguments and return codes
 * (kernels/shannon_entropy_bposit16.cu:124-146): d_p and d_out are device
 * pointers, *d_out = bposit32(H) (truncating quire256 -> bposit32).  Returns
 * -1 for n == 0, -2 when the library cannot set up the device, -3 on a launch
 * or execution error, 0 on success.  Like the reference (whose cudaFree of its
 * scratch waits for the device), it returns once the result is written: it
 * runs on the legacy default stream and synchronises it. */
int shannon_entropy_bposit16_cuda(const uint16_t* d_p, size_t n, uint32_t* d_out);

/* kernels/test_determinism_headline.cu:56-60: fp32 atomicAdd control sum
 * into *acc (not zeroed by the call). */
int mosyne_bposit_fp32_atomic_sum(const float* x, size_t n, float* acc, mosyne_stream_t stream);

/* kernels/bposit16_encode.cuh:113-418: element-wise quire256 -> bposit. */
int mosyne_bposit_quire_to_bp16(const mosyne_quire256* q, size_t n, uint16_t* out, int rtne,
                                mosyne_stream_t stream);
int mosyne_bposit_quire_to_bp32(const mosyne_quire256* q, size_t n, uint32_t* out, int rtne,
                                mosyne_stream_t stream);

/* kernels/bposit16_encode.cuh:424-431: element-wise bposit16 -> quire256. */
int mosyne_bposit_bp16_to_quire(const uint16_t* x, size_t n, mosyne_quire256* out,
                                mosyne_stream_t stream);

/* kernels/test_int32_to_bposit32.cu:94-126: value = in / 2^scale_shift. */
int mosyne_bposit_int32_to_bp32(const int32_t* in, size_t n, int scale_shift, uint32_t* out,
                                int rtne, mosyne_stream_t stream);

/* The W8A8 SwiGLU FFN of kernels/test_ffn_layer_real_qwen.cu:300-334
 * (per-token int8 x, gate and up IMMA + dequant, silu(gate) * up in fp32 with
 * silu(v) = v / (1 + expf(-v)), per-token re-quantisation, down IMMA +
 * dequant) in four launches:
 *   x       row-major [M, D] (MOSYNE_DT_F32/BF16/F16)
 *   w_gu_i8 [2F, D] int8 (K contiguous): gate and up weights quantised per
 *           channel and interleaved in blocks of 32 channels -- rows
 *           64b .. 64b+31 are gate channels 32b .. 32b+31, rows 64b+32 ..
 *           64b+63 the same up channels; w_gu_scale [2F] likewise
 *   w_down_i8 [D, F] int8 (K contiguous), w_down_scale [D]
 *   y       row-major [M, D] of y_dtype
 *   act     optional fp32 row-major [M, F] output of the activation (NULL:
 *           library scratch)
 * F must be a multiple of 32 and D, F multiples of 16.  flags: reserved (0). */
int mosyne_bposit_ffn_swiglu_w8a8(const void* x, int x_dtype, int M, int D,
                                  const int8_t* w_gu_i8, const float* w_gu_scale, int F,
                                  const int8_t* w_down_i8, const float* w_down_scale, void* y,
                                  int y_dtype, float* act, int flags, mosyne_stream_t stream);

/* kernels/test_mera_isometry_imma.cu:43-69, 166-197: bposit8 codes -> int8
 * fixed point with 6 fraction bits, clamp(floor(value * 64), -128, 127); NaR
 * and zero give 0.  The decode pass of the bposit8 IMMA path. */
int mosyne_bposit_bposit8_to_int8(const uint8_t* in, size_t n, int8_t* out,
                                  mosyne_stream_t stream);

/* kernels/test_mera_isometry_imma.cu:224-352 (the bposit8 IMMA path) as one
 * call: bposit8 A [M,K] and B [N,K] (K contiguous) are decoded to int8 (6
 * fraction bits) in one launch into library scratch, then the fused GEMM
 * writes bposit32 of acc / 2^12 (truncate, or RTNE with MOSYNE_RTNE_BP32)
 * and/or the raw INT32 accumulator; column-major [M,N] unless
 * MOSYNE_OUT_ROW_MAJOR.  Calls share the scratch: order them on one stream. */
int mosyne_bposit_gemm_bposit8(const uint8_t* A, const uint8_t* B, int M, int N, int K,
                               uint32_t* out_bp32, int32_t* out_i32, int flags,
                               mosyne_stream_t stream);

/* kernels/bposit16_reference.py:485-503 (exact value of each binary float):
 * x of dtype MOSYNE_DT_F32 or MOSYNE_DT_F64 -> bposit16 (nbits 16, uint16
 * out) or bposit32 (nbits 32, uint32 out). */
int mosyne_bposit_float_to_bposit(const void* x, int dtype, size_t n, void* out, int nbits,
                                  int rtne, mosyne_stream_t stream);

/* Standalone W8A8 epilogue over an INT32 accumulator acc [M,N] (column-major),
 * used after an exact cross-GPU INT32 reduction (K-split): same outputs and
 * flags as mosyne_bposit_gemm_i8. */
int mosyne_bposit_epilogue_i32(const int32_t* acc, int M, int N, const float* x_scale,
                               const float* w_scale, uint32_t* out_bp32, uint16_t* out_bp16,
                               void* out_y, int y_dtype, int flags, mosyne_stream_t stream);

/* No counterpart in the reference (its quire argument, whitepaper.tex:495-507,
 * at the width the value needs): exact INT64 accumulators for sums of INT32
 * partials that may exceed INT32 -- the K-split across GPUs when
 * 127^2 * K >= 2^31.  widen: dst[i] = (int64) src[i], or dst[i] += src[i]
 * with accumulate != 0.  epilogue_i64: as mosyne_bposit_epilogue_i32 over an
 * INT64 accumulator acc [M,N] (column-major); bposit outputs encode
 * acc / 2^s with flags MOSYNE_BP_SHIFT(s), y = (float)acc / (xs[m] * ws[n]). */
int mosyne_bposit_widen_i32(const int32_t* src, size_t n, int64_t* dst, int accumulate,
                            mosyne_stream_t stream);
int mosyne_bposit_epilogue_i64(const int64_t* acc, int M, int N, const float* x_scale,
                               const float* w_scale, uint32_t* out_bp32, uint16_t* out_bp16,
                               void* out_y, int y_dtype, int flags, mosyne_stream_t stream);

/* bposit16 ALU, element-wise over n codes.
 * add: kernels/bposit16_encode.cuh:472-483 (exact via quire256);
 * mul: bposit16_encode.cuh:491-537 (log2 + quire add + exp2 tables);
 * mul_exact: kernels/bposit16_reference.py:507-516 (exact product, truncated);
 * neg: bposit16_encode.cuh:437-443 (two's complement) or, with
 *      ones_complement != 0, 461-467;
 * recip/sqrt/log2/exp2: the 65,536-entry tables of
 *      kernels/build_bposit_luts.py:34-259. */
int mosyne_bposit16_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,
                        mosyne_stream_t stream);
int mosyne_bposit16_mul(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,
                        mosyne_stream_t stream);
int mosyne_bposit16_mul_exact(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,
                              mosyne_stream_t stream);
int mosyne_bposit16_neg(const uint16_t* a, size_t n, uint16_t* out, int ones_complement,
                        mosyne_stream_t stream);
int mosyne_bposit16_recip(const uint16_t* a, size_t n, uint16_t* out, mosyne_stream_t stream);
int mosyne_bposit16_sqrt(const uint16_t* a, size_t n, uint16_t* out, mosyne_stream_t stream);
int mosyne_bposit16_log2(const uint16_t* a, size_t n, uint16_t* out, mosyne_stream_t stream);
int mosyne_bposit16_exp2(const uint16_t* a, size_t n, uint16_t* out, mosyne_stream_t stream);

/* Return code: the input does not fit the fixed scratch of
 * mosyne_bposit_linear_w8a8_noalloc. */
#define MOSYNE_RC_SCRATCH_LIMIT (-21)

/* No counterpart in the reference: mosyne_bposit_linear_w8a8 that allocates
 * no device memory, for callers that cannot call cudaMalloc (a serving
 * process whose device memory belongs to a caching allocator or is capped, a
 * plugin host that forbids raw allocations, code that must avoid the device
 * synchronisation an allocation can cause).  Same arguments, layouts and
 * results as mosyne_bposit_linear_w8a8, plus a stream; needs no
 * mosyne_bposit_init.  Its scratch is one fixed static device array (about
 * 8.1 MiB, held by every GPU that loads the library until exit): M <= 16384
 * and M*K <= 8 MiB, else -21.  The first call on each device looks that array
 * up (cudaGetSymbolAddress) and should come before any stream capture;
 * cudaDeviceReset on a device that has used it is not supported (the looked-up
 * address is kept for the life of the process).  All calls share the array:
 * calls that may overlap on the GPU race, so order them on one stream.  The
 * return code covers arguments and launches; a device-side wait that gave up
 * (a wrong y) is reported afterwards by mosyne_bposit_last_error() as -30. */
int mosyne_bposit_linear_w8a8_noalloc(const float* d_x_fp32, int M, int K, const int8_t* d_w_i8,
                                      const float* d_w_scale, int N, float* d_y_fp32,
                                      mosyne_stream_t stream);

/* Test hook, no counterpart in the reference: the bounded wait that nothing
 * satisfies (as mosyne_bposit_debug_wait_timeout), recording into the error
 * word of mosyne_bposit_linear_w8a8_noalloc, so a test can see a give-up on
 * that path reported by mosyne_bposit_last_error().  Allocates nothing. */
int mosyne_bposit_debug_noalloc_wait_timeout(unsigned long long limit_ns, mosyne_stream_t stream);

/* Copies one of the device-resident ALU tables (0 log2, 1 exp2, 2 sqrt,
 * 3 recip; 65,536 u16) to host memory, for verification. */
int mosyne_bposit16_table_host(int which, uint16_t* host_out);

/* Test hook, no counterpart in the reference: runs the bposit16 ALU's 32-bit
 * forms -- op 0 the adder (mosyne_bposit16_add), 1 the exact multiplier
 * (mosyne_bposit16_mul_exact), 2 the truncated quire sum of two codes, 3 the
 * log2/exp2 multiplier (mosyne_bposit16_mul) -- and their int64 forms on
 * every one of the 2^32 pairs of codes, and writes host_out[0] = the number of pairs where they
 * differ, host_out[1] = the first such pair (a << 16 | b; ~0 when none).
 * op 4: the GEMM epilogue's slow-path-free dequant division against the
 * IEEE division on 2^32 pseudo-random operand pairs (host_out[1] = the first
 * differing pair's index); op 5: the same for the SwiGLU epilogue's
 * x / (1 + expf(-x)) operands; op 6: that division's reciprocal step against
 * the correctly rounded reciprocal on every normal divisor in [2^-110, 2^111)
 * (host_out[1] = the bits of the first differing one); op 7: the exact sum's per-code decode
 * (regime and integer value within the regime) against the quire image of every bposit16
 * code (host_out[1] = the first differing code).  Synchronous; allocates 16 bytes of device
 * memory. */
int mosyne_bposit_debug_alu_check(int op, unsigned long long* host_out);

#ifdef __cplusplus
}
#endif

#endif /* MOSYNE_BPOSIT_H */
