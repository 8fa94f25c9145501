// gemm.cuh -- fused INT8 GEMM / epilogue interface shared by the C ABI.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace mb {

// Outputs of the fused epilogue for acc[m,n] (exact INT32):
//   bp32 = bposit32(acc), bp16 = bposit16(acc), i32 = acc,
//   y    = (float)acc / (xs[m*xs_stride] * ws[n*ws_stride]) in y_dtype.
// Null pointers are skipped.  Index: row_major ? m*N + n : n*M + m.
struct EpiParams {
  int M = 0, N = 0;
  const float* xs = nullptr;
  const float* ws = nullptr;
  int xs_stride = 1, ws_stride = 1;
  uint32_t* bp32 = nullptr;
  uint16_t* bp16 = nullptr;
  void* y = nullptr;
  int y_dtype = MOSYNE_DT_F32;
  int32_t* i32 = nullptr;
  int row_major = 0;
  int rtne32 = 0, rtne16 = 0;
  int bp_shift = 0;        // bposit outputs encode acc / 2^bp_shift (0..31)
  // SwiGLU mode (set together with an fp32 y): the N columns come in blocks of
  // 64, 32 gate channels then the same 32 up channels; y receives the
  // row-major [M, N/2] activation silu(gate) * up and act_amax[m] the bit
  // pattern of max |activation| of row m (atomicMax; must start at zero).
  uint32_t* act_amax = nullptr;
  // Batched GEMM (CTA-pair kernel with TMA-store outputs only): A [batch][M][K],
  // B [batch][N][K], outputs and scales contiguous per entry.
  int batch = 1;
  // The GEMM may read B before the kernel it depends on (programmatic
  // dependent launch) has finished: B was final when that kernel started.
  // The single-CTA kernel then prefetches its B tiles into L2 first thing.
  int b_prefetch = 0;
};

enum GemmPath {
  GEMM_PATH_AUTO = 0,
  GEMM_PATH_TC = 1,        // tensor-core path, tile width chosen by shape
  GEMM_PATH_TC_BN128 = 2,
  GEMM_PATH_TC_BN256 = 3,
  GEMM_PATH_SIMT = 4,
  GEMM_PATH_TC_PAIR = 5,   // CTA-pair (cta_group::2) 256x256 tiles
};

// acc = A[M,K] (K contiguous) x B[N,K]^T (K contiguous), fused epilogue.
int gemm_i8_run(const int8_t* A, const int8_t* B, int K, const EpiParams& p,
                DeviceContext* ctx, cudaStream_t st, int force_path = GEMM_PATH_AUTO);

// Same epilogue over a column-major INT32 accumulator.
int epilogue_i32_run(const int32_t* acc, const EpiParams& p, DeviceContext* ctx,
                     cudaStream_t st);

// INT64 accumulators (wide.cu): dst (+)= (int64) src over n elements, and the
// epilogue over a column-major INT64 accumulator (bposit of acc / 2^bp_shift,
// (float)acc / (xs * ws) dequant).
int widen_i32_run(const int32_t* src, size_t n, int64_t* dst, int add, DeviceContext* ctx,
                  cudaStream_t st);
int epilogue_i64_run(const int64_t* acc, const EpiParams& p, DeviceContext* ctx, cudaStream_t st);

// Bounded wait that nothing satisfies; sets the device error word.
// n 32-bit words of device memory set to zero by a kernel (orders correctly
// before the programmatic-dependent GEMM launches, unlike a memset node).
int zero_words_run(uint32_t* p, size_t n, cudaStream_t st);

// All p.batch entries in one CTA-pair launch; RC_BAD_ARG when the shape or the
// outputs need the per-entry path (the caller then launches entry by entry).
int gemm_i8_batched_fused(const int8_t* A, const int8_t* B, int K, const EpiParams& p,
                          DeviceContext* ctx, cudaStream_t st);

int debug_wait_run(unsigned long long limit_ns, DeviceContext* ctx, cudaStream_t st);

// The epilogue's slow-path-free division against __fdiv_rn on 2^32
// pseudo-random operand pairs of the dequant (which 0) or of silu's divide
// (1), or its reciprocal step against __frcp_rn on every normal divisor in
// [2^-110, 2^111) (2): res[0] += mismatches, res[1] = min(first index or bits).
int div_check_run(DeviceContext* ctx, unsigned long long* res, cudaStream_t st, int which);

// Error word of the allocation-free entry point on the current device: read
// and cleared; RC_DEVICE_TIMEOUT when a bounded wait there gave up.
int noalloc_take_error();

}  // namespace mb
