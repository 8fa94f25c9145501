// quant.cuh -- quantiser entry points used by the C ABI.
#pragma once
#include "common.cuh"

namespace mb {

// Contiguous rows [R, C] -> int8 [R, C] with one scale per row
// (per-channel weights: R = N, C = K of a column-major [K,N] weight).
int quant_rows(int dtype, const void* x, int R, int C, int8_t* q, float* scale, cudaStream_t st);

// Activation x [M,K] (column-major, or row-major) -> int8 [M,K] row-major
// (K contiguous) with per-token scales x_scale[M] or one per-tensor scale.
int quant_activation(DeviceContext* ctx, int dtype, const void* x, int M, int K, int8_t* q,
                     float* scale, bool row_major, bool per_tensor, cudaStream_t st);

// |max| of every row of x [M,K] (row-major or column-major) -> out[M] (fp32).
int row_absmax(DeviceContext* ctx, int dtype, const void* x, int M, int K, float* out,
               bool row_major, cudaStream_t st);

// Per-row quantisation with caller-supplied row maxima (e.g. reduced across
// GPUs): scale[m] = 127 / row_max[m]; q row-major [M,K].
int quant_with_max(int dtype, const void* x, int M, int K, const float* row_max, int8_t* q,
                   float* scale, bool row_major, cudaStream_t st);

// Column-major per-token quantisation into caller-provided buffers, the row
// maxima included (no library scratch).
int quant_per_token_colmajor_into(int dtype, const void* x, int M, int K, int8_t* q, float* scale,
                                  uint32_t* amax_scratch, int num_sms, cudaStream_t st);

int write_scalar_scale(const uint32_t* amax, float* scale, cudaStream_t st);

// Row-major fp32 rows [R, C] -> int8 with scale[r] = 127 / max, the maxima
// given as fp32 bit patterns (e.g. accumulated by a GEMM epilogue).
int quant_rows_given_amax(const float* x, int R, int C, const uint32_t* amax, int8_t* q,
                          float* scale, cudaStream_t st);

}  // namespace mb
