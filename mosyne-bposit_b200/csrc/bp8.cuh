// bp8.cuh -- bposit8 -> int8 decode entry point used by the C ABI.
#pragma once
#include "common.cuh"

namespace mb {

int bp8_to_i8_run(const uint8_t* in, size_t n, int8_t* out, int num_sms, cudaStream_t st);
// Two byte stretches (a GEMM's A and B operands) in one launch.
int bp8_to_i8_pair_run(const uint8_t* in0, size_t n0, int8_t* out0, const uint8_t* in1,
                       size_t n1, int8_t* out1, int num_sms, cudaStream_t st);

}  // namespace mb
