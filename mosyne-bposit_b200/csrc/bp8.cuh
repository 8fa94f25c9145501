// bp8.cuh -- bposit8 -> int8 decode entry point used by the C ABI.
#pragma once
#include "common.cuh"

namespace mb {

int bp8_to_i8_run(const uint8_t* in, size_t n, int8_t* out, int num_sms, cudaStream_t st);

}  // namespace mb
