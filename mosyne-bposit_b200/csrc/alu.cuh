// alu.cuh -- bposit16 ALU entry point used by the C ABI.
#pragma once
#include "common.cuh"

namespace mb {

enum AluOp {
  ALU_ADD = 0,
  ALU_MUL = 1,
  ALU_MUL_EXACT = 2,
  ALU_NEG = 3,
  ALU_NEG_ONES = 4,
  ALU_LOG2 = 5,
  ALU_EXP2 = 6,
  ALU_SQRT = 7,
  ALU_RECIP = 8,
};

int alu_run(DeviceContext* ctx, int op, const uint16_t* a, const uint16_t* b, size_t n,
            uint16_t* out, cudaStream_t st);

}  // namespace mb
