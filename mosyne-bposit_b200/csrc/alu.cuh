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
// The values (exact floats, as the quire holds them) of the 32,768 bposit16
// magnitude codes the adder reads, and of the log2 table's entries for them
// the multiplier reads (device init; lg = the log2 table).
int alu_build_dec16(uint32_t* out, uint32_t* log_out, const uint16_t* lg);
// Exhaustive equivalence of the fast adder (op 0), exact multiplier (1),
// quire sum (2) and log/exp multiplier (3) with their int64 forms over all
// 2^32 code pairs: res[0] += mismatches, res[1] = min(first mismatching pair
// index) (the caller zeroes res[0] and sets res[1] to ~0).
int alu_check_run(DeviceContext* ctx, int op, unsigned long long* res, cudaStream_t st);

}  // namespace mb
