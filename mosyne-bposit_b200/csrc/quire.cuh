// quire.cuh -- exact-sum and conversion entry points used by the C ABI.
#pragma once
#include "common.cuh"

namespace mb {

int quire_sum_bp16_run(DeviceContext* ctx, const uint16_t* x, size_t n, mosyne_quire256* q_out,
                       uint16_t* bp16_out, uint32_t* bp32_out, int flags, cudaStream_t st,
                       int max_blocks = 0);
// H = -sum over p of quire(term[p]) (the Shannon entropy of bposit16
// probabilities, exact up to the final encode), in one exact-sum launch.
int shannon_entropy_bp16_run(DeviceContext* ctx, const uint16_t* p, size_t n,
                             mosyne_quire256* q_out, uint16_t* bp16_out, uint32_t* bp32_out,
                             int flags, cudaStream_t st, int max_blocks = 0);
// The entropy's pre-decoded summands for the 32,768 probability codes
// (device init; term = the entropy term table); `usable` false when a
// negative code's term is not NaR (the staged mode then is not used).
int term_dec_build(const uint16_t* term, int* out, bool* usable);
// The exact sum's per-code decode on the device against the quire image of
// every bposit16 code: res[0] = mismatches, res[1] = the lowest failing code.
int sum_bin_check_run(unsigned long long* res, cudaStream_t st);
int fp32_atomic_sum_run(DeviceContext* ctx, const float* x, size_t n, float* acc,
                        cudaStream_t st);
int quire_to_bp_run(DeviceContext* ctx, const mosyne_quire256* q, size_t n, void* out, int nbits,
                    int rtne, cudaStream_t st);
int bp16_to_quire_run(DeviceContext* ctx, const uint16_t* x, size_t n, mosyne_quire256* out,
                      cudaStream_t st);
int int32_to_bp32_run(DeviceContext* ctx, const int32_t* in, size_t n, int shift, uint32_t* out,
                      int rtne, cudaStream_t st);
int float_to_bposit_run(DeviceContext* ctx, const void* x, int dtype, size_t n, void* out,
                        int nbits, int rtne, cudaStream_t st);

}  // namespace mb
