// Host build of the library's encoder header (mosyne-bposit_b200/csrc/bposit.cuh)
// for CPU tests: the same source the kernels compile, exercised without a GPU.
#include <cstddef>
#include <cstdint>

#include "bposit.cuh"

extern "C" {

void h_from_int64(const int64_t* I, const int32_t* shift, size_t n, int nbits, int rtne,
                  uint32_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = nbits == 16 ? bp::from_int64<16>(I[i], shift[i], rtne) : bp::from_int64<32>(I[i], shift[i], rtne);
}

void h_from_int32(const int32_t* I, size_t n, int nbits, int rtne, uint32_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = nbits == 16 ? bp::from_int32<16>(I[i], rtne) : bp::from_int32<32>(I[i], rtne);
}

void h_from_int32_tab(const int32_t* I, size_t n, int nbits, int rtne, uint32_t* out, int shift) {
  bp::I32Entry t16[33], t32[33];
  for (int i = 0; i < 33; ++i) {
    t16[i] = bp::i32_table_entry<16>(i, shift);
    t32[i] = bp::i32_table_entry<32>(i, shift);
  }
  for (size_t i = 0; i < n; ++i) {
    if (nbits == 16)
      out[i] = rtne ? bp::from_int32_tab<16, true>(I[i], t16) : bp::from_int32_tab<16, false>(I[i], t16);
    else
      out[i] = rtne ? bp::from_int32_tab<32, true>(I[i], t32) : bp::from_int32_tab<32, false>(I[i], t32);
  }
}

void h_bp8_to_i8(int8_t* out) {
  for (int i = 0; i < 256; ++i) out[i] = bp::bposit8_to_int8((uint32_t)i);
}

void h_from_quire(const uint64_t* w, size_t n, int nbits, int rtne, uint32_t* out) {
  for (size_t i = 0; i < n; ++i) {
    bp::quire256 q{{w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]}};
    out[i] = nbits == 16 ? bp::from_quire<16>(q, rtne) : bp::from_quire<32>(q, rtne);
  }
}

void h_bp16_to_quire(const uint16_t* p, size_t n, uint64_t* w) {
  for (size_t i = 0; i < n; ++i) {
    const bp::quire256 q = bp::quire_from_bp16(p[i]);
    for (int j = 0; j < 4; ++j) w[4 * i + j] = q.w[j];
  }
}

void h_from_double(const double* x, size_t n, int nbits, int rtne, uint32_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = nbits == 16 ? bp::from_double<16>(x[i], rtne) : bp::from_double<32>(x[i], rtne);
}

void h_quire_sum(const uint16_t* p, size_t n, uint64_t* w) {
  bp::quire256 acc = bp::q_zero();
  for (size_t i = 0; i < n; ++i) acc = bp::q_add(acc, bp::quire_from_bp16(p[i]));
  for (int j = 0; j < 4; ++j) w[j] = acc.w[j];
}
}
