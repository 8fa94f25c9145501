// Host build of the library's encoder header (mosyne-bposit_b200/csrc/bposit.cuh)
// for CPU tests: the same source the kernels compile, exercised without a GPU.
#include <cstring>
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

void h_from_quire_sel(const uint64_t* w, size_t n, int nbits, int rtne, uint32_t* out) {
  for (size_t i = 0; i < n; ++i) {
    bp::quire256 q{{w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]}};
    out[i] = nbits == 16 ? bp::from_quire_sel<16>(q, rtne) : bp::from_quire_sel<32>(q, rtne);
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

void h_from_float(const float* x, size_t n, int nbits, int rtne, uint32_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = nbits == 16 ? bp::from_float<16>(x[i], rtne) : bp::from_float<32>(x[i], rtne);
}

// Mismatches of the int64 sum (bp::sum16_trunc) against the quire path over
// every code a paired with each b in bs, and with the codes next to -a and a
// (cancellation and doubling).
size_t h_sum16_check(const uint16_t* bs, size_t nb) {
  auto ref = [](uint32_t a, uint32_t b) {
    return bp::from_quire<16>(bp::q_add(bp::quire_from_bp16(a), bp::quire_from_bp16(b)), false);
  };
  size_t bad = 0;
  for (uint32_t a = 0; a < 65536; ++a) {
    for (size_t j = 0; j < nb; ++j)
      if (bp::sum16_trunc(a, bs[j]) != ref(a, bs[j])) ++bad;
    const uint32_t na = (0u - a) & 0xFFFFu;
    for (int d = -3; d <= 3; ++d) {
      const uint32_t b1 = (na + (uint32_t)d) & 0xFFFFu, b2 = (a + (uint32_t)d) & 0xFFFFu;
      if (bp::sum16_trunc(a, b1) != ref(a, b1)) ++bad;
      if (bp::sum16_trunc(a, b2) != ref(a, b2)) ++bad;
    }
  }
  return bad;
}

// Mismatches of the floating-point sum (bp::sum16_trunc_f32 of the quire
// values) and of the 32-bit exact product (bp::mul16_trunc_dec) against the
// int64 forms, over every code a paired with each b in bs and with the codes
// next to -a and a.
size_t h_alu32_check(const uint16_t* bs, size_t nb) {
  bp::S16Entry st[256];
  for (int i = 0; i < 256; ++i) st[i] = bp::s16_table_entry(i);
  auto mul_ref = [](uint32_t a, uint32_t b) -> uint32_t {
    const bp::Dec16 da = bp::decode16(a), db = bp::decode16(b);
    if (da.zero || db.zero) return 0u;
    if (da.nar || db.nar) return 0x8000u;
    const int64_t m = (int64_t)da.mant * (int64_t)db.mant;
    return bp::from_int64<16>((da.neg != db.neg) ? -m : m, -(da.exp2 + db.exp2), false);
  };
  auto mul_fast = [](uint32_t a, uint32_t b) -> uint32_t {
    const bp::Dec16 da = bp::decode16(a), db = bp::decode16(b);
    if (da.zero || db.zero) return 0u;
    if (da.nar || db.nar) return 0x8000u;
    return bp::mul16_trunc_dec(da, db);
  };
  size_t bad = 0;
  auto one = [&](uint32_t a, uint32_t b) {
    if (bp::sum16_trunc_f32(bp::quire_value16(a), bp::quire_value16(b), st) != bp::sum16_trunc(a, b))
      ++bad;
    if ((mul_fast(a, b) & 0xFFFFu) != (mul_ref(a, b) & 0xFFFFu)) ++bad;
  };
  for (uint32_t a = 0; a < 65536; ++a) {
    for (size_t j = 0; j < nb; ++j) one(a, bs[j]);
    const uint32_t na = (0u - a) & 0xFFFFu;
    for (int d = -3; d <= 3; ++d) {
      one(a, (na + (uint32_t)d) & 0xFFFFu);
      one(a, (a + (uint32_t)d) & 0xFFFFu);
    }
  }
  return bad;
}

// Mismatches of the floating-point sum against the int64 sum over all 2^32
// pairs of codes (threads when built with OpenMP).
size_t h_sum16_f32_exhaustive() {
  bp::S16Entry st[256];
  for (int i = 0; i < 256; ++i) st[i] = bp::s16_table_entry(i);
  size_t bad = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : bad)
  for (int a = 0; a < 65536; ++a) {
    const float fa = bp::quire_value16((uint32_t)a);
    for (uint32_t b = 0; b < 65536; ++b)
      if (bp::sum16_trunc_f32(fa, bp::quire_value16(b), st) != bp::sum16_trunc((uint32_t)a, b)) ++bad;
  }
  return bad;
}

// Mismatches of the two-half 32-bit bposit16 -> quire conversion against
// quire_from_bp16 over every code.
size_t h_quire_half_check() {
  size_t bad = 0;
  for (uint32_t c = 0; c < 65536; ++c) {
    const bp::quire256 q = bp::quire_from_bp16(c);
    for (int h = 0; h < 2; ++h) {
      uint32_t w[4];
      bp::quire_half_bp16(c, h, w);
      const uint64_t lo = (uint64_t)w[0] | ((uint64_t)w[1] << 32), hi = (uint64_t)w[2] | ((uint64_t)w[3] << 32);
      if (lo != q.w[2 * h] || hi != q.w[2 * h + 1]) ++bad;
    }
  }
  return bad;
}

void h_from_float_tab(const float* x, size_t n, int nbits, int rtne, uint32_t* out) {
  bp::F32Entry t16[256], t32[256];
  for (int i = 0; i < 256; ++i) {
    t16[i] = bp::f32_table_entry<16>(i);
    t32[i] = bp::f32_table_entry<32>(i);
  }
  for (size_t i = 0; i < n; ++i) {
    if (nbits == 16)
      out[i] = rtne ? bp::from_float_tab<16, true>(x[i], t16) : bp::from_float_tab<16, false>(x[i], t16);
    else
      out[i] = rtne ? bp::from_float_tab<32, true>(x[i], t32) : bp::from_float_tab<32, false>(x[i], t32);
  }
}

// Mismatches of the table encoder against the direct float encoder over every
// float bit pattern, bposit16 and bposit32, truncate and RTNE (threads when
// built with OpenMP).
size_t h_from_float_tab_exhaustive() {
  bp::F32Entry t16[256], t32[256];
  for (int i = 0; i < 256; ++i) {
    t16[i] = bp::f32_table_entry<16>(i);
    t32[i] = bp::f32_table_entry<32>(i);
  }
  size_t bad = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(+ : bad)
  for (int hi = 0; hi < 65536; ++hi) {
    for (uint32_t lo = 0; lo < 65536; ++lo) {
      const uint32_t u = ((uint32_t)hi << 16) | lo;
      float f;
      memcpy(&f, &u, 4);
      bad += bp::from_float_tab<16, true>(f, t16) != bp::from_float<16>(f, true);
      bad += bp::from_float_tab<16, false>(f, t16) != bp::from_float<16>(f, false);
      bad += bp::from_float_tab<32, true>(f, t32) != bp::from_float<32>(f, true);
      bad += bp::from_float_tab<32, false>(f, t32) != bp::from_float<32>(f, false);
    }
  }
  return bad;
}

// Mismatches of the exact sum's regime-bin decode against quire_from_bp16 over
// every code: regime k >= -12 and value v stand for v * 2^(8k + 85) in the
// quire's units; k = -15 (zero, NaR) and -14, -13 for summands the quire
// conversion maps to zero; no other k.
size_t h_sum_bin16_check() {
  size_t bad = 0;
  for (uint32_t c = 0; c < 65536; ++c) {
    int k, v;
    bp::sum_bin16((int32_t)(c << 16), k, v);
    if (k < -15 || k > 14) ++bad;
    if ((c & 0x7FFFu) == 0 && k != -15) ++bad;
    bp::quire256 r = bp::q_zero();
    if (k >= -12) {
      int sh = 8 * k + 85;
      uint64_t m = (uint64_t)(v < 0 ? -(int64_t)v : (int64_t)v);
      if (sh < 0) {
        if (m & ((1ull << -sh) - 1)) ++bad;   // the fold's right shift must be exact
        m >>= -sh;
        sh = 0;
      }
      r = bp::q_from_shifted(m, sh);
      if (v < 0) r = bp::q_neg(r);
    }
    const bp::quire256 q = bp::quire_from_bp16(c);
    if (memcmp(&q, &r, sizeof q) != 0) ++bad;
  }
  return bad;
}

void h_quire_sum(const uint16_t* p, size_t n, uint64_t* w) {
  bp::quire256 acc = bp::q_zero();
  for (size_t i = 0; i < n; ++i) acc = bp::q_add(acc, bp::quire_from_bp16(p[i]));
  for (int j = 0; j < 4; ++j) w[j] = acc.w[j];
}
}
