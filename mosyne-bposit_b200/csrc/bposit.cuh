// bposit.cuh -- bounded-posit (bposit8/16/32, es=3, useed=256) encoders,
// decoders and the quire256 exact accumulator, for device and host code.
//
// Format (kernels/bposit16_reference.py:22-36, 378-503; 93-146):
//   value = 256^k * 2^e * (1.f),  scale = 8k + e clamped to [-48, 48];
//   regime k>=0: (k+1) ones then a 0;  k<0: (-k) zeros then a 1;
//   3 exponent bits, then the fraction; negative values are the two's
//   complement of the (n-1)-bit magnitude field; 0x80..0 is NaR.
// Default rounding truncates the fraction (the reference's default,
// kernels/bposit16_encode.cuh:179-183); RTNE uses the round bit and sticky
// bits with a saturating increment (bposit16_encode.cuh:299-311).
//
// quire256 (bposit16_encode.cuh:27-30): 256-bit two's complement integer,
// four little-endian u64 words, 96 fraction bits.
#pragma once
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define BP_HD __host__ __device__ __forceinline__
#else
#define BP_HD inline
#endif

namespace bp {

constexpr int kQuireFracBits = 96;
constexpr int kScaleLimit = 48;

BP_HD int clz32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __clz(x);
#else
  return x ? __builtin_clz(x) : 32;
#endif
}
BP_HD int clz64(uint64_t x) {
#if defined(__CUDA_ARCH__)
  return __clzll(x);
#else
  return x ? __builtin_clzll(x) : 64;
#endif
}

// Magnitude field (n-1 bits) of a positive value with floor(log2) = scale,
// fraction bits frac64 (MSB-aligned: bit 63 is the first bit below the
// leading one) and `sticky` = any non-zero bit beyond those 64.
template <int NBITS>
BP_HD uint32_t encode_field(int scale, uint64_t frac64, bool sticky, bool rtne) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  if (scale > kScaleLimit) return FMASK;   // +maxpos
  if (scale < -kScaleLimit) return 1u;     // +minpos
  const int k = scale >> 3;                // floor(scale / 8)
  const int e = scale & 7;
  int rlen;
  uint32_t regime;
  if (k >= 0) {
    rlen = k + 2;
    regime = ((2u << k) - 1u) << (N1 - (k + 1));
  } else {
    rlen = 1 - k;
    regime = 1u << (N1 - rlen);
  }
  const int fw = N1 - rlen - 3;            // >= 4 for bposit16, >= 20 for bposit32
  const uint32_t f = (uint32_t)(frac64 >> (64 - fw));
  uint32_t field = regime | ((uint32_t)e << fw) | f;
  if (rtne) {
    const uint64_t rest = frac64 << fw;    // bits after the kept fraction
    const bool rbit = (rest >> 63) != 0;
    const bool st = sticky || ((rest << 1) != 0);
    if (rbit && (st || (f & 1u)) && field < FMASK) field += 1u;
  }
  return field;
}

// encode_field for a fraction that fits 32 bits (MSB-aligned, nothing
// beyond them): the same field in 32-bit arithmetic, for single-precision
// inputs (the kept fraction is at most 26 bits, so every shift is < 32).
template <int NBITS>
BP_HD uint32_t encode_field32(int scale, uint32_t frac32, bool rtne) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  if (scale > kScaleLimit) return FMASK;
  if (scale < -kScaleLimit) return 1u;
  const int k = scale >> 3;
  const int e = scale & 7;
  const int rlen = k >= 0 ? k + 2 : 1 - k;
  const uint32_t regime = k >= 0 ? ((2u << k) - 1u) << (N1 - (k + 1)) : 1u << (N1 - rlen);
  const int fw = N1 - rlen - 3;
  const uint32_t f = frac32 >> (32 - fw);
  uint32_t field = regime | ((uint32_t)e << fw) | f;
  if (rtne) {
    const uint32_t rest = frac32 << fw;
    if ((rest >> 31) && (((rest << 1) != 0u) || (f & 1u)) && field < FMASK) field += 1u;
  }
  return field;
}

template <int NBITS>
BP_HD uint32_t apply_sign(uint32_t field, bool neg) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  return neg ? ((1u << N1) | ((0u - field) & FMASK)) : field;
}

// bposit<NBITS> of the exact value I / 2^shift (I any int64, |I| <= 2^63).
template <int NBITS>
BP_HD uint32_t from_int64(int64_t I, int shift, bool rtne) {
  if (I == 0) return 0u;
  const bool neg = I < 0;
  const uint64_t a = neg ? (uint64_t)0 - (uint64_t)I : (uint64_t)I;
  const int lz = clz64(a);
  const int msb = 63 - lz;
  const uint64_t frac = (a << lz) << 1;    // drop the leading one
  return apply_sign<NBITS>(encode_field<NBITS>(msb - shift, frac, false, rtne), neg);
}

// Fast path for an INT32 accumulator (value = I, no fraction bits):
// int_to_bposit32(I, 0) of kernels/test_int32_to_bposit32.cu:94-112, equal
// to quire256_to_bposit32(I << 96).  scale = msb in [0, 31], so the regime is
// always k+1 ones (k <= 3) and nothing saturates: straight-line code with no
// branches, which lets the GEMM epilogue interleave many outputs.
template <int NBITS>
BP_HD uint32_t from_int32(int32_t I, bool rtne) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  const bool neg = I < 0;
  const uint32_t a = neg ? 0u - (uint32_t)I : (uint32_t)I;
  const int lz = clz32(a | 1u);                         // a == 0 is selected away below
  const int msb = 31 - lz;
  const int k = msb >> 3, e = msb & 7;
  const uint32_t regime = ((2u << k) - 1u) << (N1 - 1 - k);
  const int fw = N1 - 5 - k;                            // N1 - (k + 2) - 3
  const uint32_t frac = (a << lz) << 1;                 // MSB-aligned fraction bits
  uint32_t field = regime | ((uint32_t)e << fw) | (frac >> (32 - fw));
  const uint32_t rest = frac << fw;
  const uint32_t up = (uint32_t)rtne & (rest >> 31) & (uint32_t)(((rest << 1) != 0u) | (field & 1u)) &
                      (uint32_t)(field < FMASK);
  field += up;
  const uint32_t out = neg ? ((1u << N1) | ((0u - field) & FMASK)) : field;
  return a == 0u ? 0u : out;
}

// Table-driven INT32 -> bposit for the GEMM epilogue.  For lz = clz(|I|)
// the regime, exponent and fraction width depend only on lz, so a 33-entry
// table, entry lz + 1 for lz = 0..31 and entry 0 for I == 0, holds
//   prefix = (regime | e << fw) ^ 1 << fw   and   sh = 31 - fw;
// with x = |I| << lz (leading one at bit 31), x >> sh puts the leading one at
// bit fw and the kept fraction below it, and prefix ^ (x >> sh) clears the
// leading one: the magnitude field in ~10 integer operations.  Equal to
// from_int32 for every input (checked exhaustively over the scale range in
// the host tests).
struct I32Entry {
  uint32_t prefix;
  uint32_t sh;
};

// `shift` (0..31) encodes I / 2^shift instead of I: the scale becomes
// msb - shift, which may be negative (regime of -k zeros and a one).
template <int NBITS>
BP_HD I32Entry i32_table_entry(int idx, int shift = 0) {
  constexpr int N1 = NBITS - 1;
  const int lz = idx - 1;
  if (lz < 0 || lz >= 32) return I32Entry{0u, 31u};     // I == 0: x = 0, field 0
  const int scale = 31 - lz - shift;
  const int k = scale >> 3, e = scale & 7;                // floor division
  const int rlen = k >= 0 ? k + 2 : 1 - k;
  const int fw = N1 - rlen - 3;
  const uint32_t regime =
      k >= 0 ? ((2u << k) - 1u) << (N1 - 1 - k) : 1u << (N1 - 1 + k);
  return I32Entry{(regime | ((uint32_t)e << fw)) ^ (1u << fw), (uint32_t)(31 - fw)};
}

// clz(a) for a != 0, -1 for a == 0 (one bit-find on the GPU).
BP_HD int clz_or_m1(uint32_t a) {
#if defined(__CUDA_ARCH__)
  int r;
  asm("bfind.shiftamt.u32 %0, %1;" : "=r"(r) : "r"(a));
  return r;
#else
  return a ? __builtin_clz(a) : -1;
#endif
}

// a << n and a >> n for n in [0, 31], and 0 for n >= 32 taken as unsigned
// (PTX clamps the shift amount; n = -1 is 0xFFFFFFFF).
BP_HD uint32_t shl_clamped(uint32_t a, int n) {
#if defined(__CUDA_ARCH__)
  uint32_t r;
  asm("shl.b32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(n));
  return r;
#else
  return (uint32_t)n >= 32u ? 0u : a << n;
#endif
}

BP_HD uint32_t shr_clamped(uint32_t a, int n) {
#if defined(__CUDA_ARCH__)
  uint32_t r;
  asm("shr.b32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(n));
  return r;
#else
  return (uint32_t)n >= 32u ? 0u : a >> n;
#endif
}

template <int NBITS, bool RTNE>
BP_HD uint32_t from_int32_tab(int32_t I, const I32Entry* tab) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  const uint32_t m = (uint32_t)(I >> 31);                // all ones when negative
#if defined(__CUDA_ARCH__)
  uint32_t a;                                            // |INT32_MIN| reads as 2^31
  asm("abs.s32 %0, %1;" : "=r"(a) : "r"(I));
#else
  const uint32_t a = ((uint32_t)I ^ m) - m;
#endif
  const int lz = clz_or_m1(a);
  const I32Entry t = tab[lz + 1];
  const uint32_t x = shl_clamped(a, lz);
  uint32_t field = t.prefix ^ (x >> t.sh);
  if (RTNE) {
    const uint32_t rem = x << (32 - t.sh);                // round bit at 31, sticky below
    const uint32_t up = (rem >> 31) & (uint32_t)(((rem << 1) != 0u) | (field & 1u)) &
                        (uint32_t)(field != FMASK);
    field += up;
  }
  const uint32_t out = (field ^ m) - m;
  return NBITS == 32 ? out : (out & 0xFFFFu);
}

// ---------------------------------------------------------------------------
// bposit8 (es = 2, useed = 16, values 2^-24 .. 2^24; kernels/bposit16_reference.py
// 151-209) -> int8 fixed point with 6 fraction bits, the decode that feeds the
// bposit8 IMMA path (kernels/test_mera_isometry_imma.cu:43-69, 166-197): the
// reference takes the code's quire (value x 2^96), shifts it right by 90 bits
// (floor) and clamps to [-128, 127]; NaR and zero give 0.  Every bposit8 value
// is a multiple of 2^-24, so the quire is exact and the result is
// clamp(floor(value * 64)).
// ---------------------------------------------------------------------------
BP_HD int8_t bposit8_to_int8(uint32_t code) {
  code &= 0xFFu;
  if (code == 0u || code == 0x80u) return 0;
  const bool neg = (code >> 7) != 0;
  const uint32_t mag = neg ? ((0u - code) & 0x7Fu) : (code & 0x7Fu);
  const uint32_t lead = (mag >> 6) & 1u;
  int run = 1;
  while (run < 7 && ((mag >> (6 - run)) & 1u) == lead) ++run;
  int k, e = 0, fw = 0;
  uint32_t frac = 0;
  if (run == 7) {
    k = lead ? 6 : -7;
  } else {
    k = lead ? run - 1 : -run;
    const int left = 6 - run;                  // bits after the regime terminator
    const int ew = left < 2 ? left : 2;
    e = ew ? (int)(((mag >> (left - ew)) & ((1u << ew) - 1u)) << (2 - ew)) : 0;
    fw = left - ew;
    frac = mag & ((1u << fw) - 1u);
  }
  // value * 64 = ((1 << fw) + frac) * 2^(4k + e + 6 - fw)
  const int64_t m = (int64_t)((1u << fw) + frac);
  const int sh = 4 * k + e + 6 - fw;
  int64_t v;
  if (sh >= 0) {
    v = sh > 40 ? (int64_t)1 << 40 : m << sh;   // far above the clamp either way
    if (neg) v = -v;
  } else {
    v = neg ? -((m + ((int64_t)1 << -sh) - 1) >> -sh) : (m >> -sh);   // floor
  }
  return (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
}

// ---------------------------------------------------------------------------
// quire256
// ---------------------------------------------------------------------------
struct quire256 {
  uint64_t w[4];
};

BP_HD quire256 q_zero() { return quire256{{0, 0, 0, 0}}; }

BP_HD quire256 q_add(const quire256& a, const quire256& b) {
  quire256 r;
#if defined(__CUDA_ARCH__)
  asm("add.cc.u64 %0, %4, %8;\n\t"
      "addc.cc.u64 %1, %5, %9;\n\t"
      "addc.cc.u64 %2, %6, %10;\n\t"
      "addc.u64 %3, %7, %11;\n\t"
      : "=l"(r.w[0]), "=l"(r.w[1]), "=l"(r.w[2]), "=l"(r.w[3])
      : "l"(a.w[0]), "l"(a.w[1]), "l"(a.w[2]), "l"(a.w[3]),
        "l"(b.w[0]), "l"(b.w[1]), "l"(b.w[2]), "l"(b.w[3]));
#else
  uint64_t c = 0;
  for (int i = 0; i < 4; ++i) {
    const uint64_t s = a.w[i] + b.w[i];
    const uint64_t c1 = s < a.w[i];
    r.w[i] = s + c;
    c = c1 | (r.w[i] < s);
  }
#endif
  return r;
}

BP_HD quire256 q_sub(const quire256& a, const quire256& b) {
  quire256 r;
#if defined(__CUDA_ARCH__)
  asm("sub.cc.u64 %0, %4, %8;\n\t"
      "subc.cc.u64 %1, %5, %9;\n\t"
      "subc.cc.u64 %2, %6, %10;\n\t"
      "subc.u64 %3, %7, %11;\n\t"
      : "=l"(r.w[0]), "=l"(r.w[1]), "=l"(r.w[2]), "=l"(r.w[3])
      : "l"(a.w[0]), "l"(a.w[1]), "l"(a.w[2]), "l"(a.w[3]),
        "l"(b.w[0]), "l"(b.w[1]), "l"(b.w[2]), "l"(b.w[3]));
#else
  uint64_t br = 0;
  for (int i = 0; i < 4; ++i) {
    const uint64_t d = a.w[i] - b.w[i];
    const uint64_t b1 = a.w[i] < b.w[i];
    r.w[i] = d - br;
    br = b1 | (d < br);
  }
#endif
  return r;
}

BP_HD quire256 q_neg(const quire256& a) { return q_sub(q_zero(), a); }

BP_HD bool q_is_zero(const quire256& q) { return (q.w[0] | q.w[1] | q.w[2] | q.w[3]) == 0; }

BP_HD uint64_t q_word(const quire256& q, int i) {
  // branch-free word select (avoids local-memory indexing on the device)
  uint64_t r = 0;
  r = (i == 0) ? q.w[0] : r;
  r = (i == 1) ? q.w[1] : r;
  r = (i == 2) ? q.w[2] : r;
  r = (i == 3) ? q.w[3] : r;
  return r;
}

// Unsigned magnitude value m * 2^sh placed into a quire (0 <= sh, m < 2^63,
// sh + bitlen(m) <= 255).
BP_HD quire256 q_from_shifted(uint64_t m, int sh) {
  const int wi = sh >> 6, o = sh & 63;
  const uint64_t lo = m << o;
  const uint64_t hi = o ? (m >> (64 - o)) : 0ull;
  quire256 r;
  r.w[0] = (wi == 0) ? lo : 0ull;
  r.w[1] = (wi == 1) ? lo : ((wi == 0) ? hi : 0ull);
  r.w[2] = (wi == 2) ? lo : ((wi == 1) ? hi : 0ull);
  r.w[3] = (wi == 3) ? lo : ((wi == 2) ? hi : 0ull);
  return r;
}

// quire256 -> bposit<NBITS> (bposit16_encode.cuh:113-204 truncate,
// 221-321 RTNE, 333-418 bposit32 truncate; bposit16_reference.py:616-631,
// 775-794).
template <int NBITS>
BP_HD uint32_t from_quire(quire256 q, bool rtne) {
  if (q_is_zero(q)) return 0u;
  const bool neg = (q.w[3] >> 63) != 0;
  if (neg) q = q_neg(q);
  int msb;
  if (q.w[3]) msb = 192 + 63 - clz64(q.w[3]);
  else if (q.w[2]) msb = 128 + 63 - clz64(q.w[2]);
  else if (q.w[1]) msb = 64 + 63 - clz64(q.w[1]);
  else msb = 63 - clz64(q.w[0]);
  // 64-bit window of the bits just below the msb, and the sticky remainder.
  const int lo = msb - 64;                 // window covers [lo, msb-1]
  uint64_t win;
  bool sticky = false;
  if (lo < 0) {
    win = q.w[0] << (-lo);
  } else {
    const int wi = lo >> 6, b = lo & 63;
    const uint64_t x0 = q_word(q, wi), x1 = q_word(q, wi + 1);
    win = b ? ((x0 >> b) | (x1 << (64 - b))) : x0;
    uint64_t below = 0;
    for (int j = 0; j < 4; ++j) {
      const int base = 64 * j;
      const uint64_t wj = q.w[j];
      if (lo >= base + 64) below |= wj;
      else if (lo > base) below |= wj & ((1ull << (lo - base)) - 1ull);
    }
    sticky = below != 0;
  }
  return apply_sign<NBITS>(encode_field<NBITS>(msb - kQuireFracBits, win, sticky, rtne), neg);
}

// from_quire with selects instead of branches and word indexing: the
// magnitude (two's complement of a negative quire), its leading word by a
// select cascade, the 64 bits below the leading one taken from that word and
// the next lower one, and the sticky OR of everything beneath -- the same
// scale, window and sticky bit from_quire hands to encode_field, so the same
// code.  For the element-wise kernels, which are bound by the integer pipe.
template <int NBITS>
BP_HD uint32_t from_quire_sel(quire256 q, bool rtne) {
  const bool neg = (q.w[3] >> 63) != 0;
  if (neg) q = q_neg(q);
  const bool n3 = q.w[3] != 0, n2 = q.w[2] != 0, n1 = q.w[1] != 0;
  const int hi = n3 ? 3 : (n2 ? 2 : (n1 ? 1 : 0));
  const uint64_t h = n3 ? q.w[3] : (n2 ? q.w[2] : (n1 ? q.w[1] : q.w[0]));
  const uint64_t l = n3 ? q.w[2] : (n2 ? q.w[1] : (n1 ? q.w[0] : 0ull));
  const uint64_t below = n3 ? (q.w[1] | q.w[0]) : (n2 ? q.w[0] : 0ull);
  const int lz = clz64(h | 1ull);            // h == 0 only for the zero quire
  const int msb = 64 * hi + 63 - lz;
  // the 64 bits after the leading one: h's bits below it, then l's top bits
  const uint64_t hs = (h << lz) << 1;
  const uint64_t win = hs | (lz == 63 ? l : (l >> (63 - lz)));
  const uint64_t lrest = lz == 63 ? 0ull : (l << (lz + 1));
  const bool sticky = (lrest | below) != 0ull;
  const uint32_t r = apply_sign<NBITS>(encode_field<NBITS>(msb - kQuireFracBits, win, sticky, rtne), neg);
  return h == 0ull ? 0u : r;
}

// bposit16 decode: value = (-1)^neg * mant * 2^exp2 (bposit16_reference.py:302-374).
struct Dec16 {
  uint32_t mant;   // hidden one included, <= 13 bits
  int exp2;        // exponent of the mantissa's LSB
  bool neg;
  bool zero;
  bool nar;
};

BP_HD Dec16 decode16(uint32_t p) {
  Dec16 d;
  p &= 0xFFFFu;
  d.zero = p == 0u;
  d.nar = p == 0x8000u;
  d.neg = (p >> 15) != 0;
  uint32_t rest = p & 0x7FFFu;
  if (d.neg) rest = (0u - rest) & 0x7FFFu;
  const uint32_t lead = (rest >> 14) & 1u;
  const uint32_t x = lead ? (~rest & 0x7FFFu) : rest;
  const int rs = clz32(x) - 17;            // run length of the regime, 1..15
  int k, e = 0, fw = 0;
  uint32_t fb = 0;
  if (rs >= 15) {
    k = lead ? 14 : -15;
  } else {
    k = lead ? rs - 1 : -rs;
    const int remaining = 14 - rs;
    const uint32_t rest2 = rest & ((1u << remaining) - 1u);
    const int ew = remaining < 3 ? remaining : 3;
    if (ew > 0) e = (int)(((rest2 >> (remaining - ew)) & ((1u << ew) - 1u)) << (3 - ew));
    fw = remaining - ew;
    fb = rest2 & ((1u << fw) - 1u);
  }
  d.mant = (1u << fw) | fb;
  d.exp2 = 8 * k + e - fw;
  return d;
}

// bposit16 -> quire256 (bposit16_reference.py:602-609: truncation toward
// zero below 2^-96; zero and NaR map to 0).
BP_HD quire256 quire_from_bp16(uint32_t p) {
  const Dec16 d = decode16(p);
  if (d.zero || d.nar) return q_zero();
  int sh = d.exp2 + kQuireFracBits;
  uint64_t m = d.mant;
  if (sh < 0) {
    m = (-sh >= 32) ? 0ull : (m >> (-sh));
    sh = 0;
  }
  const quire256 q = q_from_shifted(m, sh);
  return d.neg ? q_neg(q) : q;
}

// Regime-bin decode of one bposit16 code for the exact sum.  c32 holds the code
// in its upper 16 bits (lower 16 bits zero), so the 32-bit negate is the code's
// own two's-complement negate.  With W = 1.f scaled to an integer (2^11 + f)
// and e the exponent, a code of regime k has value * 2^96 = (W << e) *
// 2^(8k + 85): within one regime the value is the integer V = W << e < 2^19.
// Returns k and the signed V.  Real codes have k = -14 .. 14; zero and NaR
// return k = -15 (the bit at 16 stops their run of zeros there), so a caller
// with bins for k = -15 .. 14 needs no clamp and drops k < -12 (values under
// 2^-96, which the per-value quire conversion truncates to zero).  Branch-free:
// the regime run is one count of leading zeros of the bits after the sign,
// inverted when they are ones.  V is formed as a float with exponent field
// e + 138 and fraction f (exactly V), then times the code's sign plus
// 1.5 * 2^23 in one fused multiply-add, exact for |V| < 2^22 (the sum's unit
// is 1), whose bits less those of 1.5 * 2^23 are the integer +-V: the
// multiply-add pipe does what took five integer operations (the exponent,
// the fraction with its hidden bit, the shift, the conditional negate).
BP_HD void sum_bin16(int32_t c32, int& k, int& v) {
  const uint32_t a = c32 < 0 ? 0u - (uint32_t)c32 : (uint32_t)c32;   // NaR: 0x80000000
  const uint32_t xs = (uint32_t)((int32_t)(a << 1) >> 31);  // all ones: a run of ones (k >= 0)
  // run length - 1 (bit 17 caps zero and NaR at 14); the lowest bit of xs is
  // below that cap and does not matter
  const int m1 = clz32(((a << 2) ^ xs) | 0x20000u);
  const uint32_t z = (a << 3) << m1;                 // exponent (3 bits), then the fraction
  uint32_t fb;                                       // (z >> 6) + (138 << 23)
#if defined(__CUDA_ARCH__)
  asm("mad.hi.u32 %0, %1, %2, %3;" : "=r"(fb) : "r"(z), "r"(1u << 26), "r"(138u << 23));
  const float f = fmaf(__uint_as_float(fb), __uint_as_float(((uint32_t)c32 & 0x80000000u) | 0x3F800000u),
                       12582912.0f);
  v = __float_as_int(f) - 0x4B400000;
#else
  fb = (z >> 6) + (138u << 23);
  float f;
  memcpy(&f, &fb, 4);
  f = (c32 < 0 ? -f : f) + 12582912.0f;
  memcpy(&v, &f, 4);
  v -= 0x4B400000;
#endif
  k = m1 ^ (int)~xs;                                 // ones: run - 1; zeros: -run
}

// from_quire<16>(quire_from_bp16(a) + quire_from_bp16(b), truncate) without
// the 256-bit quire.  Each operand is m * 2^x (m < 2^13; zero and NaR count
// as 0, and bits below 2^-96 are dropped as the per-value quire conversion
// drops them).  Aligned at the smaller exponent the exact sum fits an int64
// while the exponents differ by at most 48.  Beyond that the smaller operand
// is below 2^(x_hi - 35), far under the last kept place of any result near
// the larger one (at least 2^(x_hi - 2)), so the truncated encoding depends
// only on its sign; it is moved up to the gap of 48, which keeps the sign and
// stays under that bound.
BP_HD uint32_t sum16_trunc(uint32_t a, uint32_t b) {
  const Dec16 da = decode16(a), db = decode16(b);
  int64_t ma = (da.zero || da.nar) ? 0 : (int64_t)da.mant;
  int64_t mb = (db.zero || db.nar) ? 0 : (int64_t)db.mant;
  int xa = da.exp2, xb = db.exp2;
  if (xa < -kQuireFracBits) {
    const int s = -kQuireFracBits - xa;
    ma = s >= 32 ? 0 : (ma >> s);
    xa = -kQuireFracBits;
  }
  if (xb < -kQuireFracBits) {
    const int s = -kQuireFracBits - xb;
    mb = s >= 32 ? 0 : (mb >> s);
    xb = -kQuireFracBits;
  }
  if (ma == 0) xa = xb;                    // a zero operand opens no gap
  if (mb == 0) xb = xa;
  if (da.neg) ma = -ma;
  if (db.neg) mb = -mb;
  const bool a_hi = xa >= xb;
  const int xh = a_hi ? xa : xb;
  int xl = a_hi ? xb : xa;
  const int64_t mh = a_hi ? ma : mb, ml = a_hi ? mb : ma;
  if (xh - xl > 48) xl = xh - 48;
  const int64_t I = (int64_t)((uint64_t)mh << (xh - xl)) + ml;
  return from_int64<16>(I, -xl, false);
}

// Packed decode of a bposit16 magnitude code (0 .. 0x7FFF) as the quire
// conversion sees it: bits 0-12 the mantissa (hidden one included), bits
// 16-23 the exponent of its last place + 128, bits below 2^-96 dropped (the
// longest regimes of the code space; a mantissa that loses every bit packs as
// 0).  Magnitude 0 (zero, and NaR) packs to 0.  The ALU kernels hold the
// 32,768 packed decodes in shared memory.
BP_HD uint32_t dec16_pack(uint32_t mag) {
  const Dec16 d = decode16(mag & 0x7FFFu);
  if (d.zero || d.nar) return 0u;
  uint32_t m = d.mant;
  int x = d.exp2;
  if (x < -kQuireFracBits) {
    const int sh = -kQuireFracBits - x;
    m = sh >= 32 ? 0u : (m >> sh);
    x = -kQuireFracBits;
  }
  return m == 0u ? 0u : (m | ((uint32_t)(x + 128) << 16));
}

// The value of a packed decode as a float (exact: at most 13 significant
// bits, exponents 2^-96 .. 2^125); packed 0 gives +0.
BP_HD float dec16_value(uint32_t packed) {
  const uint32_t m = packed & 0x1FFFu;
  if (m == 0u) return 0.f;
  const int lz = clz32(m);                                // m = 1.f * 2^(31 - lz)
  const int e = 31 - lz + (int)(packed >> 16) - 128;      // exponent of the leading bit
  const uint32_t f23 = (m << (lz + 1)) >> 9;              // fraction bits below it
  const uint32_t bits = ((uint32_t)(e + 127) << 23) | f23;
#if defined(__CUDA_ARCH__)
  return __uint_as_float(bits);
#else
  float v;
  memcpy(&v, &bits, 4);
  return v;
#endif
}

// The encoding of s in sum16_trunc_f32, indexed by s's biased exponent: the
// prefix (regime and exponent bits), the shift that keeps the fraction, the
// shift that exposes the dropped bits, and the step toward zero from a value
// on the bposit16 grid (delta0 when s's fraction is zero, delta1 otherwise;
// 0 where the encoding saturates, and the landing codes of the two
// saturation edges).
struct S16Entry {
  uint32_t enc;     // prefix | fraction shift << 16 | remainder shift << 24
  uint32_t step;    // delta0 | delta1 << 16
};

BP_HD S16Entry s16_table_entry(int bexp) {
  constexpr uint32_t FMASK = 0x7FFFu;
  const int scale = bexp - 127;
  if (bexp == 0 || scale < -kScaleLimit) return S16Entry{1u | (32u << 16) | (32u << 24), 0u};
  if (scale > kScaleLimit) {
    const uint32_t d0 = scale == kScaleLimit + 1 ? FMASK - encode_field32<16>(kScaleLimit, 0xFFFFFFFFu, false) : 0u;
    return S16Entry{FMASK | (32u << 16) | (32u << 24), d0};
  }
  const int k = scale >> 3;
  const int fw = 12 - (k >= 0 ? k + 2 : 1 - k);
  const uint32_t prefix = encode_field32<16>(scale, 0u, false);
  const uint32_t d0 = scale == -kScaleLimit ? prefix - 1u : 1u;
  return S16Entry{prefix | ((uint32_t)(32 - fw) << 16) | ((uint32_t)fw << 24), d0 | (1u << 16)};
}

// Truncated bposit16 of the exact sum of two values held exactly as floats,
// each a bposit16 value as the quire holds it (0, or a magnitude in
// [2^-96, 2^113) with at most 13 significant bits) -- sum16_trunc on the
// floating-point pipe.  s = fa + fb rounded to nearest and its exact error e
// (Knuth's TwoSum: s + e = fa + fb exactly, |e| <= half an ulp of s).  The
// bposit16 values are floats with at most 13 significant bits, so a value of
// them lies within |e| of s only if it is s itself: truncating s + e toward
// zero gives the truncation of s, except when s is a bposit16 value and e
// points toward zero, where it is the next magnitude below.  The encoder
// saturates at the scale limits: below 2^-48 every value is minpos, from 2^49
// up every value is maxpos, so the steps down from 2^-48 and from 2^49 land on
// minpos and on the largest scale-48 code.
BP_HD uint32_t sum16_trunc_f32(float fa, float fb, const S16Entry* tab) {
#if defined(__CUDA_ARCH__)
  const float s = __fadd_rn(fa, fb);
  const float bv = __fsub_rn(s, fa);
  const float e = __fadd_rn(__fsub_rn(fa, __fsub_rn(s, bv)), __fsub_rn(fb, bv));
  const uint32_t sb = __float_as_uint(s);
  const uint32_t eb = __float_as_uint(e);
#else
  volatile float vs = fa + fb;
  const float s = vs;
  volatile float vbv = s - fa;
  const float bv = vbv;
  volatile float va = s - bv;
  const float av = va;
  const float e = (fa - av) + (fb - bv);
  uint32_t sb, eb;
  memcpy(&sb, &s, 4);
  memcpy(&eb, &e, 4);
#endif
  const uint32_t mag = sb & 0x7FFFFFFFu;
  const S16Entry t = tab[mag >> 23];
  const uint32_t x = mag << 9;
  uint32_t field = (t.enc & 0xFFFFu) | shr_clamped(x, (int)((t.enc >> 16) & 0xFFu));
  const uint32_t rest = shl_clamped(x, (int)(t.enc >> 24));
  const bool tz = ((eb ^ sb) >> 31) != 0u && (eb << 1) != 0u;
  const uint32_t delta = x == 0u ? (t.step & 0xFFFFu) : (t.step >> 16);
  field -= (rest == 0u && tz) ? delta : 0u;
  const uint32_t out = apply_sign<16>(field, (sb >> 31) != 0u);
  return mag == 0u ? 0u : out;
}

// Magnitude code of a bposit16 code (two's complement of a negative one;
// zero and NaR give 0).
BP_HD uint32_t mag16(uint32_t p) {
  return ((p >> 15) & 1u) ? ((0u - p) & 0x7FFFu) : (p & 0x7FFFu);
}

// The float a bposit16 code adds to a quire (its value, bits below 2^-96
// dropped; zero and NaR give 0), with the code's sign.
BP_HD float quire_value16(uint32_t code) {
  const float v = dec16_value(dec16_pack(mag16(code)));
  return ((code >> 15) & 1u) ? -v : v;
}

// Half `half` (bits 128*half .. +127, as four 32-bit words) of the quire of a
// bposit16 code, equal to that half of quire_from_bp16(code): the
// magnitude m * 2^sh (m < 2^13, sh = its last place + 96 in [0, 208], bits
// below 2^-96 dropped) occupies 32-bit words sh/32 and sh/32 + 1 of the eight;
// a negative code is the 256-bit two's complement, whose carry enters the high
// half only when the low half of the magnitude is zero.  32-bit arithmetic
// and selects only.
BP_HD void quire_half_bp16(uint32_t code, int half, uint32_t w[4]) {
  // branch-free decode of the magnitude: after the regime run (rs bits) and
  // its terminating bit, the top three bits are the exponent and the rest the
  // fraction, so the value is (2^12 + f12) * 2^(8k + e - 12) (fewer fraction
  // bits read as zeros below them)
  const uint32_t rest = mag16(code);
  const uint32_t y = rest << 17;
  const int rs = clz32(y ^ (y << 1)) + 1;                 // regime run length
  const uint32_t z = shl_clamped(y, rs + 1);
  const int k = (int)y < 0 ? rs - 1 : -rs;
  const int x = 8 * k + (int)(z >> 29) - 12;              // exponent of the last place
  uint32_t m = rest == 0u ? 0u : (0x1000u | ((z << 3) >> 20));
  int sh = x + kQuireFracBits;
  if (sh < 0) {                                           // below 2^-96: dropped
    m = shr_clamped(m, -sh);
    sh = 0;
  }
  const int wi = sh >> 5, off = sh & 31;
  const uint32_t lo = m << off, hi = shr_clamped(m, 32 - off);
  const int base = 4 * half;
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = (base + k == wi) ? lo : ((base + k == wi + 1) ? hi : 0u);
  if ((code & 0x8000u) && m != 0u) {
    // carry into this half: all of it for the low half; for the high half
    // only when the magnitude has no bit in the low half
    const bool low_nonzero = (wi <= 3 && lo != 0u) || (wi + 1 <= 3 && hi != 0u);
    uint32_t c = (half == 0 || !low_nonzero) ? 1u : 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t x = ~w[k];
      w[k] = x + c;
      c = (c != 0u && w[k] == 0u) ? 1u : 0u;
    }
  }
}

// Exact product of two decoded nonzero bposit16 values, truncated: the
// mantissa product has at most 26 bits, so from_int64's encoding of it runs
// in 32-bit arithmetic.
BP_HD uint32_t mul16_trunc_dec(const Dec16& da, const Dec16& db) {
  const uint32_t m = da.mant * db.mant;
  const int lz = clz32(m);
  return apply_sign<16>(encode_field32<16>(31 - lz + da.exp2 + db.exp2, (m << lz) << 1, false),
                        da.neg != db.neg);
}

// Exact binary float (value = m * 2^(e)) -> bposit<NBITS>: the exact
// rational the float denotes (bposit16_reference.py:485-503 given a Fraction).
template <int NBITS>
BP_HD uint32_t from_double(double x, bool rtne) {
  union { double d; uint64_t u; } v;
  v.d = x;
  const bool neg = (v.u >> 63) != 0;
  const int bexp = (int)((v.u >> 52) & 0x7FF);
  uint64_t man = v.u & ((1ull << 52) - 1);
  if (bexp == 0 && man == 0) return 0u;
  if (bexp == 0x7FF) return 1u << (NBITS - 1);           // inf/nan -> NaR
  int scale;
  uint64_t frac;
  if (bexp == 0) {                                          // subnormal
    const int lz = clz64(man);
    scale = -1074 + (63 - lz);
    frac = (man << lz) << 1;
  } else {
    scale = bexp - 1023;
    frac = man << 12;
  }
  return apply_sign<NBITS>(encode_field<NBITS>(scale, frac, false, rtne), neg);
}

// from_double of a single-precision value, in 32-bit integer arithmetic
// (every float is exactly a double, so the two agree on every input).
template <int NBITS>
BP_HD uint32_t from_float(float x, bool rtne) {
  uint32_t u;
#if defined(__CUDA_ARCH__)
  u = __float_as_uint(x);
#else
  std::memcpy(&u, &x, sizeof(u));
#endif
  const bool neg = (u >> 31) != 0;
  const int bexp = (int)((u >> 23) & 0xFFu);
  const uint32_t man = u & 0x7FFFFFu;
  if (bexp == 0 && man == 0) return 0u;
  if (bexp == 0xFF) return 1u << (NBITS - 1);             // inf/nan -> NaR
  int scale;
  uint32_t frac;
  if (bexp == 0) {                                          // subnormal
    const int lz = clz32(man);
    scale = -149 + (31 - lz);
    frac = (man << lz) << 1;
  } else {
    scale = bexp - 127;
    frac = man << 9;
  }
  return apply_sign<NBITS>(encode_field32<NBITS>(scale, frac, rtne), neg);
}

// Table-driven form of from_float for streaming kernels.  For a normal
// float the regime, exponent and fraction width depend only on the biased
// exponent, so a 256-entry table (entry bexp) holds prefix = regime | e << fw
// and the shifts 32 - fw (fraction) and fw (rounding remainder); exponents
// outside the +-48 range (and subnormals, all below 2^-126) hold the
// saturated field with both shifts 32, which clears fraction and remainder.
// Zero and inf/nan are selected separately.
struct F32Entry {
  uint32_t prefix;
  uint32_t sh;     // shift of the fraction | shift of the remainder << 8
};

template <int NBITS>
BP_HD F32Entry f32_table_entry(int bexp) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  const int scale = bexp - 127;
  if (bexp == 0xFF) return F32Entry{1u << N1, 32u | (32u << 8)};   // inf / NaN -> NaR
  if (bexp == 0 || scale < -kScaleLimit) return F32Entry{1u, 32u | (32u << 8)};
  if (scale > kScaleLimit) return F32Entry{FMASK, 32u | (32u << 8)};
  const int k = scale >> 3, e = scale & 7;
  const int rlen = k >= 0 ? k + 2 : 1 - k;
  const uint32_t regime = k >= 0 ? ((2u << k) - 1u) << (N1 - (k + 1)) : 1u << (N1 - rlen);
  const int fw = N1 - rlen - 3;
  return F32Entry{regime | ((uint32_t)e << fw), (uint32_t)(32 - fw) | ((uint32_t)fw << 8)};
}

template <int NBITS, bool RTNE>
BP_HD uint32_t from_float_tab(float xf, const F32Entry* tab) {
  constexpr int N1 = NBITS - 1;
  constexpr uint32_t FMASK = (1u << N1) - 1u;
  constexpr uint32_t NMASK = NBITS == 32 ? 0xFFFFFFFFu : ((1u << NBITS) - 1u);
  uint32_t u;
#if defined(__CUDA_ARCH__)
  u = __float_as_uint(xf);
#else
  std::memcpy(&u, &xf, sizeof(u));
#endif
  const uint32_t bexp = (u >> 23) & 0xFFu;
  const F32Entry t = tab[bexp];
  const uint32_t x = u << 9;                              // fraction, MSB-aligned
  uint32_t field = t.prefix | shr_clamped(x, (int)(t.sh & 0xFFu));
  if (RTNE) {
    // round up when the dropped bits exceed half a place, or equal it with
    // the kept field odd; never past maxpos (the NaR entry drops nothing)
    const uint32_t rest = shl_clamped(x, (int)(t.sh >> 8));
    field += (uint32_t)((rest > 0x80000000u - (field & 1u)) && field != FMASK);
  }
  // a negative value is the two's complement of its magnitude's code (NaR's
  // code is its own complement)
  const uint32_t m = (uint32_t)((int32_t)u >> 31);
  const uint32_t out = ((field ^ m) - m) & NMASK;
  return (u & 0x7FFFFFFFu) == 0u ? 0u : out;
}

}  // namespace bp
