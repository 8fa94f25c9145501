// quire.cu -- exact quire256 reductions and element-wise bposit conversions.
//
// The exact sum replaces the reference's single-warp reduction
// (kernels/test_determinism_headline.cu:65-91, <<<1,32>>>, which is only
// correct for one warp) and the <=32-block entropy reduction
// (kernels/shannon_entropy_bposit16.cu:45-119) with a grid-wide one:
// 16-byte streaming loads of 8 codes, an arithmetic bposit16 decode (no
// 2 MiB table) into per-regime int32 sums kept in shared memory, folded once
// per thread into a 256-bit quire, then warp shuffles, a shared-memory block
// step, per-block partials and a last-block finish.  Integer addition is
// associative, so the quire (and every encoding of it) is identical for any
// grid, schedule or GPU.
#include "bposit.cuh"
#include "common.cuh"
#include "quire.cuh"

namespace mb {
namespace {

using bp::quire256;

// Per-regime integer sums.  Within one regime k a bposit16 code's value is
// the integer V = W << e (W = 1.f with 11 fraction bits, e the exponent) times
// 2^(8k + 85 - 96) (bp::sum_bin16).  Each thread keeps one int32 sum per
// regime k = -15 .. 14 in its own shared-memory column (exact for
// 4096 values; folded into the 256-bit quire every 2048 values and at the
// end), the decode is branch-free and the same for every code: zero and NaR
// (k = -15) and the regimes k = -14, -13 (below 2^-96, adding nothing, as in
// the per-value conversion, which truncates there) have bins that are never
// folded, so every code takes one unconditional shared atomic at its own k.
// For k = -12 and -11 every V is a multiple of the 2^11 / 2^3 the fold
// divides out, so the sum stays exact.
constexpr int kGroups = 30;          // k = -15 .. 14
constexpr int kGroupLow = -15;
constexpr int kKeptLow = -12;        // bins below: zero, NaR, values under 2^-96
constexpr int kFoldIters = 256;                          // x 8 codes per iteration

// c32: the summand's code in the upper 16 bits (bp::sum_bin16); gk: this
// thread's sum for k = 0, the sum for k at gk[k * BS].
template <int BS>   // the block size: stride between one thread's group sums
__device__ __forceinline__ void group_accumulate_bp16(int* gk, int32_t c32) {
  int k, v;
  bp::sum_bin16(c32, k, v);
  atomicAdd(gk + k * BS, v);
}

// -code in the upper 16 bits (the 32-bit negate of code << 16 is the
// code's own negate; NaR stays NaR).
__device__ __forceinline__ int32_t neg_hi(uint32_t code) { return (int32_t)(0u - (code << 16)); }

// The entropy's summands pre-decoded: entry c (a probability code 0 .. 0x7FFF)
// = the regime and signed value of -term[c], packed as v << 5 | (k + 13)
// (0: a summand that adds nothing); negative probability codes have the NaR term, which adds
// nothing.  One shared load and one shared atomic per code in place of the
// table load and the decode.
__device__ __forceinline__ int term_dec_entry(uint32_t c, const uint16_t* term) {
  int k, v;
  bp::sum_bin16(neg_hi(term[c]), k, v);
  return k < kKeptLow ? 0 : (int)((uint32_t)v << 5) | (k - kKeptLow + 1);
}

__device__ __forceinline__ int dec_entry(uint32_t code, const int* dec) {
  return (code & 0x8000u) ? 0 : dec[code & 0x7FFFu];
}

// g0: this thread's sum for k = kKeptLow - 1 (a dropped bin, entry 0)
template <int BS>
__device__ __forceinline__ void group_add_dec(int* g0, int e) {
  atomicAdd(g0 + (e & 31) * BS, e >> 5);
}

// Also counts the negative probability codes whose term is not NaR (none in
// the table this library generates; the staged mode relies on it).
__global__ void term_dec_build_kernel(const uint16_t* __restrict__ term, int* __restrict__ out,
                                      unsigned* __restrict__ bad) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < 32768u) {
    out[c] = term_dec_entry(c, term);
    if (term[c + 32768u] != 0x8000u) atomicAdd(bad, 1u);
  }
}

template <int BS>
__device__ __forceinline__ quire256 fold_groups(int* gk, quire256 q) {
  for (int k = kGroupLow; k < kKeptLow; ++k) gk[k * BS] = 0;   // the dropped bins
  for (int k = kKeptLow; k < kGroupLow + kGroups; ++k) {
    const int s = gk[k * BS];
    if (s == 0) continue;
    gk[k * BS] = 0;
    const int sh = 8 * k + 85;                            // -11 .. 197
    uint64_t mag = s < 0 ? (uint64_t)(-(long long)s) : (uint64_t)s;
    int shp = sh;
    if (shp < 0) {
      mag >>= -shp;                                       // exact: every V is a multiple
      shp = 0;
    }
    const quire256 t = bp::q_from_shifted(mag, shp);
    q = s < 0 ? bp::q_sub(q, t) : bp::q_add(q, t);
  }
  return q;
}

__device__ __forceinline__ quire256 shfl_down_q(const quire256& q, int off) {
  quire256 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.w[i] = __shfl_down_sync(0xffffffffu, q.w[i], off);
  return r;
}

__device__ __forceinline__ quire256 block_reduce_q(quire256 q, quire256* sh /*[32]*/) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) q = bp::q_add(q, shfl_down_q(q, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = q;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (warp == 0) {
    q = lane < nw ? sh[lane] : bp::q_zero();
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q = bp::q_add(q, shfl_down_q(q, off));
  }
  return q;  // valid in thread 0
}

// The block's sum, valid in thread 0: each kept regime's sums over all the
// block's threads added in int64 by one warp (exact: a thread's sum is below
// 2^19 * 4096, the block's below 2^40) and placed into that warp's quire
// once, plus the quires of threads that folded during the loop.  In place of
// every thread folding its own 27 sums into a quire -- as many instructions
// as summing ~60 codes, when an input of 2^24 codes gives each thread ~70.
// g: the block's group sums ([kGroups][BS] int); sh: 32 quires of scratch,
// which may alias g.
template <int BS>
__device__ __forceinline__ quire256 block_fold_q(const int* g, quire256 acc, quire256* sh) {
  constexpr int NW = BS / 32;
  const bool any_acc = __syncthreads_or(!bp::q_is_zero(acc));   // also: every sum final
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  quire256 qb = bp::q_zero();
  for (int k = kKeptLow + warp; k < kGroupLow + kGroups; k += NW) {
    const int* col = g + (k - kGroupLow) * BS;
    long long s = 0;
#pragma unroll
    for (int j = 0; j < BS / 32; ++j) s += col[lane + 32 * j];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (s != 0) {
      uint64_t mag = s < 0 ? (uint64_t)(-s) : (uint64_t)s;
      int sh8 = 8 * k + 85;                               // -11 .. 197
      if (sh8 < 0) {
        mag >>= -sh8;                                     // exact: every V is a multiple
        sh8 = 0;
      }
      const quire256 t = bp::q_from_shifted(mag, sh8);
      qb = s < 0 ? bp::q_sub(qb, t) : bp::q_add(qb, t);
    }
  }
  quire256 q = lane == 0 ? qb : bp::q_zero();
  if (any_acc) {
    q = bp::q_add(q, acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q = bp::q_add(q, shfl_down_q(q, off));
  }
  __syncthreads();                                        // every sum read before sh is written
  if (lane == 0) sh[warp] = q;
  __syncthreads();
  if (warp == 0) {
    q = lane < NW ? sh[lane] : bp::q_zero();
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q = bp::q_add(q, shfl_down_q(q, off));
  }
  return q;
}

// The grid step: thread 0 of each block publishes the block's quire (acc,
// valid in thread 0), and the last block to arrive (ticket) adds all of them
// in a fixed order and writes the quire and its encodings.
__device__ __forceinline__ void grid_finish(const quire256& acc, quire256* sh, bool* is_last,
                                            quire256* __restrict__ partials,
                                            unsigned int* __restrict__ ticket,
                                            quire256* __restrict__ q_out, uint16_t* bp16_out,
                                            uint32_t* bp32_out, int rtne16, int rtne32) {
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    const unsigned int t = atomicAdd(ticket, 1u);
    *is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!*is_last) return;
  __threadfence();
  quire256 q = bp::q_zero();
  for (unsigned int i = threadIdx.x; i < gridDim.x; i += blockDim.x) {
    const volatile uint64_t* pw = reinterpret_cast<volatile uint64_t*>(&partials[i]);
    const quire256 v = {{pw[0], pw[1], pw[2], pw[3]}};
    q = bp::q_add(q, v);
  }
  __syncthreads();
  q = block_reduce_q(q, sh);
  if (threadIdx.x == 0) {
    if (q_out) *q_out = q;
    if (bp16_out) *bp16_out = (uint16_t)bp::from_quire<16>(q, rtne16);
    if (bp32_out) *bp32_out = bp::from_quire<32>(q, rtne32);
    *ticket = 0u;  // ready for the next call
  }
}

// Summand modes.  SUM_PLAIN: the codes themselves.  SUM_TERM_L2 /
// SUM_TERM_SMEM: each code p is replaced by -term[p] before it is summed, so
// the quire holds H = -sum p log2(p) (kernels/shannon_entropy_bposit16.cu:
// 63-119, bposit16_reference.py:813-824: the term table lookup, its quire
// value, negation, accumulation); NaR terms add nothing, as bposit16 ->
// quire maps NaR to zero (bposit16_reference.py:602-605).  The table is
// read through L1/L2 (small inputs) or first copied whole into the block's
// shared memory (one 512-thread block per SM), so every lookup is on chip.
enum SumMode { SUM_PLAIN = 0, SUM_TERM_L2 = 1, SUM_TERM_SMEM = 2 };
constexpr int kTermTableBytes = 65536 * 2;

template <int MODE>
__device__ __forceinline__ int32_t summand(uint32_t code, const uint16_t* __restrict__ tab) {
  if (MODE == SUM_TERM_L2) return neg_hi(__ldg(tab + code));
  return neg_hi(tab[code]);
}

template <int MODE>
constexpr size_t sum_smem(int bs) {
  return (size_t)kGroups * bs * sizeof(int) + (MODE == SUM_TERM_SMEM ? kTermTableBytes : 0);
}

// Registers: at most 40 a thread for the decoding modes (6 blocks of 256
// could be resident; the launch uses 3 per SM); the staged-table mode runs
// one 512-thread block per SM and may use 78 (its 32 lookups held before the
// atomics).
template <int MODE, int BS>
__global__ void __launch_bounds__(BS, MODE == SUM_TERM_SMEM ? 1 : 6) quire_sum_bp16_kernel(
    const uint16_t* __restrict__ x, size_t n, const uint16_t* __restrict__ term,
    quire256* __restrict__ partials,
    unsigned int* __restrict__ ticket, quire256* __restrict__ q_out, uint16_t* bp16_out,
    uint32_t* bp32_out, int rtne16, int rtne32) {
  // launched as a programmatic dependent: the set-up below (the group sums
  // cleared, the staged table copied: constant since the device was set up)
  // overlaps the previous kernel's tail; griddepcontrol.wait then waits for
  // that kernel to complete before the codes, the partials or the ticket are
  // touched.  The next kernel may start its own set-up at once.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ bool is_last;
  extern __shared__ __align__(16) uint8_t sum_smem_raw[];   // [kGroups][BS] int, then the table
  int* g = reinterpret_cast<int*>(sum_smem_raw) + threadIdx.x;
  int* gk = g - kGroupLow * BS;                             // this thread's sum for k = 0
  int* g0 = g + (kKeptLow - 1 - kGroupLow) * BS;            // k = kKeptLow - 1
  const uint16_t* tab = term;
  if (MODE == SUM_TERM_SMEM) {
    uint4* dst = reinterpret_cast<uint4*>(sum_smem_raw + (size_t)kGroups * BS * sizeof(int));
    const uint4* src = reinterpret_cast<const uint4*>(term);
    for (int i = threadIdx.x; i < kTermTableBytes / 16; i += BS) dst[i] = __ldg(src + i);
    tab = reinterpret_cast<const uint16_t*>(dst);
  }
#pragma unroll
  for (int i = 0; i < kGroups; ++i) g[i * BS] = 0;
  if (MODE == SUM_TERM_SMEM) __syncthreads();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  quire256 acc = bp::q_zero();
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  size_t done = 0;
  if (vec) {
    const size_t nv = n / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    // U independent 16-byte loads in flight per thread: the staged-table
    // mode runs one 512-thread block per SM and needs them to cover the
    // load latency; positions past the end read as code 0, which adds
    // nothing in every mode (zero, or the NaR term of zero)
    constexpr int U = MODE == SUM_TERM_SMEM ? 4 : 1;
    int iters = 0;
    // the next iteration's loads are issued before this one's codes are
    // summed, so the HBM latency overlaps the integer work
    uint4 nx[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      nx[u] = tid + u * stride < nv ? __ldcs(xv + tid + u * stride) : make_uint4(0u, 0u, 0u, 0u);
    for (size_t i0 = tid; i0 < nv; i0 += U * stride) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        r[u] = nx[u];
        const size_t in = i0 + (U + u) * stride;
        nx[u] = in < nv ? __ldcs(xv + in) : make_uint4(0u, 0u, 0u, 0u);
      }
      if (MODE == SUM_TERM_SMEM) {
        // every lookup first, then the atomics: table and sums share the
        // shared memory, so the compiler keeps program order between a
        // lookup and an earlier atomic, and interleaved they would wait on
        // one another
        const int* dec = reinterpret_cast<const int*>(tab);
        int e[U * 8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            e[u * 8 + 2 * j] = dec_entry(w[j] & 0xFFFFu, dec);
            e[u * 8 + 2 * j + 1] = dec_entry(w[j] >> 16, dec);
          }
        }
#pragma unroll
        for (int i = 0; i < U * 8; ++i) group_add_dec<BS>(g0, e[i]);
      } else {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (MODE != SUM_PLAIN) {
              group_accumulate_bp16<BS>(gk, summand<MODE>(w[j] & 0xFFFFu, tab));
              group_accumulate_bp16<BS>(gk, summand<MODE>(w[j] >> 16, tab));
            } else {
              group_accumulate_bp16<BS>(gk, (int32_t)(w[j] << 16));
              group_accumulate_bp16<BS>(gk, (int32_t)(w[j] & 0xFFFF0000u));
            }
          }
        }
      }
      if (++iters == kFoldIters / U) {     // every 2048 codes per thread
        acc = fold_groups<BS>(gk, acc);
        iters = 0;
      }
    }
    done = nv * 8;
  }
  for (size_t i = done + tid; i < n; i += stride) {
    if (MODE == SUM_TERM_SMEM)
      group_add_dec<BS>(g0, dec_entry(x[i], reinterpret_cast<const int*>(tab)));
    else
      group_accumulate_bp16<BS>(gk, MODE != SUM_PLAIN ? summand<MODE>(x[i], tab)
                                                     : (int32_t)((uint32_t)x[i] << 16));
  }
  // the block step's 32 quires reuse the start of the (now dead) group sums
  quire256* sh = reinterpret_cast<quire256*>(sum_smem_raw);
  acc = block_fold_q<BS>(g - threadIdx.x, acc, sh);
  grid_finish(acc, sh, &is_last, partials, ticket, q_out, bp16_out, bp32_out, rtne16, rtne32);
}

// Every bposit16 code through the exact sum's device decode (bp::sum_bin16)
// against its quire image (bp::quire_from_bp16), as a regime sum folds it:
// res[0] = mismatches, res[1] = the lowest failing code.
__global__ void sum_bin_check_kernel(unsigned long long* res) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 65536u) return;
  int k, v;
  bp::sum_bin16((int32_t)(c << 16), k, v);
  quire256 r = bp::q_zero();
  bool ok = k >= kGroupLow && k < kGroupLow + kGroups && ((c & 0x7FFFu) != 0u || k < kKeptLow);
  if (k >= kKeptLow) {
    int sh = 8 * k + 85;
    uint64_t m = (uint64_t)(v < 0 ? -(long long)v : (long long)v);
    if (sh < 0) {
      ok = ok && (m & ((1ull << -sh) - 1)) == 0;
      m >>= -sh;
      sh = 0;
    }
    r = bp::q_from_shifted(m, sh);
    if (v < 0) r = bp::q_neg(r);
  }
  const quire256 q = bp::quire_from_bp16(c);
  for (int i = 0; i < 4; ++i) ok = ok && q.w[i] == r.w[i];
  if (!ok) {
    atomicAdd(res, 1ull);
    atomicMin(res + 1, (unsigned long long)c);
  }
}

__global__ void fp32_atomic_sum_kernel(const float* __restrict__ x, size_t n, float* acc) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    atomicAdd(acc, x[i]);
}

// ---------------------------------------------------------------------------
// Element-wise conversions.  All are HBM streams: every thread keeps several
// independent 16-byte loads in flight (an unrolled grid stride), and memory
// is touched in whole 32-byte sectors per warp instruction wherever the
// element size allows.
// ---------------------------------------------------------------------------
constexpr int kEwUnroll = 4;

// quire256 -> bposit<NB>.  Each quire is two 16-byte loads (the array is
// 16-byte aligned: the host checks and falls back to the scalar form).
template <int NB, bool RTNE, bool VEC>
__global__ void __launch_bounds__(256) quire_to_bp_kernel(const quire256* __restrict__ q, size_t n,
                                                          void* out) {
  pdl_release();
  pdl_wait();
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i0 = tid; i0 < n; i0 += kEwUnroll * stride) {
    quire256 v[kEwUnroll];
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < n) {
        if (VEC) {
          const ulonglong2* p = reinterpret_cast<const ulonglong2*>(q + i);
          const ulonglong2 a = __ldcs(p), b = __ldcs(p + 1);
          v[u] = quire256{{a.x, a.y, b.x, b.y}};
        } else {
          v[u] = q[i];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < n) {
        const uint32_t r = bp::from_quire_sel<NB>(v[u], RTNE);
        if (NB == 16) static_cast<uint16_t*>(out)[i] = (uint16_t)r;
        else static_cast<uint32_t*>(out)[i] = r;
      }
    }
  }
}

// bposit16 -> quire256.  Lanes 2j and 2j+1 of a warp decode the same code
// and store its low and high 16 bytes, so every store instruction of the
// warp writes 512 contiguous bytes (whole sectors); an output that is not
// 16-byte aligned takes two 8-byte stores per lane instead.
template <bool VEC>
__global__ void __launch_bounds__(256) bp16_to_quire_kernel(const uint16_t* __restrict__ x,
                                                            size_t n, quire256* __restrict__ out) {
  pdl_release();
  pdl_wait();
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t tid = t >> 1;                                // code index of this lane pair
  const int half = (int)(t & 1);
  const size_t stride = ((size_t)gridDim.x * blockDim.x) >> 1;
  for (size_t i0 = tid; i0 < n; i0 += kEwUnroll * stride) {
    uint32_t c[kEwUnroll];
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      c[u] = i < n ? (uint32_t)__ldcs(x + i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < n) {
        uint32_t w[4];
        bp::quire_half_bp16(c[u], half, w);
        const uint4 v = make_uint4(w[0], w[1], w[2], w[3]);
        if (VEC) {
          __stcs(reinterpret_cast<uint4*>(out + i) + half, v);
        } else {
          uint64_t* p = reinterpret_cast<uint64_t*>(out + i) + 2 * half;
          p[0] = (uint64_t)v.x | ((uint64_t)v.y << 32);
          p[1] = (uint64_t)v.z | ((uint64_t)v.w << 32);
        }
      }
    }
  }
}

// int32 -> bposit32 of I / 2^shift for shift in [0, 31], through the
// 33-entry table of bp::i32_table_entry (four values per 16-byte vector).
template <bool RTNE>
__device__ __forceinline__ uint4 enc4_i32(int4 r, const bp::I32Entry* tab) {
  return make_uint4(bp::from_int32_tab<32, RTNE>(r.x, tab), bp::from_int32_tab<32, RTNE>(r.y, tab),
                    bp::from_int32_tab<32, RTNE>(r.z, tab), bp::from_int32_tab<32, RTNE>(r.w, tab));
}

template <bool RTNE>
__global__ void __launch_bounds__(256) int32_to_bp32_tab_kernel(const int32_t* __restrict__ in,
                                                                size_t n, size_t nv, int shift,
                                                                uint32_t* __restrict__ out) {
  pdl_release();
  __shared__ bp::I32Entry tab[33];
  if (threadIdx.x < 33) tab[threadIdx.x] = bp::i32_table_entry<32>(threadIdx.x, shift);
  __syncthreads();
  pdl_wait();
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const int4* iv = reinterpret_cast<const int4*>(in);
  uint4* ov = reinterpret_cast<uint4*>(out);
  for (size_t i0 = tid; i0 < nv; i0 += kEwUnroll * stride) {
    int4 r[kEwUnroll];
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) r[u] = __ldcs(iv + i);
    }
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) __stcs(ov + i, enc4_i32<RTNE>(r[u], tab));
    }
  }
  for (size_t i = nv * 4 + tid; i < n; i += stride) out[i] = bp::from_int32_tab<32, RTNE>(in[i], tab);
}

// Any other shift: the general int64 path.
__global__ void int32_to_bp32_kernel(const int32_t* __restrict__ in, size_t n, int shift,
                                     uint32_t* __restrict__ out, int rtne) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = bp::from_int64<32>(in[i], shift, rtne != 0);
}

// float -> bposit<NB> through the 256-entry exponent table of
// bp::f32_table_entry (shared memory), four values per 16-byte load.
template <int NB, bool RTNE>
__device__ __forceinline__ void store4_bp(void* out, size_t i, float4 f, const bp::F32Entry* t) {
  const uint32_t a = bp::from_float_tab<NB, RTNE>(f.x, t), b = bp::from_float_tab<NB, RTNE>(f.y, t);
  const uint32_t c = bp::from_float_tab<NB, RTNE>(f.z, t), d = bp::from_float_tab<NB, RTNE>(f.w, t);
  if (NB == 16) __stcs(reinterpret_cast<uint2*>(out) + i, make_uint2(a | (b << 16), c | (d << 16)));
  else __stcs(reinterpret_cast<uint4*>(out) + i, make_uint4(a, b, c, d));
}

template <int NB, bool RTNE>
__global__ void __launch_bounds__(256) float_to_bp_f32_kernel(const float* __restrict__ x, size_t n,
                                                              size_t nv, void* out) {
  pdl_release();
  __shared__ bp::F32Entry tab[256];
  tab[threadIdx.x] = bp::f32_table_entry<NB>((int)threadIdx.x);   // 256 threads
  __syncthreads();
  pdl_wait();
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const float4* xv = reinterpret_cast<const float4*>(x);
  for (size_t i0 = tid; i0 < nv; i0 += kEwUnroll * stride) {
    float4 r[kEwUnroll];
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) r[u] = __ldcs(xv + i);
    }
#pragma unroll
    for (int u = 0; u < kEwUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) store4_bp<NB, RTNE>(out, i, r[u], tab);
    }
  }
  for (size_t i = nv * 4 + tid; i < n; i += stride) {
    const uint32_t r = bp::from_float_tab<NB, RTNE>(x[i], tab);
    if (NB == 16) static_cast<uint16_t*>(out)[i] = (uint16_t)r;
    else static_cast<uint32_t*>(out)[i] = r;
  }
}

template <typename F, int NB>
__global__ void float_to_bp_kernel(const F* __restrict__ x, size_t n, void* out, int rtne) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t r = bp::from_double<NB>((double)x[i], rtne != 0);
    if (NB == 16)
      static_cast<uint16_t*>(out)[i] = (uint16_t)r;
    else
      static_cast<uint32_t*>(out)[i] = r;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned grid_for(size_t n, int num_sms, int per_sm = 8) {
  size_t b = (n + 255) / 256;
  const size_t cap = (size_t)num_sms * per_sm;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

}  // namespace

namespace {

template <int MODE, int BS>
int quire_sum_launch(DeviceContext* ctx, const uint16_t* x, size_t n, const uint16_t* term,
                     mosyne_quire256* q_out, uint16_t* bp16_out, uint32_t* bp32_out, int flags,
                     cudaStream_t st, int max_blocks) {
  if (n > 0 && !x) return RC_BAD_ARG;
  // group sums 30 KiB per 256 threads (+ the 128 KiB term table when staged)
  constexpr int kSumSmem = (int)sum_smem<MODE>(BS);
  static_assert(kSumSmem <= 227 * 1024, "shared memory");
  if (ensure_smem_attr((const void*)quire_sum_bp16_kernel<MODE, BS>, kSumSmem) != RC_OK)
    return RC_LAUNCH;
  size_t blocks = (n + 8 * BS - 1) / (8 * BS);  // >= 8 codes per thread
  // every block resident at once (shared memory bounds the blocks per SM)
  size_t cap = (size_t)resident_blocks((const void*)quire_sum_bp16_kernel<MODE, BS>, BS, kSumSmem,
                                       ctx->num_sms);
  // decoding modes: 3 blocks (24 warps) per SM, with the next load in flight,
  // cover the HBM latency; more threads only add their per-thread set-up
  // and fold (2^24 codes: 26.7 us with 6 blocks per SM, 24.8 with 3, 27.9
  // with 2, measured on B200)
  if (MODE != SUM_TERM_SMEM && cap > (size_t)ctx->num_sms * 3) cap = (size_t)ctx->num_sms * 3;
  if (max_blocks > 0 && (size_t)max_blocks < cap) cap = (size_t)max_blocks;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  if (ensure_scratch(&ctx->partials, &ctx->partials_bytes, blocks * sizeof(quire256)))
    return RC_ALLOC;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(BS, 1, 1);
  cfg.dynamicSmemBytes = kSumSmem;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const uint16_t* xc = x;
  quire256* part = static_cast<quire256*>(ctx->partials);
  quire256* qo = reinterpret_cast<quire256*>(q_out);
  const int r16 = (flags & MOSYNE_RTNE_BP16) != 0, r32 = (flags & MOSYNE_RTNE_BP32) != 0;
  if (cudaLaunchKernelEx(&cfg, quire_sum_bp16_kernel<MODE, BS>, xc, n, term, part, ctx->ticket, qo,
                         bp16_out, bp32_out, r16, r32) != cudaSuccess) {
    cudaGetLastError();            // a refused launch must not fail the next one
    return RC_LAUNCH;
  }
  return RC_OK;
}

}  // namespace

int quire_sum_bp16_run(DeviceContext* ctx, const uint16_t* x, size_t n, mosyne_quire256* q_out,
                       uint16_t* bp16_out, uint32_t* bp32_out, int flags, cudaStream_t st,
                       int max_blocks) {
  return quire_sum_launch<SUM_PLAIN, 256>(ctx, x, n, nullptr, q_out, bp16_out, bp32_out, flags,
                                          st, max_blocks);
}

int shannon_entropy_bp16_run(DeviceContext* ctx, const uint16_t* p, size_t n,
                             mosyne_quire256* q_out, uint16_t* bp16_out, uint32_t* bp32_out,
                             int flags, cudaStream_t st, int max_blocks) {
  // the staged table pays once its copy (128 KiB per SM, from L2) is small
  // beside the gathers it saves
  const uint16_t* term = ctx->lut + (size_t)LUT_TERM * 65536;
  if (n >= ((size_t)1 << 20) && ctx->term_dec_ok)   // staged: the pre-decoded summands
    return quire_sum_launch<SUM_TERM_SMEM, 512>(ctx, p, n,
                                                reinterpret_cast<const uint16_t*>(ctx->term_dec),
                                                q_out, bp16_out, bp32_out, flags, st, max_blocks);
  return quire_sum_launch<SUM_TERM_L2, 256>(ctx, p, n, term, q_out, bp16_out, bp32_out, flags, st,
                                            max_blocks);
}

int term_dec_build(const uint16_t* term, int* out, bool* usable) {
  unsigned* bad = nullptr;
  if (cudaMalloc(&bad, sizeof(unsigned)) != cudaSuccess) return RC_ALLOC;
  unsigned h = 0;
  int rc = cudaMemset(bad, 0, sizeof(unsigned)) == cudaSuccess ? RC_OK : RC_LAUNCH;
  if (rc == RC_OK) {
    term_dec_build_kernel<<<32, 1024>>>(term, out, bad);
    rc = (cudaGetLastError() == cudaSuccess &&
          cudaMemcpy(&h, bad, sizeof(unsigned), cudaMemcpyDeviceToHost) == cudaSuccess)
             ? RC_OK
             : RC_LAUNCH;
  }
  cudaFree(bad);
  *usable = rc == RC_OK && h == 0;
  return rc;
}

int sum_bin_check_run(unsigned long long* res, cudaStream_t st) {
  sum_bin_check_kernel<<<256, 256, 0, st>>>(res);
  return launch_rc();
}

int fp32_atomic_sum_run(DeviceContext* ctx, const float* x, size_t n, float* acc,
                        cudaStream_t st) {
  fp32_atomic_sum_kernel<<<grid_for(n, ctx->num_sms), 256, 0, st>>>(x, n, acc);
  return launch_rc();
}

int quire_to_bp_run(DeviceContext* ctx, const mosyne_quire256* q, size_t n, void* out, int nbits,
                    int rtne, cudaStream_t st) {
  if (n == 0) return RC_OK;
  const auto* qq = reinterpret_cast<const quire256*>(q);
  auto sg = [&](const void* k) { return stream_grid(k, 256, 0, ctx->num_sms, (n + 255) / 256); };
  const bool v = aligned16(q);
#define MB_Q2B(NB, R)                                                                          \
  (v ? launch_dependent(quire_to_bp_kernel<NB, R, true>,                                       \
                        sg((const void*)quire_to_bp_kernel<NB, R, true>), 256, st, qq, n, out) \
     : launch_dependent(quire_to_bp_kernel<NB, R, false>,                                      \
                        sg((const void*)quire_to_bp_kernel<NB, R, false>), 256, st, qq, n, out))
  if (nbits == 16) {
    if (rtne) MB_Q2B(16, true); else MB_Q2B(16, false);
  } else {
    if (rtne) MB_Q2B(32, true); else MB_Q2B(32, false);
  }
#undef MB_Q2B
  return launch_rc();
}

int bp16_to_quire_run(DeviceContext* ctx, const uint16_t* x, size_t n, mosyne_quire256* out,
                      cudaStream_t st) {
  if (n == 0) return RC_OK;
  auto* o = reinterpret_cast<quire256*>(out);
  const size_t work = (2 * n + 255) / 256;                 // two lanes per code
  if (aligned16(out))
    launch_dependent(bp16_to_quire_kernel<true>,
                     stream_grid((const void*)bp16_to_quire_kernel<true>, 256, 0, ctx->num_sms, work),
                     256, st, x, n, o);
  else
    launch_dependent(bp16_to_quire_kernel<false>,
                     stream_grid((const void*)bp16_to_quire_kernel<false>, 256, 0, ctx->num_sms, work),
                     256, st, x, n, o);
  return launch_rc();
}

int int32_to_bp32_run(DeviceContext* ctx, const int32_t* in, size_t n, int shift, uint32_t* out,
                      int rtne, cudaStream_t st) {
  if (n == 0) return RC_OK;
  if (shift < 0 || shift > 31) {
    int32_to_bp32_kernel<<<grid_for(n, ctx->num_sms), 256, 0, st>>>(in, n, shift, out, rtne);
    return launch_rc();
  }
  const size_t nv = (aligned16(in) && aligned16(out)) ? n / 4 : 0;
  const size_t work = ((nv ? nv : n) + 255) / 256;
  if (rtne)
    launch_dependent(int32_to_bp32_tab_kernel<true>,
                     stream_grid((const void*)int32_to_bp32_tab_kernel<true>, 256, 0, ctx->num_sms, work),
                     256, st, in, n, nv, shift, out);
  else
    launch_dependent(int32_to_bp32_tab_kernel<false>,
                     stream_grid((const void*)int32_to_bp32_tab_kernel<false>, 256, 0, ctx->num_sms, work),
                     256, st, in, n, nv, shift, out);
  return launch_rc();
}

int float_to_bposit_run(DeviceContext* ctx, const void* x, int dtype, size_t n, void* out,
                        int nbits, int rtne, cudaStream_t st) {
  if (n == 0) return RC_OK;
  if (dtype == MOSYNE_DT_F32) {
    const float* xf = static_cast<const float*>(x);
    // 16-byte input vectors; the output vector is 8 (bposit16) or 16 bytes
    const bool v = aligned16(x) && (reinterpret_cast<uintptr_t>(out) & (nbits == 16 ? 7u : 15u)) == 0;
    const size_t nv = v ? n / 4 : 0;
    const size_t work = ((nv ? nv : n) + 255) / 256;
#define MB_F2B(NB, R)                                                                          \
  launch_dependent(float_to_bp_f32_kernel<NB, R>,                                              \
                   stream_grid((const void*)float_to_bp_f32_kernel<NB, R>, 256, 0, ctx->num_sms, work), \
                   256, st, xf, n, nv, out)
    if (nbits == 16) {
      if (rtne) MB_F2B(16, true); else MB_F2B(16, false);
    } else {
      if (rtne) MB_F2B(32, true); else MB_F2B(32, false);
    }
#undef MB_F2B
  } else if (dtype == MOSYNE_DT_F64) {
    const unsigned g = grid_for(n, ctx->num_sms);
    if (nbits == 16)
      float_to_bp_kernel<double, 16><<<g, 256, 0, st>>>(static_cast<const double*>(x), n, out, rtne);
    else
      float_to_bp_kernel<double, 32><<<g, 256, 0, st>>>(static_cast<const double*>(x), n, out, rtne);
  } else {
    return RC_BAD_ARG;
  }
  return launch_rc();
}

}  // namespace mb
