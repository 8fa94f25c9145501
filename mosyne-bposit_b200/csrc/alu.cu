// alu.cu -- element-wise bposit16 ALU kernels.
//
// The reference bakes ~9.6 MB of tables into a generated header as
// __device__ const arrays (kernels/build_bposit_luts.py:34-335), including a
// 2 MiB bposit16 -> quire table.  Here:
//  * bposit16 -> quire is arithmetic (bp::quire_from_bp16), no table;
//  * the four transcendental tables (log2, exp2, sqrt, recip; 128 KiB each)
//    are uploaded once per device at init and, for large launches, staged
//    into shared memory per CTA (one persistent CTA per SM) so every lookup
//    is an on-chip access; small launches read them through L2.
#include "alu.cuh"
#include "bposit.cuh"
#include "common.cuh"

namespace mb {
namespace {

constexpr uint32_t NAR = 0x8000u;
constexpr uint32_t ONE = 0x4000u;
constexpr int TAB_BYTES = 65536 * 2;

// add = truncating encode of the exact quire sum (bposit16_encode.cuh:472-483;
// bposit16_reference.py:758-772), the sum taken in an int64 (bp::sum16_trunc)
__device__ __forceinline__ uint32_t add16(uint32_t a, uint32_t b) {
  if (a == NAR || b == NAR) return NAR;
  if (a == 0) return b;
  if (b == 0) return a;
  return bp::sum16_trunc(a, b);
}

// exact product, truncated (bposit16_reference.py:507-516; zero before NaR)
__device__ __forceinline__ uint32_t mul16_exact(uint32_t a, uint32_t b) {
  const bp::Dec16 da = bp::decode16(a), db = bp::decode16(b);
  if (da.zero || db.zero) return 0u;
  if (da.nar || db.nar) return NAR;
  const int64_t m = (int64_t)da.mant * (int64_t)db.mant;
  return bp::from_int64<16>((da.neg != db.neg) ? -m : m, -(da.exp2 + db.exp2), false);
}

__device__ __forceinline__ uint32_t abs16(uint32_t x) {
  return (x >> 15) ? ((0u - x) & 0x7FFFu) : x;
}

// mul via log2 + quire add + exp2 (bposit16_encode.cuh:491-537)
__device__ __forceinline__ uint32_t mul16_logexp(uint32_t a, uint32_t b, const uint16_t* lg,
                                                 const uint16_t* ex) {
  if (a == NAR || b == NAR) return NAR;
  if (a == 0 || b == 0) return 0u;
  if (a == ONE) return b;
  if (b == ONE) return a;
  const bool rs = ((a ^ b) >> 15) & 1u;
  const uint32_t la = lg[abs16(a)], lb = lg[abs16(b)];
  const uint32_t ls = bp::sum16_trunc(la, lb);           // quire add of the logarithms
  const uint32_t mag = __ldg(ex + ls);
  if (mag == NAR || mag == 0) return mag;
  return rs ? ((0u - mag) & 0xFFFFu) : mag;
}

enum Op { OP_ADD, OP_MUL, OP_MUL_EXACT, OP_NEG, OP_NEG1, OP_LUT };

template <Op OP>
__device__ __forceinline__ uint32_t apply(uint32_t a, uint32_t b, const uint16_t* t0,
                                          const uint16_t* t1) {
  if (OP == OP_ADD) return add16(a, b);
  if (OP == OP_MUL) return mul16_logexp(a, b, t0, t1);
  if (OP == OP_MUL_EXACT) return mul16_exact(a, b);
  if (OP == OP_NEG) return (a == 0 || a == NAR) ? a : ((0u - a) & 0xFFFFu);
  if (OP == OP_NEG1) return (a == 0 || a == NAR) ? a : (~a & 0xFFFFu);
  return t0[a];  // OP_LUT
}

// Element-wise kernel; STAGE copies table t0 into shared memory first.
// Each thread keeps U independent 16-byte vectors (8 codes each) in flight.
template <Op OP>
__device__ __forceinline__ uint4 apply8(uint4 ra, uint4 rb, const uint16_t* tab,
                                        const uint16_t* t1) {
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
  uint32_t wo[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = apply<OP>(wa[j] & 0xFFFFu, wb[j] & 0xFFFFu, tab, t1);
    const uint32_t hi = apply<OP>(wa[j] >> 16, wb[j] >> 16, tab, t1);
    wo[j] = (lo & 0xFFFFu) | (hi << 16);
  }
  return make_uint4(wo[0], wo[1], wo[2], wo[3]);
}

template <Op OP>
__host__ __device__ constexpr int ew_unroll() {
  return (OP == OP_ADD || OP == OP_MUL || OP == OP_MUL_EXACT) ? 2 : 4;
}

template <Op OP, bool STAGE>
__global__ void __launch_bounds__(1024) ew_kernel(const uint16_t* __restrict__ a,
                                                  const uint16_t* __restrict__ b, size_t n,
                                                  uint16_t* __restrict__ out,
                                                  const uint16_t* __restrict__ t0,
                                                  const uint16_t* __restrict__ t1) {
  constexpr int U = ew_unroll<OP>();
  extern __shared__ __align__(16) uint16_t s_tab[];
  const uint16_t* tab = t0;
  if (STAGE) {
    const uint4* src = reinterpret_cast<const uint4*>(t0);
    uint4* dst = reinterpret_cast<uint4*>(s_tab);
    for (int i = threadIdx.x; i < TAB_BYTES / 16; i += blockDim.x) dst[i] = __ldg(src + i);
    __syncthreads();
    tab = s_tab;
  }
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(out) |
                     (b ? reinterpret_cast<uintptr_t>(b) : 0)) &
                    15) == 0;
  size_t done = 0;
  if (vec) {
    const size_t nv = n / 8;
    const uint4* av = reinterpret_cast<const uint4*>(a);
    const uint4* bv = reinterpret_cast<const uint4*>(b);
    uint4* ov = reinterpret_cast<uint4*>(out);
    for (size_t i0 = tid; i0 < nv; i0 += U * stride) {
      uint4 ra[U], rb[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const size_t i = i0 + u * stride;
        ra[u] = make_uint4(0, 0, 0, 0);
        rb[u] = make_uint4(0, 0, 0, 0);
        if (i < nv) {
          ra[u] = __ldcs(av + i);
          if (b) rb[u] = __ldcs(bv + i);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const size_t i = i0 + u * stride;
        if (i < nv) __stcs(ov + i, apply8<OP>(ra[u], rb[u], tab, t1));
      }
    }
    done = nv * 8;
  }
  for (size_t i = done + tid; i < n; i += stride)
    out[i] = (uint16_t)apply<OP>(a[i], b ? b[i] : 0u, tab, t1);
}

template <Op OP>
int launch_ew(DeviceContext* ctx, const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,
              const uint16_t* t0, const uint16_t* t1, cudaStream_t st) {
  if (n == 0) return RC_OK;
  if (!a || !out) return RC_BAD_ARG;
  const bool table_op = (OP == OP_LUT || OP == OP_MUL);
  const bool stage = table_op && n >= (size_t)ctx->num_sms * 16384;
  if (stage) {
    // one CTA of 1024 threads per SM holding the 128 KiB table
    if (ensure_smem_attr((const void*)ew_kernel<OP, true>, TAB_BYTES) != RC_OK) return RC_LAUNCH;
    ew_kernel<OP, true><<<ctx->num_sms, 1024, TAB_BYTES, st>>>(a, b, n, out, t0, t1);
  } else {
    const unsigned blocks = stream_grid((const void*)ew_kernel<OP, false>, 256, 0, ctx->num_sms,
                                        (n + 8 * 256 - 1) / (8 * 256));
    ew_kernel<OP, false><<<blocks, 256, 0, st>>>(a, b, n, out, t0, t1);
  }
  return launch_rc();
}

}  // namespace

int alu_run(DeviceContext* ctx, int op, const uint16_t* a, const uint16_t* b, size_t n,
            uint16_t* out, cudaStream_t st) {
  const uint16_t* lut = ctx->lut;
  switch (op) {
    case ALU_ADD: return launch_ew<OP_ADD>(ctx, a, b, n, out, nullptr, nullptr, st);
    case ALU_MUL:
      return launch_ew<OP_MUL>(ctx, a, b, n, out, lut + LUT_LOG2 * 65536, lut + LUT_EXP2 * 65536, st);
    case ALU_MUL_EXACT: return launch_ew<OP_MUL_EXACT>(ctx, a, b, n, out, nullptr, nullptr, st);
    case ALU_NEG: return launch_ew<OP_NEG>(ctx, a, nullptr, n, out, nullptr, nullptr, st);
    case ALU_NEG_ONES: return launch_ew<OP_NEG1>(ctx, a, nullptr, n, out, nullptr, nullptr, st);
    case ALU_LOG2: return launch_ew<OP_LUT>(ctx, a, nullptr, n, out, lut + LUT_LOG2 * 65536, nullptr, st);
    case ALU_EXP2: return launch_ew<OP_LUT>(ctx, a, nullptr, n, out, lut + LUT_EXP2 * 65536, nullptr, st);
    case ALU_SQRT: return launch_ew<OP_LUT>(ctx, a, nullptr, n, out, lut + LUT_SQRT * 65536, nullptr, st);
    case ALU_RECIP: return launch_ew<OP_LUT>(ctx, a, nullptr, n, out, lut + LUT_RECIP * 65536, nullptr, st);
    default: return RC_BAD_ARG;
  }
}

}  // namespace mb
