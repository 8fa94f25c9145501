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
// bposit16_reference.py:758-772): the two values as exact floats (`vt`: the
// value of each of the 32,768 magnitude codes, in shared memory for large
// launches), their sum and its exact error on the floating-point pipe
// (bp::sum16_trunc_f32; equal to the int64 bp::sum16_trunc for every pair of
// codes, checked exhaustively on the GPU by mosyne_bposit_debug_alu_check).
// Special codes by selects, so the warp does not diverge.
__device__ __forceinline__ float tab_value(const uint32_t* vt, uint32_t code) {
  return __uint_as_float(vt[bp::mag16(code)] | ((code & 0x8000u) << 16));
}

__device__ __forceinline__ uint32_t add16(uint32_t a, uint32_t b, const uint32_t* vt,
                                          const bp::S16Entry* st) {
  uint32_t r = bp::sum16_trunc_f32(tab_value(vt, a), tab_value(vt, b), st);
  r = b == 0 ? a : r;
  r = a == 0 ? b : r;
  return (a == NAR || b == NAR) ? NAR : r;
}

// exact product, truncated (bposit16_reference.py:507-516; zero before NaR),
// encoded in 32-bit arithmetic (the mantissa product has <= 26 bits)
__device__ __forceinline__ uint32_t mul16_exact(uint32_t a, uint32_t b) {
  const bp::Dec16 da = bp::decode16(a), db = bp::decode16(b);
  if (da.zero || db.zero) return 0u;
  if (da.nar || db.nar) return NAR;
  return bp::mul16_trunc_dec(da, db);
}

// The int64 forms the fast ones replace, kept as the reference of the
// exhaustive equivalence check.
__device__ __forceinline__ uint32_t add16_int64(uint32_t a, uint32_t b) {
  if (a == NAR || b == NAR) return NAR;
  if (a == 0) return b;
  if (b == 0) return a;
  return bp::sum16_trunc(a, b);
}

__device__ __forceinline__ uint32_t mul16_exact_int64(uint32_t a, uint32_t b) {
  const bp::Dec16 da = bp::decode16(a), db = bp::decode16(b);
  if (da.zero || db.zero) return 0u;
  if (da.nar || db.nar) return NAR;
  const int64_t m = (int64_t)da.mant * (int64_t)db.mant;
  return bp::from_int64<16>((da.neg != db.neg) ? -m : m, -(da.exp2 + db.exp2), false);
}

__device__ __forceinline__ uint32_t abs16(uint32_t x) {
  return (x >> 15) ? ((0u - x) & 0x7FFFu) : x;
}

// mul via log2 + quire add + exp2 (bposit16_encode.cuh:491-537), from the
// logarithms as exact floats (`lv`: entry m = the quire value of the log2
// code of magnitude code m, signed; in shared memory for large launches): the
// truncated quire sum of the two logarithms on the floating-point pipe, the
// exp2 table read through L1.  Special codes by selects.
__device__ __forceinline__ uint32_t mul16_logexp_f32(uint32_t a, uint32_t b, const uint32_t* lv,
                                                     const uint16_t* ex, const bp::S16Entry* st) {
  const uint32_t ls = bp::sum16_trunc_f32(__uint_as_float(lv[abs16(a)]),
                                          __uint_as_float(lv[abs16(b)]), st);
  const uint32_t mag = __ldg(ex + ls);
  const bool rs = ((a ^ b) >> 15) & 1u;
  uint32_t r = (mag == NAR || mag == 0 || !rs) ? mag : ((0u - mag) & 0xFFFFu);
  r = b == ONE ? a : r;
  r = a == ONE ? b : r;
  r = (a == 0 || b == 0) ? 0u : r;
  return (a == NAR || b == NAR) ? NAR : r;
}

// The int64 form of the same (the reference of the exhaustive check).
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
__device__ __forceinline__ uint32_t apply(uint32_t a, uint32_t b, const bp::S16Entry* st,
                                          const uint16_t* t0,
                                          const uint16_t* t1) {
  if (OP == OP_ADD) return add16(a, b, reinterpret_cast<const uint32_t*>(t0), st);
  if (OP == OP_MUL) return mul16_logexp_f32(a, b, reinterpret_cast<const uint32_t*>(t0), t1, st);
  if (OP == OP_MUL_EXACT) return mul16_exact(a, b);
  if (OP == OP_NEG) return (a == 0 || a == NAR) ? a : ((0u - a) & 0xFFFFu);
  if (OP == OP_NEG1) return (a == 0 || a == NAR) ? a : (~a & 0xFFFFu);
  return t0[a];  // OP_LUT
}

// Element-wise kernel; STAGE copies table t0 into shared memory first.
// Each thread keeps U independent 16-byte vectors (8 codes each) in flight.
template <Op OP>
__device__ __forceinline__ uint4 apply8(uint4 ra, uint4 rb, const bp::S16Entry* st,
                                        const uint16_t* tab,
                                        const uint16_t* t1) {
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
  uint32_t wo[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = apply<OP>(wa[j] & 0xFFFFu, wb[j] & 0xFFFFu, st, tab, t1);
    const uint32_t hi = apply<OP>(wa[j] >> 16, wb[j] >> 16, st, tab, t1);
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
  // launched as a programmatic dependent: the tables (built when the device
  // was set up, constant since) are staged while the previous kernel drains;
  // griddepcontrol.wait precedes every read of the operands and every write
  // of the output.  The next kernel may start its own staging at once.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int U = ew_unroll<OP>();
  extern __shared__ __align__(16) uint16_t s_tab[];
  // the truncated-sum encoder's table (add and the log/exp multiplier)
  __shared__ bp::S16Entry s16[(OP == OP_ADD || OP == OP_MUL) ? 256 : 1];
  if (OP == OP_ADD || OP == OP_MUL) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s16[i] = bp::s16_table_entry(i);
    if (!STAGE) __syncthreads();
  }
  const uint16_t* tab = t0;
  if (STAGE) {
    const uint4* src = reinterpret_cast<const uint4*>(t0);
    uint4* dst = reinterpret_cast<uint4*>(s_tab);
    for (int i = threadIdx.x; i < TAB_BYTES / 16; i += blockDim.x) dst[i] = __ldg(src + i);
    __syncthreads();
    tab = s_tab;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
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
        if (i < nv) __stcs(ov + i, apply8<OP>(ra[u], rb[u], s16, tab, t1));
      }
    }
    done = nv * 8;
  }
  for (size_t i = done + tid; i < n; i += stride)
    out[i] = (uint16_t)apply<OP>(a[i], b ? b[i] : 0u, s16, tab, t1);
}

template <Op OP>
int launch_ew(DeviceContext* ctx, const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,
              const uint16_t* t0, const uint16_t* t1, cudaStream_t st) {
  if (n == 0) return RC_OK;
  if (!a || !out) return RC_BAD_ARG;
  const bool table_op = (OP == OP_LUT || OP == OP_MUL || OP == OP_ADD);
  const bool stage = table_op && n >= (size_t)ctx->num_sms * 16384;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (stage) {
    // one CTA of 1024 threads per SM holding the 128 KiB table
    if (ensure_smem_attr((const void*)ew_kernel<OP, true>, TAB_BYTES) != RC_OK) return RC_LAUNCH;
    cfg.gridDim = dim3((unsigned)ctx->num_sms, 1, 1);
    cfg.blockDim = dim3(1024, 1, 1);
    cfg.dynamicSmemBytes = TAB_BYTES;
    e = cudaLaunchKernelEx(&cfg, ew_kernel<OP, true>, a, b, n, out, t0, t1);
  } else {
    cfg.gridDim = dim3(stream_grid((const void*)ew_kernel<OP, false>, 256, 0, ctx->num_sms,
                                   (n + 8 * 256 - 1) / (8 * 256)), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = 0;
    e = cudaLaunchKernelEx(&cfg, ew_kernel<OP, false>, a, b, n, out, t0, t1);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();            // a refused launch must not fail the next one
    return RC_LAUNCH;
  }
  return RC_OK;
}

__global__ void dec16_build_kernel(uint32_t* out, uint32_t* log_out, const uint16_t* lg) {
  const uint32_t m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m < 32768u) {
    out[m] = __float_as_uint(bp::quire_value16(m));
    log_out[m] = __float_as_uint(bp::quire_value16(lg[m]));
  }
}

// Every (a, b) pair of 16-bit codes, a = the high half of the pair index:
// the fast form against the int64 form; counts mismatches and records the
// first (lowest) mismatching pair index.
__global__ void alu_check_kernel(int op, const uint32_t* dec, const uint32_t* logdec,
                                 const uint16_t* lg, const uint16_t* ex, unsigned long long* res) {
  __shared__ bp::S16Entry st[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) st[i] = bp::s16_table_entry(i);
  __syncthreads();
  const uint64_t total = 1ull << 32;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t a = (uint32_t)(i >> 16), b = (uint32_t)(i & 0xFFFFu);
    uint32_t f, r;
    if (op == 0) {
      f = add16(a, b, dec, st);
      r = add16_int64(a, b);
    } else if (op == 1) {
      f = mul16_exact(a, b);
      r = mul16_exact_int64(a, b);
    } else if (op == 2) {
      f = bp::sum16_trunc_f32(bp::quire_value16(a), bp::quire_value16(b), st);
      r = bp::sum16_trunc(a, b);
    } else {
      f = mul16_logexp_f32(a, b, logdec, ex, st);
      r = mul16_logexp(a, b, lg, ex);
    }
    if ((f & 0xFFFFu) != (r & 0xFFFFu)) {
      atomicAdd(res, 1ull);
      atomicMin(res + 1, (unsigned long long)i);
    }
  }
}

}  // namespace

int alu_build_dec16(uint32_t* out, uint32_t* log_out, const uint16_t* lg) {
  dec16_build_kernel<<<32, 1024>>>(out, log_out, lg);
  if (cudaGetLastError() != cudaSuccess) return RC_LAUNCH;
  return cudaDeviceSynchronize() == cudaSuccess ? RC_OK : RC_LAUNCH;
}

int alu_check_run(DeviceContext* ctx, int op, unsigned long long* res, cudaStream_t st) {
  if (op < 0 || op > 3 || !res) return RC_BAD_ARG;
  alu_check_kernel<<<ctx->num_sms * 8, 256, 0, st>>>(op, ctx->dec16, ctx->logdec16,
                                                     ctx->lut + LUT_LOG2 * 65536,
                                                     ctx->lut + LUT_EXP2 * 65536, res);
  return launch_rc();
}

int alu_run(DeviceContext* ctx, int op, const uint16_t* a, const uint16_t* b, size_t n,
            uint16_t* out, cudaStream_t st) {
  const uint16_t* lut = ctx->lut;
  switch (op) {
    case ALU_ADD:
      return launch_ew<OP_ADD>(ctx, a, b, n, out, reinterpret_cast<const uint16_t*>(ctx->dec16),
                               nullptr, st);
    case ALU_MUL:
      return launch_ew<OP_MUL>(ctx, a, b, n, out, reinterpret_cast<const uint16_t*>(ctx->logdec16),
                               lut + LUT_EXP2 * 65536, st);
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
