// wide.cu -- INT64 accumulators for exact sums of INT32 partials that may not
// fit INT32: the K-split across GPUs when 127^2 * K >= 2^31.
//
// The reference's quire argument (docs/whitepaper/mosyne_bposit_whitepaper.tex
// :495-507: integer addition is associative, so an exact accumulator gives
// one answer for any order) is carried at the width the value needs.  An
// INT8 dot product of length K is below 127^2 * K in magnitude, so an INT64
// lane is exact for K < 5.7e14; its quire256 is the same integer shifted
// left by 96 bits, so the bposit encodings of the two agree.
//
//   widen:     dst[i] (+)= (int64) src[i]          -- INT32 partial tiles in
//   epilogue:  acc (int64, column-major [M,N]) -> bposit32 / bposit16 of
//              acc / 2^shift and (float)acc / (xs[m] * ws[n]) in fp32 / bf16 /
//              fp16, as the INT32 epilogue does for INT32 accumulators.
#include "bposit.cuh"
#include "common.cuh"
#include "gemm.cuh"

namespace mb {
namespace {

// Grid-stride over n elements, four per thread per step with 16-byte loads of
// the INT32 source when both pointers allow it.
__global__ void __launch_bounds__(256) widen_i32_kernel(const int32_t* __restrict__ src, size_t n,
                                                        int64_t* __restrict__ dst, int add,
                                                        int vec) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (vec) {
    const size_t n4 = n / 4;
    const int4* s4 = reinterpret_cast<const int4*>(src);
    longlong2* d2 = reinterpret_cast<longlong2*>(dst);
    for (size_t i = t; i < n4; i += stride) {
      const int4 v = __ldcs(s4 + i);
      longlong2 lo = make_longlong2(v.x, v.y), hi = make_longlong2(v.z, v.w);
      if (add) {
        const longlong2 a = d2[2 * i], b = d2[2 * i + 1];
        lo.x += a.x;
        lo.y += a.y;
        hi.x += b.x;
        hi.y += b.y;
      }
      d2[2 * i] = lo;
      d2[2 * i + 1] = hi;
    }
    for (size_t i = n4 * 4 + t; i < n; i += stride) dst[i] = (add ? dst[i] : 0) + (int64_t)src[i];
  } else {
    for (size_t i = t; i < n; i += stride) dst[i] = (add ? dst[i] : 0) + (int64_t)src[i];
  }
}

// One output channel's M accumulators per block row of the grid: blocks of
// 1024 rows, each thread four rows 256 apart (coalesced), columns strided.
__global__ void __launch_bounds__(256) epilogue_i64_kernel(const int64_t* __restrict__ acc,
                                                           EpiParams p) {
  const int m0 = blockIdx.x * 1024 + threadIdx.x;
  for (int n = blockIdx.y; n < p.N; n += gridDim.y) {
    const int64_t* col = acc + (size_t)n * p.M;
    const float wsn = p.y ? p.ws[(size_t)n * p.ws_stride] : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + i * 256;
      if (m >= p.M) continue;
      const int64_t v = __ldcs(col + m);
      const size_t idx = p.row_major ? (size_t)m * p.N + n : (size_t)n * p.M + m;
      if (p.bp32) p.bp32[idx] = bp::from_int64<32>(v, p.bp_shift, p.rtne32 != 0);
      if (p.bp16) p.bp16[idx] = (uint16_t)bp::from_int64<16>(v, p.bp_shift, p.rtne16 != 0);
      if (p.y) {
        const float y = __fdiv_rn(__ll2float_rn(v), __fmul_rn(p.xs[(size_t)m * p.xs_stride], wsn));
        if (p.y_dtype == MOSYNE_DT_F32) static_cast<float*>(p.y)[idx] = y;
        else if (p.y_dtype == MOSYNE_DT_BF16)
          static_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(y);
        else static_cast<__half*>(p.y)[idx] = __float2half_rn(y);
      }
    }
  }
}

}  // namespace

int widen_i32_run(const int32_t* src, size_t n, int64_t* dst, int add, DeviceContext* ctx,
                  cudaStream_t st) {
  if (n == 0) return RC_OK;
  if (!src || !dst) return RC_BAD_ARG;
  const int vec = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) ? 1 : 0;
  const unsigned blocks = stream_grid((const void*)widen_i32_kernel, 256, 0, ctx->num_sms,
                                      (n + 4 * 256 - 1) / (4 * 256));
  widen_i32_kernel<<<blocks, 256, 0, st>>>(src, n, dst, add, vec);
  return launch_rc();
}

int epilogue_i64_run(const int64_t* acc, const EpiParams& p, DeviceContext* ctx, cudaStream_t st) {
  if (p.M <= 0 || p.N <= 0 || !acc) return RC_BAD_ARG;
  const unsigned gx = (unsigned)((p.M + 1023) / 1024);
  unsigned gy = (unsigned)p.N;
  const unsigned cap = (unsigned)ctx->num_sms * 16;
  if (gx * gy > cap) gy = cap / gx > 0 ? cap / gx : 1;
  epilogue_i64_kernel<<<dim3(gx, gy), 256, 0, st>>>(acc, p);
  return launch_rc();
}

}  // namespace mb
