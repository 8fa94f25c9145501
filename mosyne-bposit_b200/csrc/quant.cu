// quant.cu -- symmetric int8 quantisers (per-channel, per-token, per-tensor).
//
// Arithmetic is the reference's, bit for bit (libmosyne_bposit.cu:162-244):
// scale = 127.f / max|slice| (1.0 when max <= 1e-8), q = rint(clamp(v*scale,
// +-127)).  The layouts differ from the reference on purpose: activations
// always leave here K-contiguous ([M,K] row-major), the operand layout the
// tensor-core GEMM's TMA loads, and every read is coalesced (the reference's
// per-token kernel walks column-major x with stride M, libmosyne_bposit.cu:218).
#include <atomic>
#include "common.cuh"
#include "quant.cuh"

// kPdlNote: the activation quantisers let a programmatic dependent launch
// (the W8A8 GEMM that follows them) start at once.  The dependent waits
// (griddepcontrol.wait) before it loads any operand; before that it at most
// prefetches its weights into L2, which is coherent, so no stale data can
// result.  Each quantiser's own griddepcontrol.wait, before its first global
// access, waits for the kernel before it to complete, so the GEMM's wait
// covers every earlier kernel.  The row quantisers (registers, a warp or a
// block per row) are themselves launched as programmatic dependents, so
// their launch overlaps the previous
// kernel's tail (e.g. the previous layer's GEMM, which reads the int8
// activations this kernel is about to write).
// The one-row-per-block quantiser is launched so (8192 x 4096 bf16 per token
// 20.5 -> 19.2 us, per-channel 14336 x 4096 fp32 40.8 -> 39.2 us, B200); the
// one-cluster per-tensor quantiser is not: its cluster of 16 CTAs waiting
// beside the previous GEMM made the 128 x 2048 x 11008 linear layer 0.4 us
// slower.  Its griddepcontrol.wait then returns at once.
namespace mb {
namespace {

template <typename T>
struct Vec;  // 16-byte vectors
template <>
struct Vec<float> {
  static constexpr int N = 4;
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per contiguous row: max over the row, then quantise it.  Used for
// per-channel weights (column-major [K,N] = N contiguous rows of K) and for
// row-major activations.  `given_amax` (nullable) supplies a per-tensor max.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) quant_rows_kernel(const T* __restrict__ x, int R, int C,
                                                         int8_t* __restrict__ q,
                                                         float* __restrict__ scale,
                                                         const uint32_t* __restrict__ given_amax,
                                                         int amax_stride, int reverse) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  pdl_wait();
  constexpr int V = Vec<T>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = (reverse ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x) * 8 + warp;
  if (row >= R) return;
  const T* xr = x + (size_t)row * C;
  int8_t* qr = q + (size_t)row * C;
  float m = 0.f;
  if (given_amax) {
    m = __uint_as_float(given_amax[(size_t)row * amax_stride]);
  } else {
    if (VEC) {
      for (int c = lane * V; c < C; c += 32 * V) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
        const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32<T>(v[i])));
      }
    } else {
      for (int c = lane; c < C; c += 32) m = fmaxf(m, fabsf(to_f32<T>(xr[c])));
    }
    m = warp_max(m);
  }
  const float s = quant_scale_from_max(m);
  if (lane == 0 && scale) scale[row] = s;
  if (VEC) {
    for (int c = lane * V; c < C; c += 32 * V) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
      const T* v = reinterpret_cast<const T*>(&raw);
      int8_t o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = quantize1(to_f32<T>(v[i]), s);
      if (V == 4) {
        *reinterpret_cast<uint32_t*>(qr + c) = *reinterpret_cast<uint32_t*>(o);
      } else {
        *reinterpret_cast<uint2*>(qr + c) = *reinterpret_cast<uint2*>(o);
      }
    }
  } else {
    for (int c = lane; c < C; c += 32) qr[c] = quantize1(to_f32<T>(xr[c]), s);
  }
}

// One block per contiguous row, for few and long rows (activations of a few
// hundred tokens): block-wide max, then quantise.  `given_amax` as above;
// `scalar_scale` (nullable) receives the per-tensor scale from row 0.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) quant_row_block_kernel(
    const T* __restrict__ x, int C, int8_t* __restrict__ q, float* __restrict__ scale,
    const uint32_t* __restrict__ given_amax, int amax_stride, float* __restrict__ scalar_scale,
    int reverse) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  pdl_wait();
  constexpr int V = Vec<T>::N;
  __shared__ float red[8];
  const int row = reverse ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
  const T* xr = x + (size_t)row * C;
  int8_t* qr = q + (size_t)row * C;
  float m = 0.f;
  if (given_amax) {
    m = __uint_as_float(given_amax[(size_t)row * amax_stride]);
  } else {
    if (VEC) {
      for (int c = threadIdx.x * V; c < C; c += 256 * V) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
        const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32<T>(v[i])));
      }
    } else {
      for (int c = threadIdx.x; c < C; c += 256) m = fmaxf(m, fabsf(to_f32<T>(xr[c])));
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])),
              fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
  }
  const float s = quant_scale_from_max(m);
  if (threadIdx.x == 0) {
    if (scale) scale[row] = s;
    if (scalar_scale && row == 0) *scalar_scale = s;
  }
  if (VEC) {
    for (int c = threadIdx.x * V; c < C; c += 256 * V) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
      const T* v = reinterpret_cast<const T*>(&raw);
      int8_t o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = quantize1(to_f32<T>(v[i]), s);
      if (V == 4) *reinterpret_cast<uint32_t*>(qr + c) = *reinterpret_cast<uint32_t*>(o);
      else *reinterpret_cast<uint2*>(qr + c) = *reinterpret_cast<uint2*>(o);
    }
  } else {
    for (int c = threadIdx.x; c < C; c += 256) qr[c] = quantize1(to_f32<T>(xr[c]), s);
  }
}

// One CTA per row with the whole row held in registers between the max and
// the quantise step, so the row is read from HBM once (a two-pass kernel
// re-reads it, and with thousands of rows in flight the second read misses
// L2).  NV 16-byte vectors per thread cover rows of up to 256 * NV * V
// elements; each of the NV loads is one 4 KiB coalesced block read.
//
// PT: one scale for the whole tensor, in the same single launch.  Launched
// cooperatively (every block resident), one block per row: each block adds
// its row |max| to the call's slot and arrives at a grid barrier; the last
// to arrive reads the maximum, writes the scalar scale, clears the next
// call's slot and the arrival count, and opens the next generation, which
// releases the others.  The state is self-resetting (graph replays work) and
// the wait is bounded (a give-up sets the device error word).
template <typename T, int NV, bool PT>
__global__ void __launch_bounds__(256) quant_row_reg_kernel(const T* __restrict__ x, int C,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale,
                                                            unsigned int* bar, int* err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int V = Vec<T>::N;
  __shared__ float red[8];
  __shared__ float gmax;
  const int row = blockIdx.x;
  const T* xr = x + (size_t)row * C;
  int8_t* qr = q + (size_t)row * C;
  uint4 raw[NV];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 256 + (int)threadIdx.x) * V;
    raw[j] = c < C ? __ldcs(reinterpret_cast<const uint4*>(xr + c)) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const T* v = reinterpret_cast<const T*>(&raw[j]);
#pragma unroll
    for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32<T>(v[i])));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])),
            fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
  if (PT) {
    if (threadIdx.x == 0) {
      unsigned g;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
      unsigned int* slot = bar + 2 + (g & 1u);
      atomicMax(slot, __float_as_uint(m));
      __threadfence();
      if (atomicAdd(bar, 1u) == gridDim.x - 1) {
        const float mx = __uint_as_float(atomicAdd(slot, 0u));
        bar[2 + ((g + 1u) & 1u)] = 0u;             // the next call's slot starts at zero
        bar[0] = 0u;
        if (scale) *scale = quant_scale_from_max(mx);
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(bar + 1), "r"(g + 1u) : "memory");
        gmax = mx;
      } else {
        unsigned cur = g;
        const unsigned long long t0 = globaltimer_ns();
        while (cur == g) {
          __nanosleep(100);
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar + 1) : "memory");
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            set_error(err, ERR_GRID_BARRIER);
            break;
          }
        }
        gmax = __uint_as_float(atomicAdd(slot, 0u));
      }
    }
    __syncthreads();
    m = gmax;
  }
  const float s = quant_scale_from_max(m);
  if (!PT && threadIdx.x == 0 && scale) scale[row] = s;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 256 + (int)threadIdx.x) * V;
    if (c < C) {
      const T* v = reinterpret_cast<const T*>(&raw[j]);
      int8_t o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = quantize1(to_f32<T>(v[i]), s);
      if (V == 4) __stcs(reinterpret_cast<unsigned int*>(qr + c), *reinterpret_cast<unsigned int*>(o));
      else __stcs(reinterpret_cast<uint2*>(qr + c), *reinterpret_cast<uint2*>(o));
    }
  }
}

// Per-tensor quantisation of a small row-major tensor by ONE thread-block
// cluster (the activation of a decode-sized W8A8 linear).  Each thread loads
// its NV 16-byte vectors into registers (element vector v = j * CTAs * 1024 +
// CTA * 1024 + thread, coalesced); the CTA maxima meet through distributed
// shared memory behind the cluster's hardware barrier, so there is no grid
// barrier in global memory, no spin and no second read; each CTA then
// quantises what it holds.  The second cluster barrier keeps every CTA's
// shared memory alive until all peers have read its maximum.
constexpr int kPtThreads = 1024;
constexpr int kPtMaxNv = 8;        // 1024 threads x 8 vectors: <= 64 registers a thread

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
               "memory");
}

template <typename T, int NV>
__global__ void __launch_bounds__(kPtThreads, 1) quant_pt_cluster_kernel(const T* __restrict__ x,
                                                                        unsigned nvec,
                                                                        int8_t* __restrict__ q,
                                                                        float* __restrict__ scale) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int V = Vec<T>::N;
  __shared__ float red[32];
  __shared__ float cta_max, all_max;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned stride = gridDim.x * kPtThreads;
  const unsigned base = blockIdx.x * kPtThreads + threadIdx.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint4 raw[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const unsigned v = base + (unsigned)j * stride;
    raw[j] = v < nvec ? __ldcs(xv + v) : make_uint4(0u, 0u, 0u, 0u);
  }
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const T* e = reinterpret_cast<const T*>(&raw[j]);
#pragma unroll
    for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32<T>(e[i])));
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = warp_max(red[lane]);
    if (lane == 0) cta_max = m;
  }
  cluster_barrier();                       // every CTA's maximum is in its shared memory
  if (warp == 0) {
    float v = 0.f;
    if ((unsigned)lane < gridDim.x) {
      uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(&cta_max)), remote;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(lane));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    }
    v = warp_max(v);
    if (lane == 0) all_max = v;
  }
  __syncthreads();
  const float s = quant_scale_from_max(all_max);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale) *scale = s;
  uint8_t* qb = reinterpret_cast<uint8_t*>(q);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const unsigned v = base + (unsigned)j * stride;
    if (v < nvec) {
      const T* e = reinterpret_cast<const T*>(&raw[j]);
      int8_t o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = quantize1(to_f32<T>(e[i]), s);
      if (V == 4) __stcs(reinterpret_cast<unsigned int*>(qb + (size_t)v * V), *reinterpret_cast<unsigned int*>(o));
      else __stcs(reinterpret_cast<uint2*>(qb + (size_t)v * V), *reinterpret_cast<uint2*>(o));
    }
  }
  cluster_barrier();                       // no CTA leaves while a peer may read cta_max
}

// Column-major x [M,K] (m contiguous): per-row |max| via coalesced reads of
// 64 consecutive rows, reduced with atomicMax on the fp32 bit pattern (exact
// and order independent for non-negative values).
template <typename T>
__global__ void __launch_bounds__(256) colmajor_rowmax_kernel(const T* __restrict__ x, int M,
                                                              int K, int k_chunk,
                                                              uint32_t* __restrict__ amax) {
  __shared__ float red[4][64];
  const int ml = threadIdx.x & 63, kl = threadIdx.x >> 6;
  const int m = blockIdx.x * 64 + ml;
  const int k_begin = blockIdx.y * k_chunk;
  const int k_end = min(K, k_begin + k_chunk);
  float v = 0.f;
  if (m < M) {
    for (int k = k_begin + kl; k < k_end; k += 4) v = fmaxf(v, fabsf(to_f32<T>(x[(size_t)k * M + m])));
  }
  red[kl][ml] = v;
  __syncthreads();
  if (kl == 0 && m < M) {
    v = fmaxf(fmaxf(red[0][ml], red[1][ml]), fmaxf(red[2][ml], red[3][ml]));
    atomicMax(&amax[m], __float_as_uint(v));
  }
}

// Column-major x [M,K] -> int8 [M,K] row-major through a 64x64 shared tile.
// amax_stride = 1: per-row max (per token); 0: one max (per tensor).
template <typename T>
__global__ void __launch_bounds__(256) colmajor_quant_kernel(const T* __restrict__ x, int M,
                                                             int K,
                                                             const uint32_t* __restrict__ amax,
                                                             int amax_stride,
                                                             int8_t* __restrict__ q,
                                                             float* __restrict__ scale) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  pdl_wait();
  __shared__ __align__(16) int8_t tile[64][64 + 16];
  __shared__ float srow[64];
  const int m0 = blockIdx.x * 64, k0 = blockIdx.y * 64;
  const int ml = threadIdx.x & 63, kl = threadIdx.x >> 6;
  if (threadIdx.x < 64) {
    const int m = m0 + threadIdx.x;
    const float s = m < M ? quant_scale_from_max(__uint_as_float(amax[(size_t)m * amax_stride])) : 1.f;
    srow[threadIdx.x] = s;
    if (scale && blockIdx.y == 0 && m < M && (amax_stride || m == 0)) scale[m] = s;
  }
  __syncthreads();
  const int m = m0 + ml;
  const float s = srow[ml];
#pragma unroll 4
  for (int kk = kl; kk < 64; kk += 4) {
    const int k = k0 + kk;
    int8_t v = 0;
    if (m < M && k < K) v = quantize1(to_f32<T>(x[(size_t)k * M + m]), s);
    tile[ml][kk] = v;
  }
  __syncthreads();
  // 64 rows x 4 chunks of 16 bytes
  const int r = threadIdx.x >> 2, c = (threadIdx.x & 3) * 16;
  const int mo = m0 + r;
  if (mo < M) {
    int8_t* dst = q + (size_t)mo * K + k0 + c;
    if (((K & 15) == 0) && (k0 + c + 16 <= K)) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&tile[r][c]);
    } else {
      for (int i = 0; i < 16 && k0 + c + i < K; ++i) dst[i] = tile[r][c + i];
    }
  }
}

// Four consecutive elements of T as floats (16 bytes of fp32, 8 of bf16/fp16).
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}
template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
  const uint2 r = __ldcs(reinterpret_cast<const uint2*>(p));
  const T* v = reinterpret_cast<const T*>(&r);
  return make_float4(to_f32<T>(v[0]), to_f32<T>(v[1]), to_f32<T>(v[2]), to_f32<T>(v[3]));
}

// Column-major x [M,K] with M % 4 == 0 (every column 4-element aligned):
// each lane takes 4 consecutive rows m, a warp 128 rows of one column k; the
// 8 warps of a block walk the block's K range 8 columns apart with four
// loads in flight each; per-row maxima go through shared memory to one
// atomicMax per row and block.
template <typename T>
__global__ void __launch_bounds__(256) colmajor_rowmax_vec_kernel(const T* __restrict__ x, int M,
                                                                  int K, int k_chunk,
                                                                  uint32_t* __restrict__ amax) {
  __shared__ float red[8][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.x * 128 + lane * 4;
  const int k_begin = blockIdx.y * k_chunk;
  const int k_end = min(K, k_begin + k_chunk);
  float4 mx = make_float4(0.f, 0.f, 0.f, 0.f);
  if (m < M) {
    for (int k = k_begin + warp; k < k_end; k += 32) {
      float4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int kk = k + 8 * u;
        r[u] = kk < k_end ? load4<T>(x + (size_t)kk * M + m) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        mx.x = fmaxf(mx.x, fabsf(r[u].x));
        mx.y = fmaxf(mx.y, fabsf(r[u].y));
        mx.z = fmaxf(mx.z, fabsf(r[u].z));
        mx.w = fmaxf(mx.w, fabsf(r[u].w));
      }
    }
  }
  red[warp][lane * 4 + 0] = mx.x;
  red[warp][lane * 4 + 1] = mx.y;
  red[warp][lane * 4 + 2] = mx.z;
  red[warp][lane * 4 + 3] = mx.w;
  __syncthreads();
  if (threadIdx.x < 128) {
    float v = red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < 8; ++w) v = fmaxf(v, red[w][threadIdx.x]);
    const int mo = blockIdx.x * 128 + threadIdx.x;
    if (mo < M) atomicMax(&amax[mo], __float_as_uint(v));
  }
}

// Column-major x [M,K] (M % 4 == 0) -> int8 [M,K] row-major, 64x64 tiles:
// each thread loads a 4x4 block (4 rows m at 4 columns k; four loads in
// flight), quantises it and transposes it in registers into four 32-bit
// words of 4 consecutive k for one m; a padded shared tile of words then
// gives each output row as 16-byte stores.  With `reverse` the tiles run
// last to first, so the columns the max pass read last are still in L2.
template <typename T>
__global__ void __launch_bounds__(256) colmajor_quant_vec_kernel(const T* __restrict__ x, int M,
                                                                 int K,
                                                                 const uint32_t* __restrict__ amax,
                                                                 int amax_stride,
                                                                 int8_t* __restrict__ q,
                                                                 float* __restrict__ scale,
                                                                 int reverse) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // see kPdlNote
  pdl_wait();
  __shared__ uint32_t tile[64][17];
  __shared__ float srow[64];
  const unsigned nb = gridDim.x * gridDim.y;
  const unsigned b = blockIdx.y * gridDim.x + blockIdx.x;
  const unsigned rb = reverse ? nb - 1 - b : b;
  const int m0 = (int)(rb % gridDim.x) * 64, k0 = (int)(rb / gridDim.x) * 64;
  if (threadIdx.x < 64) {
    const int m = m0 + threadIdx.x;
    const float s = m < M ? quant_scale_from_max(__uint_as_float(amax[(size_t)m * amax_stride])) : 1.f;
    srow[threadIdx.x] = s;
    if (scale && k0 == 0 && m < M && (amax_stride || m == 0)) scale[m] = s;
  }
  __syncthreads();
  const int mq = threadIdx.x & 15, kq = threadIdx.x >> 4;   // 4-row group, 4-column group
  const int m = m0 + 4 * mq, kb = k0 + 4 * kq;
  float4 r[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int k = kb + u;
    r[u] = (m < M && k < K) ? load4<T>(x + (size_t)k * M + m) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float s0 = srow[4 * mq], s1 = srow[4 * mq + 1], s2 = srow[4 * mq + 2], s3 = srow[4 * mq + 3];
  uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;                  // row m+i, columns kb..kb+3
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    w0 |= (uint32_t)(uint8_t)quantize1(r[u].x, s0) << (8 * u);
    w1 |= (uint32_t)(uint8_t)quantize1(r[u].y, s1) << (8 * u);
    w2 |= (uint32_t)(uint8_t)quantize1(r[u].z, s2) << (8 * u);
    w3 |= (uint32_t)(uint8_t)quantize1(r[u].w, s3) << (8 * u);
  }
  tile[4 * mq + 0][kq] = w0;
  tile[4 * mq + 1][kq] = w1;
  tile[4 * mq + 2][kq] = w2;
  tile[4 * mq + 3][kq] = w3;
  __syncthreads();
  // 64 rows x 4 chunks of 16 bytes
  const int rr = threadIdx.x >> 2, c = threadIdx.x & 3;
  const int mo = m0 + rr, ko = k0 + 16 * c;
  if (mo < M && ko < K) {
    int8_t* dst = q + (size_t)mo * K + ko;
    const uint4 v = make_uint4(tile[rr][4 * c], tile[rr][4 * c + 1], tile[rr][4 * c + 2],
                               tile[rr][4 * c + 3]);
    if (((K & 15) == 0) && (ko + 16 <= K)) {
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(&v);
      for (int i = 0; i < 16 && ko + i < K; ++i) dst[i] = (int8_t)vb[i];
    }
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(256) absmax_kernel(const T* __restrict__ x, size_t n,
                                                     uint32_t* __restrict__ amax) {
  __shared__ float red[8];
  float m = 0.f;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (V > 1) {
    const size_t nv = n / V;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    constexpr int U = 4;                     // independent 16-byte loads in flight
    for (size_t i0 = tid; i0 < nv; i0 += U * stride) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const size_t i = i0 + u * stride;
        raw[u] = i < nv ? __ldcs(xv + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T* v = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int j = 0; j < V; ++j) m = fmaxf(m, fabsf(to_f32<T>(v[j])));
      }
    }
    for (size_t i = nv * V + tid; i < n; i += stride) m = fmaxf(m, fabsf(to_f32<T>(x[i])));
  } else {
    for (size_t i = tid; i < n; i += stride) m = fmaxf(m, fabsf(to_f32<T>(x[i])));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) atomicMax(amax, __float_as_uint(m));
  }
}

template <typename T>
bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// Row-major [R, C]: |max| of each row into amax[R] (fp32 bit patterns).
template <typename T>
__global__ void __launch_bounds__(256) rowmax_rows_kernel(const T* __restrict__ x, int R, int C,
                                                          uint32_t* __restrict__ amax) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= R) return;
  const T* xr = x + (size_t)row * C;
  float m = 0.f;
  for (int c = lane; c < C; c += 32) m = fmaxf(m, fabsf(to_f32<T>(xr[c])));
  m = warp_max(m);
  if (lane == 0) amax[row] = __float_as_uint(m);
}

// Rows per launch below which each row gets a whole block instead of a warp
// (a warp per row would leave most SMs idle).
constexpr int kBlockPerRowMax = 2048;

template <typename T, int NV>
void launch_row_reg(const void* x, int R, int C, int8_t* q, float* scale, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see kPdlNote
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)R);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  unsigned int* no_bar = nullptr;
  int* no_err = nullptr;
  cudaLaunchKernelEx(&cfg, quant_row_reg_kernel<T, NV, false>, static_cast<const T*>(x), C, q,
                     scale, no_bar, no_err);   // a refused launch is reported by launch_rc()
}

// The one-launch per-tensor quantiser (rows held in registers, grid barrier);
// false when the rows cannot all be resident or the launch is refused.
template <typename T, int NV>
bool launch_row_reg_pt(DeviceContext* ctx, const void* x, int R, int C, int8_t* q, float* scale,
                       cudaStream_t st) {
  auto kern = quant_row_reg_kernel<T, NV, true>;
  if (R > resident_blocks((const void*)kern, 256, 0, ctx->num_sms)) return false;
  const T* xx = static_cast<const T*>(x);
  unsigned int* bar = ctx->pt_bar;
  int* err = ctx->err;
  void* args[] = {(void*)&xx, (void*)&C, (void*)&q, (void*)&scale, (void*)&bar, (void*)&err};
  if (cudaLaunchCooperativeKernel((const void*)kern, dim3((unsigned)R), dim3(256), args, 0, st) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

// The one-cluster per-tensor quantiser: false when the tensor is too large
// for one cluster or the cluster launch is refused (the caller falls back).
// Cluster of 16 CTAs (non-portable size) where the device schedules it, else 8.
template <typename T, int NV>
bool launch_pt_cluster_nv(const void* x, unsigned nvec, int cl, int8_t* q, float* scale,
                          cudaStream_t st) {
  auto kern = quant_pt_cluster_kernel<T, NV>;
  // whether the 16-CTA cluster is schedulable: asked once (every device of a
  // process is the same part)
  static std::atomic<int> big_ok{-1};
  if (cl > 8 && big_ok.load() == 0) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cl);
  cfg.blockDim = dim3(kPtThreads);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)cl;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cl > 8 && big_ok.load() < 0) {
    int clusters = 0;
    const bool ok =
        cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1) == cudaSuccess &&
        cudaOccupancyMaxActiveClusters(&clusters, (const void*)kern, &cfg) == cudaSuccess &&
        clusters >= 1;
    if (!ok) cudaGetLastError();
    big_ok.store(ok ? 1 : 0);
    if (!ok) return false;
  }
  if (cudaLaunchKernelEx(&cfg, kern, static_cast<const T*>(x), nvec, q, scale) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

template <typename T>
bool launch_pt_cluster(const void* x, size_t n, int8_t* q, float* scale, cudaStream_t st) {
  constexpr int V = Vec<T>::N;
  if (n % V != 0 || !aligned16<T>(x) || (reinterpret_cast<uintptr_t>(q) % V) != 0) return false;
  const size_t nvec = n / V;
  for (int cl : {16, 8}) {
    const size_t per = (size_t)cl * kPtThreads;
    if (nvec > per * kPtMaxNv) continue;
    const int nv = (int)((nvec + per - 1) / per);
    const bool ok = nv <= 1   ? launch_pt_cluster_nv<T, 1>(x, (unsigned)nvec, cl, q, scale, st)
                    : nv <= 2 ? launch_pt_cluster_nv<T, 2>(x, (unsigned)nvec, cl, q, scale, st)
                    : nv <= 4 ? launch_pt_cluster_nv<T, 4>(x, (unsigned)nvec, cl, q, scale, st)
                              : launch_pt_cluster_nv<T, 8>(x, (unsigned)nvec, cl, q, scale, st);
    if (ok) return true;
  }
  return false;
}

// `reverse` walks the rows last to first: after a pass that streamed the
// whole tensor (the per-tensor max), the rows it read last are still in L2.
template <typename T>
int quant_rows_t(const void* x, int R, int C, int8_t* q, float* scale, const uint32_t* amax,
                 cudaStream_t st, int amax_stride = 0, float* scalar_scale = nullptr,
                 int reverse = 0) {
  constexpr int V = Vec<T>::N;
  const bool vec = (C % V == 0) && aligned16<T>(x) && ((reinterpret_cast<uintptr_t>(q) % V) == 0);
  if (!amax && !scalar_scale && vec && C <= 256 * V * 16) {
    const int nv = (C + 256 * V - 1) / (256 * V);     // 16-byte vectors per thread
    if (nv <= 1) launch_row_reg<T, 1>(x, R, C, q, scale, st);
    else if (nv <= 2) launch_row_reg<T, 2>(x, R, C, q, scale, st);
    else if (nv <= 4) launch_row_reg<T, 4>(x, R, C, q, scale, st);
    else if (nv <= 8) launch_row_reg<T, 8>(x, R, C, q, scale, st);
    else launch_row_reg<T, 16>(x, R, C, q, scale, st);
    return launch_rc();
  }
  if (R <= kBlockPerRowMax || scalar_scale) {
    if (vec)
      launch_dependent(quant_row_block_kernel<T, true>, (unsigned)R, 256, st,
                       static_cast<const T*>(x), C, q, scale, amax, amax_stride, scalar_scale,
                       reverse);
    else
      launch_dependent(quant_row_block_kernel<T, false>, (unsigned)R, 256, st,
                       static_cast<const T*>(x), C, q, scale, amax, amax_stride, scalar_scale,
                       reverse);
    return launch_rc();
  }
  // warps per row; a partial last block only when R % 8 != 0, so reversing
  // whole blocks still covers every row once
  const unsigned blocks = (unsigned)((R + 7) / 8);
  if (vec)
    launch_dependent(quant_rows_kernel<T, true>, blocks, 256, st, static_cast<const T*>(x), R, C,
                     q, scale, amax, amax_stride, reverse);
  else
    launch_dependent(quant_rows_kernel<T, false>, blocks, 256, st, static_cast<const T*>(x), R, C,
                     q, scale, amax, amax_stride, reverse);
  return launch_rc();
}

// Column-major max pass + quantise pass; the vector kernels when every
// column starts 4-element aligned.
template <typename T>
bool colmajor_vec_ok(const void* x, int M) {
  return (M % 4) == 0 && (reinterpret_cast<uintptr_t>(x) % (4 * sizeof(T))) == 0;
}

template <typename T>
void colmajor_rowmax_launch(const void* x, int M, int K, uint32_t* amax, int num_sms,
                            cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  if (colmajor_vec_ok<T>(x, M)) {
    // enough K slices that every SM holds its full complement of blocks
    const int gm = (M + 127) / 128;
    const int target = resident_blocks((const void*)colmajor_rowmax_vec_kernel<T>, 256, 0, num_sms);
    int splits = (target + gm - 1) / gm;
    splits = max(1, min(splits, (K + 31) / 32));
    const int k_chunk = (K + splits - 1) / splits;
    colmajor_rowmax_vec_kernel<T><<<dim3(gm, (K + k_chunk - 1) / k_chunk), 256, 0, st>>>(
        xt, M, K, k_chunk, amax);
    return;
  }
  const int gm = (M + 63) / 64;
  int splits = (2 * num_sms + gm - 1) / gm;
  splits = max(1, min(splits, (K + 63) / 64));
  const int k_chunk = (K + splits - 1) / splits;
  colmajor_rowmax_kernel<T><<<dim3(gm, (K + k_chunk - 1) / k_chunk), 256, 0, st>>>(
      xt, M, K, k_chunk, amax);
}

template <typename T>
void colmajor_quant_launch(const void* x, int M, int K, const uint32_t* amax, int amax_stride,
                           int8_t* q, float* scale, int reverse, cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  const dim3 grid((M + 63) / 64, (K + 63) / 64);
  // the quantise pass follows the max pass as a programmatic dependent
  if (colmajor_vec_ok<T>(x, M))
    launch_dependent_smem(colmajor_quant_vec_kernel<T>, grid, 256, 0, st, xt, M, K, amax,
                          amax_stride, q, scale, reverse);
  else
    launch_dependent_smem(colmajor_quant_kernel<T>, grid, 256, 0, st, xt, M, K, amax,
                          amax_stride, q, scale);
}

template <typename T>
int colmajor_per_token_t(DeviceContext* ctx, const void* x, int M, int K, int8_t* q,
                         float* scale, cudaStream_t st) {
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->amax), &ctx->amax_bytes,
                     (size_t)M * sizeof(uint32_t)))
    return RC_ALLOC;
  cudaMemsetAsync(ctx->amax, 0, (size_t)M * sizeof(uint32_t), st);
  colmajor_rowmax_launch<T>(x, M, K, ctx->amax, ctx->num_sms, st);
  colmajor_quant_launch<T>(x, M, K, ctx->amax, 1, q, scale, /*reverse=*/1, st);
  return launch_rc();
}

template <typename T>
int per_tensor_t(DeviceContext* ctx, const void* t, int rows, int cols, int8_t* q, float* scale,
                 bool row_major, cudaStream_t st) {
  constexpr int V = Vec<T>::N;
  // small tensors: one cluster, no grid barrier
  if (row_major && launch_pt_cluster<T>(t, (size_t)rows * (size_t)cols, q, scale, st)) return RC_OK;
  if (row_major && ctx->pt_bar && cols % V == 0 && aligned16<T>(t) &&
      (reinterpret_cast<uintptr_t>(q) % V) == 0 && cols <= 256 * V * 16) {
    const int nv = (cols + 256 * V - 1) / (256 * V);
    const bool ok = nv <= 1   ? launch_row_reg_pt<T, 1>(ctx, t, rows, cols, q, scale, st)
                    : nv <= 2 ? launch_row_reg_pt<T, 2>(ctx, t, rows, cols, q, scale, st)
                    : nv <= 4 ? launch_row_reg_pt<T, 4>(ctx, t, rows, cols, q, scale, st)
                    : nv <= 8 ? launch_row_reg_pt<T, 8>(ctx, t, rows, cols, q, scale, st)
                              : launch_row_reg_pt<T, 16>(ctx, t, rows, cols, q, scale, st);
    if (ok) return RC_OK;
  }
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->amax), &ctx->amax_bytes, sizeof(uint32_t)))
    return RC_ALLOC;
  cudaMemsetAsync(ctx->amax, 0, sizeof(uint32_t), st);
  const size_t n = (size_t)rows * (size_t)cols;
  const size_t work = (n + 2047) / 2048;
  if (aligned16<T>(t))
    absmax_kernel<T, Vec<T>::N><<<stream_grid((const void*)absmax_kernel<T, Vec<T>::N>, 256, 0,
                                              ctx->num_sms, work), 256, 0, st>>>(
        static_cast<const T*>(t), n, ctx->amax);
  else
    absmax_kernel<T, 1><<<stream_grid((const void*)absmax_kernel<T, 1>, 256, 0, ctx->num_sms, work),
                          256, 0, st>>>(static_cast<const T*>(t), n, ctx->amax);
  int rc = launch_rc();
  if (rc) return rc;
  if (row_major)   // the quantiser's row 0 also writes the per-tensor scale
    return quant_rows_t<T>(t, rows, cols, q, nullptr, ctx->amax, st, 0, scale, /*reverse=*/1);
  colmajor_quant_launch<T>(t, rows, cols, ctx->amax, 0, q, scale, /*reverse=*/1, st);
  return launch_rc();
}

__global__ void scalar_scale_kernel(const uint32_t* amax, float* scale) {
  *scale = quant_scale_from_max(__uint_as_float(*amax));
}

}  // namespace

int write_scalar_scale(const uint32_t* amax, float* scale, cudaStream_t st) {
  if (!scale) return RC_OK;
  scalar_scale_kernel<<<1, 1, 0, st>>>(amax, scale);
  return launch_rc();
}

int quant_rows(int dtype, const void* x, int R, int C, int8_t* q, float* scale, cudaStream_t st) {
  if (R <= 0 || C <= 0) return R == 0 || C == 0 ? RC_OK : RC_BAD_ARG;
  switch (dtype) {
    case MOSYNE_DT_F32: return quant_rows_t<float>(x, R, C, q, scale, nullptr, st);
    case MOSYNE_DT_BF16: return quant_rows_t<__nv_bfloat16>(x, R, C, q, scale, nullptr, st);
    case MOSYNE_DT_F16: return quant_rows_t<__half>(x, R, C, q, scale, nullptr, st);
    default: return RC_BAD_ARG;
  }
}

int row_absmax(DeviceContext* ctx, int dtype, const void* x, int M, int K, float* out,
               bool row_major, cudaStream_t st) {
  if (M <= 0 || K <= 0) return RC_BAD_ARG;
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
  if (row_major) {
    const unsigned blocks = (unsigned)((M + 7) / 8);
    switch (dtype) {
      case MOSYNE_DT_F32: rowmax_rows_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), M, K, o); break;
      case MOSYNE_DT_BF16: rowmax_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), M, K, o); break;
      case MOSYNE_DT_F16: rowmax_rows_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x), M, K, o); break;
      default: return RC_BAD_ARG;
    }
    return launch_rc();
  }
  cudaMemsetAsync(o, 0, (size_t)M * sizeof(uint32_t), st);
  switch (dtype) {
    case MOSYNE_DT_F32: colmajor_rowmax_launch<float>(x, M, K, o, ctx->num_sms, st); break;
    case MOSYNE_DT_BF16: colmajor_rowmax_launch<__nv_bfloat16>(x, M, K, o, ctx->num_sms, st); break;
    case MOSYNE_DT_F16: colmajor_rowmax_launch<__half>(x, M, K, o, ctx->num_sms, st); break;
    default: return RC_BAD_ARG;
  }
  return launch_rc();
}

template <typename T>
int quant_given_t(const void* x, int M, int K, const float* row_max, int8_t* q, float* scale,
                  bool row_major, cudaStream_t st) {
  const uint32_t* am = reinterpret_cast<const uint32_t*>(row_max);
  if (row_major) return quant_rows_t<T>(x, M, K, q, scale, am, st, 1);
  colmajor_quant_launch<T>(x, M, K, am, 1, q, scale, 0, st);
  return launch_rc();
}

int quant_rows_given_amax(const float* x, int R, int C, const uint32_t* amax, int8_t* q,
                          float* scale, cudaStream_t st) {
  if (R <= 0 || C <= 0) return RC_BAD_ARG;
  return quant_rows_t<float>(x, R, C, q, scale, amax, st, 1);
}

int quant_with_max(int dtype, const void* x, int M, int K, const float* row_max, int8_t* q,
                   float* scale, bool row_major, cudaStream_t st) {
  if (M <= 0 || K <= 0) return RC_BAD_ARG;
  switch (dtype) {
    case MOSYNE_DT_F32: return quant_given_t<float>(x, M, K, row_max, q, scale, row_major, st);
    case MOSYNE_DT_BF16: return quant_given_t<__nv_bfloat16>(x, M, K, row_max, q, scale, row_major, st);
    case MOSYNE_DT_F16: return quant_given_t<__half>(x, M, K, row_max, q, scale, row_major, st);
    default: return RC_BAD_ARG;
  }
}

template <typename T>
int colmajor_per_token_into_t(const void* x, int M, int K, int8_t* q, float* scale, uint32_t* amax,
                              int num_sms, cudaStream_t st) {
  if (cudaMemsetAsync(amax, 0, (size_t)M * sizeof(uint32_t), st) != cudaSuccess) return RC_LAUNCH;
  colmajor_rowmax_launch<T>(x, M, K, amax, num_sms, st);
  colmajor_quant_launch<T>(x, M, K, amax, 1, q, scale, /*reverse=*/1, st);
  return launch_rc();
}

int quant_per_token_colmajor_into(int dtype, const void* x, int M, int K, int8_t* q, float* scale,
                                  uint32_t* amax_scratch, int num_sms, cudaStream_t st) {
  if (M <= 0 || K <= 0) return RC_BAD_ARG;
  switch (dtype) {
    case MOSYNE_DT_F32: return colmajor_per_token_into_t<float>(x, M, K, q, scale, amax_scratch, num_sms, st);
    case MOSYNE_DT_BF16: return colmajor_per_token_into_t<__nv_bfloat16>(x, M, K, q, scale, amax_scratch, num_sms, st);
    case MOSYNE_DT_F16: return colmajor_per_token_into_t<__half>(x, M, K, q, scale, amax_scratch, num_sms, st);
    default: return RC_BAD_ARG;
  }
}

int quant_activation(DeviceContext* ctx, int dtype, const void* x, int M, int K, int8_t* q,
                     float* scale, bool row_major, bool per_tensor, cudaStream_t st) {
  if (M <= 0 || K <= 0) return RC_BAD_ARG;
  if (per_tensor) {
    switch (dtype) {
      case MOSYNE_DT_F32: return per_tensor_t<float>(ctx, x, M, K, q, scale, row_major, st);
      case MOSYNE_DT_BF16: return per_tensor_t<__nv_bfloat16>(ctx, x, M, K, q, scale, row_major, st);
      case MOSYNE_DT_F16: return per_tensor_t<__half>(ctx, x, M, K, q, scale, row_major, st);
      default: return RC_BAD_ARG;
    }
  }
  if (row_major) return quant_rows(dtype, x, M, K, q, scale, st);
  switch (dtype) {
    case MOSYNE_DT_F32: return colmajor_per_token_t<float>(ctx, x, M, K, q, scale, st);
    case MOSYNE_DT_BF16: return colmajor_per_token_t<__nv_bfloat16>(ctx, x, M, K, q, scale, st);
    case MOSYNE_DT_F16: return colmajor_per_token_t<__half>(ctx, x, M, K, q, scale, st);
    default: return RC_BAD_ARG;
  }
}

}  // namespace mb
