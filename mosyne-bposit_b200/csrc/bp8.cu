// bp8.cu -- bposit8 -> int8 fixed-point decode (kernels/test_mera_isometry_imma.cu:
// 43-69, 166-197): the pre-pass of the bposit8 IMMA path, one byte in, one
// byte out, HBM-bound.
//
// The 256-entry table travels in the kernel's parameter space; each block
// spreads it over shared memory as 32 copies of 256 words, copy l in bank l,
// so the 32 lanes of a warp look up 32 arbitrary codes in one conflict-free
// wavefront.  Each thread keeps four 16-byte loads in flight and stores
// 16 bytes per vector; a head/tail pass handles unaligned ends.
#include <cstdint>

#include "bp8.cuh"
#include "bposit.cuh"

namespace mb {
namespace {

struct Bp8Table {
  int8_t v[256];
};

constexpr int kBp8Threads = 256;
constexpr int kBp8SmemBytes = 256 * 32 * 4;   // 32 KiB

__device__ __forceinline__ uint32_t lut_word(const uint32_t* lut, uint32_t lane4, uint32_t w,
                                             int j) {
  // entry idx of copy `lane` sits at byte (idx * 32 + lane) * 4
  const uint32_t idx = (w >> (8 * j)) & 0xFFu;
  return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(lut) +
                                            ((idx << 7) | lane4));
}

__device__ __forceinline__ uint32_t decode4(const uint32_t* lut, uint32_t lane4, uint32_t w) {
  const uint32_t b0 = lut_word(lut, lane4, w, 0), b1 = lut_word(lut, lane4, w, 1);
  const uint32_t b2 = lut_word(lut, lane4, w, 2), b3 = lut_word(lut, lane4, w, 3);
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

__global__ void __launch_bounds__(kBp8Threads) bp8_to_i8_kernel(
    const __grid_constant__ Bp8Table tab, const uint8_t* __restrict__ in,
    int8_t* __restrict__ out, size_t n, size_t head, size_t nvec) {
  extern __shared__ uint32_t lut[];
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x)
    lut[i] = (uint32_t)(uint8_t)tab.v[i >> 5];
  __syncthreads();
  const uint32_t lane4 = (threadIdx.x & 31u) * 4u;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  // unaligned head and tail, one byte per thread
  const size_t tail0 = head + nvec * 16;
  for (size_t i = tid; i < head; i += stride) out[i] = tab.v[in[i]];
  for (size_t i = tail0 + tid; i < n; i += stride) out[i] = tab.v[in[i]];
  const uint4* src = reinterpret_cast<const uint4*>(in + head);
  uint4* dst = reinterpret_cast<uint4*>(out + head);
  constexpr int U = 4;                       // independent 16-byte loads in flight
  for (size_t i0 = tid; i0 < nvec; i0 += U * stride) {
    uint4 w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nvec) w[u] = __ldcs(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nvec) {
        uint4 r;
        r.x = decode4(lut, lane4, w[u].x);
        r.y = decode4(lut, lane4, w[u].y);
        r.z = decode4(lut, lane4, w[u].z);
        r.w = decode4(lut, lane4, w[u].w);
        __stcs(dst + i, r);
      }
    }
  }
}

Bp8Table g_bp8_table;
bool g_bp8_ready = false;

}  // namespace

int bp8_to_i8_run(const uint8_t* in, size_t n, int8_t* out, int num_sms, cudaStream_t st) {
  if (!g_bp8_ready) {                 // 256 host-side decodes, same on every device
    for (int i = 0; i < 256; ++i) g_bp8_table.v[i] = bp::bposit8_to_int8((uint32_t)i);
    g_bp8_ready = true;
  }
  if (n == 0) return RC_OK;
  // 16-byte vectors need the same alignment phase on both sides
  const uintptr_t ai = reinterpret_cast<uintptr_t>(in), ao = reinterpret_cast<uintptr_t>(out);
  size_t head = n, nvec = 0;
  if ((ai & 15u) == (ao & 15u)) {
    head = (16u - (ai & 15u)) & 15u;
    if (head > n) head = n;
    nvec = (n - head) / 16;
  }
  if (ensure_smem_attr((const void*)bp8_to_i8_kernel, kBp8SmemBytes) != RC_OK) return RC_LAUNCH;
  const size_t work = nvec ? nvec : n;
  const unsigned blocks = stream_grid((const void*)bp8_to_i8_kernel, kBp8Threads, kBp8SmemBytes,
                                      num_sms, (work + kBp8Threads - 1) / kBp8Threads);
  bp8_to_i8_kernel<<<blocks, kBp8Threads, kBp8SmemBytes, st>>>(g_bp8_table, in, out, n, head,
                                                              nvec);
  return launch_rc();
}

}  // namespace mb
