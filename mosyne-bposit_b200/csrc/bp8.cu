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

// One stretch of bytes to decode: an unaligned head and tail, 16-byte vectors
// between them.
struct Bp8Seg {
  const uint8_t* in;
  int8_t* out;
  size_t n, head, nvec;
};

__device__ __forceinline__ void bp8_seg_ends(const Bp8Table& tab, const Bp8Seg& sg, size_t tid,
                                             size_t stride) {
  const size_t tail0 = sg.head + sg.nvec * 16;
  for (size_t i = tid; i < sg.head; i += stride) sg.out[i] = tab.v[sg.in[i]];
  for (size_t i = tail0 + tid; i < sg.n; i += stride) sg.out[i] = tab.v[sg.in[i]];
}

// Up to two stretches in one launch (the A and B operands of a bposit8 GEMM):
// the grid strides over the vectors of both in turn.
__global__ void __launch_bounds__(kBp8Threads) bp8_to_i8_kernel(
    const __grid_constant__ Bp8Table tab, Bp8Seg s0, Bp8Seg s1) {
  // a GEMM launched after this kernel as a programmatic dependent waits for
  // it before reading anything; it may set itself up meanwhile.  This kernel
  // is launched the same way: its table is spread while the previous kernel
  // drains, and it waits for that kernel before touching global memory.
  pdl_release();
  extern __shared__ uint32_t lut[];
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x)
    lut[i] = (uint32_t)(uint8_t)tab.v[i >> 5];
  __syncthreads();
  pdl_wait();
  const uint32_t lane4 = (threadIdx.x & 31u) * 4u;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  bp8_seg_ends(tab, s0, tid, stride);
  bp8_seg_ends(tab, s1, tid, stride);
  const size_t nv = s0.nvec + s1.nvec;
  constexpr int U = 4;                       // independent 16-byte loads in flight
  for (size_t i0 = tid; i0 < nv; i0 += U * stride) {
    uint4 w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) {
        const Bp8Seg& sg = i < s0.nvec ? s0 : s1;
        const size_t j = i < s0.nvec ? i : i - s0.nvec;
        w[u] = __ldcs(reinterpret_cast<const uint4*>(sg.in + sg.head) + j);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const size_t i = i0 + u * stride;
      if (i < nv) {
        const Bp8Seg& sg = i < s0.nvec ? s0 : s1;
        const size_t j = i < s0.nvec ? i : i - s0.nvec;
        uint4 r;
        r.x = decode4(lut, lane4, w[u].x);
        r.y = decode4(lut, lane4, w[u].y);
        r.z = decode4(lut, lane4, w[u].z);
        r.w = decode4(lut, lane4, w[u].w);
        __stcs(reinterpret_cast<uint4*>(sg.out + sg.head) + j, r);
      }
    }
  }
}

Bp8Table g_bp8_table;
bool g_bp8_ready = false;

}  // namespace

namespace {

Bp8Seg bp8_seg(const uint8_t* in, size_t n, int8_t* out) {
  // 16-byte vectors need the same alignment phase on both sides
  const uintptr_t ai = reinterpret_cast<uintptr_t>(in), ao = reinterpret_cast<uintptr_t>(out);
  Bp8Seg sg{in, out, n, n, 0};
  if ((ai & 15u) == (ao & 15u)) {
    sg.head = (16u - (ai & 15u)) & 15u;
    if (sg.head > n) sg.head = n;
    sg.nvec = (n - sg.head) / 16;
  }
  return sg;
}

}  // namespace

int bp8_to_i8_pair_run(const uint8_t* in0, size_t n0, int8_t* out0, const uint8_t* in1,
                       size_t n1, int8_t* out1, int num_sms, cudaStream_t st) {
  if (!g_bp8_ready) {                 // 256 host-side decodes, same on every device
    for (int i = 0; i < 256; ++i) g_bp8_table.v[i] = bp::bposit8_to_int8((uint32_t)i);
    g_bp8_ready = true;
  }
  if (n0 + n1 == 0) return RC_OK;
  const Bp8Seg s0 = bp8_seg(in0, n0, out0), s1 = bp8_seg(in1, n1, out1);
  if (ensure_smem_attr((const void*)bp8_to_i8_kernel, kBp8SmemBytes) != RC_OK) return RC_LAUNCH;
  const size_t nv = s0.nvec + s1.nvec;
  const size_t work = nv ? nv : n0 + n1;
  const unsigned blocks = stream_grid((const void*)bp8_to_i8_kernel, kBp8Threads, kBp8SmemBytes,
                                      num_sms, (work + kBp8Threads - 1) / kBp8Threads);
  launch_dependent_smem(bp8_to_i8_kernel, blocks, kBp8Threads, kBp8SmemBytes, st, g_bp8_table, s0,
                        s1);
  return launch_rc();
}

int bp8_to_i8_run(const uint8_t* in, size_t n, int8_t* out, int num_sms, cudaStream_t st) {
  return bp8_to_i8_pair_run(in, n, out, nullptr, 0, nullptr, num_sms, st);
}

}  // namespace mb
