// common.cuh -- library-wide state, error codes and small device helpers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

#include "mosyne_bposit.h"

namespace mb {

// Per-device library state.  The reference keeps one process-global state for
// the device current at init (libmosyne_bposit.cu:49-77); this build keeps
// one context per device ordinal so multi-GPU processes work.
struct DeviceContext {
  bool ready = false;
  int device = -1;
  int num_sms = 0;
  int* err = nullptr;              // device error word (first failure code)
  // grow-only scratch for the W8A8 path (libmosyne_bposit.cu:56-61)
  int8_t* x_i8 = nullptr;
  size_t x_i8_bytes = 0;
  float* x_scale = nullptr;
  size_t x_scale_bytes = 0;
  uint32_t* amax = nullptr;        // per-row / per-tensor |max| bit patterns
  size_t amax_bytes = 0;
  void* partials = nullptr;        // exact-sum block partials
  size_t partials_bytes = 0;
  unsigned int* ticket = nullptr;  // last-block ticket for grid reductions
  // grid barrier of the one-launch per-tensor quantiser: [0] arrivals,
  // [1] generation, [2 + (generation & 1)] that call's |max| (fp32 bits)
  unsigned int* pt_bar = nullptr;
  // decoded int8 operands of the bposit8 GEMM (A, then B at a 256-byte boundary)
  int8_t* bp8_buf = nullptr;
  size_t bp8_buf_bytes = 0;
  // SwiGLU FFN intermediates: activation [M,F] fp32, its int8 codes, scales
  // and row maxima
  float* ffn_act = nullptr;
  size_t ffn_act_bytes = 0;
  int8_t* ffn_h_i8 = nullptr;
  size_t ffn_h_i8_bytes = 0;
  float* ffn_h_scale = nullptr;
  size_t ffn_h_scale_bytes = 0;
  uint32_t* ffn_amax = nullptr;
  size_t ffn_amax_bytes = 0;
  bool scratch_ok = true;          // false: entry points that must not allocate
  int sm_target = 0;               // GEMM grids use at most this many SMs (0: all)
  // stream-K partial tiles of the CTA-pair GEMM ([pair][cta][256 cols][128 rows]
  // int32) and their per-CTA ready flags (zero between launches)
  int32_t* sk_ws = nullptr;
  size_t sk_ws_bytes = 0;
  unsigned* sk_flags = nullptr;
  // bposit16 ALU tables, 65,536 x u16 each, device resident
  uint16_t* lut = nullptr;         // [MB_LUT_COUNT][65536]
  // values (float bits) of the 32,768 bposit16 magnitude codes (the adder's
  // table) and of the log2 table's entries for those codes (the multiplier's)
  uint32_t* dec16 = nullptr;
  uint32_t* logdec16 = nullptr;
  // the entropy's summands -term[p] pre-decoded into (group, value), p < 0x8000
  int* term_dec = nullptr;
  bool term_dec_ok = false;
};

enum LutId { LUT_LOG2 = 0, LUT_EXP2 = 1, LUT_SQRT = 2, LUT_RECIP = 3, LUT_TERM = 4, MB_LUT_COUNT = 5 };

constexpr int kMaxDevices = 64;

DeviceContext* ctx_current();       // context of the current device, or nullptr
DeviceContext* ctx_get_or_init();   // initialise lazily (for the new entry points)
int ensure_scratch(void** ptr, size_t* cur, size_t need);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device),
// under a lock, so concurrent first calls from several host threads are safe.
int ensure_smem_attr(const void* kernel, int bytes);

// Blocks of `kernel` (with `threads` threads and `smem` dynamic shared bytes)
// that are resident at once on the current device: num_sms times the
// occupancy limit, cached per kernel.  Grid-stride kernels launch at most
// this many, so every block runs in the first and only wave.
int resident_blocks(const void* kernel, int threads, size_t smem, int num_sms);

// min(work, resident_blocks(...)), at least 1.
inline unsigned stream_grid(const void* kernel, int threads, size_t smem, int num_sms,
                            size_t work_blocks) {
  const size_t cap = (size_t)resident_blocks(kernel, threads, smem, num_sms);
  size_t b = work_blocks < cap ? work_blocks : cap;
  return (unsigned)(b == 0 ? 1 : b);
}

// error codes (reference: libmosyne_bposit.cu:95-143, 322-348)
constexpr int RC_OK = 0;
constexpr int RC_LAUNCH = -1;
constexpr int RC_GEMM = -2;
constexpr int RC_NOT_INIT = -10;
constexpr int RC_ALLOC = -11;
constexpr int RC_BAD_ARG = -20;
constexpr int RC_DEVICE_TIMEOUT = -30;

// device error-word codes (which wait gave up)
constexpr int ERR_PRODUCER_WAIT = 1;
constexpr int ERR_MMA_WAIT_FULL = 2;
constexpr int ERR_MMA_WAIT_TMEM = 3;
constexpr int ERR_EPI_WAIT = 4;
constexpr int ERR_DRAIN_WAIT = 5;
constexpr int ERR_TEST_WAIT = 6;
constexpr int ERR_SK_WAIT = 7;        // a stream-K partial tile did not arrive
constexpr int ERR_GRID_BARRIER = 8;   // the one-launch per-tensor quantiser's grid barrier

// Upper bound on CTA pairs of the pair GEMM (stream-K flag array size).
constexpr int kSkMaxPairs = 128;

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

inline cudaStream_t as_stream(mosyne_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline int launch_rc() { return cudaGetLastError() == cudaSuccess ? RC_OK : RC_LAUNCH; }

// Programmatic dependent launch of a stream kernel: it may start (and run its
// set-up) while the previous kernel in the stream drains.  The kernel calls
// pdl_release() first (so the next kernel may start the same way) and
// pdl_wait() before its first global-memory access, which waits for the
// previous kernel to complete and its writes to be visible.  A refused launch
// is reported by launch_rc().
__device__ __forceinline__ void pdl_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline void launch_dependent_smem(void (*kern)(KArgs...), dim3 grid, unsigned block,
                                  size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename... KArgs, typename... Args>
inline void launch_dependent(void (*kern)(KArgs...), unsigned grid, unsigned block,
                             cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// 127 / max in fp32, 1.0 for an all-zero slice (libmosyne_bposit.cu:170, 234).
__device__ __forceinline__ float quant_scale_from_max(float amax) {
  return (amax > 1e-8f) ? __fdiv_rn(127.f, amax) : 1.f;
}

// rint(clamp(v*s, +-127)) (libmosyne_bposit.cu:178-180, 240-242).
__device__ __forceinline__ int8_t quantize1(float v, float s) {
  float t = __fmul_rn(v, s);
  t = fminf(127.f, fmaxf(-127.f, t));
  return (int8_t)__float2int_rn(t);
}

// Wall-clock bound for every device-side wait (ns).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace mb
