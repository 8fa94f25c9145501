// noalloc.cu -- a W8A8 linear entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a serving process whose memory is
// owned by a caching allocator or capped by its operator, a plugin host that
// forbids raw device allocations, or code that must not trigger the implicit
// device synchronisation a cudaMalloc/cudaFree can cause.  The regular entry
// points grow their scratch with cudaMalloc (and mosyne_bposit_init allocates
// the library state).  This entry point instead keeps its scratch -- the int8
// activations, the per-token scales and row maxima -- in one file-scope
// static __device__ array of fixed size, reserved when the library is loaded
// and held by every GPU that loads the library until the process exits.
//
// Limits: M <= kNoAllocMaxRows and M * K <= kNoAllocMaxQuantBytes; larger
// inputs are rejected with MOSYNE_RC_SCRATCH_LIMIT (-21).
//
// Set-up: the first call on each device (with that device current) looks the
// array's device address up with cudaGetSymbolAddress; make that first call
// before any stream capture.  The address is cached for the life of the
// process: cudaDeviceReset on a device that has used this entry point is not
// supported (the cached address would belong to the destroyed context).  All
// calls share the array and each call overwrites it, so calls that overlap on
// the GPU (concurrent streams, or launches that may run at the same time)
// race; order them on one stream.
//
// Errors: every device-side wait of the GEMM is bounded; a wait that gives up
// records its code in an error word that lives in the same static array, and
// mosyne_bposit_last_error() reports it (-30) and clears it.  The entry point
// itself returns before its kernels run, so its return code covers argument
// and launch errors only.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "quant.cuh"

namespace mb {
namespace {

constexpr int kNoAllocMaxRows = 16384;
constexpr size_t kNoAllocMaxQuantBytes = size_t(8) << 20;   // 8 MiB of int8 activations

struct NoAllocScratch {
  int8_t x_i8[kNoAllocMaxQuantBytes];
  float x_scale[kNoAllocMaxRows];
  uint32_t amax[kNoAllocMaxRows];
  int err;                 // device error word of this path (0: no wait gave up)
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

struct NoAllocDevice {
  NoAllocScratch* scratch = nullptr;   // device address of g_noalloc_scratch
  int num_sms = 0;
};

NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current.  In host code the symbol is only
// a host-side stand-in; the kernels get the address returned here.
int noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.scratch) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return RC_LAUNCH;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return RC_LAUNCH;
    d.num_sms = sms;
    d.scratch = static_cast<NoAllocScratch*>(ptr);
  }
  *out = &d;
  return RC_OK;
}

}  // namespace

// Reads and clears the error word of the allocation-free path on the current
// device (0 when that path has not run there).  No allocation: a copy from the
// static array to a host int and a kernel-free memset of one word.
int noalloc_take_error() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RC_OK;
  NoAllocScratch* s = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    s = g_noalloc_dev[dev].scratch;
  }
  if (!s) return RC_OK;
  int h = 0;
  if (cudaMemcpy(&h, &s->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return RC_LAUNCH;
  if (h == 0) return RC_OK;
  if (cudaMemset(&s->err, 0, sizeof(int)) != cudaSuccess) return RC_LAUNCH;
  return RC_DEVICE_TIMEOUT;
}

// The bounded wait that nothing satisfies, recording into this path's error
// word: lets a test see a give-up reported without hanging or faulting a GPU.
int noalloc_debug_wait(unsigned long long limit_ns, cudaStream_t st) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RC_LAUNCH;
  NoAllocDevice* d = nullptr;
  if (noalloc_setup(dev, &d) != RC_OK) return RC_LAUNCH;
  DeviceContext ctx;
  ctx.ready = true;
  ctx.device = dev;
  ctx.num_sms = d->num_sms;
  ctx.err = &d->scratch->err;
  return debug_wait_run(limit_ns, &ctx, st);
}

}  // namespace mb

using namespace mb;

extern "C" int mosyne_bposit_debug_noalloc_wait_timeout(unsigned long long limit_ns,
                                                        mosyne_stream_t stream) {
  return noalloc_debug_wait(limit_ns, as_stream(stream));
}

extern "C" int mosyne_bposit_linear_w8a8_noalloc(const float* x, int M, int K, const int8_t* w_i8,
                                                 const float* w_scale, int N, float* y,
                                                 mosyne_stream_t stream) {
  if (M <= 0 || K <= 0 || N <= 0 || !x || !w_i8 || !w_scale || !y) return RC_BAD_ARG;
  if (M > kNoAllocMaxRows || (size_t)M * (size_t)K > kNoAllocMaxQuantBytes) {
    std::fprintf(stderr,
                 "mosyne_bposit_linear_w8a8_noalloc: M=%d K=%d exceeds the static scratch "
                 "(M <= %d, M*K <= %zu)\n",
                 M, K, kNoAllocMaxRows, kNoAllocMaxQuantBytes);
    return MOSYNE_RC_SCRATCH_LIMIT;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RC_LAUNCH;
  NoAllocDevice* d = nullptr;
  if (noalloc_setup(dev, &d) != RC_OK) return RC_LAUNCH;
  cudaStream_t st = as_stream(stream);
  NoAllocScratch* s = d->scratch;
  // Row maxima must start at zero for every call (the array keeps the last
  // call's contents).
  if (quant_per_token_colmajor_into(MOSYNE_DT_F32, x, M, K, s->x_i8, s->x_scale, s->amax,
                                    d->num_sms, st) != RC_OK)
    return RC_LAUNCH;
  DeviceContext ctx;             // launch parameters only; no library state touched
  ctx.ready = true;
  ctx.device = dev;
  ctx.num_sms = d->num_sms;
  ctx.err = &s->err;             // a bounded wait that gives up is reported by last_error
  ctx.scratch_ok = false;        // no split-K workspace: one K slice per tile
  EpiParams p;
  p.M = M;
  p.N = N;
  p.xs = s->x_scale;
  p.xs_stride = 1;
  p.ws = w_scale;
  p.ws_stride = 1;
  p.y = y;
  p.y_dtype = MOSYNE_DT_F32;
  const int rc = gemm_i8_run(s->x_i8, w_i8, K, p, &ctx, st);
  return rc == RC_BAD_ARG ? RC_BAD_ARG : (rc ? RC_GEMM : RC_OK);
}
