// capi.cu -- the extern "C" surface of libmosyne_bposit.so and the per-device
// library state behind it.
//
// The reference's nine exports (libmosyne_bposit.cu:95-495) keep their
// names, signatures, column-major layouts, return codes and stream
// behaviour (legacy default stream, no synchronisation).  Their bodies are
// this build's pipeline: coalesced quantiser -> tcgen05 INT8 GEMM with the
// dequant fused into the epilogue (no INT32 tensor in HBM, no cuBLASLt).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "alu.cuh"
#include "bp8.cuh"
#include "bposit.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "quant.cuh"
#include "quire.cuh"

#include "_gen/bposit16_tables.inc"  // kBposit16Tables[MB_LUT_COUNT][65536], generated at build time
static_assert(sizeof(kBposit16Tables) == sizeof(uint16_t) * 65536 * mb::MB_LUT_COUNT,
              "the generated tables and the device table ids disagree");

#ifndef MOSYNE_BPOSIT_VERSION
#define MOSYNE_BPOSIT_VERSION "0.1.0-b200"
#endif

namespace mb {

namespace {
DeviceContext g_ctx[kMaxDevices];
std::mutex g_mu;

// Grow-only device staging for the host-pointer entry points.
struct HostStage {
  void* buf[6] = {};
  size_t bytes[6] = {};
};
HostStage g_stage[kMaxDevices];
// The host-buffer entry points share a device's staging buffers: one call at
// a time per device (each returns only after its last copy).
std::mutex g_stage_mu[kMaxDevices];

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return (d >= 0 && d < kMaxDevices) ? d : -1;
}

void free_ctx(DeviceContext& c) {
  cudaFree(c.err);
  cudaFree(c.x_i8);
  cudaFree(c.x_scale);
  cudaFree(c.amax);
  cudaFree(c.partials);
  cudaFree(c.ticket);
  cudaFree(c.lut);
  cudaFree(c.dec16);
  cudaFree(c.logdec16);
  cudaFree(c.term_dec);
  cudaFree(c.ffn_act);
  cudaFree(c.ffn_h_i8);
  cudaFree(c.ffn_h_scale);
  cudaFree(c.ffn_amax);
  cudaFree(c.sk_ws);
  cudaFree(c.sk_flags);
  cudaFree(c.pt_bar);
  cudaFree(c.bp8_buf);
  c = DeviceContext();
}

int init_device(int d) {
  DeviceContext& c = g_ctx[d];
  if (c.ready) return RC_OK;
  c.device = d;
  if (cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess)
    return -1;
  if (cudaMalloc(&c.err, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&c.ticket, sizeof(unsigned int)) != cudaSuccess ||
      cudaMalloc(&c.lut, sizeof(kBposit16Tables)) != cudaSuccess ||
      cudaMalloc(&c.dec16, 32768 * sizeof(uint32_t)) != cudaSuccess ||
      cudaMalloc(&c.logdec16, 32768 * sizeof(uint32_t)) != cudaSuccess ||
      cudaMalloc(&c.term_dec, 32768 * sizeof(int)) != cudaSuccess ||
      cudaMalloc(&c.sk_flags, 2 * kSkMaxPairs * sizeof(unsigned)) != cudaSuccess ||
      cudaMalloc(&c.pt_bar, 4 * sizeof(unsigned)) != cudaSuccess) {
    free_ctx(c);
    return -2;
  }
  if (cudaMemset(c.err, 0, sizeof(int)) != cudaSuccess ||
      cudaMemset(c.ticket, 0, sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(c.sk_flags, 0, 2 * kSkMaxPairs * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(c.pt_bar, 0, 4 * sizeof(unsigned)) != cudaSuccess ||
      cudaMemcpy(c.lut, kBposit16Tables, sizeof(kBposit16Tables), cudaMemcpyHostToDevice) !=
          cudaSuccess ||
      alu_build_dec16(c.dec16, c.logdec16, c.lut + LUT_LOG2 * 65536) != RC_OK ||
      term_dec_build(c.lut + LUT_TERM * 65536, c.term_dec, &c.term_dec_ok) != RC_OK) {
    free_ctx(c);
    return -3;
  }
  c.ready = true;
  return RC_OK;
}

}  // namespace

DeviceContext* ctx_current() {
  const int d = current_device();
  if (d < 0) return nullptr;
  return g_ctx[d].ready ? &g_ctx[d] : nullptr;
}

DeviceContext* ctx_get_or_init() {
  const int d = current_device();
  if (d < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ctx[d].ready && init_device(d) != RC_OK) return nullptr;
  return &g_ctx[d];
}

int ensure_scratch(void** ptr, size_t* cur, size_t need) {
  if (*cur >= need) return 0;
  if (*ptr) {
    cudaFree(*ptr);
    *ptr = nullptr;
    *cur = 0;
  }
  if (cudaMalloc(ptr, need) != cudaSuccess) return -1;
  *cur = need;
  return 0;
}

int resident_blocks(const void* kernel, int threads, size_t smem, int num_sms) {
  struct Key {
    const void* k;
    int threads;
    size_t smem;
    int sms;
  };
  static std::mutex mu;
  static Key keys[128];
  static int vals[128];
  static int used = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i].k == kernel && keys[i].threads == threads && keys[i].smem == smem &&
        keys[i].sms == num_sms)
      return vals[i];
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int v = per_sm * num_sms;
  if (used < 128) {
    keys[used] = Key{kernel, threads, smem, num_sms};
    vals[used] = v;
    ++used;
  }
  return v;
}

int ensure_smem_attr(const void* kernel, int bytes) {
  struct Key {
    const void* k;
    int dev;
    int bytes;
  };
  static std::mutex mu;
  static Key keys[256];
  static int used = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RC_LAUNCH;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i].k == kernel && keys[i].dev == dev && keys[i].bytes >= bytes) return RC_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return RC_LAUNCH;
  if (used < 256) keys[used++] = Key{kernel, dev, bytes};
  return RC_OK;
}

namespace {

// Streams and events of the pipelined host-buffer GEMM, per device, made on
// first use.  Each call returns only after its last download, so the next
// call's uploads never overwrite staging buffers still in use.
struct HostPipe {
  bool ready = false;
  // downloads alternate between two streams (two copy engines in flight)
  cudaStream_t up = nullptr, compute = nullptr, down = nullptr, down2 = nullptr;
  // [0, 8): blocks of B; [8, 12): pieces of A
  cudaEvent_t uploaded[12] = {}, computed[12] = {};
};
HostPipe g_pipe[kMaxDevices];
std::mutex g_pipe_mu;

HostPipe* host_pipe(int d) {
  std::lock_guard<std::mutex> lk(g_pipe_mu);
  HostPipe& h = g_pipe[d];
  if (!h.ready) {
    if (cudaStreamCreateWithFlags(&h.up, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h.compute, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h.down, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h.down2, cudaStreamNonBlocking) != cudaSuccess)
      return nullptr;
    for (int i = 0; i < 12; ++i)
      if (cudaEventCreateWithFlags(&h.uploaded[i], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&h.computed[i], cudaEventDisableTiming) != cudaSuccess)
        return nullptr;
    h.ready = true;
  }
  return &h;
}

void* stage_buf(int d, int slot, size_t need) {
  HostStage& s = g_stage[d];
  if (ensure_scratch(&s.buf[slot], &s.bytes[slot], need ? need : 1)) return nullptr;
  return s.buf[slot];
}

bool dtype_ok(int dt) { return dt == MOSYNE_DT_F32 || dt == MOSYNE_DT_BF16 || dt == MOSYNE_DT_F16; }

}  // namespace

int linear_impl(const void* x, int x_dtype, int M, int K, const int8_t* w_i8,
                const float* w_scale, int N, void* y, int y_dtype, uint32_t* y_bp32,
                uint16_t* y_bp16, int flags, cudaStream_t st) {
  DeviceContext* ctx = ctx_current();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || K <= 0 || N <= 0 || !x || !w_i8 || !dtype_ok(x_dtype)) return RC_BAD_ARG;
  if (y && (!w_scale || !dtype_ok(y_dtype))) return RC_BAD_ARG;
  const bool per_tensor = (flags & MOSYNE_X_PER_TENSOR) != 0;
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->x_scale), &ctx->x_scale_bytes,
                     (size_t)M * sizeof(float)))
    return RC_ALLOC;
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->x_i8), &ctx->x_i8_bytes,
                     (size_t)M * (size_t)K))
    return RC_ALLOC;
  int rc = quant_activation(ctx, x_dtype, x, M, K, ctx->x_i8, ctx->x_scale,
                            (flags & MOSYNE_X_ROW_MAJOR) != 0, per_tensor, st);
  if (rc) return rc == RC_ALLOC ? RC_ALLOC : RC_LAUNCH;
  EpiParams p;
  p.M = M;
  p.N = N;
  p.xs = ctx->x_scale;
  p.xs_stride = per_tensor ? 0 : 1;
  p.ws = w_scale;
  p.ws_stride = (flags & MOSYNE_WS_SCALAR) ? 0 : 1;
  p.y = y;
  p.y_dtype = y_dtype;
  p.bp32 = y_bp32;
  p.bp16 = y_bp16;
  p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
  p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
  p.rtne16 = (flags & MOSYNE_RTNE_BP16) ? 1 : 0;
  // the quantiser just launched started after every earlier kernel of the
  // stream finished, and lets the GEMM start early: the weights are final
  // then, so the GEMM may pull them into L2 while the activation is quantised
  p.b_prefetch = 1;
  rc = gemm_i8_run(ctx->x_i8, w_i8, K, p, ctx, st);
  return rc == RC_BAD_ARG ? RC_BAD_ARG : (rc ? RC_GEMM : RC_OK);
}

}  // namespace mb

using namespace mb;

extern "C" {

// ---------------------------------------------------------------- reference ABI

int mosyne_bposit_init(void) {
  const int d = current_device();
  if (d < 0) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  return init_device(d);
}

void mosyne_bposit_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  int cur = -1;
  cudaGetDevice(&cur);
  for (int d = 0; d < kMaxDevices; ++d) {
    const bool has_stage = g_stage[d].buf[0] || g_stage[d].buf[1] || g_stage[d].buf[2] ||
                           g_stage[d].buf[3] || g_stage[d].buf[4] || g_stage[d].buf[5];
    if (!g_ctx[d].ready && !has_stage) continue;
    cudaSetDevice(d);
    free_ctx(g_ctx[d]);
    for (int i = 0; i < 6; ++i) {
      cudaFree(g_stage[d].buf[i]);
      g_stage[d].buf[i] = nullptr;
      g_stage[d].bytes[i] = 0;
    }
  }
  if (cur >= 0) cudaSetDevice(cur);
}

int mosyne_bposit_quantize_weight_per_channel(const float* w_fp32, int K, int N, int8_t* w_i8_out,
                                              float* w_scale_out) {
  if (K <= 0 || N <= 0 || !w_fp32 || !w_i8_out || !w_scale_out) return RC_LAUNCH;
  return quant_rows(MOSYNE_DT_F32, w_fp32, N, K, w_i8_out, w_scale_out, 0) ? RC_LAUNCH : RC_OK;
}

int mosyne_bposit_linear_w8a8(const float* x, int M, int K, const int8_t* w_i8,
                              const float* w_scale, int N, float* y) {
  return linear_impl(x, MOSYNE_DT_F32, M, K, w_i8, w_scale, N, y, MOSYNE_DT_F32, nullptr,
                     nullptr, 0, 0);
}

int mosyne_bposit_linear_w8a8_bf16(const mosyne_bf16_t* x, int M, int K, const int8_t* w_i8,
                                   const float* w_scale, int N, float* y) {
  return linear_impl(x, MOSYNE_DT_BF16, M, K, w_i8, w_scale, N, y, MOSYNE_DT_F32, nullptr,
                     nullptr, 0, 0);
}

int mosyne_bposit_linear_w8a8_bf16_io(const mosyne_bf16_t* x, int M, int K, const int8_t* w_i8,
                                      const float* w_scale, int N, mosyne_bf16_t* y) {
  return linear_impl(x, MOSYNE_DT_BF16, M, K, w_i8, w_scale, N, y, MOSYNE_DT_BF16, nullptr,
                     nullptr, 0, 0);
}

int mosyne_bposit_linear_w8a8_fp16(const mosyne_fp16_t* x, int M, int K, const int8_t* w_i8,
                                   const float* w_scale, int N, float* y) {
  return linear_impl(x, MOSYNE_DT_F16, M, K, w_i8, w_scale, N, y, MOSYNE_DT_F32, nullptr,
                     nullptr, 0, 0);
}

int mosyne_bposit_linear_w8a8_fp16_io(const mosyne_fp16_t* x, int M, int K, const int8_t* w_i8,
                                      const float* w_scale, int N, mosyne_fp16_t* y) {
  return linear_impl(x, MOSYNE_DT_F16, M, K, w_i8, w_scale, N, y, MOSYNE_DT_F16, nullptr,
                     nullptr, 0, 0);
}

int mosyne_bposit_linear_w8a8_host(const float* host_x, int M, int K, const float* host_w, int N,
                                   float* host_y) {
  if (!ctx_current()) {
    const int rc = mosyne_bposit_init();
    if (rc != 0) return rc;
  }
  if (M <= 0 || K <= 0 || N <= 0 || !host_x || !host_w || !host_y) return RC_BAD_ARG;
  const int d = current_device();
  if (d < 0) return RC_NOT_INIT;
  std::lock_guard<std::mutex> stage_lock(g_stage_mu[d]);
  float* dx = static_cast<float*>(stage_buf(d, 0, (size_t)M * K * sizeof(float)));
  float* dw = static_cast<float*>(stage_buf(d, 1, (size_t)K * N * sizeof(float)));
  float* dy = static_cast<float*>(stage_buf(d, 2, (size_t)M * N * sizeof(float)));
  int8_t* dwi8 = static_cast<int8_t*>(stage_buf(d, 3, (size_t)K * N));
  float* dws = static_cast<float*>(stage_buf(d, 4, (size_t)N * sizeof(float)));
  if (!dx || !dw || !dy || !dwi8 || !dws) return RC_ALLOC;
  if (cudaMemcpy(dx, host_x, (size_t)M * K * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dw, host_w, (size_t)K * N * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
    return RC_LAUNCH;
  int rc = mosyne_bposit_quantize_weight_per_channel(dw, K, N, dwi8, dws);
  if (rc == 0) rc = mosyne_bposit_linear_w8a8(dx, M, K, dwi8, dws, N, dy);
  if (rc == 0 && cudaMemcpy(host_y, dy, (size_t)M * N * sizeof(float), cudaMemcpyDeviceToHost) !=
                     cudaSuccess)
    rc = RC_LAUNCH;
  return rc;
}

// ---------------------------------------------------------------- additions

const char* mosyne_bposit_version(void) { return MOSYNE_BPOSIT_VERSION " sm_100a tcgen05"; }

int mosyne_bposit_last_error(void) {
  DeviceContext* ctx = ctx_current();
  if (cudaDeviceSynchronize() != cudaSuccess) return RC_LAUNCH;
  // the allocation-free path keeps its own error word (no library state)
  const int rc_noalloc = noalloc_take_error();
  if (rc_noalloc == RC_LAUNCH) return RC_LAUNCH;
  if (!ctx) return rc_noalloc;
  int h = 0;
  if (cudaMemcpy(&h, ctx->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return RC_LAUNCH;
  if (h != 0) {
    cudaMemset(ctx->err, 0, sizeof(int));
    // a wait that gave up may have left stream-K ready flags set
    cudaMemset(ctx->sk_flags, 0, 2 * kSkMaxPairs * sizeof(unsigned));
    return RC_DEVICE_TIMEOUT;
  }
  return rc_noalloc;
}

int mosyne_bposit_set_sm_count_target(int sms) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (sms < 0) return RC_BAD_ARG;
  ctx->sm_target = sms >= ctx->num_sms ? 0 : sms;
  return RC_OK;
}

int mosyne_bposit_debug_wait_timeout(unsigned long long limit_ns, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  return debug_wait_run(limit_ns, ctx, as_stream(stream));
}

int mosyne_bposit_gemm_i8(const int8_t* A, const int8_t* B, int M, int N, int K,
                          const float* x_scale, const float* w_scale, uint32_t* out_bp32,
                          uint16_t* out_bp16, void* out_y, int y_dtype, int32_t* out_i32,
                          int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B) return RC_BAD_ARG;
  if (out_y && (!x_scale || !w_scale || !dtype_ok(y_dtype))) return RC_BAD_ARG;
  EpiParams p;
  p.M = M;
  p.N = N;
  p.xs = x_scale;
  p.ws = w_scale;
  p.xs_stride = (flags & MOSYNE_XS_SCALAR) ? 0 : 1;
  p.ws_stride = (flags & MOSYNE_WS_SCALAR) ? 0 : 1;
  p.bp32 = out_bp32;
  p.bp16 = out_bp16;
  p.y = out_y;
  p.y_dtype = y_dtype;
  p.i32 = out_i32;
  p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
  p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
  p.rtne16 = (flags & MOSYNE_RTNE_BP16) ? 1 : 0;
  p.bp_shift = (flags >> 24) & 31;
  // test hooks: force a GEMM path / tail cut (bits 16-21) / stream-K phase off
  // (bit 22) or on (bit 23) / K slices (bits 29-31)
  const int path = ((flags >> 16) & 0xFF) | ((int)(((unsigned)flags >> 29) & 0x7u) << 8);
  return gemm_i8_run(A, B, K, p, ctx, as_stream(stream), path);
}

int mosyne_bposit_gemm_i8_batched(const int8_t* A, const int8_t* B, int batch, int M, int N,
                                  int K, const float* x_scale, const float* w_scale,
                                  uint32_t* out_bp32, uint16_t* out_bp16, void* out_y,
                                  int y_dtype, int32_t* out_i32, int flags,
                                  mosyne_stream_t stream) {
  if (batch < 0 || M <= 0 || N <= 0 || K <= 0) return RC_BAD_ARG;
  if (batch == 0) return RC_OK;
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (!A || !B || (out_y && (!x_scale || !w_scale || !dtype_ok(y_dtype)))) return RC_BAD_ARG;
  {
    EpiParams p;
    p.M = M;
    p.N = N;
    p.batch = batch;
    p.xs = x_scale;
    p.ws = w_scale;
    p.xs_stride = (flags & MOSYNE_XS_SCALAR) ? 0 : 1;
    p.ws_stride = (flags & MOSYNE_WS_SCALAR) ? 0 : 1;
    p.bp32 = out_bp32;
    p.bp16 = out_bp16;
    p.y = out_y;
    p.y_dtype = y_dtype;
    p.i32 = out_i32;
    p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
    p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
    p.rtne16 = (flags & MOSYNE_RTNE_BP16) ? 1 : 0;
    p.bp_shift = (flags >> 24) & 31;
    if (gemm_i8_batched_fused(A, B, K, p, ctx, as_stream(stream)) == RC_OK) return RC_OK;
  }
  // Otherwise one launch per entry, back to back on one stream: each is
  // launched as a programmatic dependent, so its set-up overlaps the
  // previous one's tail.
  const size_t mk = (size_t)M * K, nk = (size_t)N * K, mn = (size_t)M * N;
  const size_t ysz = y_dtype == MOSYNE_DT_F32 ? 4 : 2;
  const bool xs1 = (flags & MOSYNE_XS_SCALAR) != 0, ws1 = (flags & MOSYNE_WS_SCALAR) != 0;
  for (int b = 0; b < batch; ++b) {
    const int rc = mosyne_bposit_gemm_i8(
        A + b * mk, B + b * nk, M, N, K, x_scale ? x_scale + (xs1 ? 0 : (size_t)b * M) : nullptr,
        w_scale ? w_scale + (ws1 ? 0 : (size_t)b * N) : nullptr,
        out_bp32 ? out_bp32 + b * mn : nullptr, out_bp16 ? out_bp16 + b * mn : nullptr,
        out_y ? static_cast<char*>(out_y) + b * mn * ysz : nullptr, y_dtype,
        out_i32 ? out_i32 + b * mn : nullptr, flags, stream);
    if (rc) return rc;
  }
  return RC_OK;
}

int mosyne_bposit_gemm_i8_host(const int8_t* A, const int8_t* B, int M, int N, int K,
                               uint32_t* out_bp32, int32_t* out_i32, int flags) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B) return RC_BAD_ARG;
  const int d = ctx->device;
  std::lock_guard<std::mutex> stage_lock(g_stage_mu[d]);
  const size_t mk = (size_t)M * K, nk = (size_t)N * K, mn = (size_t)M * N;
  int8_t* dA = static_cast<int8_t*>(stage_buf(d, 0, mk));
  int8_t* dB = static_cast<int8_t*>(stage_buf(d, 1, nk));
  uint32_t* dbp = out_bp32 ? static_cast<uint32_t*>(stage_buf(d, 2, mn * 4)) : nullptr;
  int32_t* di = out_i32 ? static_cast<int32_t*>(stage_buf(d, 3, mn * 4)) : nullptr;
  if (!dA || !dB || (out_bp32 && !dbp) || (out_i32 && !di)) return RC_ALLOC;
  HostPipe* hp = host_pipe(d);
  if (!hp) return RC_LAUNCH;
  // Pipelined over blocks of output channels: B rows [n0, n1) are contiguous
  // in B and their outputs are contiguous in the column-major result, so the
  // upload of block c + 1, the GEMM of block c and the download of block
  // c - 1 run at the same time (host->device and device->host on their own
  // copy engines).  The first block is also cut along M, so its first piece
  // needs only a quarter of A: the downloads, which bound the call, start
  // after A's first piece and B's first block instead of after all of A.  A
  // piece's outputs sit contiguously in device scratch ([channels][piece
  // rows]) and come down with one strided copy into the host result.
  const int nblk = N >= 8 * 512 ? 8 : (N >= 2 * 512 ? N / 512 : 1);
  const int step = ((N + nblk - 1) / nblk + 255) / 256 * 256;
  const int R = (M >= 4 * 512 && nblk > 1) ? 4 : 1;
  const int mstep = ((M + R - 1) / R + 127) / 128 * 128;
  const int gflags = flags & ~(MOSYNE_XS_SCALAR | MOSYNE_WS_SCALAR);
  const int nc0 = N < step ? N : step;
  auto up = [&](void* dst, const void* src, size_t bytes, cudaEvent_t ev) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, hp->up) == cudaSuccess &&
           cudaEventRecord(ev, hp->up) == cudaSuccess;
  };
  int ndown = 0;
  auto down = [&](int m0, int mc, int n0, int nc, size_t doff, cudaEvent_t ev) {
    cudaStream_t ds = (ndown++ & 1) ? hp->down2 : hp->down;
    if (cudaEventRecord(ev, hp->compute) != cudaSuccess ||
        cudaStreamWaitEvent(ds, ev, 0) != cudaSuccess)
      return false;
    const size_t hoff = (size_t)n0 * M + m0;
    if (dbp && cudaMemcpy2DAsync(out_bp32 + hoff, (size_t)M * 4, dbp + doff, (size_t)mc * 4,
                                 (size_t)mc * 4, (size_t)nc, cudaMemcpyDeviceToHost,
                                 ds) != cudaSuccess)
      return false;
    if (di && cudaMemcpy2DAsync(out_i32 + hoff, (size_t)M * 4, di + doff, (size_t)mc * 4,
                                (size_t)mc * 4, (size_t)nc, cudaMemcpyDeviceToHost,
                                ds) != cudaSuccess)
      return false;
    return true;
  };
  // uploads in the order they are needed: A piece 0, B block 0, the other
  // pieces of A, the other blocks of B
  if (!up(dA, A, (size_t)(M < mstep ? M : mstep) * K, hp->uploaded[8]) ||
      !up(dB, B, (size_t)nc0 * K, hp->uploaded[0]))
    return RC_LAUNCH;
  for (int r = 1; r < R && r * mstep < M; ++r) {
    const int m0 = r * mstep, mc = M - m0 < mstep ? M - m0 : mstep;
    if (!up(dA + (size_t)m0 * K, A + (size_t)m0 * K, (size_t)mc * K, hp->uploaded[8 + r]))
      return RC_LAUNCH;
  }
  int c = 0;
  for (int n0 = 0; n0 < N; n0 += step, ++c) {
    const int nc = N - n0 < step ? N - n0 : step;
    const size_t boff = (size_t)n0 * K, ooff = (size_t)n0 * M;
    if (c > 0 && !up(dB + boff, B + boff, (size_t)nc * K, hp->uploaded[c])) return RC_LAUNCH;
    if (cudaStreamWaitEvent(hp->compute, hp->uploaded[c], 0) != cudaSuccess) return RC_LAUNCH;
    const int pieces = c == 0 ? R : 1;
    for (int r = 0; r < pieces && r * mstep < M; ++r) {
      const int m0 = pieces > 1 ? r * mstep : 0;
      const int mc = pieces > 1 ? (M - m0 < mstep ? M - m0 : mstep) : M;
      // every piece of A this GEMM reads is up (block 0: its own piece)
      for (int q = (pieces > 1 ? r : 0); q < (pieces > 1 ? r + 1 : R); ++q)
        if (q * mstep < M && cudaStreamWaitEvent(hp->compute, hp->uploaded[8 + q], 0) != cudaSuccess)
          return RC_LAUNCH;
      const size_t doff = ooff + (size_t)nc * m0;
      const int rc = mosyne_bposit_gemm_i8(dA + (size_t)m0 * K, dB + boff, mc, nc, K, nullptr,
                                           nullptr, dbp ? dbp + doff : nullptr, nullptr, nullptr,
                                           MOSYNE_DT_F32, di ? di + doff : nullptr, gflags,
                                           hp->compute);
      if (rc) return rc;
      if (!down(m0, mc, n0, nc, doff, hp->computed[pieces > 1 ? 8 + r : c])) return RC_LAUNCH;
    }
  }
  return cudaStreamSynchronize(hp->down) == cudaSuccess &&
                 cudaStreamSynchronize(hp->down2) == cudaSuccess
             ? RC_OK
             : RC_LAUNCH;
}

int mosyne_bposit_ffn_swiglu_w8a8(const void* x, int x_dtype, int M, int D,
                                  const int8_t* w_gu_i8, const float* w_gu_scale, int F,
                                  const int8_t* w_down_i8, const float* w_down_scale, void* y,
                                  int y_dtype, float* act, int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || D <= 0 || F <= 0 || (F % 32) != 0 || !x || !w_gu_i8 || !w_gu_scale ||
      !w_down_i8 || !w_down_scale || !y || !dtype_ok(x_dtype) || !dtype_ok(y_dtype))
    return RC_BAD_ARG;
  if ((D % 16) != 0 || (F % 16) != 0) return RC_BAD_ARG;   // TMA row strides
  cudaStream_t st = as_stream(stream);
  const size_t mf = (size_t)M * F;
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->x_scale), &ctx->x_scale_bytes, M * sizeof(float)) ||
      ensure_scratch(reinterpret_cast<void**>(&ctx->x_i8), &ctx->x_i8_bytes, (size_t)M * D) ||
      (!act && ensure_scratch(reinterpret_cast<void**>(&ctx->ffn_act), &ctx->ffn_act_bytes,
                              mf * sizeof(float))) ||
      ensure_scratch(reinterpret_cast<void**>(&ctx->ffn_h_i8), &ctx->ffn_h_i8_bytes, mf) ||
      ensure_scratch(reinterpret_cast<void**>(&ctx->ffn_h_scale), &ctx->ffn_h_scale_bytes,
                     M * sizeof(float)) ||
      ensure_scratch(reinterpret_cast<void**>(&ctx->ffn_amax), &ctx->ffn_amax_bytes,
                     M * sizeof(uint32_t)))
    return RC_ALLOC;
  float* a = act ? act : ctx->ffn_act;
  // 1. per-token int8 of x (row-major [M, D])
  int rc = quant_activation(ctx, x_dtype, x, M, D, ctx->x_i8, ctx->x_scale, true, false, st);
  if (rc) return rc == RC_ALLOC ? RC_ALLOC : RC_LAUNCH;
  // 2. gate and up in one GEMM (N = 2F, interleaved channel blocks); the
  //    epilogue writes silu(gate) * up and each row's |max|
  if (zero_words_run(ctx->ffn_amax, (size_t)M, st) != RC_OK) return RC_LAUNCH;
  EpiParams p;
  p.M = M;
  p.N = 2 * F;
  p.xs = ctx->x_scale;
  p.ws = w_gu_scale;
  p.y = a;
  p.y_dtype = MOSYNE_DT_F32;
  p.row_major = 1;
  p.act_amax = ctx->ffn_amax;
  rc = gemm_i8_run(ctx->x_i8, w_gu_i8, D, p, ctx, st);
  if (rc) return rc == RC_BAD_ARG ? RC_BAD_ARG : RC_GEMM;
  // 3. per-token int8 of the activation with those maxima
  rc = quant_rows_given_amax(a, M, F, ctx->ffn_amax, ctx->ffn_h_i8, ctx->ffn_h_scale, st);
  if (rc) return RC_LAUNCH;
  // 4. down projection, dequantised into y (row-major [M, D])
  EpiParams q;
  q.M = M;
  q.N = D;
  q.xs = ctx->ffn_h_scale;
  q.ws = w_down_scale;
  q.y = y;
  q.y_dtype = y_dtype;
  q.row_major = 1;
  (void)flags;
  rc = gemm_i8_run(ctx->ffn_h_i8, w_down_i8, F, q, ctx, st);
  return rc == RC_BAD_ARG ? RC_BAD_ARG : (rc ? RC_GEMM : RC_OK);
}

int mosyne_bposit_linear_w8a8_ex(const void* x, int x_dtype, int M, int K, const int8_t* w_i8,
                                 const float* w_scale, int N, void* y, int y_dtype,
                                 uint32_t* y_bp32, uint16_t* y_bp16, int flags,
                                 mosyne_stream_t stream) {
  return linear_impl(x, x_dtype, M, K, w_i8, w_scale, N, y, y_dtype, y_bp32, y_bp16, flags,
                     as_stream(stream));
}

int mosyne_bposit_quantize_per_token(const void* x, int x_dtype, int M, int K, int8_t* x_i8,
                                     float* x_scale, int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || K <= 0 || !x || !x_i8 || !dtype_ok(x_dtype)) return RC_BAD_ARG;
  return quant_activation(ctx, x_dtype, x, M, K, x_i8, x_scale, (flags & MOSYNE_X_ROW_MAJOR) != 0,
                          false, as_stream(stream));
}

int mosyne_bposit_quantize_per_tensor(const void* t, int dtype, int rows, int cols, int8_t* q,
                                      float* scale, int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (rows <= 0 || cols <= 0 || !t || !q || !dtype_ok(dtype)) return RC_BAD_ARG;
  return quant_activation(ctx, dtype, t, rows, cols, q, scale, (flags & MOSYNE_X_ROW_MAJOR) != 0,
                          true, as_stream(stream));
}

int mosyne_bposit_row_absmax(const void* x, int x_dtype, int M, int K, float* row_max, int flags,
                             mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || K <= 0 || !x || !row_max || !dtype_ok(x_dtype)) return RC_BAD_ARG;
  return row_absmax(ctx, x_dtype, x, M, K, row_max, (flags & MOSYNE_X_ROW_MAJOR) != 0,
                    as_stream(stream));
}

int mosyne_bposit_quantize_with_max(const void* x, int x_dtype, int M, int K, const float* row_max,
                                    int8_t* x_i8, float* x_scale, int flags,
                                    mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || K <= 0 || !x || !row_max || !x_i8 || !dtype_ok(x_dtype)) return RC_BAD_ARG;
  return quant_with_max(x_dtype, x, M, K, row_max, x_i8, x_scale,
                        (flags & MOSYNE_X_ROW_MAJOR) != 0, as_stream(stream));
}

int mosyne_bposit_quantize_weight_per_channel_ex(const void* w, int dtype, int K, int N,
                                                 int8_t* w_i8_out, float* w_scale_out,
                                                 mosyne_stream_t stream) {
  if (K <= 0 || N <= 0 || !w || !w_i8_out || !w_scale_out || !dtype_ok(dtype)) return RC_BAD_ARG;
  return quant_rows(dtype, w, N, K, w_i8_out, w_scale_out, as_stream(stream));
}

int mosyne_bposit_quire_sum_bp16(const uint16_t* x, size_t n, mosyne_quire256* q_out,
                                 uint16_t* bp16_out, uint32_t* bp32_out, int flags,
                                 mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  return quire_sum_bp16_run(ctx, x, n, q_out, bp16_out, bp32_out, flags, as_stream(stream),
                            (flags >> 16) & 0xFFFF);
}

int mosyne_bposit_shannon_entropy_bp16(const uint16_t* p, size_t n, mosyne_quire256* q_out,
                                       uint32_t* bp32_out, uint16_t* bp16_out, int flags,
                                       mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  return shannon_entropy_bp16_run(ctx, p, n, q_out, bp16_out, bp32_out, flags, as_stream(stream),
                                  (flags >> 16) & 0xFFFF);
}

int shannon_entropy_bposit16_cuda(const uint16_t* d_p, size_t n, uint32_t* d_out) {
  if (n == 0) return -1;
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return -2;
  if (!d_p || !d_out) return -3;
  if (shannon_entropy_bp16_run(ctx, d_p, n, nullptr, nullptr, d_out, 0, nullptr) != RC_OK)
    return -3;
  return cudaStreamSynchronize(nullptr) == cudaSuccess ? 0 : -3;
}

int mosyne_bposit_fp32_atomic_sum(const float* x, size_t n, float* acc, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (!acc || (n && !x)) return RC_BAD_ARG;
  return fp32_atomic_sum_run(ctx, x, n, acc, as_stream(stream));
}

int mosyne_bposit_quire_to_bp16(const mosyne_quire256* q, size_t n, uint16_t* out, int rtne,
                                mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (n && (!q || !out)) return RC_BAD_ARG;
  return quire_to_bp_run(ctx, q, n, out, 16, rtne, as_stream(stream));
}

int mosyne_bposit_quire_to_bp32(const mosyne_quire256* q, size_t n, uint32_t* out, int rtne,
                                mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (n && (!q || !out)) return RC_BAD_ARG;
  return quire_to_bp_run(ctx, q, n, out, 32, rtne, as_stream(stream));
}

int mosyne_bposit_bp16_to_quire(const uint16_t* x, size_t n, mosyne_quire256* out,
                                mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (n && (!x || !out)) return RC_BAD_ARG;
  return bp16_to_quire_run(ctx, x, n, out, as_stream(stream));
}

int mosyne_bposit_int32_to_bp32(const int32_t* in, size_t n, int scale_shift, uint32_t* out,
                                int rtne, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (n && (!in || !out)) return RC_BAD_ARG;
  return int32_to_bp32_run(ctx, in, n, scale_shift, out, rtne, as_stream(stream));
}

int mosyne_bposit_bposit8_to_int8(const uint8_t* in, size_t n, int8_t* out,
                                  mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (n && (!in || !out)) return RC_BAD_ARG;
  return bp8_to_i8_run(in, n, out, ctx->num_sms, as_stream(stream));
}

int mosyne_bposit_gemm_bposit8(const uint8_t* A, const uint8_t* B, int M, int N, int K,
                               uint32_t* out_bp32, int32_t* out_i32, int flags,
                               mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || (!out_bp32 && !out_i32)) return RC_BAD_ARG;
  const size_t na = (size_t)M * K, nb = (size_t)N * K;
  const size_t boff = (na + 255) & ~(size_t)255;
  if (ensure_scratch(reinterpret_cast<void**>(&ctx->bp8_buf), &ctx->bp8_buf_bytes, boff + nb))
    return RC_ALLOC;
  cudaStream_t st = as_stream(stream);
  int8_t* a8 = ctx->bp8_buf;
  int8_t* b8 = ctx->bp8_buf + boff;
  if (bp8_to_i8_pair_run(A, na, a8, B, nb, b8, ctx->num_sms, st) != RC_OK) return RC_LAUNCH;
  EpiParams p;
  p.M = M;
  p.N = N;
  p.bp32 = out_bp32;
  p.i32 = out_i32;
  p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
  p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
  p.bp_shift = 12;                 // two operands with 6 fraction bits each
  const int rc = gemm_i8_run(a8, b8, K, p, ctx, st);
  return rc == RC_BAD_ARG ? RC_BAD_ARG : (rc ? RC_GEMM : RC_OK);
}

int mosyne_bposit_float_to_bposit(const void* x, int dtype, size_t n, void* out, int nbits,
                                  int rtne, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if ((n && (!x || !out)) || (nbits != 16 && nbits != 32)) return RC_BAD_ARG;
  return float_to_bposit_run(ctx, x, dtype, n, out, nbits, rtne, as_stream(stream));
}

int mosyne_bposit_epilogue_i32(const int32_t* acc, int M, int N, const float* x_scale,
                               const float* w_scale, uint32_t* out_bp32, uint16_t* out_bp16,
                               void* out_y, int y_dtype, int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || N <= 0 || !acc) return RC_BAD_ARG;
  if (out_y && (!x_scale || !w_scale || !dtype_ok(y_dtype))) return RC_BAD_ARG;
  EpiParams p;
  p.M = M;
  p.N = N;
  p.xs = x_scale;
  p.ws = w_scale;
  p.xs_stride = (flags & MOSYNE_XS_SCALAR) ? 0 : 1;
  p.ws_stride = (flags & MOSYNE_WS_SCALAR) ? 0 : 1;
  p.bp32 = out_bp32;
  p.bp16 = out_bp16;
  p.y = out_y;
  p.y_dtype = y_dtype;
  p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
  p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
  p.rtne16 = (flags & MOSYNE_RTNE_BP16) ? 1 : 0;
  return epilogue_i32_run(acc, p, ctx, as_stream(stream));
}

int mosyne_bposit_epilogue_i64(const int64_t* acc, int M, int N, const float* x_scale,
                               const float* w_scale, uint32_t* out_bp32, uint16_t* out_bp16,
                               void* out_y, int y_dtype, int flags, mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (M <= 0 || N <= 0 || !acc) return RC_BAD_ARG;
  if (out_y && (!x_scale || !w_scale || !dtype_ok(y_dtype))) return RC_BAD_ARG;
  EpiParams p;
  p.M = M;
  p.N = N;
  p.xs = x_scale;
  p.ws = w_scale;
  p.xs_stride = (flags & MOSYNE_XS_SCALAR) ? 0 : 1;
  p.ws_stride = (flags & MOSYNE_WS_SCALAR) ? 0 : 1;
  p.bp32 = out_bp32;
  p.bp16 = out_bp16;
  p.y = out_y;
  p.y_dtype = y_dtype;
  p.row_major = (flags & MOSYNE_OUT_ROW_MAJOR) ? 1 : 0;
  p.rtne32 = (flags & MOSYNE_RTNE_BP32) ? 1 : 0;
  p.rtne16 = (flags & MOSYNE_RTNE_BP16) ? 1 : 0;
  p.bp_shift = (int)(((unsigned)flags >> 24) & 31u);
  return epilogue_i64_run(acc, p, ctx, as_stream(stream));
}

int mosyne_bposit_widen_i32(const int32_t* src, size_t n, int64_t* dst, int accumulate,
                            mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  return widen_i32_run(src, n, dst, accumulate ? 1 : 0, ctx, as_stream(stream));
}

#define MB_ALU_ENTRY(name, op)                                                           \
  int name(const uint16_t* a, size_t n, uint16_t* out, mosyne_stream_t stream) {         \
    DeviceContext* ctx = ctx_get_or_init();                                              \
    if (!ctx) return RC_NOT_INIT;                                                        \
    return alu_run(ctx, op, a, nullptr, n, out, as_stream(stream));                      \
  }
#define MB_ALU_ENTRY2(name, op)                                                          \
  int name(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out,               \
           mosyne_stream_t stream) {                                                     \
    DeviceContext* ctx = ctx_get_or_init();                                              \
    if (!ctx) return RC_NOT_INIT;                                                        \
    if (n && !b) return RC_BAD_ARG;                                                      \
    return alu_run(ctx, op, a, b, n, out, as_stream(stream));                            \
  }

MB_ALU_ENTRY2(mosyne_bposit16_add, ALU_ADD)
MB_ALU_ENTRY2(mosyne_bposit16_mul, ALU_MUL)
MB_ALU_ENTRY2(mosyne_bposit16_mul_exact, ALU_MUL_EXACT)
MB_ALU_ENTRY(mosyne_bposit16_recip, ALU_RECIP)
MB_ALU_ENTRY(mosyne_bposit16_sqrt, ALU_SQRT)
MB_ALU_ENTRY(mosyne_bposit16_log2, ALU_LOG2)
MB_ALU_ENTRY(mosyne_bposit16_exp2, ALU_EXP2)

int mosyne_bposit16_neg(const uint16_t* a, size_t n, uint16_t* out, int ones_complement,
                        mosyne_stream_t stream) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  return alu_run(ctx, ones_complement ? ALU_NEG_ONES : ALU_NEG, a, nullptr, n, out,
                 as_stream(stream));
}

int mosyne_bposit16_table_host(int which, uint16_t* host_out) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (which < 0 || which >= MB_LUT_COUNT || !host_out) return RC_BAD_ARG;
  return cudaMemcpy(host_out, ctx->lut + (size_t)which * 65536, 65536 * sizeof(uint16_t),
                    cudaMemcpyDeviceToHost) == cudaSuccess
             ? RC_OK
             : RC_LAUNCH;
}

int mosyne_bposit_debug_alu_check(int op, unsigned long long* host_out) {
  DeviceContext* ctx = ctx_get_or_init();
  if (!ctx) return RC_NOT_INIT;
  if (op < 0 || op > 7 || !host_out) return RC_BAD_ARG;
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(unsigned long long)) != cudaSuccess) return RC_ALLOC;
  const unsigned long long init[2] = {0ull, ~0ull};
  int rc = cudaMemcpy(d, init, sizeof(init), cudaMemcpyHostToDevice) == cudaSuccess ? RC_OK
                                                                                    : RC_LAUNCH;
  if (rc == RC_OK)
    rc = op == 7 ? sum_bin_check_run(d, 0)
                 : op >= 4 ? div_check_run(ctx, d, 0, op - 4) : alu_check_run(ctx, op, d, 0);
  if (rc == RC_OK && cudaMemcpy(host_out, d, sizeof(init), cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = RC_LAUNCH;
  cudaFree(d);
  return rc;
}

}  // extern "C"
