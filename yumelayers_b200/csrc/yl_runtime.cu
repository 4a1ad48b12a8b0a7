// yl_runtime.cu -- context, session and tensor lifecycle of the backend.
//
// Replaces MetalEngine's device/queue/pools (MetalEngine.swift:6-193), the
// GpuSession begin/commit/end recording (GpuTraining.swift:4-151) and
// GPUTensor (GPUTensor.swift:9-143).  Waits are bounded and return
// YL_ERR_TIMEOUT where the reference calls exit(70).
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "yl_internal.h"

namespace yl {

static thread_local std::string t_last_error;

yl_status set_error(yl_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return st;
}

static std::atomic<unsigned long long> g_launches{0};

yl_status check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(YL_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
  return YL_OK;
}

yl_status scratch_get(yl_ctx* ctx, size_t bytes, void** out, int slot) {
  if (bytes == 0) bytes = 256;
  if (bytes > ctx->scratch_bytes[slot]) {
    if (ctx->scratch[slot]) YL_CUDA(cudaFreeAsync(ctx->scratch[slot], ctx->stream));
    ctx->scratch[slot] = nullptr;
    ctx->scratch_bytes[slot] = 0;
    size_t want = bytes + bytes / 4;
    cudaError_t e = cudaMallocAsync(&ctx->scratch[slot], want, ctx->stream);
    if (e != cudaSuccess)
      return set_error(YL_ERR_OOM, "scratch allocation of %zu bytes failed: %s", want,
                       cudaGetErrorString(e));
    ctx->scratch_bytes[slot] = want;
  }
  *out = ctx->scratch[slot];
  return YL_OK;
}

}  // namespace yl

using namespace yl;

extern "C" {

const char* yl_last_error_message(void) { return t_last_error.c_str(); }

const char* yl_version(void) { return "yumelayers_b200 0.1 (sm_100a, tcgen05/TMA)"; }

unsigned long long yl_kernel_launch_count(void) { return g_launches.load(); }

yl_status yl_ctx_create(int device, yl_ctx** out) {
  YL_CHECK(out != nullptr, YL_ERR_INVALID, "yl_ctx_create: out is NULL");
  int count = 0;
  YL_CUDA(cudaGetDeviceCount(&count));
  YL_CHECK(device >= 0 && device < count, YL_ERR_INVALID, "yl_ctx_create: device %d of %d",
           device, count);
  YL_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  YL_CUDA(cudaGetDeviceProperties(&prop, device));
  YL_CHECK(prop.major == 10, YL_ERR_UNSUPPORTED,
           "yl_ctx_create: device %d is sm_%d%d; this build targets sm_100a (B200)", device,
           prop.major, prop.minor);
  yl_ctx* c = new yl_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  YL_CUDA(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking));
  c->stream = c->own_stream;
  YL_CUDA(cudaEventCreate(&c->ev_begin));
  YL_CUDA(cudaEventCreate(&c->ev_end));
  YL_CUDA(cudaMalloc(&c->dev_err, 16));
  YL_CUDA(cudaMemset(c->dev_err, 0, 16));
  YL_CUDA(cudaMalloc(&c->sched, sizeof(int) * 2 * kSchedSlots));
  YL_CUDA(cudaMemset(c->sched, 0, sizeof(int) * 2 * kSchedSlots));
  *out = c;
  return YL_OK;
}

yl_status yl_ctx_destroy(yl_ctx* ctx) {
  if (!ctx) return YL_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (int s = 0; s < 3; ++s)
    if (ctx->scratch[s]) cudaFreeAsync(ctx->scratch[s], ctx->stream);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->dev_err);
  cudaFree(ctx->sched);
  cudaEventDestroy(ctx->ev_begin);
  cudaEventDestroy(ctx->ev_end);
  cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return YL_OK;
}

yl_status yl_ctx_set_stream(yl_ctx* ctx, void* s) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_ctx_set_stream: ctx is NULL");
  ctx->stream = s ? (cudaStream_t)s : ctx->own_stream;
  return YL_OK;
}

void* yl_ctx_get_stream(yl_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

yl_status yl_session_begin(yl_ctx* ctx) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_session_begin: ctx is NULL");
  YL_CUDA(cudaEventRecord(ctx->ev_begin, ctx->stream));
  ctx->wall_begin = std::chrono::steady_clock::now();
  ctx->session_open = true;
  return YL_OK;
}

yl_status yl_session_commit(yl_ctx* ctx) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_session_commit: ctx is NULL");
  YL_CUDA(cudaEventRecord(ctx->ev_end, ctx->stream));
  return YL_OK;
}

// Polls the end event against a deadline (gpuWaitOutcome, GpuWaitPolicy.swift:54-61):
// done -> OK, deadline passed -> YL_ERR_TIMEOUT; never blocks without bound.
static yl_status wait_event(cudaEvent_t ev, double timeout_s) {
  auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return YL_OK;
    if (e != cudaErrorNotReady)
      return set_error(YL_ERR_CUDA, "session wait: %s", cudaGetErrorString(e));
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el >= timeout_s)
      return set_error(YL_ERR_TIMEOUT, "session wait exceeded %.1f s", timeout_s);
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

yl_status yl_session_end(yl_ctx* ctx, double timeout_s, double* gpu_ms) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_session_end: ctx is NULL");
  YL_CUDA(cudaEventRecord(ctx->ev_end, ctx->stream));
  if (timeout_s <= 0) timeout_s = 30.0;  // the reference's 30 s deadline (GpuTraining.swift:30)
  YL_TRY(wait_event(ctx->ev_end, timeout_s));
  double wall_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - ctx->wall_begin)
          .count();
  if (gpu_ms) {
    float ms = 0.f;
    double rep = 0.0;
    if (ctx->session_open && cudaEventElapsedTime(&ms, ctx->ev_begin, ctx->ev_end) == cudaSuccess)
      rep = ms;
    // boundedGpuMs (GpuWaitPolicy.swift:75-87): never report more than the wall time.
    if (wall_ms <= 0) *gpu_ms = rep > 0 ? rep : 0;
    else if (rep <= 0) *gpu_ms = wall_ms;
    else if (rep > wall_ms + 50.0) *gpu_ms = wall_ms;
    else *gpu_ms = rep;
  }
  ctx->session_open = false;
  return yl_ctx_check_device_errors(ctx);
}

yl_status yl_ctx_check_device_errors(yl_ctx* ctx) {
  YL_CHECK(ctx, YL_ERR_INVALID, "ctx is NULL");
  int h = 0;
  YL_CUDA(cudaMemcpyAsync(&h, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  if (h != 0) {
    YL_CUDA(cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), ctx->stream));
    YL_CUDA(cudaStreamSynchronize(ctx->stream));
    // a bounded device wait that gave up is the GPU-side hang guard's
    // timeout (the reference exits with 70 there, GpuTraining.swift:92-97)
    if (h == 1)
      return set_error(YL_ERR_TIMEOUT, "a kernel's bounded wait timed out (device error 1)");
    return set_error(YL_ERR_DEVICE_ASSERT, "a kernel reported device error %d (%s)", h,
                     "device-side check failed");
  }
  return YL_OK;
}

yl_status yl_ctx_set_wait_limit(yl_ctx* ctx, long long cycles) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_ctx_set_wait_limit: ctx is NULL");
  const long long v = cycles > 0 ? cycles : 0;
  YL_CUDA(cudaMemcpyAsync(reinterpret_cast<char*>(ctx->dev_err) + 8, &v, sizeof(v),
                          cudaMemcpyHostToDevice, ctx->stream));
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  return YL_OK;
}

const char* yl_ctx_last_kernel(yl_ctx* ctx, int which) {
  if (!ctx || which < 0 || which > 1) return "";
  return ctx->last_kernel[which];
}

// ------------------------------------------------------------------ tensors

struct yl_tensor {
  yl_ctx* ctx;
  int rows, cols;
  float* data;
};

yl_status yl_tensor_create(yl_ctx* ctx, int rows, int cols, const float* host, yl_tensor** out) {
  YL_CHECK(ctx && out, YL_ERR_INVALID, "yl_tensor_create: NULL argument");
  YL_CHECK(rows >= 0 && cols >= 0, YL_ERR_SHAPE, "yl_tensor_create: %d x %d", rows, cols);
  size_t n = (size_t)rows * cols;
  float* p = nullptr;
  cudaError_t e = cudaMallocAsync((void**)&p, n ? n * sizeof(float) : 256, ctx->stream);
  if (e != cudaSuccess)
    return set_error(YL_ERR_OOM, "yl_tensor_create %d x %d: %s", rows, cols,
                     cudaGetErrorString(e));
  if (host && n) {
    YL_CUDA(cudaMemcpyAsync(p, host, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    YL_CUDA(cudaStreamSynchronize(ctx->stream));
  }
  *out = new yl_tensor{ctx, rows, cols, p};
  return YL_OK;
}

yl_status yl_tensor_release(yl_tensor* t) {
  if (!t) return YL_OK;
  YL_CUDA(cudaFreeAsync(t->data, t->ctx->stream));
  delete t;
  return YL_OK;
}

float* yl_tensor_data(yl_tensor* t) { return t ? t->data : nullptr; }
int yl_tensor_rows(const yl_tensor* t) { return t ? t->rows : 0; }
int yl_tensor_cols(const yl_tensor* t) { return t ? t->cols : 0; }

yl_status yl_tensor_upload(yl_tensor* t, const float* host, size_t n) {
  YL_CHECK(t && host, YL_ERR_INVALID, "yl_tensor_upload: NULL argument");
  YL_CHECK(n == (size_t)t->rows * t->cols, YL_ERR_SHAPE, "yl_tensor_upload: %zu != %d x %d", n,
           t->rows, t->cols);
  YL_CUDA(cudaMemcpyAsync(t->data, host, n * sizeof(float), cudaMemcpyHostToDevice,
                          t->ctx->stream));
  YL_CUDA(cudaStreamSynchronize(t->ctx->stream));
  return YL_OK;
}

yl_status yl_tensor_download(yl_tensor* t, float* host, size_t n) {
  YL_CHECK(t && host, YL_ERR_INVALID, "yl_tensor_download: NULL argument");
  YL_CHECK(n == (size_t)t->rows * t->cols, YL_ERR_SHAPE, "yl_tensor_download: %zu != %d x %d",
           n, t->rows, t->cols);
  YL_CUDA(cudaMemcpyAsync(host, t->data, n * sizeof(float), cudaMemcpyDeviceToHost,
                          t->ctx->stream));
  YL_CUDA(cudaStreamSynchronize(t->ctx->stream));
  return YL_OK;
}

yl_status yl_tensor_get_value(yl_tensor* t, size_t i, float* v) {
  YL_CHECK(t && v, YL_ERR_INVALID, "yl_tensor_get_value: NULL argument");
  YL_CHECK(i < (size_t)t->rows * t->cols, YL_ERR_SHAPE, "yl_tensor_get_value: index %zu", i);
  YL_CUDA(cudaMemcpyAsync(v, t->data + i, sizeof(float), cudaMemcpyDeviceToHost, t->ctx->stream));
  YL_CUDA(cudaStreamSynchronize(t->ctx->stream));
  return YL_OK;
}

yl_status yl_tensor_set_value(yl_tensor* t, size_t i, float v) {
  YL_CHECK(t, YL_ERR_INVALID, "yl_tensor_set_value: NULL argument");
  YL_CHECK(i < (size_t)t->rows * t->cols, YL_ERR_SHAPE, "yl_tensor_set_value: index %zu", i);
  YL_CUDA(cudaMemcpyAsync(t->data + i, &v, sizeof(float), cudaMemcpyHostToDevice, t->ctx->stream));
  YL_CUDA(cudaStreamSynchronize(t->ctx->stream));
  return YL_OK;
}

yl_status yl_copy(yl_ctx* ctx, float* dst, const float* src, size_t n) {
  YL_CHECK(ctx && dst && src, YL_ERR_INVALID, "yl_copy: NULL argument");
  YL_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
  return YL_OK;
}

yl_status yl_memcpy_htod(yl_ctx* ctx, void* dst, const void* src, size_t bytes) {
  YL_CHECK(ctx && dst && src, YL_ERR_INVALID, "yl_memcpy_htod: NULL argument");
  YL_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  return YL_OK;
}

yl_status yl_memcpy_dtoh(yl_ctx* ctx, void* dst, const void* src, size_t bytes) {
  YL_CHECK(ctx && dst && src, YL_ERR_INVALID, "yl_memcpy_dtoh: NULL argument");
  YL_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  return YL_OK;
}

yl_status yl_zero_fill(yl_ctx* ctx, float* dst, size_t n) {
  YL_CHECK(ctx && dst, YL_ERR_INVALID, "yl_zero_fill: NULL argument");
  YL_CUDA(cudaMemsetAsync(dst, 0, n * sizeof(float), ctx->stream));
  return YL_OK;
}

}  // extern "C"
