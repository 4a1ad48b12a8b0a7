// yl_diag.cu -- kernel-level diagnostics: the B200 counterpart of the
// reference's profileConv / runGpuBench (Diagnostics.swift:83-201), timing
// one conv shape's forward, dX and dW kernels (and GroupNorm+SiLU) with CUDA
// events on NHWC buffers the call allocates itself.
#include <algorithm>
#include <vector>

#include "yl_kernels.h"
#include "yl_ptx.cuh"
#include "yl_norm.h"
#include "yume_c.h"

using namespace yl;

namespace {

__global__ void fill_kernel(float* p, long long n, uint32_t seed, float scale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    uint32_t x = (uint32_t)i * 2654435761u ^ seed;
    x ^= x >> 15;
    x *= 2246822519u;
    x ^= x >> 13;
    p[i] = scale * ((float)(x & 0xFFFFFF) / 8388608.0f - 1.0f);
  }
}

struct DevBufs {
  std::vector<void*> ptrs;
  ~DevBufs() {
    for (void* p : ptrs) cudaFree(p);
  }
  yl_status get(size_t floats, float** out) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, floats * sizeof(float));
    if (e != cudaSuccess)
      return set_error(YL_ERR_OOM, "profile buffer of %zu floats: %s", floats,
                       cudaGetErrorString(e));
    ptrs.push_back(p);
    *out = (float*)p;
    return YL_OK;
  }
};

// One thread waits on an mbarrier initialised for one arrival that nothing
// ever makes: the wait runs out after the context's wait limit and records
// YL_DEVERR_TIMEOUT, exactly as a conv kernel's pipeline wait would.
__global__ void wait_probe_kernel(int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  if (!mbar_wait(&bar, 0, wait_limit(err))) report_error(err, YL_DEVERR_TIMEOUT);
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Busy for `ns` nanoseconds of the global timer; also bounded by `max_cycles`
// SM clock cycles so it ends even if the timer were to stall.
__global__ void spin_kernel(unsigned long long ns, long long max_cycles) {
  const unsigned long long t0 = global_ns();
  const long long c0 = clock64();
  while (global_ns() - t0 < ns && clock64() - c0 < max_cycles) {
  }
}

}  // namespace

extern "C" {

yl_status yl_debug_wait_probe(yl_ctx* ctx) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_debug_wait_probe: ctx is NULL");
  wait_probe_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_err);
  return check_launch("wait_probe_kernel");
}

yl_status yl_debug_spin(yl_ctx* ctx, double seconds) {
  YL_CHECK(ctx && seconds >= 0.0 && seconds <= 10.0, YL_ERR_INVALID,
           "yl_debug_spin: seconds must be in [0, 10]");
  const unsigned long long ns = (unsigned long long)(seconds * 1e9);
  // 3 GHz is above any SM clock of this part: the cycle bound only backs up
  // the timer and never cuts a healthy spin short
  spin_kernel<<<1, 32, 0, ctx->stream>>>(ns, (long long)(seconds * 3e9) + 1000000LL);
  return check_launch("spin_kernel");
}

yl_status yl_profile_conv(yl_ctx* ctx, int n, int c, int h, int w, int oc, int k, int stride,
                          int up, int reps, yl_conv_profile* out) {
  YL_CHECK(ctx && out && reps >= 1, YL_ERR_INVALID, "yl_profile_conv: bad argument");
  YL_CHECK(c % 4 == 0 && oc % 4 == 0, YL_ERR_SHAPE, "yl_profile_conv: channels multiple of 4");
  const int pad = k / 2;
  const int ih = up ? 2 * h : h, iw = up ? 2 * w : w;
  const int oh = (ih + 2 * pad - k) / stride + 1, ow = (iw + 2 * pad - k) / stride + 1;
  DevBufs b;
  float *x = nullptr, *wt = nullptr, *wd = nullptr, *y = nullptr, *dy = nullptr, *dx = nullptr,
        *dw = nullptr;
  YL_TRY(b.get((size_t)n * h * w * c, &x));
  YL_TRY(b.get((size_t)oc * k * k * c, &wt));
  YL_TRY(b.get((size_t)oc * k * k * c, &wd));
  YL_TRY(b.get((size_t)n * oh * ow * oc, &y));
  YL_TRY(b.get((size_t)n * oh * ow * oc, &dy));
  YL_TRY(b.get((size_t)n * ih * iw * c, &dx));
  YL_TRY(b.get((size_t)oc * k * k * c, &dw));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(x, (long long)n * h * w * c, 1, 1.f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(wt, (long long)oc * k * k * c, 2, 0.05f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(wd, (long long)oc * k * k * c, 3, 0.05f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(dy, (long long)n * oh * ow * oc, 4, 1.f);
  YL_TRY(check_launch("fill_kernel"));
  ConvGather g;
  g.src = x;
  g.img_stride = (long long)h * w * c;
  g.row_stride = w * c;
  g.ps = c;
  g.cin = c;
  g.hv = ih;
  g.wv = iw;
  g.up = up;
  g.mode = MODE_FPROP;
  g.ksize = k;
  g.stride = stride;
  g.pad = pad;
  g.oh = oh;
  g.ow = ow;
  g.m_total = n * oh * ow;
  g.k_total = k * k * c;
  ConvEpilogue e;
  e.out = y;
  e.ldo = oc;
  e.n_total = oc;
  ConvGather gd;
  gd.src = dy;
  gd.img_stride = (long long)oh * ow * oc;
  gd.row_stride = ow * oc;
  gd.ps = oc;
  gd.cin = oc;
  gd.hv = oh;
  gd.wv = ow;
  gd.mode = MODE_DGRAD;
  gd.ksize = k;
  gd.stride = stride;
  gd.pad = pad;
  gd.oh = ih;
  gd.ow = iw;
  gd.m_total = n * ih * iw;
  gd.k_total = k * k * oc;
  ConvEpilogue ed;
  ed.out = dx;
  ed.ldo = c;
  ed.n_total = c;
  const int splits = conv_wgrad_pick_splits(ctx, oc, g, dy, oc);
  float* ws;
  YL_TRY(b.get(conv_wgrad_ws_floats(g, oc, dy, oc, splits), &ws));
  cudaEvent_t e0, e1;
  YL_CUDA(cudaEventCreate(&e0));
  YL_CUDA(cudaEventCreate(&e1));
  double ms[3] = {0, 0, 0};
  for (int mode = 0; mode < 3; ++mode) {
    for (int r = -1; r < reps; ++r) {  // r = -1 is an untimed warm-up
      if (r == 0) YL_CUDA(cudaEventRecord(e0, ctx->stream));
      if (mode == 0) YL_TRY(conv_fprop(ctx, g, wt, oc, e));
      if (mode == 1) {
        // an upsample conv's dX at the source resolution, as the executor runs it
        yl_status st = up ? conv_dgrad_upsampled(ctx, dy, oc, oc, n, h, w, 2 * h, 2 * w, wd, c, ed)
                          : YL_ERR_UNSUPPORTED;
        if (st == YL_ERR_UNSUPPORTED) st = conv_fprop(ctx, gd, wd, c, ed);
        YL_TRY(st);
      }
      if (mode == 2) YL_TRY(conv_wgrad_ws(ctx, dy, oc, oc, g, dw, 0, ws, splits));
    }
    YL_CUDA(cudaEventRecord(e1, ctx->stream));
    YL_CUDA(cudaEventSynchronize(e1));
    float t = 0.f;
    YL_CUDA(cudaEventElapsedTime(&t, e0, e1));
    ms[mode] = t / reps;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  out->fprop_ms = ms[0];
  out->dgrad_ms = ms[1];
  out->wgrad_ms = ms[2];
  out->flops = 2.0 * n * oh * ow * (double)oc * c * k * k;
  out->wgrad_splits = splits;
  return yl_ctx_check_device_errors(ctx);
}

yl_status yl_profile_adam(yl_ctx* ctx, long long n, int tensors, int reps, double* ms_out) {
  YL_CHECK(ctx && ms_out && reps >= 1 && n > 0 && tensors >= 1 && tensors <= 48, YL_ERR_INVALID,
           "yl_profile_adam: bad argument");
  DevBufs b;
  float *p = nullptr, *g = nullptr, *m = nullptr, *v = nullptr;
  YL_TRY(b.get((size_t)n, &p));
  YL_TRY(b.get((size_t)n, &g));
  YL_TRY(b.get((size_t)n, &m));
  YL_TRY(b.get((size_t)n, &v));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(p, n, 9, 1.f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(g, n, 10, 0.1f);
  YL_CUDA(cudaMemsetAsync(m, 0, (size_t)n * sizeof(float), ctx->stream));
  YL_CUDA(cudaMemsetAsync(v, 0, (size_t)n * sizeof(float), ctx->stream));
  YL_TRY(check_launch("fill_kernel"));
  // the flat buffer split into `tensors` consecutive tensors, like a model's table
  AdamTensor table[48];
  // tensor sizes rounded up to 4 floats, as every tensor of the models is
  const long long per = ((n + tensors - 1) / tensors + 3) & ~3LL;
  int count = 0;
  for (long long o = 0; o < n; o += per, ++count)
    table[count] = AdamTensor{p + o, g + o, m + o, v + o, std::min(per, n - o)};
  cudaEvent_t e0, e1;
  YL_CUDA(cudaEventCreate(&e0));
  YL_CUDA(cudaEventCreate(&e1));
  for (int rr = -1; rr < reps; ++rr) {
    if (rr == 0) YL_CUDA(cudaEventRecord(e0, ctx->stream));
    YL_TRY(adam_multi(ctx, table, count, 2e-4f, 0.9f, 0.999f, 1e-8f, rr + 2, 1.f, 0.f, 0, nullptr));
  }
  YL_CUDA(cudaEventRecord(e1, ctx->stream));
  YL_CUDA(cudaEventSynchronize(e1));
  float t = 0.f;
  YL_CUDA(cudaEventElapsedTime(&t, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms_out = t / reps;
  return yl_ctx_check_device_errors(ctx);
}

yl_status yl_profile_groupnorm(yl_ctx* ctx, int n, int c, int h, int w, int reps, double* fwd_ms,
                               double* bwd_ms, double* apply_ms) {
  YL_CHECK(ctx && fwd_ms && bwd_ms && reps >= 1, YL_ERR_INVALID, "yl_profile_groupnorm");
  const long long e = (long long)n * h * w * c;
  DevBufs b;
  float *x = nullptr, *y = nullptr, *dy = nullptr, *dx = nullptr, *g = nullptr, *bt = nullptr,
        *dg = nullptr, *db = nullptr, *m = nullptr, *r = nullptr;
  YL_TRY(b.get(e, &x));
  YL_TRY(b.get(e, &y));
  YL_TRY(b.get(e, &dy));
  YL_TRY(b.get(e, &dx));
  YL_TRY(b.get(c, &g));
  YL_TRY(b.get(c, &bt));
  YL_TRY(b.get(c, &dg));
  YL_TRY(b.get(c, &db));
  YL_TRY(b.get((size_t)n * 32, &m));
  YL_TRY(b.get((size_t)n * 32, &r));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(x, e, 5, 1.f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(dy, e, 6, 1.f);
  fill_kernel<<<4, 256, 0, ctx->stream>>>(g, c, 7, 1.f);
  fill_kernel<<<4, 256, 0, ctx->stream>>>(bt, c, 8, 0.1f);
  YL_TRY(check_launch("fill_kernel"));
  cudaEvent_t e0, e1;
  YL_CUDA(cudaEventCreate(&e0));
  YL_CUDA(cudaEventCreate(&e1));
  double ms[3];
  for (int mode = 0; mode < 3; ++mode) {
    for (int rr = -1; rr < reps; ++rr) {
      if (rr == 0) YL_CUDA(cudaEventRecord(e0, ctx->stream));
      if (mode == 0)
        YL_TRY(gn_silu_forward(ctx, x, n, c, 32, (long long)h * w, c, 1e-6f, 0, g, bt, 1, y, c, 1,
                               m, r));
      else if (mode == 2)  // the apply pass alone, statistics from mode 0
        YL_TRY(gn_silu_apply(ctx, x, n, c, 32, (long long)h * w, c, m, r, g, bt, 1, y, c, 1));
      else
        YL_TRY(gn_silu_backward(ctx, x, dy, c, n, c, 32, (long long)h * w, c, m, r, g, bt, 1, y, c,
                                dx, c, 1, dg, db, 0));
    }
    YL_CUDA(cudaEventRecord(e1, ctx->stream));
    YL_CUDA(cudaEventSynchronize(e1));
    float t = 0.f;
    YL_CUDA(cudaEventElapsedTime(&t, e0, e1));
    ms[mode] = t / reps;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *fwd_ms = ms[0];
  *bwd_ms = ms[1];
  if (apply_ms) *apply_ms = ms[2];
  return yl_ctx_check_device_errors(ctx);
}

yl_status yl_profile_layered(yl_ctx* ctx, int n, long long plane, int reps, double* ms_out) {
  YL_CHECK(ctx && ms_out && reps >= 1 && n >= 1 && plane >= 1, YL_ERR_INVALID,
           "yl_profile_layered: bad argument");
  DevBufs b;
  float *r = nullptr, *t = nullptr, *c = nullptr, *g = nullptr, *l = nullptr;
  const long long e8 = (long long)n * 8 * plane, e3 = (long long)n * 3 * plane;
  YL_TRY(b.get((size_t)e8, &r));
  YL_TRY(b.get((size_t)e8, &t));
  YL_TRY(b.get((size_t)e3, &c));
  YL_TRY(b.get((size_t)e8, &g));
  YL_TRY(b.get((size_t)n, &l));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(r, e8, 11, 1.f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(t, e8, 12, 1.f);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(c, e3, 13, 1.f);
  YL_TRY(check_launch("fill_kernel"));
  cudaEvent_t e0, e1;
  YL_CUDA(cudaEventCreate(&e0));
  YL_CUDA(cudaEventCreate(&e1));
  for (int rr = -1; rr < reps; ++rr) {
    if (rr == 0) YL_CUDA(cudaEventRecord(e0, ctx->stream));
    YL_TRY(yl_layered_loss(ctx, r, t, c, n, plane, 1.f, 1.f, g, l));
  }
  YL_CUDA(cudaEventRecord(e1, ctx->stream));
  YL_CUDA(cudaEventSynchronize(e1));
  float tm = 0.f;
  YL_CUDA(cudaEventElapsedTime(&tm, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms_out = tm / reps;
  return yl_ctx_check_device_errors(ctx);
}

}  // extern "C"
