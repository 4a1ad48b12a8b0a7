// yl_norm.cu -- fused GroupNorm(+affine) + SiLU, forward and backward, on
// NHWC activations.
//
// Replaces groupNorm / encodeGroupNormGrad (GpuSessionOps.swift:121-131,
// GpuSessionNormGrad.swift:10-24; kernels MetalKernelSourcesC.swift:10-101,
// one thread per group with serial loops) plus the separate activation and
// activation-gradient passes (relu/sigmoid kernels B:191-224).  The target
// op is torch.nn.GroupNorm (affine, eps) followed by SiLU; `mode` 1 selects
// the reference's own variance rule (var = max(E[x^2]-E[x]^2, 1e-5), no eps).
//
// Forward:  (1) statistics: many CTAs per image, each thread owns one
//               channel quad and streams pixels with 16-byte loads,
//               accumulating in double; per-(image, chunk) partials are
//               merged in a fixed order -> mean, rstd per (image, group).
//           (2) apply: y = silu((x - mean) * rstd * gamma + beta), rounded to
//               tf32 because the next consumer is a convolution.
// Backward: (1) per-(image, chunk) partials of sum(dxh), sum(dxh*xh) per
//               group and of dgamma/dbeta per channel, dxh = dy*silu'(a)*gamma;
//           (2) dx = rstd*(dxh - mean(dxh) - xh*mean(dxh*xh)) (+ addend).
// Memory traffic per element: forward 2 reads + 1 write, backward 4 reads +
// 1 write (+1 read for the addend).
#include <mutex>

#include "yl_kernels.h"
#include "yl_norm.h"
#include "yl_ptx.cuh"

namespace yl {

__device__ __forceinline__ float silu_f(float a) { return a / (1.f + __expf(-a)); }

struct GnGeom {
  int n, c, g, ps;
  long long hw;
  int chunks;
  int quads, rows;  // block = quads * rows threads
};

static GnGeom gn_geom(int n, int c, int g, long long hw, int ps) {
  GnGeom q;
  q.n = n;
  q.c = c;
  q.g = g;
  q.ps = ps;
  q.hw = hw;
  q.quads = c / 4;
  q.rows = q.quads >= 256 ? 1 : 256 / q.quads;
  long long per_img_threads = (long long)q.rows;
  long long chunks = (hw + 4 * per_img_threads - 1) / (4 * per_img_threads);  // >= 4 px per thread
  if (chunks > 148 * 4 / (n > 0 ? n : 1) + 1) chunks = 148 * 4 / (n > 0 ? n : 1) + 1;
  if (chunks < 1) chunks = 1;
  q.chunks = (int)chunks;
  return q;
}

// partial[img][chunk][g] = (sum, sumsq)
__global__ void gn_stats_partial_kernel(const float* __restrict__ x, GnGeom q,
                                        double* __restrict__ part) {
  extern __shared__ double sh[];  // [g][2]
  const int img = blockIdx.y, chunk = blockIdx.x;
  const int t = threadIdx.x;
  for (int i = t; i < 2 * q.g; i += blockDim.x) sh[i] = 0.0;
  __syncthreads();
  const int quad = t % q.quads, row = t / q.quads;
  const int cg = q.c / q.g;
  const int grp = (quad * 4) / cg;
  const long long per = (q.hw + q.chunks - 1) / q.chunks;
  const long long p0 = chunk * per, p1 = min(q.hw, p0 + per);
  const float* base = x + (long long)img * q.hw * q.ps + quad * 4;
  double s = 0.0, ss = 0.0;
  for (long long p = p0 + row; p < p1; p += q.rows) {
    const float4 v = *reinterpret_cast<const float4*>(base + p * q.ps);
    s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  atomicAdd(&sh[2 * grp], s);
  atomicAdd(&sh[2 * grp + 1], ss);
  __syncthreads();
  double* out = part + ((long long)img * q.chunks + chunk) * 2 * q.g;
  for (int i = t; i < 2 * q.g; i += blockDim.x) out[i] = sh[i];
}

__global__ void gn_stats_final_kernel(const double* __restrict__ part, GnGeom q, float eps,
                                      int mode, float* __restrict__ mean,
                                      float* __restrict__ rstd) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // img * g + grp
  if (idx >= q.n * q.g) return;
  const int img = idx / q.g, grp = idx % q.g;
  double s = 0.0, ss = 0.0;
  for (int k = 0; k < q.chunks; ++k) {
    const double* pp = part + ((long long)img * q.chunks + k) * 2 * q.g;
    s += pp[2 * grp];
    ss += pp[2 * grp + 1];
  }
  const double cnt = (double)q.hw * (q.c / q.g);
  const double m = s / cnt;
  double var = ss / cnt - m * m;
  double r;
  if (mode == 1) {
    if (var < 1e-5) var = 1e-5;  // groupnorm_kernel's clamp (MetalKernelSourcesC.swift:36-38)
    r = 1.0 / sqrt(var);
  } else {
    if (var < 0) var = 0;
    r = 1.0 / sqrt(var + (double)eps);
  }
  mean[idx] = (float)m;
  rstd[idx] = (float)r;
}

__global__ void gn_apply_kernel(const float* __restrict__ x, GnGeom q,
                                const float* __restrict__ mean, const float* __restrict__ rstd,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                int silu, int round, float* __restrict__ y, int ldy) {
  const long long total = (long long)q.n * q.hw * q.quads;
  const int cg = q.c / q.g;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int quad = (int)(i % q.quads);
    const long long pix = i / q.quads;  // img * hw + p
    const int img = (int)(pix / q.hw);
    const int c = quad * 4;
    const int grp = c / cg;
    const float m = mean[img * q.g + grp], r = rstd[img * q.g + grp];
    const float4 v = *reinterpret_cast<const float4*>(x + pix * q.ps + c);
    float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float a = (o[k] - m) * r;
      if (gamma) a = a * __ldg(gamma + c + k);
      if (beta) a = a + __ldg(beta + c + k);
      if (silu) a = silu_f(a);
      o[k] = round ? round_tf32(a) : a;
    }
    *reinterpret_cast<float4*>(y + pix * ldy + c) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// Backward partials: per (img, chunk): group sums [g][2] then channel sums [c][2].
__global__ void gn_bwd_partial_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                      int lddy, GnGeom q, const float* __restrict__ mean,
                                      const float* __restrict__ rstd,
                                      const float* __restrict__ gamma,
                                      const float* __restrict__ beta, int silu,
                                      double* __restrict__ part) {
  extern __shared__ double sh[];  // [g][2] + [c][2]
  const int img = blockIdx.y, chunk = blockIdx.x;
  const int t = threadIdx.x;
  const int nsh = 2 * q.g + 2 * q.c;
  for (int i = t; i < nsh; i += blockDim.x) sh[i] = 0.0;
  __syncthreads();
  const int quad = t % q.quads, row = t / q.quads;
  const int cg = q.c / q.g;
  const int c = quad * 4;
  const int grp = c / cg;
  const float m = mean[img * q.g + grp], r = rstd[img * q.g + grp];
  float ga[4], be[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    ga[k] = gamma ? gamma[c + k] : 1.f;
    be[k] = beta ? beta[c + k] : 0.f;
  }
  const long long per = (q.hw + q.chunks - 1) / q.chunks;
  const long long p0 = chunk * per, p1 = min(q.hw, p0 + per);
  const float* xb = x + (long long)img * q.hw * q.ps + c;
  const float* db = dy + (long long)img * q.hw * lddy + c;
  double sd = 0, sdx = 0, dg[4] = {0, 0, 0, 0}, dbt[4] = {0, 0, 0, 0};
  for (long long p = p0 + row; p < p1; p += q.rows) {
    const float4 xv = *reinterpret_cast<const float4*>(xb + p * q.ps);
    const float4 dv = *reinterpret_cast<const float4*>(db + p * lddy);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const float ds[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float xh = (xs[k] - m) * r;
      float da = ds[k];
      if (silu) {
        const float a = xh * ga[k] + be[k];
        const float sg = 1.f / (1.f + __expf(-a));
        da *= sg * (1.f + a * (1.f - sg));
      }
      dg[k] += (double)da * xh;
      dbt[k] += da;
      const float dxh = da * ga[k];
      sd += dxh;
      sdx += (double)dxh * xh;
    }
  }
  atomicAdd(&sh[2 * grp], sd);
  atomicAdd(&sh[2 * grp + 1], sdx);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    atomicAdd(&sh[2 * q.g + 2 * (c + k)], dg[k]);
    atomicAdd(&sh[2 * q.g + 2 * (c + k) + 1], dbt[k]);
  }
  __syncthreads();
  double* out = part + ((long long)img * q.chunks + chunk) * nsh;
  for (int i = t; i < nsh; i += blockDim.x) out[i] = sh[i];
}

// Reduces the partials: per (img, grp) -> coef[img][grp][2] = (mean(dxh), mean(dxh*xh));
// per channel -> dgamma, dbeta (fixed order over images and chunks).
__global__ void gn_bwd_final_kernel(const double* __restrict__ part, GnGeom q,
                                    float* __restrict__ coef, float* dgamma, float* dbeta,
                                    int accumulate) {
  const int nsh = 2 * q.g + 2 * q.c;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const double cnt = (double)q.hw * (q.c / q.g);
  if (idx < q.n * q.g) {
    const int img = idx / q.g, grp = idx % q.g;
    double a = 0, b = 0;
    for (int k = 0; k < q.chunks; ++k) {
      const double* pp = part + ((long long)img * q.chunks + k) * nsh;
      a += pp[2 * grp];
      b += pp[2 * grp + 1];
    }
    coef[2 * idx] = (float)(a / cnt);
    coef[2 * idx + 1] = (float)(b / cnt);
  }
  if (idx < q.c) {
    double a = 0, b = 0;
    for (int img = 0; img < q.n; ++img)
      for (int k = 0; k < q.chunks; ++k) {
        const double* pp = part + ((long long)img * q.chunks + k) * nsh + 2 * q.g;
        a += pp[2 * idx];
        b += pp[2 * idx + 1];
      }
    if (dgamma) dgamma[idx] = accumulate ? dgamma[idx] + (float)a : (float)a;
    if (dbeta) dbeta[idx] = accumulate ? dbeta[idx] + (float)b : (float)b;
  }
}

__global__ void gn_bwd_apply_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                    int lddy, GnGeom q, const float* __restrict__ mean,
                                    const float* __restrict__ rstd,
                                    const float* __restrict__ gamma,
                                    const float* __restrict__ beta, int silu,
                                    const float* __restrict__ coef,
                                    const float* __restrict__ addend, int ldadd,
                                    float* __restrict__ dx, int lddx, int round) {
  const long long total = (long long)q.n * q.hw * q.quads;
  const int cg = q.c / q.g;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int quad = (int)(i % q.quads);
    const long long pix = i / q.quads;
    const int img = (int)(pix / q.hw);
    const int c = quad * 4;
    const int gi = img * q.g + c / cg;
    const float m = mean[gi], r = rstd[gi];
    const float md = coef[2 * gi], mdx = coef[2 * gi + 1];
    const float4 xv = *reinterpret_cast<const float4*>(x + pix * q.ps + c);
    const float4 dv = *reinterpret_cast<const float4*>(dy + pix * lddy + c);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const float ds[4] = {dv.x, dv.y, dv.z, dv.w};
    float4 av = make_float4(0.f, 0.f, 0.f, 0.f);
    if (addend) av = *reinterpret_cast<const float4*>(addend + pix * ldadd + c);
    const float adds[4] = {av.x, av.y, av.z, av.w};
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float ga = gamma ? __ldg(gamma + c + k) : 1.f;
      const float xh = (xs[k] - m) * r;
      float da = ds[k];
      if (silu) {
        const float a = xh * ga + (beta ? __ldg(beta + c + k) : 0.f);
        const float sg = 1.f / (1.f + __expf(-a));
        da *= sg * (1.f + a * (1.f - sg));
      }
      const float v = r * (da * ga - md - xh * mdx) + adds[k];
      o[k] = round ? round_tf32(v) : v;
    }
    *reinterpret_cast<float4*>(dx + pix * lddx + c) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

static yl_status gn_check(int n, int c, int g, long long hw, int ps) {
  YL_CHECK(n > 0 && hw > 0 && g > 0 && c % g == 0, YL_ERR_SHAPE,
           "groupnorm: channels %d not divisible by groups %d", c, g);
  YL_CHECK(c % 4 == 0 && (c / g) % 4 == 0 && ps % 4 == 0 && ps >= c, YL_ERR_SHAPE,
           "groupnorm: channels per group (%d) and pixel stride (%d) must be multiples of 4",
           c / g, ps);
  YL_CHECK(c / 4 <= 1024, YL_ERR_SHAPE, "groupnorm: at most 4096 channels");
  return YL_OK;
}

yl_status gn_stats(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                   float eps, int mode, float* mean, float* rstd) {
  YL_TRY(gn_check(n, c, g, hw, ps));
  GnGeom q = gn_geom(n, c, g, hw, ps);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)n * q.chunks * 2 * g * sizeof(double), &ws));
  dim3 grid(q.chunks, n);
  gn_stats_partial_kernel<<<grid, q.quads * q.rows, 2 * g * sizeof(double), ctx->stream>>>(
      x, q, (double*)ws);
  YL_TRY(check_launch("gn_stats_partial_kernel"));
  gn_stats_final_kernel<<<(n * g + 127) / 128, 128, 0, ctx->stream>>>((double*)ws, q, eps, mode,
                                                                     mean, rstd);
  return check_launch("gn_stats_final_kernel");
}

yl_status gn_silu_forward(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                          float eps, int mode, const float* gamma, const float* beta, int silu,
                          float* y, int ldy, int round, float* mean, float* rstd) {
  YL_TRY(gn_stats(ctx, x, n, c, g, hw, ps, eps, mode, mean, rstd));
  GnGeom q = gn_geom(n, c, g, hw, ps);
  long long total = (long long)n * hw * q.quads;
  gn_apply_kernel<<<grid_1d(total, 256, ctx->num_sms * 16), 256, 0, ctx->stream>>>(
      x, q, mean, rstd, gamma, beta, silu, round, y, ldy);
  return check_launch("gn_apply_kernel");
}

yl_status gn_silu_backward(yl_ctx* ctx, const float* x, const float* dy, int lddy, int n, int c,
                           int g, long long hw, int ps, const float* mean, const float* rstd,
                           const float* gamma, const float* beta, int silu, const float* addend,
                           int ldadd, float* dx, int lddx, int round, float* dgamma, float* dbeta,
                           int accumulate_params) {
  YL_TRY(gn_check(n, c, g, hw, ps));
  YL_CHECK(lddy % 4 == 0 && lddx % 4 == 0 && (!addend || ldadd % 4 == 0), YL_ERR_SHAPE,
           "groupnorm backward: strides must be multiples of 4");
  GnGeom q = gn_geom(n, c, g, hw, ps);
  const int nsh = 2 * g + 2 * c;
  size_t part_bytes = (size_t)n * q.chunks * nsh * sizeof(double);
  size_t coef_off = (part_bytes + 255) & ~size_t(255);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, coef_off + (size_t)n * g * 2 * sizeof(float), &ws));
  double* part = (double*)ws;
  float* coef = (float*)((char*)ws + coef_off);
  dim3 grid(q.chunks, n);
  gn_bwd_partial_kernel<<<grid, q.quads * q.rows, nsh * sizeof(double), ctx->stream>>>(
      x, dy, lddy, q, mean, rstd, gamma, beta, silu, part);
  YL_TRY(check_launch("gn_bwd_partial_kernel"));
  int m = n * g > c ? n * g : c;
  gn_bwd_final_kernel<<<(m + 127) / 128, 128, 0, ctx->stream>>>(part, q, coef, dgamma, dbeta,
                                                               accumulate_params);
  YL_TRY(check_launch("gn_bwd_final_kernel"));
  long long total = (long long)n * hw * q.quads;
  gn_bwd_apply_kernel<<<grid_1d(total, 256, ctx->num_sms * 16), 256, 0, ctx->stream>>>(
      x, dy, lddy, q, mean, rstd, gamma, beta, silu, coef, addend, ldadd, dx, lddx, round);
  return check_launch("gn_bwd_apply_kernel");
}

// ---------------------------------------------------------------------------
// GroupNorm(+affine)+SiLU forward that allocates no device memory.
//
// yl_groupnorm_silu_fwd takes its per-(image, chunk, group) statistics
// partials from the context's stream-ordered scratch, which grows with
// cudaMallocAsync whenever a call needs more than it holds.  Some callers may
// not allocate inside the call: a host that fixes the process's device
// footprint at start-up (its pool or allocator refuses later growth), or code
// that must not add allocation nodes or synchronisation to the work it is
// recording.  This variant keeps the partials in a fixed array compiled into
// the library instead.
//
// Limits and rules:
//  * the partials need n * chunks * 2 * groups doubles, chunks being the
//    pixel split of gn_geom (at most 592 / n + 1); calls that need more than
//    kGnNoAllocDoubles (131072 doubles = 1 MiB) are rejected with
//    YL_ERR_SHAPE before anything is launched;
//  * NHWC layout only, channels and channels per group multiples of 4, and
//    the caller provides mean_out / rstd_out (no other temporaries exist);
//  * the first call on each device looks the array up with
//    cudaGetSymbolAddress (which may load the library's device code), so make
//    one call on every device before recording the calls into a graph;
//  * nothing has to start at zero: each call overwrites every partial it
//    reads;
//  * one array per device: calls that overlap on the same device (two
//    streams, two threads, two contexts) race on it.  Serialise them.
constexpr size_t kGnNoAllocDoubles = 131072;
static __device__ __align__(256) double g_gn_noalloc_partials[kGnNoAllocDoubles];

namespace {
constexpr int kMaxNoAllocDevices = 64;
std::mutex g_noalloc_mu;
double* g_noalloc_ptr[kMaxNoAllocDevices] = {};
}  // namespace

static yl_status gn_noalloc_scratch(int device, double** out) {
  YL_CHECK(device >= 0 && device < kMaxNoAllocDevices, YL_ERR_INVALID,
           "no-alloc groupnorm: device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    int cur = -1;
    YL_CUDA(cudaGetDevice(&cur));
    YL_CHECK(cur == device, YL_ERR_INVALID,
             "no-alloc groupnorm: the context's device %d must be current (current is %d)",
             device, cur);
    void* p = nullptr;
    YL_CUDA(cudaGetSymbolAddress(&p, g_gn_noalloc_partials));
    g_noalloc_ptr[device] = static_cast<double*>(p);
  }
  *out = g_noalloc_ptr[device];
  return YL_OK;
}

}  // namespace yl

extern "C" yl_status yl_groupnorm_silu_fwd_noalloc(yl_ctx* ctx, const float* x, int n, int c,
                                                   int h, int w, int groups, float eps, int mode,
                                                   const float* gamma, const float* beta,
                                                   int apply_silu, float* y, float* mean_out,
                                                   float* rstd_out) {
  using namespace yl;
  YL_CHECK(ctx && x && y && mean_out && rstd_out, YL_ERR_INVALID,
           "yl_groupnorm_silu_fwd_noalloc: NULL argument (mean_out and rstd_out are required)");
  const long long hw = (long long)h * w;
  YL_CHECK(h > 0 && w > 0, YL_ERR_SHAPE, "yl_groupnorm_silu_fwd_noalloc: empty image");
  YL_TRY(gn_check(n, c, groups, hw, c));
  GnGeom q = gn_geom(n, c, groups, hw, c);
  const size_t need = (size_t)n * q.chunks * 2 * groups;
  YL_CHECK(need <= kGnNoAllocDoubles, YL_ERR_SHAPE,
           "yl_groupnorm_silu_fwd_noalloc: n=%d groups=%d needs %zu statistics doubles, above "
           "the fixed %zu; use yl_groupnorm_silu_fwd",
           n, groups, need, kGnNoAllocDoubles);
  double* part = nullptr;
  YL_TRY(gn_noalloc_scratch(ctx->device, &part));
  dim3 grid(q.chunks, n);
  gn_stats_partial_kernel<<<grid, q.quads * q.rows, 2 * groups * sizeof(double), ctx->stream>>>(
      x, q, part);
  YL_TRY(check_launch("gn_stats_partial_kernel"));
  gn_stats_final_kernel<<<(n * groups + 127) / 128, 128, 0, ctx->stream>>>(part, q, eps, mode,
                                                                          mean_out, rstd_out);
  YL_TRY(check_launch("gn_stats_final_kernel"));
  const long long total = (long long)n * hw * q.quads;
  gn_apply_kernel<<<grid_1d(total, 256, ctx->num_sms * 16), 256, 0, ctx->stream>>>(
      x, q, mean_out, rstd_out, gamma, beta, apply_silu, 0, y, c);
  return check_launch("gn_apply_kernel");
}
