// yl_train_ops.cu -- the small, memory-bound training ops: multi-tensor
// Adam with the gradient sanitize/clip folded in, the VAE latent and loss
// heads, Linear layers, the timestep embedding and SiLU.
#include <cmath>

#include "yl_kernels.h"
#include "yl_norm.h"
#include "yl_ptx.cuh"

namespace yl {

// ------------------------------------------------------------------ Adam
// adam_kernel (MetalKernelSourcesA.swift:271-287) ran one launch per
// parameter tensor with pow() per element, after sanitizeGrads
// (GradSanitize.swift:18-101) copied every gradient to the CPU and back.
// Here: one launch computes the global squared norm of the (scaled,
// sanitized) gradients into a device scalar, and one launch updates all
// tensors, reading that scalar to apply the clip factor -- no host round trip.
constexpr int kMaxAdamTensors = 48;
struct AdamPack {
  AdamTensor t[kMaxAdamTensors];
  long long start[kMaxAdamTensors + 1];   // element prefix sums
  long long istart[kMaxAdamTensors + 1];  // work-item prefix sums (update kernel)
  int count;
};

__device__ __forceinline__ int adam_find(const AdamPack& p, long long i) {
  int lo = 0, hi = p.count - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (p.start[mid] <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float sanitize_scale(float g, float scale, int sanitize) {
  float v = g * scale;
  if (sanitize && !isfinite(v)) v = 0.f;
  return v;
}

__global__ void adam_norm_partial_kernel(const __grid_constant__ AdamPack p, float scale,
                                         int sanitize, double* part) {
  const long long total = p.start[p.count];
  double s = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = adam_find(p, i);
    const float v = sanitize_scale(p.t[k].grad[i - p.start[k]], scale, sanitize);
    s += (double)v * v;
  }
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

__global__ void adam_norm_final_kernel(const double* part, int nb, float* norm) {
  if (threadIdx.x == 0) {
    double s = 0;
    for (int i = 0; i < nb; ++i) s += part[i];
    norm[0] = (float)sqrt(s);
  }
}

__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float graw, float lr,
                                          float b1, float b2, float eps, float c1, float c2,
                                          float scale, int sanitize, float clipf) {
  const float g = sanitize_scale(graw, scale, sanitize) * clipf;
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  p -= lr * (m / c1) / (sqrtf(v / c2) + eps);
}

// Work items of kAdamChunk consecutive elements of one tensor; a block walks
// items with a grid stride and updates four elements per thread and step
// (16-byte loads) when the item's four arrays are 16-byte aligned.
constexpr long long kAdamChunk = 8192;

__global__ void adam_update_kernel(const __grid_constant__ AdamPack p, float lr, float b1, float b2,
                                   float eps, float c1, float c2, float scale, int sanitize,
                                   float clip, const float* norm) {
  float clipf = 1.f;
  if (clip > 0.f && norm) {
    const float nv = *norm;
    if (nv > clip) clipf = clip / nv;
  }
  const long long items = p.istart[p.count];
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    int k = 0;
    while (k + 1 < p.count && p.istart[k + 1] <= it) ++k;
    const AdamTensor& t = p.t[k];
    const long long c0 = (it - p.istart[k]) * kAdamChunk;
    const long long c1e = min(t.n, c0 + kAdamChunk);
    // the four arrays of a tensor never overlap: let the loads run ahead of the stores
    float* __restrict__ pp = t.param + c0;
    float* __restrict__ mp = t.m + c0;
    float* __restrict__ vp = t.v + c0;
    const float* __restrict__ gp = t.grad + c0;
    const long long len = c1e - c0;
    const bool vec = ((reinterpret_cast<uintptr_t>(pp) | reinterpret_cast<uintptr_t>(mp) |
                       reinterpret_cast<uintptr_t>(vp) | reinterpret_cast<uintptr_t>(gp)) &
                      15) == 0;
    long long done = 0;
    if (vec) {
      const long long n4 = len >> 2;
#pragma unroll 2
      for (long long q = threadIdx.x; q < n4; q += blockDim.x) {
        float4 P = reinterpret_cast<float4*>(pp)[q], M = reinterpret_cast<float4*>(mp)[q];
        float4 V = reinterpret_cast<float4*>(vp)[q];
        const float4 G = __ldg(reinterpret_cast<const float4*>(gp) + q);
        adam_elem(P.x, M.x, V.x, G.x, lr, b1, b2, eps, c1, c2, scale, sanitize, clipf);
        adam_elem(P.y, M.y, V.y, G.y, lr, b1, b2, eps, c1, c2, scale, sanitize, clipf);
        adam_elem(P.z, M.z, V.z, G.z, lr, b1, b2, eps, c1, c2, scale, sanitize, clipf);
        adam_elem(P.w, M.w, V.w, G.w, lr, b1, b2, eps, c1, c2, scale, sanitize, clipf);
        reinterpret_cast<float4*>(pp)[q] = P;
        reinterpret_cast<float4*>(mp)[q] = M;
        reinterpret_cast<float4*>(vp)[q] = V;
      }
      done = n4 << 2;
    }
    for (long long j = done + threadIdx.x; j < len; j += blockDim.x)
      adam_elem(pp[j], mp[j], vp[j], gp[j], lr, b1, b2, eps, c1, c2, scale, sanitize, clipf);
  }
}

yl_status adam_multi(yl_ctx* ctx, const AdamTensor* tensors, int count, float lr, float b1,
                     float b2, float eps, int t, float grad_scale, float clip_max_norm,
                     int sanitize, float* norm_out) {
  YL_CHECK(count >= 0, YL_ERR_INVALID, "adam_multi: negative tensor count");
  if (t < 1) t = 1;
  const float c1 = 1.f - powf(b1, (float)t), c2 = 1.f - powf(b2, (float)t);
  const int nb = ctx->num_sms * 4;
  float* norm = norm_out;
  void* ws = nullptr;
  const bool need_norm = clip_max_norm > 0.f || norm_out;
  if (need_norm) {
    YL_TRY(scratch_get(ctx, nb * sizeof(double) + 256, &ws));
    if (!norm) norm = (float*)((char*)ws + nb * sizeof(double));
  }
  for (int base = 0; base < count; base += kMaxAdamTensors) {
    AdamPack p;
    p.count = count - base < kMaxAdamTensors ? count - base : kMaxAdamTensors;
    p.start[0] = 0;
    p.istart[0] = 0;
    for (int k = 0; k < p.count; ++k) {
      p.t[k] = tensors[base + k];
      YL_CHECK(p.t[k].param && p.t[k].grad && p.t[k].m && p.t[k].v, YL_ERR_INVALID,
               "adam_multi: NULL pointer in tensor %d", base + k);
      p.start[k + 1] = p.start[k] + p.t[k].n;
      p.istart[k + 1] = p.istart[k] + (p.t[k].n + kAdamChunk - 1) / kAdamChunk;
    }
    if (p.start[p.count] == 0) continue;
    if (need_norm) {
      YL_CHECK(count <= kMaxAdamTensors, YL_ERR_UNSUPPORTED,
               "adam_multi: global-norm clipping supports at most %d tensors per call",
               kMaxAdamTensors);
      adam_norm_partial_kernel<<<nb, 256, 0, ctx->stream>>>(p, grad_scale, sanitize, (double*)ws);
      YL_TRY(check_launch("adam_norm_partial_kernel"));
      adam_norm_final_kernel<<<1, 32, 0, ctx->stream>>>((double*)ws, nb, norm);
      YL_TRY(check_launch("adam_norm_final_kernel"));
    }
    const long long items = p.istart[p.count];
    const int grid = (int)std::min<long long>(items, (long long)ctx->num_sms * 8);
    adam_update_kernel<<<grid, 256, 0, ctx->stream>>>(
        p, lr, b1, b2, eps, c1, c2, grad_scale, sanitize, clip_max_norm, need_norm ? norm : nullptr);
    YL_TRY(check_launch("adam_update_kernel"));
  }
  return YL_OK;
}

// ------------------------------------------------------------------ Linear
// LinearGPU (DenoiserMLP.swift:20-71): Y = X W^T + b; dX = dY W; dW = dY^T X;
// db = sumCols(dY).  Shapes here are tiny (batch <= 64, width <= 512).
__global__ void linear_fwd_kernel(const float* __restrict__ X, const float* __restrict__ W,
                                  const float* __restrict__ b, float* __restrict__ Y, int n,
                                  int ic, int oc) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= n * oc) return;
  const int r = wid / oc, o = wid % oc;
  const float* x = X + (long long)r * ic;
  const float* w = W + (long long)o * ic;
  float s = 0.f;
  for (int i = lane; i < ic; i += 32) s = fmaf(x[i], w[i], s);
#pragma unroll
  for (int d = 16; d; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if (lane == 0) Y[(long long)r * oc + o] = s + (b ? b[o] : 0.f);
}

__global__ void linear_dx_kernel(const float* __restrict__ W, const float* __restrict__ dY,
                                 float* __restrict__ dX, int n, int ic, int oc, int acc) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * ic) return;
  const int r = idx / ic, i = idx % ic;
  float s = 0.f;
  for (int o = 0; o < oc; ++o) s = fmaf(dY[(long long)r * oc + o], W[(long long)o * ic + i], s);
  dX[idx] = acc ? dX[idx] + s : s;
}

__global__ void linear_dw_kernel(const float* __restrict__ X, const float* __restrict__ dY,
                                 float* __restrict__ dW, float* __restrict__ db, int n, int ic,
                                 int oc, int acc) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx < oc * ic) {
    const int o = idx / ic, i = idx % ic;
    float s = 0.f;
    for (int r = 0; r < n; ++r) s = fmaf(dY[(long long)r * oc + o], X[(long long)r * ic + i], s);
    dW[idx] = acc ? dW[idx] + s : s;
  }
  if (db && idx < oc) {
    float s = 0.f;
    for (int r = 0; r < n; ++r) s += dY[(long long)r * oc + idx];
    db[idx] = acc ? db[idx] + s : s;
  }
}

yl_status linear_forward(yl_ctx* ctx, const float* X, const float* W, const float* b, float* Y,
                         int n, int ic, int oc) {
  YL_CHECK(X && W && Y, YL_ERR_INVALID, "linear_forward: NULL argument");
  long long threads = (long long)n * oc * 32;
  if (threads == 0) return YL_OK;
  linear_fwd_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(X, W, b, Y, n, ic,
                                                                               oc);
  return check_launch("linear_fwd_kernel");
}

yl_status linear_backward(yl_ctx* ctx, const float* X, const float* W, const float* dY, float* dX,
                          float* dW, float* db, int n, int ic, int oc, int accumulate) {
  YL_CHECK(dY, YL_ERR_INVALID, "linear_backward: dY is NULL");
  if (dX) {
    YL_CHECK(W, YL_ERR_INVALID, "linear_backward: W is NULL");
    linear_dx_kernel<<<(n * ic + 255) / 256, 256, 0, ctx->stream>>>(W, dY, dX, n, ic, oc,
                                                                   accumulate);
    YL_TRY(check_launch("linear_dx_kernel"));
  }
  if (dW) {
    YL_CHECK(X, YL_ERR_INVALID, "linear_backward: X is NULL");
    int m = oc * ic > oc ? oc * ic : oc;
    linear_dw_kernel<<<(m + 255) / 256, 256, 0, ctx->stream>>>(X, dY, dW, db, n, ic, oc,
                                                              accumulate);
    YL_TRY(check_launch("linear_dw_kernel"));
  } else if (db) {
    linear_dw_kernel<<<(oc + 255) / 256, 256, 0, ctx->stream>>>(X, dY, nullptr, db, n, 0, oc,
                                                               accumulate);
    YL_TRY(check_launch("linear_dw_kernel"));
  }
  return YL_OK;
}

// ------------------------------------------------------------------ embedding / SiLU
// motionTimeEmbedding (MotionPlanner.swift:155-165) in double, like the
// reference's host loop; variant 1 is timestep_embedding (src/diffusion.py:6-10).
__global__ void time_embedding_kernel(const float* __restrict__ t, int n, int dim, int variant,
                                      float* __restrict__ out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * (dim / 2)) return;
  const int b = idx / (dim / 2), j = idx % (dim / 2);
  if (variant == 0) {
    double tt = (double)t[b];
    if (!isfinite(tt)) tt = 0.0;
    tt = fmin(fmax(tt, 0.0), 1.0);
    const int i = 2 * j;
    const double w = pow(1000.0, (double)i / (double)dim);
    out[(long long)b * dim + i] = (float)sin(tt * w);
    out[(long long)b * dim + i + 1] = (float)cos(tt * w);
  } else {
    const int half = dim / 2;
    const float f = expf(-logf(10000.f) * (float)j / (float)half);
    const float a = t[b] * f;
    out[(long long)b * dim + j] = cosf(a);
    out[(long long)b * dim + half + j] = sinf(a);
  }
}

yl_status time_embedding(yl_ctx* ctx, const float* t, int n, int dim, int variant, float* out) {
  YL_CHECK(t && out, YL_ERR_INVALID, "time_embedding: NULL argument");
  YL_CHECK(dim > 0 && dim % 2 == 0, YL_ERR_SHAPE, "time_embedding: dim must be even and > 0");
  YL_CHECK(variant == 0 || variant == 1, YL_ERR_INVALID, "time_embedding: unknown variant");
  int total = n * (dim / 2);
  if (total == 0) return YL_OK;
  time_embedding_kernel<<<(total + 255) / 256, 256, 0, ctx->stream>>>(t, n, dim, variant, out);
  return check_launch("time_embedding_kernel");
}

__global__ void silu_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                            float* __restrict__ out, long long n, int bwd, int acc) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float a = x[i];
    const float s = 1.f / (1.f + expf(-a));
    float r = bwd ? dy[i] * s * (1.f + a * (1.f - s)) : a * s;
    out[i] = acc ? out[i] + r : r;
  }
}

yl_status silu_forward(yl_ctx* ctx, const float* x, float* y, long long n) {
  silu_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(x, nullptr, y, n, 0, 0);
  return check_launch("silu_kernel");
}
yl_status silu_backward(yl_ctx* ctx, const float* x, const float* dy, float* dx, long long n,
                        int accumulate) {
  silu_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(x, dy, dx, n, 1, accumulate);
  return check_launch("silu_kernel");
}

// ------------------------------------------------------------------ VAE heads
__device__ __forceinline__ uint32_t yhash(uint32_t x) {
  x = ((x >> ((x >> 28u) + 4u)) ^ x) * 277803737u;
  return (x >> 22u) ^ x;
}
// randn_kernel (MetalKernelSourcesB.swift:385-402).
__device__ __forceinline__ float yrandn(uint32_t seed, uint32_t gid) {
  const uint32_t h1 = yhash(gid * 747796405u + seed * 2891336453u + 1u);
  const uint32_t h2 = yhash(gid * 2654435761u + seed * 1013904223u + 0x9E3779B9u);
  const float u1 = fmaxf((float)(h1 >> 8) / 16777216.0f, 1e-7f);
  const float u2 = (float)(h2 >> 8) / 16777216.0f;
  return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
}
// trainingNoiseSeed (ConvVAEHelpers.swift:33-37).
__host__ __device__ __forceinline__ uint32_t noise_seed(int64_t step, int64_t b) {
  const uint64_t a = (uint64_t)step * 0x9E3779B97F4A7C15ull;
  const uint64_t bb = (uint64_t)b * 0xC2B2AE3D27D4EB4Full;
  return (uint32_t)((a ^ (bb + 0x165667B19E3779F9ull)) >> 32);
}

__global__ void latent_fwd_kernel(const float* __restrict__ e, int lde, int n, long long hw, int c,
                                  int64_t step, float* __restrict__ z, int ldz) {
  const long long total = (long long)n * hw * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    const long long pix = i / c;
    const int img = (int)(pix / hw);
    const long long p = pix - (long long)img * hw;
    const float mu = e[pix * lde + ch];
    const float lv = fminf(fmaxf(e[pix * lde + c + ch], -10.f), 10.f);
    const float ep = yrandn(noise_seed(step, img), (uint32_t)(ch * hw + p));
    z[pix * ldz + ch] = mu + expf(0.5f * lv) * ep;
  }
}

__global__ void latent_bwd_kernel(const float* __restrict__ e, int lde,
                                  const float* __restrict__ dz, int lddz, int n, long long hw,
                                  int c, int64_t step, float betaN, float betaHalfN,
                                  float* __restrict__ de, int ldde) {
  const long long total = (long long)n * hw * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    const long long pix = i / c;
    const int img = (int)(pix / hw);
    const long long p = pix - (long long)img * hw;
    const float mu = e[pix * lde + ch];
    const float lv = fminf(fmaxf(e[pix * lde + c + ch], -10.f), 10.f);
    const float ep = yrandn(noise_seed(step, img), (uint32_t)(ch * hw + p));
    const float d = dz[pix * lddz + ch];
    // vae_grad_kernel (MetalKernelSourcesB.swift:365-380)
    de[pix * ldde + ch] = round_tf32(d + betaN * mu);
    de[pix * ldde + c + ch] = round_tf32(d * ep * 0.5f * expf(0.5f * lv) + betaHalfN * (expf(lv) - 1.f));
  }
}

yl_status latent_head_forward(yl_ctx* ctx, const float* e, int lde, int n, long long hw, int c,
                              int64_t step, float* z, int ldz) {
  long long total = (long long)n * hw * c;
  latent_fwd_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(e, lde, n, hw, c, step, z, ldz);
  return check_launch("latent_fwd_kernel");
}

yl_status latent_head_backward(yl_ctx* ctx, const float* e, int lde, const float* dz, int lddz,
                               int n, long long hw, int c, int64_t step, float betaN,
                               float betaHalfN, float* de, int ldde) {
  long long total = (long long)n * hw * c;
  latent_bwd_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(e, lde, dz, lddz, n, hw, c, step,
                                                                 betaN, betaHalfN, de, ldde);
  return check_launch("latent_bwd_kernel");
}

// L1 (l1grad_kernel B:453-461) + KL (kl_reduce_kernel B:334-357) head.
__global__ void l1_kl_partial_kernel(const float* __restrict__ r, const float* __restrict__ t,
                                     long long n_pix, int ld, int ch, float inv,
                                     float* __restrict__ dr, const float* __restrict__ e, int lde,
                                     long long n_lat, int c_lat, double* part) {
  double l1 = 0, kl = 0;
  const long long nr = n_pix * ld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nr;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % ld);
    float g = 0.f;
    if (k < ch) {
      const float d = r[i] - t[i];
      l1 += fabs((double)d);
      g = (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f)) * inv;
    }
    if (dr) dr[i] = g;
  }
  const long long nl = n_lat * c_lat;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nl;
       i += (long long)gridDim.x * blockDim.x) {
    const long long pix = i / c_lat;
    const int k = (int)(i % c_lat);
    const float mu = e[pix * lde + k];
    const float lv = fminf(fmaxf(e[pix * lde + c_lat + k], -10.f), 10.f);
    kl += 0.5 * ((double)mu * mu + exp((double)lv) - 1.0 - lv);
  }
  __shared__ double ra[32], rb[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    kl += __shfl_xor_sync(0xffffffffu, kl, o);
  }
  if ((threadIdx.x & 31) == 0) {
    ra[threadIdx.x >> 5] = l1;
    rb[threadIdx.x >> 5] = kl;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0, b = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      a += ra[w];
      b += rb[w];
    }
    part[2 * blockIdx.x] = a;
    part[2 * blockIdx.x + 1] = b;
  }
}

__global__ void loss_final_kernel(const double* part, int nb, double sa, double sb, float* out) {
  if (threadIdx.x == 0) {
    double a = 0, b = 0;
    for (int i = 0; i < nb; ++i) {
      a += part[2 * i];
      b += part[2 * i + 1];
    }
    out[0] = (float)(a * sa + b * sb);
  }
}

yl_status l1_kl_head(yl_ctx* ctx, const float* recon, const float* target, long long n_pix, int ld,
                     int ch, const float* e, int lde, long long n_lat_pix, int c_lat, float beta,
                     float* drecon, float* loss_out) {
  const int nb = ctx->num_sms * 2;
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, 2 * nb * sizeof(double), &ws));
  const double nr = (double)n_pix * ch;
  const float inv = (float)(1.0 / nr);
  l1_kl_partial_kernel<<<nb, 256, 0, ctx->stream>>>(recon, target, n_pix, ld, ch, inv, drecon, e,
                                                    lde, e ? n_lat_pix : 0, c_lat, (double*)ws);
  YL_TRY(check_launch("l1_kl_partial_kernel"));
  if (loss_out) {
    const double nl = (double)n_lat_pix * c_lat;
    loss_final_kernel<<<1, 32, 0, ctx->stream>>>((double*)ws, nb, 1.0 / nr,
                                                 nl > 0 ? (double)beta / nl : 0.0, loss_out);
    YL_TRY(check_launch("loss_final_kernel"));
  }
  return YL_OK;
}

__global__ void mse_partial_kernel(const float* __restrict__ p, const float* __restrict__ t,
                                   long long n_pix, int ld, int ch, float scale,
                                   float* __restrict__ dp, double* part) {
  double s = 0;
  const long long n = n_pix * ld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % ld);
    float g = 0.f;
    if (k < ch) {
      const float d = p[i] - t[i];
      s += (double)d * d;
      g = scale * d;
    }
    if (dp) dp[i] = round_tf32(g);
  }
  __shared__ double ra[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) ra[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a += ra[w];
    part[2 * blockIdx.x] = a;
    part[2 * blockIdx.x + 1] = 0.0;
  }
}

yl_status mse_head(yl_ctx* ctx, const float* pred, const float* target, long long n_pix, int ld,
                   int ch, float* dpred, float* loss_out) {
  const int nb = ctx->num_sms * 2;
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, 2 * nb * sizeof(double), &ws));
  const double cnt = (double)n_pix * ch;
  mse_partial_kernel<<<nb, 256, 0, ctx->stream>>>(pred, target, n_pix, ld, ch, (float)(2.0 / cnt),
                                                  dpred, (double*)ws);
  YL_TRY(check_launch("mse_partial_kernel"));
  if (loss_out) {
    loss_final_kernel<<<1, 32, 0, ctx->stream>>>((double*)ws, nb, 1.0 / cnt, 0.0, loss_out);
    YL_TRY(check_launch("loss_final_kernel"));
  }
  return YL_OK;
}

}  // namespace yl

// ------------------------------------------------------------------ Sobel edge loss
// encodeSobelEdgeGrad (GpuSessionEdgeLoss.swift:10-41; kernels
// MetalKernelSourcesB.swift:466-551; CPU reference LossFunctions.swift:29-66,
// 194-235): L = (1/(h*w)) sum_q (|grad luma R|_q - |grad luma T|_q)^2 over the
// interior pixels, per image; dL/dR through the 3x3 Sobel windows.
namespace yl {

struct ImgView {  // channel c of pixel p of image i: base + i*istride + p*pstride + c*cstride
  const float* base;
  long long istride, pstride, cstride;
  __device__ __forceinline__ float at(long long i, long long p, int c) const {
    return base[i * istride + p * pstride + c * cstride];
  }
};

// One pass per 64 x 16 tile of output pixels: the luma of both images over
// the tile and a 2-pixel halo goes to shared memory once; each pixel of the
// tile and a 1-pixel ring gets its two Sobel magnitudes there, its share of
// the loss, and the coefficients its window hands back to the pixels under
// it; the tile's gradient then sums the 3x3 neighbours' coefficients.
// Global traffic: read both images once (halo re-reads hit L1/L2) and write
// the gradient -- 36 bytes per RGB pixel.
constexpr int kSobTW = 64, kSobTH = 16;

__device__ __forceinline__ float luma_at(const ImgView& v, long long img, long long q) {
  return 0.2126f * v.at(img, q, 0) + 0.7152f * v.at(img, q, 1) + 0.0722f * v.at(img, q, 2);
}

__global__ void __launch_bounds__(256)
    sobel_tile_kernel(ImgView r, ImgView t, int h, int w, int tiles_x, float scale, float* grad,
                      long long gi, long long gp, long long gc, double* __restrict__ part) {
  __shared__ float lr[kSobTH + 4][kSobTW + 4], lt[kSobTH + 4][kSobTW + 4];
  __shared__ float ax[kSobTH + 2][kSobTW + 2], ay[kSobTH + 2][kSobTW + 2];
  __shared__ double red[256];
  // Sobel taps, row by row (dy = -1..1, dx = -1..1)
  const float KX[9] = {-1.f, 0.f, 1.f, -2.f, 0.f, 2.f, -1.f, 0.f, 1.f};
  const float KY[9] = {-1.f, -2.f, -1.f, 0.f, 0.f, 0.f, 1.f, 2.f, 1.f};
  const int img = blockIdx.y;
  const int x0 = (blockIdx.x % tiles_x) * kSobTW, y0 = (blockIdx.x / tiles_x) * kSobTH;
  for (int i = threadIdx.x; i < (kSobTH + 4) * (kSobTW + 4); i += blockDim.x) {
    const int yy = i / (kSobTW + 4), xx = i % (kSobTW + 4);
    const int y = y0 - 2 + yy, x = x0 - 2 + xx;
    float a = 0.f, b = 0.f;
    if (y >= 0 && y < h && x >= 0 && x < w) {
      const long long q = (long long)y * w + x;
      a = luma_at(r, img, q);
      b = luma_at(t, img, q);
    }
    lr[yy][xx] = a;
    lt[yy][xx] = b;
  }
  __syncthreads();
  double acc = 0.0;
  for (int i = threadIdx.x; i < (kSobTH + 2) * (kSobTW + 2); i += blockDim.x) {
    const int yy = i / (kSobTW + 2), xx = i % (kSobTW + 2);
    const int y = y0 - 1 + yy, x = x0 - 1 + xx;
    float cx = 0.f, cy = 0.f;
    if (y >= 1 && y < h - 1 && x >= 1 && x < w - 1) {
      float sxr = 0.f, syr = 0.f, sxt = 0.f, syt = 0.f;
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const float vr = lr[yy + k / 3][xx + k % 3], vt = lt[yy + k / 3][xx + k % 3];
        sxr += KX[k] * vr;
        syr += KY[k] * vr;
        sxt += KX[k] * vt;
        syt += KY[k] * vt;
      }
      const float mr = sqrtf(sxr * sxr + syr * syr), mt = sqrtf(sxt * sxt + syt * syt);
      const float d0 = mr - mt;
      if (yy >= 1 && yy <= kSobTH && xx >= 1 && xx <= kSobTW) acc += (double)d0 * d0;
      const float inv = mr > 1e-6f ? 1.f / mr : 0.f;
      cx = d0 * inv * scale * sxr;
      cy = d0 * inv * scale * syr;
    }
    ax[yy][xx] = cx;
    ay[yy][xx] = cy;
  }
  __syncthreads();
  if (grad) {
    for (int i = threadIdx.x; i < kSobTH * kSobTW; i += blockDim.x) {
      const int yy = i / kSobTW, xx = i % kSobTW;
      const int y = y0 + yy, x = x0 + xx;
      if (y >= h || x >= w) continue;
      // pixel p sits at tap (1 - dy, 1 - dx) of the window centred at p + (dy, dx)
      float c = 0.f;
#pragma unroll
      for (int dy = -1; dy <= 1; ++dy)
#pragma unroll
        for (int dx = -1; dx <= 1; ++dx) {
          const int k = (1 - dy) * 3 + (1 - dx);
          c += ax[yy + 1 + dy][xx + 1 + dx] * KX[k] + ay[yy + 1 + dy][xx + 1 + dx] * KY[k];
        }
      float* g = grad + img * gi + ((long long)y * w + x) * gp;
      g[0] = c * 0.2126f;
      g[gc] = c * 0.7152f;
      g[2 * gc] = c * 0.0722f;
    }
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[(long long)img * gridDim.x + blockIdx.x] = red[0];
}

__global__ void sobel_loss_final_kernel(const double* __restrict__ part, int blocks, int n,
                                        double inv_hw, float* __restrict__ loss) {
  const int img = blockIdx.x * blockDim.x + threadIdx.x;
  if (img >= n) return;
  double s = 0.0;
  for (int b = 0; b < blocks; ++b) s += part[(long long)img * blocks + b];
  loss[img] = (float)(s * inv_hw);
}

}  // namespace yl

extern "C" yl_status yl_sobel_edge_loss(yl_ctx* ctx, const float* recon, const float* target,
                                        int n, int h, int w, int layout, int ld, float* grad,
                                        float* loss) {
  using namespace yl;
  YL_CHECK(ctx && recon && target && (grad || loss), YL_ERR_INVALID,
           "yl_sobel_edge_loss: NULL argument");
  YL_CHECK(n >= 1 && h >= 1 && w >= 1, YL_ERR_SHAPE, "yl_sobel_edge_loss: empty input");
  YL_CHECK(layout == YL_LAYOUT_NCHW || (layout == YL_LAYOUT_NHWC && ld >= 3), YL_ERR_INVALID,
           "yl_sobel_edge_loss: layout %d, pixel stride %d", layout, ld);
  const long long hw = (long long)h * w;
  const bool nchw = layout == YL_LAYOUT_NCHW;
  const long long istr = nchw ? 3 * hw : hw * ld, pstr = nchw ? 1 : ld, cstr = nchw ? hw : 1;
  ImgView r{recon, istr, pstr, cstr}, t{target, istr, pstr, cstr};
  const int tiles_x = (w + kSobTW - 1) / kSobTW, tiles_y = (h + kSobTH - 1) / kSobTH;
  const long long tiles = (long long)tiles_x * tiles_y;
  YL_CHECK(tiles < (1LL << 31) && n <= 65535, YL_ERR_SHAPE, "yl_sobel_edge_loss: %d x %d x %d",
           n, h, w);
  const int blocks = (int)tiles;
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)n * blocks * sizeof(double), &ws));
  double* part = (double*)ws;
  sobel_tile_kernel<<<dim3(blocks, n), 256, 0, ctx->stream>>>(
      r, t, h, w, tiles_x, (float)(2.0 / (double)hw), grad, istr, pstr, cstr, part);
  YL_TRY(check_launch("sobel_tile_kernel"));
  if (!loss) return YL_OK;
  sobel_loss_final_kernel<<<(n + 127) / 128, 128, 0, ctx->stream>>>(part, blocks, n,
                                                                     1.0 / (double)hw, loss);
  return check_launch("sobel_loss_final_kernel");
}

// ------------------------------------------------------------------ layered 8-channel loss
// layered_grad_kernel (MetalKernelSourcesB.swift:414-449) with the loss of
// layeredLoss (LayeredVAELoss.swift:129-149) in the same pass: per image, 8
// CHW planes (bg RGB | obj RGB | mask | light) against the target planes and
// the composed frame clamp((bg*(1-m) + obj*m) * light, 0, 1) against comp.
// One pass reads recon, target and comp once and writes the gradient (108 B
// per pixel); V = 4 moves four pixels of every plane per thread in float4.
namespace yl {

template <int V>
struct Vec;
template <>
struct Vec<1> {
  static __device__ __forceinline__ void ld(const float* p, float* o) { o[0] = __ldg(p); }
  static __device__ __forceinline__ void st(float* p, const float* v) { p[0] = v[0]; }
};
template <>
struct Vec<4> {
  static __device__ __forceinline__ void ld(const float* p, float* o) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = t.x;
    o[1] = t.y;
    o[2] = t.z;
    o[3] = t.w;
  }
  static __device__ __forceinline__ void st(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};

template <int V>
__global__ void __launch_bounds__(256, 4) layered_loss_kernel(
    const float* __restrict__ recon, const float* __restrict__ target,
    const float* __restrict__ comp, long long plane, float dl, float dc,
    float* __restrict__ grad, double* __restrict__ part) {
  const int img = blockIdx.y;
  const float* r = recon + (long long)img * 8 * plane;
  const float* t = target + (long long)img * 8 * plane;
  const float* cp = comp + (long long)img * 3 * plane;
  float* g = grad ? grad + (long long)img * 8 * plane : nullptr;
  const long long nv = plane / V;
  float sl = 0.f, sc = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i * V;
    float m[V], l[V], dm[V], dlt[V];
    Vec<V>::ld(r + 6 * plane + p, m);
    Vec<V>::ld(r + 7 * plane + p, l);
#pragma unroll
    for (int k = 0; k < V; ++k) dm[k] = dlt[k] = 0.f;
    // one colour channel at a time: background and object planes, their
    // targets and the frame channel in, both gradient planes out
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float bg[V], ob[V], tb[V], to[V], y[V], gb[V], go[V];
      Vec<V>::ld(r + c * plane + p, bg);
      Vec<V>::ld(r + (3 + c) * plane + p, ob);
      Vec<V>::ld(t + c * plane + p, tb);
      Vec<V>::ld(t + (3 + c) * plane + p, to);
      Vec<V>::ld(cp + c * plane + p, y);
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float im = 1.f - m[k];
        const float base = bg[k] * im + ob[k] * m[k];
        const float v = base * l[k];
        const float e = fminf(fmaxf(v, 0.f), 1.f) - y[k];
        sc = fmaf(e, e, sc);
        // the clamp passes the gradient only strictly inside (0, 1)
        const float gc = (v > 0.f && v < 1.f) ? dc * e : 0.f;
        const float db = bg[k] - tb[k], dob = ob[k] - to[k];
        sl = fmaf(db, db, fmaf(dob, dob, sl));
        gb[k] = dl * db + gc * l[k] * im;
        go[k] = dl * dob + gc * l[k] * m[k];
        dm[k] += gc * l[k] * (ob[k] - bg[k]);
        dlt[k] += gc * base;
      }
      if (g) {
        Vec<V>::st(g + c * plane + p, gb);
        Vec<V>::st(g + (3 + c) * plane + p, go);
      }
    }
    float tm[V], tl[V];
    Vec<V>::ld(t + 6 * plane + p, tm);
    Vec<V>::ld(t + 7 * plane + p, tl);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float d6 = m[k] - tm[k], d7 = l[k] - tl[k];
      sl = fmaf(d6, d6, fmaf(d7, d7, sl));
      tm[k] = dl * d6 + dm[k];
      tl[k] = dl * d7 + dlt[k];
    }
    if (g) {
      Vec<V>::st(g + 6 * plane + p, tm);
      Vec<V>::st(g + 7 * plane + p, tl);
    }
  }
  // block sums in double, fixed order
  __shared__ double red[2][256];
  red[0][threadIdx.x] = sl;
  red[1][threadIdx.x] = sc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      red[0][threadIdx.x] += red[0][threadIdx.x + o];
      red[1][threadIdx.x] += red[1][threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double* q = part + 2 * ((long long)img * gridDim.x + blockIdx.x);
    q[0] = red[0][0];
    q[1] = red[1][0];
  }
}

__global__ void layered_loss_final_kernel(const double* __restrict__ part, int blocks, int n,
                                          double wl_8n, double wc_3n, float* __restrict__ loss) {
  const int img = blockIdx.x * blockDim.x + threadIdx.x;
  if (img >= n) return;
  double sl = 0.0, sc = 0.0;
  for (int b = 0; b < blocks; ++b) {
    sl += part[2 * ((long long)img * blocks + b)];
    sc += part[2 * ((long long)img * blocks + b) + 1];
  }
  loss[img] = (float)(wl_8n * sl + wc_3n * sc);
}

template <int V>
__global__ void __launch_bounds__(256) layered_compose_kernel(const float* __restrict__ recon,
                                                              long long plane,
                                                              float* __restrict__ out) {
  const int img = blockIdx.y;
  const float* r = recon + (long long)img * 8 * plane;
  float* o = out + (long long)img * 3 * plane;
  const long long nv = plane / V;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i * V;
    float R[8][V], Y[3][V];
#pragma unroll
    for (int c = 0; c < 8; ++c) Vec<V>::ld(r + c * plane + p, R[c]);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float m = R[6][k], l = R[7][k], im = 1.f - m;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        Y[c][k] = fminf(fmaxf((R[c][k] * im + R[3 + c][k] * m) * l, 0.f), 1.f);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) Vec<V>::st(o + c * plane + p, Y[c]);
  }
}

static bool aligned16(const void* p) { return p == nullptr || ((uintptr_t)p & 15) == 0; }

// blocks per image: one wave of 4 resident 256-thread blocks per SM over the batch
static int layered_blocks(yl_ctx* ctx, long long nv, int n) {
  const long long want = (nv + 255) / 256;
  const long long cap = std::max(1LL, (long long)ctx->num_sms * 4 / n);
  return (int)std::max(1LL, std::min(want, cap));
}

}  // namespace yl

extern "C" yl_status yl_layered_loss(yl_ctx* ctx, const float* recon, const float* target,
                                     const float* comp, int n, long long plane, float layer_weight,
                                     float compose_weight, float* grad, float* loss) {
  using namespace yl;
  YL_CHECK(ctx && recon && target && comp && (grad || loss), YL_ERR_INVALID,
           "yl_layered_loss: NULL argument");
  YL_CHECK(n >= 1 && plane >= 1 && n <= 65535, YL_ERR_SHAPE,
           "yl_layered_loss: %d images of %lld pixels", n, plane);
  const bool v4 = plane % 4 == 0 && aligned16(recon) && aligned16(target) && aligned16(comp) &&
                  aligned16(grad);
  const long long nv = v4 ? plane / 4 : plane;
  const int blocks = layered_blocks(ctx, nv, n);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)n * blocks * 2 * sizeof(double), &ws));
  double* part = (double*)ws;
  const float dl = (float)(2.0 * layer_weight / (8.0 * (double)plane));
  const float dc = (float)(2.0 * compose_weight / (3.0 * (double)plane));
  if (v4)
    layered_loss_kernel<4><<<dim3(blocks, n), 256, 0, ctx->stream>>>(recon, target, comp, plane,
                                                                     dl, dc, grad, part);
  else
    layered_loss_kernel<1><<<dim3(blocks, n), 256, 0, ctx->stream>>>(recon, target, comp, plane,
                                                                     dl, dc, grad, part);
  YL_TRY(check_launch("layered_loss_kernel"));
  if (!loss) return YL_OK;
  layered_loss_final_kernel<<<(n + 127) / 128, 128, 0, ctx->stream>>>(
      part, blocks, n, (double)layer_weight / (8.0 * (double)plane),
      (double)compose_weight / (3.0 * (double)plane), loss);
  return check_launch("layered_loss_final_kernel");
}

extern "C" yl_status yl_layered_compose(yl_ctx* ctx, const float* recon, int n, long long plane,
                                        float* out) {
  using namespace yl;
  YL_CHECK(ctx && recon && out, YL_ERR_INVALID, "yl_layered_compose: NULL argument");
  YL_CHECK(n >= 1 && plane >= 1 && n <= 65535, YL_ERR_SHAPE,
           "yl_layered_compose: %d images of %lld pixels", n, plane);
  const bool v4 = plane % 4 == 0 && aligned16(recon) && aligned16(out);
  const long long nv = v4 ? plane / 4 : plane;
  const int blocks = layered_blocks(ctx, nv, n);
  if (v4)
    layered_compose_kernel<4><<<dim3(blocks, n), 256, 0, ctx->stream>>>(recon, plane, out);
  else
    layered_compose_kernel<1><<<dim3(blocks, n), 256, 0, ctx->stream>>>(recon, plane, out);
  return check_launch("layered_compose_kernel");
}
