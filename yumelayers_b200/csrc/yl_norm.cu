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
#include <algorithm>
#include <mutex>

#include "yl_kernels.h"
#include "yl_norm.h"
#include "yl_ptx.cuh"

namespace yl {

// SiLU and the logistic function with the approximate divide (2 ulp): the
// GroupNorm passes are bandwidth kernels that the IEEE divide's extra
// instructions would otherwise make issue-bound.
__device__ __forceinline__ float silu_f(float a) { return __fdividef(a, 1.f + __expf(-a)); }
__device__ __forceinline__ float sigmoid_f(float a) { return __fdividef(1.f, 1.f + __expf(-a)); }

// Launch geometry shared by all GroupNorm kernels.  A block is quads x rows
// threads; thread (quad, row) owns channels [4*quad, 4*quad+4) and walks the
// pixels p0 + row, p0 + row + rows, ... of its block's chunk, so every
// per-channel constant (group statistics, gamma, beta) is loop-invariant and
// no index needs a division.  Reductions use `chunks` pixel chunks per image
// (one wave of 4 blocks per SM over all images, at least 16 pixels per
// thread); the elementwise passes split each image into `achunks` work items
// that a grid of resident blocks walks (no partial last wave).
struct GnGeom {
  int n, c, g, ps;
  long long hw;
  int chunks, achunks;
  int quads, rows;
};

constexpr int kGnBlocksPerWave = 148 * 4;

static GnGeom gn_geom(int n, int c, int g, long long hw, int ps) {
  GnGeom q;
  q.n = n;
  q.c = c;
  q.g = g;
  q.ps = ps;
  q.hw = hw;
  q.quads = c / 4;
  q.rows = q.quads >= 256 ? 1 : 256 / q.quads;
  const long long per_img = n > 0 ? n : 1;
  long long cap = hw / (16LL * q.rows);
  if (cap < 1) cap = 1;
  q.chunks = (int)std::max(1LL, std::min((long long)kGnBlocksPerWave / per_img, cap));
  q.achunks = (int)std::max(1LL, std::min(4096LL / per_img, cap));
  return q;
}

__device__ __forceinline__ void chunk_range(const GnGeom& q, int chunk, int nchunks, long long* p0,
                                            long long* p1) {
  const long long per = (q.hw + nchunks - 1) / nchunks;
  *p0 = chunk * per;
  *p1 = min(q.hw, *p0 + per);
}

// partial[img][chunk][g] = (sum, sumsq).  Four pixels per iteration are summed
// in float, then added to the thread's double accumulators.
__global__ void gn_stats_partial_kernel(const float* __restrict__ x, GnGeom q,
                                        double* __restrict__ part) {
  extern __shared__ double sh[];  // [g][2]
  const int img = blockIdx.y, chunk = blockIdx.x;
  const int t = threadIdx.x;
  for (int i = t; i < 2 * q.g; i += blockDim.x) sh[i] = 0.0;
  __syncthreads();
  const int quad = t % q.quads, row = t / q.quads;
  const int grp = (quad * 4) / (q.c / q.g);
  long long p0, p1;
  chunk_range(q, chunk, q.chunks, &p0, &p1);
  const float* base = x + (long long)img * q.hw * q.ps + quad * 4;
  const long long step = (long long)q.rows * q.ps;
  double s = 0.0, ss = 0.0;
  long long p = p0 + row;
  const float* xp = base + p * q.ps;
  for (; p + 3LL * q.rows < p1; p += 4LL * q.rows, xp += 4 * step) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(xp));
    const float4 b = __ldg(reinterpret_cast<const float4*>(xp + step));
    const float4 c = __ldg(reinterpret_cast<const float4*>(xp + 2 * step));
    const float4 d = __ldg(reinterpret_cast<const float4*>(xp + 3 * step));
    const float fs = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w)) +
                     ((c.x + c.y) + (c.z + c.w)) + ((d.x + d.y) + (d.z + d.w));
    const float fq = ((a.x * a.x + a.y * a.y) + (a.z * a.z + a.w * a.w)) +
                     ((b.x * b.x + b.y * b.y) + (b.z * b.z + b.w * b.w)) +
                     ((c.x * c.x + c.y * c.y) + (c.z * c.z + c.w * c.w)) +
                     ((d.x * d.x + d.y * d.y) + (d.z * d.z + d.w * d.w));
    s += fs;
    ss += fq;
  }
  for (; p < p1; p += q.rows, xp += step) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(xp));
    s += (double)((a.x + a.y) + (a.z + a.w));
    ss += (double)((a.x * a.x + a.y * a.y) + (a.z * a.z + a.w * a.w));
  }
  if (p0 + row < p1) {
    atomicAdd(&sh[2 * grp], s);
    atomicAdd(&sh[2 * grp + 1], ss);
  }
  __syncthreads();
  double* out = part + ((long long)img * q.chunks + chunk) * 2 * q.g;
  for (int i = t; i < 2 * q.g; i += blockDim.x) out[i] = sh[i];
}

// One warp per (image, group): lanes sum the chunk partials in a fixed
// strided order, then a fixed shuffle tree (deterministic).
__global__ void gn_stats_final_kernel(const double* __restrict__ part, GnGeom q, float eps,
                                      int mode, float* __restrict__ mean,
                                      float* __restrict__ rstd) {
  const int idx = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // img * g + grp
  const int lane = threadIdx.x & 31;
  if (idx >= q.n * q.g) return;
  const int img = idx / q.g, grp = idx % q.g;
  double s = 0.0, ss = 0.0;
  for (int k = lane; k < q.chunks; k += 32) {
    const double* pp = part + ((long long)img * q.chunks + k) * 2 * q.g;
    s += pp[2 * grp];
    ss += pp[2 * grp + 1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if (lane) return;
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

__device__ __forceinline__ float4 gn_act4(float4 v, const float (&sc)[4], const float (&sh)[4],
                                          int silu, int round) {
  float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float a = fmaf(o[k], sc[k], sh[k]);
    if (silu) a = silu_f(a);
    o[k] = round ? round_tf32(a) : a;
  }
  return make_float4(o[0], o[1], o[2], o[3]);
}

// y = [silu]((x - mean) * rstd * gamma + beta) = [silu](x * scale + shift).
__global__ void __launch_bounds__(256, 4)
    gn_apply_kernel(const float* __restrict__ x, GnGeom q, const float* __restrict__ mean,
                    const float* __restrict__ rstd, const float* __restrict__ gamma,
                    const float* __restrict__ beta, int silu, int round, float* __restrict__ y,
                    int ldy) {
  const int quad = threadIdx.x % q.quads, row = threadIdx.x / q.quads;
  const int c = quad * 4;
  const int grp = c / (q.c / q.g);
  float ga[4], be[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    ga[k] = gamma ? __ldg(gamma + c + k) : 1.f;
    be[k] = beta ? __ldg(beta + c + k) : 0.f;
  }
  const long long R = q.rows;
  for (int item = blockIdx.x; item < q.n * q.achunks; item += gridDim.x) {
    const int img = item / q.achunks;
    const float m = mean[img * q.g + grp], r = rstd[img * q.g + grp];
    float sc[4], sf[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sc[k] = r * ga[k];
      sf[k] = be[k] - m * r * ga[k];
    }
    long long p0, p1;
    chunk_range(q, item - img * q.achunks, q.achunks, &p0, &p1);
    const float* xb = x + (long long)img * q.hw * q.ps + c;
    float* yb = y + (long long)img * q.hw * ldy + c;
    long long p = p0 + row;
    // three pixels per iteration: three 16-byte loads in flight per thread
    // (measured on 8x128x480x856: 6.0 TB/s, against 5.7 with four and 5.1
    // with eight -- fewer registers leave room for more resident blocks)
    for (; p + 2 * R < p1; p += 3 * R) {
      float4 a[3];
#pragma unroll
      for (int u = 0; u < 3; ++u)
        a[u] = __ldg(reinterpret_cast<const float4*>(xb + (p + u * R) * q.ps));
#pragma unroll
      for (int u = 0; u < 3; ++u)
        *reinterpret_cast<float4*>(yb + (p + u * R) * ldy) = gn_act4(a[u], sc, sf, silu, round);
    }
    for (; p < p1; p += R) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(xb + p * q.ps));
      *reinterpret_cast<float4*>(yb + p * ldy) = gn_act4(a, sc, sf, silu, round);
    }
  }
}

// Per element of the backward: xh = (x - mean) * rstd, a = xh * gamma + beta,
// da = dy * silu'(a) (or dy), dxh = da * gamma.
struct GnBwdConst {
  float m, r, ga[4], be[4];
};

__device__ __forceinline__ void gn_bwd_elem(float x, float dy, float ga, float be, float m, float r,
                                            int silu, float* xh, float* da) {
  *xh = (x - m) * r;
  float d = dy;
  if (silu) {
    const float a = fmaf(*xh, ga, be);
    const float sg = sigmoid_f(a);
    d *= sg * fmaf(a, 1.f - sg, 1.f);
  }
  *da = d;
}

// Backward partials per (img, chunk): group sums [g][2] of (dxh, dxh*xh), then
// channel sums [c][2] of (da*xh, da) for dgamma, dbeta.  Each thread sums its
// pixels in float (a few hundred per chunk at most); the block and chunk
// reductions are in double.  At most 64 registers, so four blocks fit per SM
// and the reduction grid is exactly one wave.
__global__ void __launch_bounds__(256, 4)
    gn_bwd_partial_kernel(const float* __restrict__ x, const float* __restrict__ dy, int lddy,
                          GnGeom q, const float* __restrict__ mean, const float* __restrict__ rstd,
                          const float* __restrict__ gamma, const float* __restrict__ beta,
                          int silu, double* __restrict__ part) {
  extern __shared__ double sh[];  // [g][2] + [c][2]
  const int img = blockIdx.y, chunk = blockIdx.x;
  const int t = threadIdx.x;
  const int nsh = 2 * q.g + 2 * q.c;
  for (int i = t; i < nsh; i += blockDim.x) sh[i] = 0.0;
  __syncthreads();
  const int quad = t % q.quads, row = t / q.quads;
  const int c = quad * 4;
  const int grp = c / (q.c / q.g);
  const float m = mean[img * q.g + grp], r = rstd[img * q.g + grp];
  float ga[4], be[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    ga[k] = gamma ? __ldg(gamma + c + k) : 1.f;
    be[k] = beta ? __ldg(beta + c + k) : 0.f;
  }
  long long p0, p1;
  chunk_range(q, chunk, q.chunks, &p0, &p1);
  const float* xb = x + (long long)img * q.hw * q.ps + c;
  const float* db = dy + (long long)img * q.hw * lddy + c;
  float sd = 0.f, sdx = 0.f, dg[4] = {0.f, 0.f, 0.f, 0.f}, dbt[4] = {0.f, 0.f, 0.f, 0.f};
  const long long R = q.rows;
  long long p = p0 + row;
  // four pixels per iteration: eight 16-byte loads in flight per thread
  for (; p < p1; p += 4 * R) {
    float4 xv[4], dv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long pp = p + u * R;
      xv[u] = dv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (pp < p1) {
        xv[u] = __ldg(reinterpret_cast<const float4*>(xb + pp * q.ps));
        dv[u] = __ldg(reinterpret_cast<const float4*>(db + pp * lddy));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (p + u * R >= p1) break;
      const float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
      const float ds[4] = {dv[u].x, dv[u].y, dv[u].z, dv[u].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float xh, dd;
        gn_bwd_elem(xs[k], ds[k], ga[k], be[k], m, r, silu, &xh, &dd);
        dg[k] = fmaf(dd, xh, dg[k]);
        dbt[k] += dd;
      }
    }
  }
  // the group sums of gamma*da and gamma*da*xh follow from the channel sums
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    sd = fmaf(ga[k], dbt[k], sd);
    sdx = fmaf(ga[k], dg[k], sdx);
  }
  if (p0 + row < p1) {
    atomicAdd(&sh[2 * grp], (double)sd);
    atomicAdd(&sh[2 * grp + 1], (double)sdx);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      atomicAdd(&sh[2 * q.g + 2 * (c + k)], (double)dg[k]);
      atomicAdd(&sh[2 * q.g + 2 * (c + k) + 1], (double)dbt[k]);
    }
  }
  __syncthreads();
  double* out = part + ((long long)img * q.chunks + chunk) * nsh;
  for (int i = t; i < nsh; i += blockDim.x) out[i] = sh[i];
}

// One warp per (img, grp) -> coef[img][grp][2] = (mean(dxh), mean(dxh*xh)),
// then one warp per channel -> dgamma, dbeta; fixed-order sums.
__global__ void gn_bwd_final_kernel(const double* __restrict__ part, GnGeom q,
                                    float* __restrict__ coef, float* dgamma, float* dbeta,
                                    int accumulate) {
  const int nsh = 2 * q.g + 2 * q.c;
  const int wid = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const double cnt = (double)q.hw * (q.c / q.g);
  double a = 0, b = 0;
  if (wid < q.n * q.g) {
    const int img = wid / q.g, grp = wid % q.g;
    for (int k = lane; k < q.chunks; k += 32) {
      const double* pp = part + ((long long)img * q.chunks + k) * nsh;
      a += pp[2 * grp];
      b += pp[2 * grp + 1];
    }
  } else if (wid < q.n * q.g + q.c) {
    const int ch = wid - q.n * q.g;
    for (int k = lane; k < q.n * q.chunks; k += 32) {
      const double* pp = part + (long long)k * nsh + 2 * q.g;
      a += pp[2 * ch];
      b += pp[2 * ch + 1];
    }
  } else {
    return;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (lane) return;
  if (wid < q.n * q.g) {
    coef[2 * wid] = (float)(a / cnt);
    coef[2 * wid + 1] = (float)(b / cnt);
  } else {
    const int ch = wid - q.n * q.g;
    if (dgamma) dgamma[ch] = accumulate ? dgamma[ch] + (float)a : (float)a;
    if (dbeta) dbeta[ch] = accumulate ? dbeta[ch] + (float)b : (float)b;
  }
}

// dx = rstd * (dxh - mean(dxh) - xh * mean(dxh*xh)) (+ addend).
__global__ void __launch_bounds__(256, 4)
    gn_bwd_apply_kernel(const float* __restrict__ x, const float* __restrict__ dy, int lddy,
                        GnGeom q, const float* __restrict__ mean, const float* __restrict__ rstd,
                        const float* __restrict__ gamma, const float* __restrict__ beta, int silu,
                        const float* __restrict__ coef, const float* __restrict__ addend,
                        int ldadd, float* __restrict__ dx, int lddx, int round) {
  const int quad = threadIdx.x % q.quads, row = threadIdx.x / q.quads;
  const int c = quad * 4;
  const int grp = c / (q.c / q.g);
  float ga[4], be[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    ga[k] = gamma ? __ldg(gamma + c + k) : 1.f;
    be[k] = beta ? __ldg(beta + c + k) : 0.f;
  }
  const long long R = q.rows;
  for (int item = blockIdx.x; item < q.n * q.achunks; item += gridDim.x) {
    const int img = item / q.achunks;
    const int gi = img * q.g + grp;
    const float m = mean[gi], r = rstd[gi];
    const float md = coef[2 * gi], mdx = coef[2 * gi + 1];
    long long p0, p1;
    chunk_range(q, item - img * q.achunks, q.achunks, &p0, &p1);
    const float* xb = x + (long long)img * q.hw * q.ps + c;
    const float* dyb = dy + (long long)img * q.hw * lddy + c;
    const float* ab = addend ? addend + (long long)img * q.hw * ldadd + c : nullptr;
    float* dxb = dx + (long long)img * q.hw * lddx + c;
    for (long long p = p0 + row; p < p1; p += 2 * R) {
      const bool two = p + R < p1;
      float4 xv[2], dv[2], av[2];
  #pragma unroll
      for (int u = 0; u < 2; ++u) {
        xv[u] = dv[u] = av[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u == 0 || two) {
          const long long pp = p + u * R;
          xv[u] = __ldg(reinterpret_cast<const float4*>(xb + pp * q.ps));
          dv[u] = __ldg(reinterpret_cast<const float4*>(dyb + pp * lddy));
          if (ab) av[u] = __ldg(reinterpret_cast<const float4*>(ab + pp * ldadd));
        }
      }
  #pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && !two) break;
        const float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
        const float ds[4] = {dv[u].x, dv[u].y, dv[u].z, dv[u].w};
        const float adds[4] = {av[u].x, av[u].y, av[u].z, av[u].w};
        float o[4];
  #pragma unroll
        for (int k = 0; k < 4; ++k) {
          float xh, da;
          gn_bwd_elem(xs[k], ds[k], ga[k], be[k], m, r, silu, &xh, &da);
          const float v = r * (da * ga[k] - md - xh * mdx) + adds[k];
          o[k] = round ? round_tf32(v) : v;
        }
        *reinterpret_cast<float4*>(dxb + (p + u * R) * lddx) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
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

// The two launches of the statistics pass, with the partials in `part`
// (n * chunks * 2 * g doubles).
static yl_status gn_stats_launch(yl_ctx* ctx, const float* x, const GnGeom& q, float eps, int mode,
                                 double* part, float* mean, float* rstd) {
  dim3 grid(q.chunks, q.n);
  gn_stats_partial_kernel<<<grid, q.quads * q.rows, 2 * q.g * sizeof(double), ctx->stream>>>(
      x, q, part);
  YL_TRY(check_launch("gn_stats_partial_kernel"));
  const int warps = q.n * q.g;
  gn_stats_final_kernel<<<(warps + 7) / 8, 256, 0, ctx->stream>>>(part, q, eps, mode, mean, rstd);
  return check_launch("gn_stats_final_kernel");
}

// Blocks of `kernel` that stay resident on the device at once (at least one).
template <typename K>
static int resident_grid(yl_ctx* ctx, K kernel, int threads, long long items) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const long long g = (long long)per_sm * ctx->num_sms;
  return (int)std::max(1LL, std::min(g, items));
}

static yl_status gn_apply_launch(yl_ctx* ctx, const float* x, const GnGeom& q, const float* mean,
                                 const float* rstd, const float* gamma, const float* beta,
                                 int silu, int round, float* y, int ldy) {
  const int threads = q.quads * q.rows;
  const int grid = resident_grid(ctx, gn_apply_kernel, threads, (long long)q.n * q.achunks);
  gn_apply_kernel<<<grid, threads, 0, ctx->stream>>>(x, q, mean, rstd, gamma, beta, silu, round, y,
                                                    ldy);
  return check_launch("gn_apply_kernel");
}

yl_status gn_stats(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                   float eps, int mode, float* mean, float* rstd) {
  YL_TRY(gn_check(n, c, g, hw, ps));
  GnGeom q = gn_geom(n, c, g, hw, ps);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)n * q.chunks * 2 * g * sizeof(double), &ws));
  return gn_stats_launch(ctx, x, q, eps, mode, (double*)ws, mean, rstd);
}

yl_status gn_silu_forward(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                          float eps, int mode, const float* gamma, const float* beta, int silu,
                          float* y, int ldy, int round, float* mean, float* rstd) {
  YL_TRY(gn_stats(ctx, x, n, c, g, hw, ps, eps, mode, mean, rstd));
  YL_CHECK(ldy % 4 == 0, YL_ERR_SHAPE, "groupnorm: output stride must be a multiple of 4");
  return gn_apply_launch(ctx, x, gn_geom(n, c, g, hw, ps), mean, rstd, gamma, beta, silu, round,
                         y, ldy);
}

yl_status gn_silu_apply(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                        const float* mean, const float* rstd, const float* gamma,
                        const float* beta, int silu, float* y, int ldy, int round) {
  YL_TRY(gn_check(n, c, g, hw, ps));
  YL_CHECK(ldy % 4 == 0, YL_ERR_SHAPE, "groupnorm: output stride must be a multiple of 4");
  return gn_apply_launch(ctx, x, gn_geom(n, c, g, hw, ps), mean, rstd, gamma, beta, silu, round,
                         y, ldy);
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
  const int warps = n * g + c;
  gn_bwd_final_kernel<<<(warps + 7) / 8, 256, 0, ctx->stream>>>(part, q, coef, dgamma, dbeta,
                                                              accumulate_params);
  YL_TRY(check_launch("gn_bwd_final_kernel"));
  const int agrid =
      resident_grid(ctx, gn_bwd_apply_kernel, q.quads * q.rows, (long long)n * q.achunks);
  gn_bwd_apply_kernel<<<agrid, q.quads * q.rows, 0, ctx->stream>>>(
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
//    one call on every device before any stream capture; the address is
//    cached for the life of the process (a cudaDeviceReset of the device
//    afterwards is not supported: it would leave the cached address stale);
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
  YL_TRY(gn_stats_launch(ctx, x, q, eps, mode, part, mean_out, rstd_out));
  return gn_apply_launch(ctx, x, q, mean_out, rstd_out, gamma, beta, apply_silu, 0, y, c);
}
