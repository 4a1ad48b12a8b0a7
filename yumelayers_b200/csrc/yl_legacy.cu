// yl_legacy.cu -- the reference-mode operators: one C entry point per
// GpuSession method with the reference kernel's exact semantics, in the
// reference's per-image CHW layout (GpuSessionOps.swift, MetalKernelSources*.swift).
// They keep fp32 arithmetic (the reference's tests pin them at 1e-5..1e-4),
// but are written as parallel kernels: grid-stride elementwise loops, a
// shared-memory tiled GEMM, and block/grid reductions where the reference
// runs one thread per group or one thread per output over a serial loop.
#include <cmath>

#include "yl_kernels.h"
#include "yl_ptx.cuh"

namespace yl {

// ------------------------------------------------------------------ GEMM
// C[M,N] = op(A) * op(B), fp32 FMA, 64x64 tile, 16x16 threads, 4x4 per thread.
// matmul_kernel / matmul_tiled_kernel (MetalKernelSourcesA.swift:11-94).
__global__ void legacy_matmul_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                     float* __restrict__ C, int M, int N, int K, int transA,
                                     int transB) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * 16 + tx;
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = tid; e < 64 * 16; e += 256) {
      int mm = e / 16, kk = e % 16;
      int r = r0 + mm, k = k0 + kk;
      float av = 0.f;
      if (r < M && k < K) av = transA ? A[(long long)k * M + r] : A[(long long)r * K + k];
      As[kk][mm] = av;
      int nn = e / 16;
      int c = c0 + nn;
      float bv = 0.f;
      if (c < N && k < K) bv = transB ? B[(long long)c * K + k] : B[(long long)k * N + c];
      Bs[kk][nn] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int i = 0; i < 4; ++i) b[i] = Bs[kk][tx * 4 + i];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(a[i], b[jj], acc[i][jj]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      int r = r0 + ty * 4 + i, c = c0 + tx * 4 + jj;
      if (r < M && c < N) C[(long long)r * N + c] = acc[i][jj];
    }
}

static yl_status legacy_matmul(yl_ctx* ctx, const float* A, const float* B, float* C, int M, int N,
                               int K, int transA, int transB) {
  if (M == 0 || N == 0) return YL_OK;
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  legacy_matmul_kernel<<<grid, dim3(16, 16), 0, ctx->stream>>>(A, B, C, M, N, K, transA, transB);
  return check_launch("legacy_matmul_kernel");
}

// gradW: C[r,c] = sum_i A[r*K+i] * B[c*K+i] (gradw_plain_kernel, A:122-137):
// one warp per output element with a shuffle reduction instead of a serial K loop.
__global__ void legacy_gradw_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                    float* __restrict__ C, int oc, int kk, int K) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= oc * kk) return;
  const int r = warp_global / kk, c = warp_global % kk;
  const float* a = A + (long long)r * K;
  const float* b = B + (long long)c * K;
  float s = 0.f;
  for (int i = lane; i < K; i += 32) s = fmaf(a[i], b[i], s);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) C[(long long)r * kk + c] = s;
}

// ------------------------------------------------------------------ conv primitives
__global__ void legacy_im2col_kernel(const float* __restrict__ X, float* __restrict__ C, int ic,
                                     int ih, int iw, int kh, int kw, int stride, int pad, int oh,
                                     int ow) {
  const long long total = (long long)ic * kh * kw * oh * ow;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int sp = (int)(idx % ((long long)oh * ow));
    const int col = (int)(idx / ((long long)oh * ow));
    const int c = col / (kh * kw), r = col % (kh * kw);
    const int ky = r / kw, kx = r % kw;
    const int oy = sp / ow, ox = sp % ow;
    const int iy = oy * stride + ky - pad, ix = ox * stride + kx - pad;
    float v = 0.f;
    if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) v = X[((long long)c * ih + iy) * iw + ix];
    C[idx] = v;
  }
}

__global__ void legacy_col2im_kernel(const float* __restrict__ C, float* __restrict__ G, int ic,
                                     int ih, int iw, int kh, int kw, int stride, int pad, int oh,
                                     int ow) {
  const long long total = (long long)ic * ih * iw;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int x = (int)(idx % iw);
    const int y = (int)((idx / iw) % ih);
    const int c = (int)(idx / ((long long)iw * ih));
    float acc = 0.f;
    for (int ky = 0; ky < kh; ++ky) {
      const int sy = y + pad - ky;
      if (sy < 0 || sy % stride != 0) continue;
      const int oy = sy / stride;
      if (oy >= oh) continue;
      for (int kx = 0; kx < kw; ++kx) {
        const int sx = x + pad - kx;
        if (sx < 0 || sx % stride != 0) continue;
        const int ox = sx / stride;
        if (ox >= ow) continue;
        acc += C[((long long)c * kh * kw + ky * kw + kx) * (oh * ow) + oy * ow + ox];
      }
    }
    G[idx] = acc;
  }
}

__global__ void legacy_conv_back_input_s1_kernel(const float* __restrict__ dOut,
                                                 const float* __restrict__ W,
                                                 float* __restrict__ dx, int ic, int oc, int ih,
                                                 int iw, int kh, int kw, int pad) {
  const int oh = ih + 2 * pad - kh + 1, ow = iw + 2 * pad - kw + 1;
  const long long total = (long long)ic * ih * iw;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int x = (int)(idx % iw);
    const int y = (int)((idx / iw) % ih);
    const int c = (int)(idx / ((long long)iw * ih));
    float acc = 0.f;
    for (int o = 0; o < oc; ++o) {
      const long long woff = (long long)o * (ic * kh * kw) + (long long)c * (kh * kw);
      for (int ky = 0; ky < kh; ++ky) {
        const int oy = y + pad - ky;
        if (oy < 0 || oy >= oh) continue;
        for (int kx = 0; kx < kw; ++kx) {
          const int ox = x + pad - kx;
          if (ox < 0 || ox >= ow) continue;
          acc += dOut[(long long)o * (oh * ow) + oy * ow + ox] * W[woff + ky * kw + kx];
        }
      }
    }
    dx[idx] = acc;
  }
}

// Row sums (biasRowGrad) and column sums (sumCols): one block per row /
// 32-column strip with a block reduction.
__global__ void legacy_row_sum_kernel(const float* __restrict__ G, float* __restrict__ out,
                                      int cols) {
  const float* row = G + (long long)blockIdx.x * cols;
  float s = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) s += row[i];
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) out[blockIdx.x] = s;
  }
}

__global__ void legacy_col_sum_kernel(const float* __restrict__ A, float* __restrict__ C, int rows,
                                      int cols) {
  __shared__ float red[8][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (col < cols)
    for (int r = threadIdx.y; r < rows; r += 8) s += A[(long long)r * cols + col];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && col < cols) {
    float t = 0.f;
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    C[col] = t;
  }
}

// ------------------------------------------------------------------ GroupNorm (reference mode)
// groupnorm_kernel / groupnorm_grad_kernel (MetalKernelSourcesC.swift:10-101):
// affine-free, var = E[x^2] - E[x]^2 clamped at >= 1e-5, no eps.  One block
// per group with a double-precision block reduction (the reference's CPU
// truth, LossFunctions.swift:97-176, accumulates in double).
template <int NT>
__device__ void block_sum2(double& a, double& b) {
  __shared__ double ra[NT / 32], rb[NT / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if ((threadIdx.x & 31) == 0) {
    ra[threadIdx.x >> 5] = a;
    rb[threadIdx.x >> 5] = b;
  }
  __syncthreads();
  a = 0;
  b = 0;
  for (int i = 0; i < NT / 32; ++i) {
    a += ra[i];
    b += rb[i];
  }
  __syncthreads();
}

__global__ void legacy_groupnorm_kernel(const float* __restrict__ in, float* __restrict__ out,
                                        int C, int P, int groups) {
  const int gsize = C / groups;
  const int g = blockIdx.x;
  const long long base = (long long)g * gsize * P, n = (long long)gsize * P;
  double s = 0, q = 0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    double v = in[base + i];
    s += v;
    q += v * v;
  }
  block_sum2<256>(s, q);
  double mean = s / n, var = q / n - mean * mean;
  if (var < 1e-5) var = 1e-5;
  const double inv = 1.0 / sqrt(var);
  for (long long i = threadIdx.x; i < n; i += blockDim.x)
    out[base + i] = (float)((in[base + i] - mean) * inv);
}

__global__ void legacy_groupnorm_grad_kernel(const float* __restrict__ in,
                                             const float* __restrict__ dy, float* __restrict__ out,
                                             int C, int P, int groups) {
  const int gsize = C / groups;
  const int g = blockIdx.x;
  const long long base = (long long)g * gsize * P, n = (long long)gsize * P;
  double s = 0, q = 0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    double v = in[base + i];
    s += v;
    q += v * v;
  }
  block_sum2<256>(s, q);
  double mean = s / n, var = q / n - mean * mean;
  if (var < 1e-5) var = 1e-5;
  const double inv = 1.0 / sqrt(var);
  double sd = 0, sdx = 0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    double d = dy[base + i];
    sd += d;
    sdx += d * (in[base + i] - mean);
  }
  block_sum2<256>(sd, sdx);
  const double md = sd / n, mdx = sdx / n;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    double xm = in[base + i] - mean;
    out[base + i] = (float)(inv * (dy[base + i] - md - xm * mdx / var));
  }
}

// ------------------------------------------------------------------ elementwise
__device__ __forceinline__ float sigmoidf_(float a) { return 1.f / (1.f + expf(-a)); }

__global__ void legacy_unary_kernel(int op, const float* __restrict__ A, float* __restrict__ C,
                                    long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float a = A[i];
    float r;
    switch (op) {
      case YL_RELU: r = fmaxf(a, 0.f); break;
      case YL_SIGMOID: r = sigmoidf_(a); break;
      case YL_TANH: r = tanhf(a); break;
      case YL_TANH_GRAD: { float t = tanhf(a); r = 1.f - t * t; } break;
      case YL_EXP: r = expf(a); break;
      case YL_EXP_HALF: r = expf(0.5f * fminf(fmaxf(a, -10.f), 10.f)); break;
      default: r = a * sigmoidf_(a); break;  // YL_SILU
    }
    C[i] = r;
  }
}

__global__ void legacy_binary_kernel(int op, const float* __restrict__ A,
                                     const float* __restrict__ B, float* __restrict__ C,
                                     long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float a = A[i], b = B[i];
    float r;
    switch (op) {
      case YL_ADD: r = a + b; break;
      case YL_SUB: r = a - b; break;
      case YL_MUL: r = a * b; break;
      case YL_RELU_GRAD: r = a > 0.f ? b : 0.f; break;
      case YL_SIGMOID_GRAD: { float s = sigmoidf_(a); r = b * s * (1.f - s); } break;
      default: { float s = sigmoidf_(a); r = b * s * (1.f + a * (1.f - s)); } break;  // SiLU'
    }
    C[i] = r;
  }
}

__global__ void legacy_affine_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                     const float* __restrict__ D, float* C, float s, float add,
                                     int mode, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    switch (mode) {
      case 0: C[i] = A[i] * s; break;           // smul
      case 1: C[i] = A[i] + add; break;         // addConst
      case 2: C[i] = A[i] + B[i] * D[i]; break; // fma
      default: C[i] = C[i] + B[i]; break;       // addInPlace (C == A)
    }
  }
}

__global__ void legacy_bias_kernel(const float* __restrict__ A, const float* __restrict__ b,
                                   float* __restrict__ C, int rows, int cols, int per_row) {
  const long long n = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    C[i] = A[i] + (per_row ? b[i / cols] : b[i % cols]);
}

__global__ void legacy_updown_kernel(const float* __restrict__ X, float* __restrict__ Y, int c,
                                     int h, int w, int up) {
  const long long n = up ? (long long)c * 4 * h * w : (long long)c * h * w;
  const int w2 = 2 * w;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    if (up) {
      const int x = (int)(i % w2);
      const int y = (int)((i / w2) % (2 * h));
      const int ch = (int)(i / ((long long)w2 * 2 * h));
      Y[i] = X[((long long)ch * h + y / 2) * w + x / 2];
    } else {
      const int x = (int)(i % w);
      const int y = (int)((i / w) % h);
      const int ch = (int)(i / ((long long)w * h));
      const long long base = ((long long)ch * h * 2 + y * 2) * w2 + x * 2;
      Y[i] = X[base] + X[base + 1] + X[base + w2] + X[base + w2 + 1];
    }
  }
}

// yume_hash + randn_kernel (MetalKernelSourcesB.swift:385-402).
__device__ __forceinline__ uint32_t yume_hash(uint32_t x) {
  x = ((x >> ((x >> 28u) + 4u)) ^ x) * 277803737u;
  return (x >> 22u) ^ x;
}
__device__ __forceinline__ float yume_randn(uint32_t seed, uint32_t gid) {
  const uint32_t h1 = yume_hash(gid * 747796405u + seed * 2891336453u + 1u);
  const uint32_t h2 = yume_hash(gid * 2654435761u + seed * 1013904223u + 0x9E3779B9u);
  const float u1 = fmaxf((float)(h1 >> 8) / 16777216.0f, 1e-7f);
  const float u2 = (float)(h2 >> 8) / 16777216.0f;
  return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
}
__global__ void legacy_randn_kernel(float* out, uint32_t seed, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = yume_randn(seed, (uint32_t)i);
}

// mse_reduce_kernel (B:236-258) / kl_reduce_kernel (B:334-357): grid-wide
// reduction in double partials, then one fixed-order final pass.
__global__ void legacy_reduce_partial_kernel(const float* __restrict__ a,
                                             const float* __restrict__ b, long long n, int mode,
                                             double* part) {
  double s = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    if (mode == 0) {
      const double d = (double)a[i] - b[i];
      s += d * d;
    } else {
      const float l = fminf(fmaxf(b[i], -10.f), 10.f);
      s += 0.5 * ((double)a[i] * a[i] + exp((double)l) - 1.0 - l);
    }
  }
  double dummy = 0;
  block_sum2<256>(s, dummy);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}
__global__ void legacy_reduce_final_kernel(const double* part, int nb, float* out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0;
    for (int i = 0; i < nb; ++i) s += part[i];
    out[0] = (float)s;
  }
}

__global__ void legacy_l1grad_kernel(const float* __restrict__ r, const float* __restrict__ t,
                                     float* __restrict__ out, float invN, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float d = r[i] - t[i];
    out[i] = (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f)) * invN;
  }
}

__global__ void legacy_vae_grad_kernel(const float* __restrict__ dz, const float* __restrict__ mu,
                                       const float* __restrict__ lv, const float* __restrict__ eps,
                                       float* __restrict__ dmu, float* __restrict__ dlv,
                                       float betaN, float betaHalfN, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float l = fminf(fmaxf(lv[i], -10.f), 10.f);
    const float d = dz[i];
    dmu[i] = d + betaN * mu[i];
    dlv[i] = d * eps[i] * 0.5f * expf(0.5f * l) + betaHalfN * (expf(l) - 1.f);
  }
}

// adam_kernel (MetalKernelSourcesA.swift:271-287); the bias corrections are
// computed once on the host instead of pow() per element.
__global__ void legacy_adam_kernel(float* __restrict__ p, const float* __restrict__ g,
                                   float* __restrict__ m, float* __restrict__ v, long long n,
                                   float lr, float c1, float c2) {
  const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gi = g[i];
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    p[i] -= lr * (mi / c1) / (sqrtf(vi / c2) + eps);
  }
}

}  // namespace yl

using namespace yl;

#define YL_NN(...)                                                              \
  do {                                                                          \
    const void* ptrs_[] = {__VA_ARGS__};                                        \
    for (const void* p_ : ptrs_)                                                \
      YL_CHECK(p_ != nullptr, YL_ERR_INVALID, "%s: NULL argument", __func__);   \
  } while (0)

extern "C" {

yl_status yl_matmul(yl_ctx* ctx, const float* A, const float* B, float* C, int M, int N, int K,
                    int transA, int transB) {
  YL_NN(ctx, A, B, C);
  YL_CHECK(M >= 0 && N >= 0 && K >= 0, YL_ERR_SHAPE, "yl_matmul: negative dimension");
  return legacy_matmul(ctx, A, B, C, M, N, K, transA, transB);
}

yl_status yl_im2col(yl_ctx* ctx, const float* X, float* cols, int ic, int ih, int iw, int kh,
                    int kw, int stride, int pad) {
  YL_NN(ctx, X, cols);
  YL_CHECK(stride > 0 && ih + 2 * pad >= kh && iw + 2 * pad >= kw, YL_ERR_SHAPE,
           "yl_im2col: bad geometry");
  int oh = (ih + 2 * pad - kh) / stride + 1, ow = (iw + 2 * pad - kw) / stride + 1;
  long long total = (long long)ic * kh * kw * oh * ow;
  legacy_im2col_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(X, cols, ic, ih, iw, kh, kw,
                                                                    stride, pad, oh, ow);
  return check_launch("legacy_im2col_kernel");
}

yl_status yl_col2im(yl_ctx* ctx, const float* cols, float* G, int ic, int ih, int iw, int kh,
                    int kw, int stride, int pad, int oh, int ow) {
  YL_NN(ctx, cols, G);
  YL_CHECK(stride > 0, YL_ERR_SHAPE, "yl_col2im: stride must be positive");
  long long total = (long long)ic * ih * iw;
  legacy_col2im_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(cols, G, ic, ih, iw, kh, kw,
                                                                    stride, pad, oh, ow);
  return check_launch("legacy_col2im_kernel");
}

yl_status yl_grad_w(yl_ctx* ctx, const float* A, const float* B, float* C, int oc, int kk, int K) {
  YL_NN(ctx, A, B, C);
  long long warps = (long long)oc * kk;
  if (warps == 0) return YL_OK;
  legacy_gradw_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(A, B, C, oc,
                                                                                    kk, K);
  return check_launch("legacy_gradw_kernel");
}

yl_status yl_conv_back_input_s1(yl_ctx* ctx, const float* dOut, const float* W, float* dx, int ic,
                                int oc, int ih, int iw, int k, int pad) {
  YL_NN(ctx, dOut, W, dx);
  long long total = (long long)ic * ih * iw;
  legacy_conv_back_input_s1_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(
      dOut, W, dx, ic, oc, ih, iw, k, k, pad);
  return check_launch("legacy_conv_back_input_s1_kernel");
}

yl_status yl_bias_row(yl_ctx* ctx, const float* A, const float* b, float* C, int rows, int cols) {
  YL_NN(ctx, A, b, C);
  legacy_bias_kernel<<<grid_1d((long long)rows * cols, 256), 256, 0, ctx->stream>>>(A, b, C, rows,
                                                                                    cols, 1);
  return check_launch("legacy_bias_kernel");
}

yl_status yl_bias_row_grad(yl_ctx* ctx, const float* G, float* out, int rows, int cols) {
  YL_NN(ctx, G, out);
  if (rows == 0) return YL_OK;
  legacy_row_sum_kernel<<<rows, 256, 0, ctx->stream>>>(G, out, cols);
  return check_launch("legacy_row_sum_kernel");
}

yl_status yl_add_bias(yl_ctx* ctx, const float* A, const float* bias, float* C, int rows,
                      int cols) {
  YL_NN(ctx, A, bias, C);
  legacy_bias_kernel<<<grid_1d((long long)rows * cols, 256), 256, 0, ctx->stream>>>(A, bias, C,
                                                                                    rows, cols, 0);
  return check_launch("legacy_bias_kernel");
}

yl_status yl_sum_cols(yl_ctx* ctx, const float* A, float* C, int rows, int cols) {
  YL_NN(ctx, A, C);
  if (cols == 0) return YL_OK;
  legacy_col_sum_kernel<<<(cols + 31) / 32, dim3(32, 8), 0, ctx->stream>>>(A, C, rows, cols);
  return check_launch("legacy_col_sum_kernel");
}

yl_status yl_group_norm(yl_ctx* ctx, const float* A, float* C, int rows, int cols, int groups) {
  YL_NN(ctx, A, C);
  YL_CHECK(groups >= 1 && rows % groups == 0, YL_ERR_SHAPE,
           "yl_group_norm: rows %d %% groups %d != 0", rows, groups);
  legacy_groupnorm_kernel<<<groups, 256, 0, ctx->stream>>>(A, C, rows, cols, groups);
  return check_launch("legacy_groupnorm_kernel");
}

yl_status yl_group_norm_grad(yl_ctx* ctx, const float* x, const float* dy, float* out, int rows,
                             int cols, int groups) {
  YL_NN(ctx, x, dy, out);
  YL_CHECK(groups >= 1 && rows % groups == 0, YL_ERR_SHAPE,
           "yl_group_norm_grad: rows %d %% groups %d != 0", rows, groups);
  legacy_groupnorm_grad_kernel<<<groups, 256, 0, ctx->stream>>>(x, dy, out, rows, cols, groups);
  return check_launch("legacy_groupnorm_grad_kernel");
}

yl_status yl_unary(yl_ctx* ctx, int op, const float* A, float* C, size_t n) {
  YL_NN(ctx, A, C);
  YL_CHECK(op >= YL_RELU && op <= YL_SILU, YL_ERR_INVALID, "yl_unary: unknown op %d", op);
  legacy_unary_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(op, A, C, (long long)n);
  return check_launch("legacy_unary_kernel");
}

yl_status yl_binary(yl_ctx* ctx, int op, const float* A, const float* B, float* C, size_t n) {
  YL_NN(ctx, A, B, C);
  YL_CHECK(op >= YL_ADD && op <= YL_SILU_GRAD, YL_ERR_INVALID, "yl_binary: unknown op %d", op);
  legacy_binary_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(op, A, B, C, (long long)n);
  return check_launch("legacy_binary_kernel");
}

yl_status yl_smul(yl_ctx* ctx, float s, const float* A, float* C, size_t n) {
  YL_NN(ctx, A, C);
  legacy_affine_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(A, nullptr, nullptr, C, s, 0.f, 0,
                                                                (long long)n);
  return check_launch("legacy_affine_kernel");
}

yl_status yl_add_const(yl_ctx* ctx, const float* A, float s, float* C, size_t n) {
  YL_NN(ctx, A, C);
  legacy_affine_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(A, nullptr, nullptr, C, 0.f, s, 1,
                                                                (long long)n);
  return check_launch("legacy_affine_kernel");
}

yl_status yl_fma(yl_ctx* ctx, const float* A, const float* B, const float* D, float* C, size_t n) {
  YL_NN(ctx, A, B, D, C);
  legacy_affine_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(A, B, D, C, 0.f, 0.f, 2,
                                                                (long long)n);
  return check_launch("legacy_affine_kernel");
}

yl_status yl_add_in_place(yl_ctx* ctx, float* A, const float* B, size_t n) {
  YL_NN(ctx, A, B);
  legacy_affine_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(A, B, nullptr, A, 0.f, 0.f, 3,
                                                                (long long)n);
  return check_launch("legacy_affine_kernel");
}

yl_status yl_upsample2x(yl_ctx* ctx, const float* X, float* Y, int c, int h, int w) {
  YL_NN(ctx, X, Y);
  legacy_updown_kernel<<<grid_1d((long long)c * 4 * h * w, 256), 256, 0, ctx->stream>>>(X, Y, c, h,
                                                                                        w, 1);
  return check_launch("legacy_updown_kernel");
}

yl_status yl_downsample2x(yl_ctx* ctx, const float* X, float* Y, int c, int h, int w) {
  YL_NN(ctx, X, Y);
  legacy_updown_kernel<<<grid_1d((long long)c * h * w, 256), 256, 0, ctx->stream>>>(X, Y, c, h, w,
                                                                                    0);
  return check_launch("legacy_updown_kernel");
}

yl_status yl_split2(yl_ctx* ctx, const float* X, float* mu, float* logvar, int c, int plane) {
  YL_NN(ctx, X, mu, logvar);
  size_t n = (size_t)c * plane * sizeof(float);
  YL_CUDA(cudaMemcpyAsync(mu, X, n, cudaMemcpyDeviceToDevice, ctx->stream));
  YL_CUDA(cudaMemcpyAsync(logvar, X + (size_t)c * plane, n, cudaMemcpyDeviceToDevice, ctx->stream));
  return YL_OK;
}

yl_status yl_merge2(yl_ctx* ctx, const float* mu, const float* logvar, float* X, int c, int plane) {
  YL_NN(ctx, X, mu, logvar);
  size_t n = (size_t)c * plane * sizeof(float);
  YL_CUDA(cudaMemcpyAsync(X, mu, n, cudaMemcpyDeviceToDevice, ctx->stream));
  YL_CUDA(cudaMemcpyAsync(X + (size_t)c * plane, logvar, n, cudaMemcpyDeviceToDevice, ctx->stream));
  return YL_OK;
}

yl_status yl_randn(yl_ctx* ctx, float* out, uint32_t seed, size_t n) {
  YL_NN(ctx, out);
  legacy_randn_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(out, seed, (long long)n);
  return check_launch("legacy_randn_kernel");
}

static yl_status reduce_to_scalar(yl_ctx* ctx, const float* a, const float* b, size_t n, int mode,
                                  float* out) {
  const int nb = (int)grid_1d(n, 256, 1024);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, nb * sizeof(double), &ws));
  legacy_reduce_partial_kernel<<<nb, 256, 0, ctx->stream>>>(a, b, (long long)n, mode, (double*)ws);
  YL_TRY(check_launch("legacy_reduce_partial_kernel"));
  legacy_reduce_final_kernel<<<1, 32, 0, ctx->stream>>>((double*)ws, nb, out);
  return check_launch("legacy_reduce_final_kernel");
}

yl_status yl_mse_sum(yl_ctx* ctx, const float* recon, const float* target, size_t n,
                     float* out_dev) {
  YL_NN(ctx, recon, target, out_dev);
  return reduce_to_scalar(ctx, recon, target, n, 0, out_dev);
}

yl_status yl_kl_sum(yl_ctx* ctx, const float* mu, const float* logvar, size_t n, float* out_dev) {
  YL_NN(ctx, mu, logvar, out_dev);
  return reduce_to_scalar(ctx, mu, logvar, n, 1, out_dev);
}

yl_status yl_l1_grad(yl_ctx* ctx, const float* recon, const float* target, float* out, size_t n) {
  YL_NN(ctx, recon, target, out);
  float inv = (float)(1.0 / (double)(n ? n : 1));
  legacy_l1grad_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(recon, target, out, inv,
                                                                (long long)n);
  return check_launch("legacy_l1grad_kernel");
}

yl_status yl_vae_grad(yl_ctx* ctx, const float* dz, const float* mu, const float* logvar,
                      const float* eps, float* dmu, float* dlogvar, float betaN, float betaHalfN,
                      size_t n) {
  YL_NN(ctx, dz, mu, logvar, eps, dmu, dlogvar);
  legacy_vae_grad_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(dz, mu, logvar, eps, dmu,
                                                                  dlogvar, betaN, betaHalfN,
                                                                  (long long)n);
  return check_launch("legacy_vae_grad_kernel");
}

yl_status yl_adam_update(yl_ctx* ctx, float* param, const float* grad, float* m, float* v, size_t n,
                         int t, float lr) {
  YL_NN(ctx, param, grad, m, v);
  if (t < 1) t = 1;  // GpuSessionOps.swift:246-248
  float c1 = 1.f - powf(0.9f, (float)t), c2 = 1.f - powf(0.999f, (float)t);
  legacy_adam_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(param, grad, m, v, (long long)n, lr,
                                                              c1, c2);
  return check_launch("legacy_adam_kernel");
}

}  // extern "C"
