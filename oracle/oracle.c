/*
 * oracle.c -- CPU restatement of YumeLayersCore's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA backend
 * (yumelayers_b200/csrc) and the timed CPU baseline; the product path never
 * links, loads or calls it.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py may use it.
 *
 * Every function below restates one piece of the reference and cites the
 * reference file:line it follows (paths are relative to the YumeLayers
 * project root).  The reference's GPU code is Metal Shading Language held in
 * Swift strings; the per-index loops below are the same arithmetic written in
 * C.  Layouts are the reference's: per-image CHW with rows = channels and
 * cols = H*W, conv weights (oc, ic*k*k), Linear weights (oc, ic).
 *
 * Parity pins: integer-pattern known-answer tests from the reference's own
 * tests (Tests/YumeLayersTests/TestGroup3.swift:345-536, TestGroup4.swift:
 * 116-221) are checked in tests/test_oracle.py; the ops that exist only in
 * the reference's PyTorch prototype (SiLU, affine GroupNorm, Conv2d,
 * timestep_embedding) are cross-checked against torch CPU there too.
 *
 * Build: see oracle/Makefile (gcc -O3 -march=native -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

ORC_API int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

ORC_API void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ======================================================================= */
/* 1. Reference kernels, restated per index (reference layout, fp32).       */
/* ======================================================================= */

/* matmul_kernel / matmul_tiled_kernel (MetalKernelSourcesA.swift:11-94):
 * C[r,c] = sum_k op(A)[r,k] * op(B)[k,c]; transA reads A[k*M+r], transB reads
 * B[c*K+k].  Accumulation order is k ascending, fp32, like the naive kernel. */
ORC_API void orc_matmul(const float* A, const float* B, float* C, int M, int N,
                        int K, int transA, int transB) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < M; ++r) {
    for (int c = 0; c < N; ++c) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) {
        float av = transA ? A[(size_t)k * M + r] : A[(size_t)r * K + k];
        float bv = transB ? B[(size_t)c * K + k] : B[(size_t)k * N + c];
        acc += av * bv;
      }
      C[(size_t)r * N + c] = acc;
    }
  }
}

/* Packed implicit-GEMM fp32 convolution core used by the conv composition
 * (orc_conv2d_fwd / orc_conv2d_bwd below), so that full-resolution layers
 * (480 x 856) check in seconds and the timed CPU baseline is a fair one.
 * It forms the same sums as im2col + matmul (forward), gradW (dW) and
 * col2im / convBackInputS1 (dX); only the association order differs.  The
 * per-index restatements above and below (orc_im2col, orc_matmul,
 * orc_col2im, orc_conv_back_input_s1, orc_gradw) stay the reference's kernels
 * one to one and pin this core in the tests.
 *
 * A tile is NB output pixels of one image: its im2col columns are gathered
 * into a K x NB panel T (K = channels * taps), then a 6 x 16 register-blocked
 * micro-kernel (twelve 8-wide fp32 accumulators, AVX2 FMA through GCC vector
 * extensions) multiplies the weight rows into it. */
typedef float v8f __attribute__((vector_size(32)));
enum { TILE_NB = 64, MK_M = 6, MK_N = 16 };

static inline v8f ld8(const float* p) { v8f v; memcpy(&v, p, sizeof v); return v; }
static inline void st8(float* p, v8f v) { memcpy(p, &v, sizeof v); }

/* acc[r][0..15] = sum_{i < len} A[r * lda + i] * B[i * ldb + 0..15] for r < mr
 * (rows >= mr read row 0 and are discarded by the caller). */
static inline void mk6x16(const float* A, long lda, int mr, const float* B, long ldb, int len,
                          float acc[MK_M][MK_N]) {
  const float* a[MK_M];
  for (int r = 0; r < MK_M; ++r) a[r] = A + (r < mr ? r : 0) * lda;
  v8f c00 = {0}, c01 = {0}, c10 = {0}, c11 = {0}, c20 = {0}, c21 = {0};
  v8f c30 = {0}, c31 = {0}, c40 = {0}, c41 = {0}, c50 = {0}, c51 = {0};
  for (int i = 0; i < len; ++i) {
    const v8f b0 = ld8(B + (long)i * ldb), b1 = ld8(B + (long)i * ldb + 8);
    v8f x;
    x = (v8f){0} + a[0][i]; c00 += x * b0; c01 += x * b1;
    x = (v8f){0} + a[1][i]; c10 += x * b0; c11 += x * b1;
    x = (v8f){0} + a[2][i]; c20 += x * b0; c21 += x * b1;
    x = (v8f){0} + a[3][i]; c30 += x * b0; c31 += x * b1;
    x = (v8f){0} + a[4][i]; c40 += x * b0; c41 += x * b1;
    x = (v8f){0} + a[5][i]; c50 += x * b0; c51 += x * b1;
  }
  st8(acc[0], c00); st8(acc[0] + 8, c01); st8(acc[1], c10); st8(acc[1] + 8, c11);
  st8(acc[2], c20); st8(acc[2] + 8, c21); st8(acc[3], c30); st8(acc[3] + 8, c31);
  st8(acc[4], c40); st8(acc[4] + 8, c41); st8(acc[5], c50); st8(acc[5] + 8, c51);
}

/* Y[m * ldy + p] = sum_k A[m * lda + k] * T[k * ldt + p] for m < M, p < np;
 * T holds whole 16-column groups (ldt >= np rounded up to 16, padding zero). */
static void gemm_a_t(const float* A, int M, long lda, const float* T, int K, long ldt, int np,
                     float* Y, long ldy) {
  float acc[MK_M][MK_N];
  for (int m0 = 0; m0 < M; m0 += MK_M) {
    const int mr = M - m0 < MK_M ? M - m0 : MK_M;
    for (int p0 = 0; p0 < np; p0 += MK_N) {
      const int pr = np - p0 < MK_N ? np - p0 : MK_N;
      mk6x16(A + (long)m0 * lda, lda, mr, T + p0, ldt, K, acc);
      for (int r = 0; r < mr; ++r) memcpy(Y + (long)(m0 + r) * ldy + p0, acc[r], sizeof(float) * pr);
    }
  }
}

/* Geometry of one conv as the core sees it.  Forward / dW: output pixel
 * (oy, ox) of oh x ow reads tap (ky, kx) at (oy*s - pad + ky, ox*s - pad + kx)
 * of the ih x iw input, which with `up` is the nearest-x2 view of the stored
 * h x w tensor.  Transposed (dX): output pixel (iy, ix) of ih x iw gathers
 * dy[(iy + pad - ky) / s][(ix + pad - kx) / s] when the division is exact. */
typedef struct {
  int C, h, w, ih, iw, k, s, pad, up, oh, ow;
} ConvGeom;

/* im2col columns of pixels [p0, p0 + np) (forward pixel order): T[c*k*k + t][j]. */
static void pack_fwd(const float* x, const ConvGeom* g, long p0, int np, float* T, int ldt) {
  const int kk = g->k * g->k;
  for (int c = 0; c < g->C; ++c) {
    const float* xc = x + (size_t)c * g->h * g->w;
    for (int t = 0; t < kk; ++t) {
      const int ky = t / g->k, kx = t % g->k;
      float* row = T + (size_t)(c * kk + t) * ldt;
      int oy = (int)(p0 / g->ow), ox = (int)(p0 % g->ow);
      for (int j = 0; j < np; ++j) {
        const int iy = oy * g->s - g->pad + ky, ix = ox * g->s - g->pad + kx;
        float v = 0.0f;
        if (iy >= 0 && iy < g->ih && ix >= 0 && ix < g->iw)
          v = g->up ? xc[(size_t)(iy >> 1) * g->w + (ix >> 1)] : xc[(size_t)iy * g->w + ix];
        row[j] = v;
        if (++ox == g->ow) { ox = 0; ++oy; }
      }
      for (int j = np; j < ldt; ++j) row[j] = 0.0f;
    }
  }
}

/* Transposed columns of input-space pixels [p0, p0 + np) of ih x iw:
 * T[o*k*k + t][j] = dy[o][oy][ox] (the col2im gather, MetalKernelSourcesB.swift:28-58). */
static void pack_tr(const float* dy, int OC, const ConvGeom* g, long p0, int np, float* T,
                    int ldt) {
  const int kk = g->k * g->k;
  for (int o = 0; o < OC; ++o) {
    const float* dyo = dy + (size_t)o * g->oh * g->ow;
    for (int t = 0; t < kk; ++t) {
      const int ky = t / g->k, kx = t % g->k;
      float* row = T + (size_t)(o * kk + t) * ldt;
      int y = (int)(p0 / g->iw), x = (int)(p0 % g->iw);
      for (int j = 0; j < np; ++j) {
        const int sy = y + g->pad - ky, sx = x + g->pad - kx;
        float v = 0.0f;
        if (sy >= 0 && sx >= 0 && sy % g->s == 0 && sx % g->s == 0) {
          const int oy = sy / g->s, ox = sx / g->s;
          if (oy < g->oh && ox < g->ow) v = dyo[(size_t)oy * g->ow + ox];
        }
        row[j] = v;
        if (++x == g->iw) { x = 0; ++y; }
      }
      for (int j = np; j < ldt; ++j) row[j] = 0.0f;
    }
  }
}

/* y (N, OC, oh, ow) = W (OC, C*k*k) * im2col(x) per image. */
static void conv_core_fwd(const float* x, int N, const ConvGeom* g, const float* w, int OC,
                          float* y) {
  const int K = g->C * g->k * g->k;
  const long P = (long)g->oh * g->ow, tiles = (P + TILE_NB - 1) / TILE_NB;
#pragma omp parallel
  {
    float* T = (float*)malloc(sizeof(float) * (size_t)K * TILE_NB);
#pragma omp for schedule(dynamic, 4)
    for (long it = 0; it < (long)N * tiles; ++it) {
      const int n = (int)(it / tiles);
      const long p0 = (it % tiles) * TILE_NB;
      const int np = (int)(P - p0 < TILE_NB ? P - p0 : TILE_NB);
      pack_fwd(x + (size_t)n * g->C * g->h * g->w, g, p0, np, T, TILE_NB);
      gemm_a_t(w, OC, K, T, K, TILE_NB, np, y + (size_t)n * OC * P + p0, P);
    }
    free(T);
  }
}

/* dx (N, C, ih, iw) = col2im(W^T dy) per image: Wt[c][o*k*k + t] = W[o][c*k*k + t]. */
static void conv_core_dgrad(const float* dy, int N, const ConvGeom* g, const float* w, int OC,
                            float* dx) {
  const int kk = g->k * g->k, K = OC * kk;
  float* wt = (float*)malloc(sizeof(float) * (size_t)g->C * K);
  for (int o = 0; o < OC; ++o)
    for (int c = 0; c < g->C; ++c)
      for (int t = 0; t < kk; ++t)
        wt[(size_t)c * K + o * kk + t] = w[(size_t)o * g->C * kk + c * kk + t];
  const long P = (long)g->ih * g->iw, tiles = (P + TILE_NB - 1) / TILE_NB;
#pragma omp parallel
  {
    float* T = (float*)malloc(sizeof(float) * (size_t)K * TILE_NB);
#pragma omp for schedule(dynamic, 4)
    for (long it = 0; it < (long)N * tiles; ++it) {
      const int n = (int)(it / tiles);
      const long p0 = (it % tiles) * TILE_NB;
      const int np = (int)(P - p0 < TILE_NB ? P - p0 : TILE_NB);
      pack_tr(dy + (size_t)n * OC * g->oh * g->ow, OC, g, p0, np, T, TILE_NB);
      gemm_a_t(wt, g->C, K, T, K, TILE_NB, np, dx + (size_t)n * g->C * P + p0, P);
    }
    free(T);
  }
  free(wt);
}

/* dw (OC, C*k*k) = sum over images and pixels of dy x im2col(x) (gradW,
 * MetalKernelSourcesA.swift:122-137, summed over the batch).  Each thread
 * sums its pixel tiles into a private [K][OC] buffer; the buffers are added
 * in thread order, so a fixed thread count gives a fixed result. */
static void conv_core_wgrad(const float* x, const float* dy, int N, const ConvGeom* g, int OC,
                            float* dw) {
  const int K = g->C * g->k * g->k;
  const int ocp = (OC + MK_N - 1) / MK_N * MK_N;
  const long P = (long)g->oh * g->ow, tiles = (P + TILE_NB - 1) / TILE_NB;
  const int nth = orc_num_threads();
  float* priv = (float*)calloc((size_t)nth * K * ocp, sizeof(float));
#pragma omp parallel num_threads(nth)
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    float* mine = priv + (size_t)tid * K * ocp;
    float* T = (float*)malloc(sizeof(float) * (size_t)K * TILE_NB);
    float* dyt = (float*)malloc(sizeof(float) * (size_t)TILE_NB * ocp);
    float acc[MK_M][MK_N];
#pragma omp for schedule(static)
    for (long it = 0; it < (long)N * tiles; ++it) {
      const int n = (int)(it / tiles);
      const long p0 = (it % tiles) * TILE_NB;
      const int np = (int)(P - p0 < TILE_NB ? P - p0 : TILE_NB);
      pack_fwd(x + (size_t)n * g->C * g->h * g->w, g, p0, np, T, TILE_NB);
      const float* dyn = dy + (size_t)n * OC * P + p0;
      for (int j = 0; j < np; ++j)
        for (int o = 0; o < ocp; ++o) dyt[(size_t)j * ocp + o] = o < OC ? dyn[(size_t)o * P + j] : 0.0f;
      for (int k0 = 0; k0 < K; k0 += MK_M) {
        const int mr = K - k0 < MK_M ? K - k0 : MK_M;
        for (int o0 = 0; o0 < ocp; o0 += MK_N) {
          mk6x16(T + (size_t)k0 * TILE_NB, TILE_NB, mr, dyt + o0, ocp, np, acc);
          for (int r = 0; r < mr; ++r) {
            float* d = mine + (size_t)(k0 + r) * ocp + o0;
            for (int q = 0; q < MK_N; ++q) d[q] += acc[r][q];
          }
        }
      }
    }
    free(T);
    free(dyt);
  }
#pragma omp parallel for schedule(static)
  for (int o = 0; o < OC; ++o)
    for (int kx = 0; kx < K; ++kx) {
      float s = 0.0f;
      for (int t = 0; t < nth; ++t) s += priv[((size_t)t * K + kx) * ocp + o];
      dw[(size_t)o * K + kx] += s;
    }
  free(priv);
}

/* im2col3d_kernel (MetalKernelSourcesA.swift:325-352): X (ic, ih, iw) ->
 * C (ic*kh*kw, oh*ow); out-of-range taps read 0. */
ORC_API void orc_im2col(const float* X, float* C, int ic, int ih, int iw, int kh,
                        int kw, int stride, int pad) {
  int oh = (ih + 2 * pad - kh) / stride + 1;
  int ow = (iw + 2 * pad - kw) / stride + 1;
  int rows = ic * kh * kw;
#pragma omp parallel for schedule(static)
  for (int col = 0; col < rows; ++col) {
    int c = col / (kh * kw), r = col % (kh * kw);
    int ky = r / kw, kx = r % kw;
    for (int oy = 0; oy < oh; ++oy)
      for (int ox = 0; ox < ow; ++ox) {
        int iy = oy * stride + ky - pad, ix = ox * stride + kx - pad;
        float v = 0.0f;
        if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) v = X[((size_t)c * ih + iy) * iw + ix];
        C[(size_t)col * (oh * ow) + oy * ow + ox] = v;
      }
  }
}

/* col2im3d_kernel (MetalKernelSourcesB.swift:28-58): gather of dcols back to
 * (ic, ih, iw) for any stride; col2im3d_s1_kernel (B:60-85) is its stride-1
 * special case and gives the same sums. */
ORC_API void orc_col2im(const float* C, float* G, int ic, int ih, int iw, int kh,
                        int kw, int stride, int pad, int oh, int ow) {
#pragma omp parallel for schedule(static)
  for (int c = 0; c < ic; ++c)
    for (int y = 0; y < ih; ++y)
      for (int x = 0; x < iw; ++x) {
        float acc = 0.0f;
        for (int ky = 0; ky < kh; ++ky) {
          int sy = y + pad - ky;
          if (sy < 0 || sy % stride != 0) continue;
          int oy = sy / stride;
          if (oy >= oh) continue;
          for (int kx = 0; kx < kw; ++kx) {
            int sx = x + pad - kx;
            if (sx < 0 || sx % stride != 0) continue;
            int ox = sx / stride;
            if (ox >= ow) continue;
            acc += C[((size_t)c * kh * kw + ky * kw + kx) * (oh * ow) + oy * ow + ox];
          }
        }
        G[((size_t)c * ih + y) * iw + x] = acc;
      }
}

/* conv_back_input_s1_kernel (MetalKernelSourcesB.swift:125-159), including the
 * output-size fix at B:139-143 (bounds on the conv OUTPUT oh/ow). */
ORC_API void orc_conv_back_input_s1(const float* dOut, const float* W, float* dx,
                                    int ic, int oc, int ih, int iw, int kh, int kw,
                                    int pad) {
  int oh = ih + 2 * pad - kh + 1;
  int ow = iw + 2 * pad - kw + 1;
#pragma omp parallel for schedule(static)
  for (int c = 0; c < ic; ++c)
    for (int y = 0; y < ih; ++y)
      for (int x = 0; x < iw; ++x) {
        float acc = 0.0f;
        for (int o = 0; o < oc; ++o) {
          size_t woff = (size_t)o * (ic * kh * kw) + (size_t)c * (kh * kw);
          for (int ky = 0; ky < kh; ++ky) {
            int oy = y + pad - ky;
            if (oy < 0 || oy >= oh) continue;
            for (int kx = 0; kx < kw; ++kx) {
              int ox = x + pad - kx;
              if (ox < 0 || ox >= ow) continue;
              acc += dOut[(size_t)o * (oh * ow) + oy * ow + ox] * W[woff + ky * kw + kx];
            }
          }
        }
        dx[((size_t)c * ih + y) * iw + x] = acc;
      }
}

/* gradw_plain_kernel (MetalKernelSourcesA.swift:122-137):
 * C[r,c] = sum_i A[r*K+i] * B[c*K+i]. */
ORC_API void orc_gradw(const float* A, const float* B, float* C, int oc, int kk, int K) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < oc; ++r)
    for (int c = 0; c < kk; ++c) {
      float acc = 0.0f;
      for (int i = 0; i < K; ++i) acc += A[(size_t)r * K + i] * B[(size_t)c * K + i];
      C[(size_t)r * kk + c] = acc;
    }
}

/* biasrow3d_kernel (MetalKernelSourcesB.swift:112-121): C[r,c] = A[r,c] + b[r]. */
ORC_API void orc_bias_row(const float* A, const float* b, float* C, int rows, int cols) {
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) C[(size_t)r * cols + c] = A[(size_t)r * cols + c] + b[r];
}

/* biasrowgrad_kernel (MetalKernelSourcesB.swift:162-171): out[r] = sum_c G[r,c]. */
ORC_API void orc_bias_row_grad(const float* G, float* out, int rows, int cols) {
  for (int r = 0; r < rows; ++r) {
    float s = 0.0f;
    for (int c = 0; c < cols; ++c) s += G[(size_t)r * cols + c];
    out[r] = s;
  }
}

/* addbias_kernel (MetalKernelSourcesA.swift:179-187): C[i] = A[i] + bias[i % cols]. */
ORC_API void orc_add_bias(const float* A, const float* bias, float* C, int n, int cols) {
  for (int i = 0; i < n; ++i) C[i] = A[i] + bias[i % cols];
}

/* sumcols_kernel (MetalKernelSourcesA.swift:253-269): C[j] = sum_i A[i*cols+j]. */
ORC_API void orc_sum_cols(const float* A, float* C, int rows, int cols) {
  for (int j = 0; j < cols; ++j) {
    float s = 0.0f;
    for (int i = 0; i < rows; ++i) s += A[(size_t)i * cols + j];
    C[j] = s;
  }
}

/* upsample3d_kernel (MetalKernelSourcesB.swift:87-97): (c,h,w) -> (c,2h,2w). */
ORC_API void orc_upsample2x(const float* X, float* Y, int c, int h, int w) {
  int w2 = 2 * w;
  for (int ch = 0; ch < c; ++ch)
    for (int y = 0; y < 2 * h; ++y)
      for (int x = 0; x < w2; ++x)
        Y[((size_t)ch * h * 2 + y) * w2 + x] = X[((size_t)ch * h + y / 2) * w + x / 2];
}

/* downsample3d_kernel (MetalKernelSourcesB.swift:99-110): 2x2 sum. */
ORC_API void orc_downsample2x(const float* X, float* Y, int c, int h, int w) {
  int w2 = 2 * w;
  for (int ch = 0; ch < c; ++ch)
    for (int y = 0; y < h; ++y)
      for (int x = 0; x < w; ++x) {
        size_t base = ((size_t)ch * h * 2 + y * 2) * w2 + x * 2;
        Y[((size_t)ch * h + y) * w + x] = X[base] + X[base + 1] + X[base + w2] + X[base + w2 + 1];
      }
}

/* groupNormCPU (LossFunctions.swift:97-126), the CPU source of truth for
 * groupnorm_kernel (MetalKernelSourcesC.swift:10-46): affine-free, var clamped
 * at >= 1e-5, no eps; double accumulation. */
ORC_API void orc_groupnorm_ref(const float* xs, float* out, int channels, int groups,
                               int plane) {
  int gsize = channels / groups;
  double count = (double)gsize * plane;
  for (int g = 0; g < groups; ++g) {
    int c0 = g * gsize;
    double sum = 0, sq = 0;
    for (int c = c0; c < c0 + gsize; ++c)
      for (int p = 0; p < plane; ++p) {
        double v = xs[(size_t)c * plane + p];
        sum += v; sq += v * v;
      }
    double mean = sum / count;
    double var = sq / count - mean * mean;
    if (var < 1e-5) var = 1e-5;
    double inv = 1.0 / sqrt(var);
    for (int c = c0; c < c0 + gsize; ++c)
      for (int p = 0; p < plane; ++p) {
        size_t idx = (size_t)c * plane + p;
        out[idx] = (float)((xs[idx] - mean) * inv);
      }
  }
}

/* groupNormGradCPU (LossFunctions.swift:132-176), source of truth for
 * groupnorm_grad_kernel (MetalKernelSourcesC.swift:51-101). */
ORC_API void orc_groupnorm_grad_ref(const float* xs, const float* dys, float* out,
                                    int channels, int groups, int plane) {
  int gsize = channels / groups;
  double n = (double)gsize * plane;
  for (int g = 0; g < groups; ++g) {
    int c0 = g * gsize;
    double sum = 0, sq = 0;
    for (int c = c0; c < c0 + gsize; ++c)
      for (int p = 0; p < plane; ++p) {
        double v = xs[(size_t)c * plane + p];
        sum += v; sq += v * v;
      }
    double mean = sum / n;
    double var = sq / n - mean * mean;
    if (var < 1e-5) var = 1e-5;
    double inv = 1.0 / sqrt(var);
    double sdy = 0, sdyxm = 0;
    for (int c = c0; c < c0 + gsize; ++c)
      for (int p = 0; p < plane; ++p) {
        size_t idx = (size_t)c * plane + p;
        sdy += dys[idx];
        sdyxm += dys[idx] * (xs[idx] - mean);
      }
    double mdy = sdy / n, mdyxm = sdyxm / n;
    for (int c = c0; c < c0 + gsize; ++c)
      for (int p = 0; p < plane; ++p) {
        size_t idx = (size_t)c * plane + p;
        double xm = xs[idx] - mean;
        out[idx] = (float)(inv * (dys[idx] - mdy - xm * mdyxm / var));
      }
  }
}

/* Elementwise kernels.  op codes follow the reference kernel list:
 *  0 relu (B:191-197)        1 sigmoid (B:208-214)    2 tanh (A:236-242)
 *  3 tanhgrad (A:244-251)    4 exp (B:273-279)        5 exphalf (B:293-299)
 *  6 silu (src/vae.py:11, torch nn.SiLU)                                    */
ORC_API void orc_unary(int op, const float* A, float* C, int n) {
  for (int i = 0; i < n; ++i) {
    float a = A[i];
    switch (op) {
      case 0: C[i] = a > 0.0f ? a : 0.0f; break;
      case 1: C[i] = 1.0f / (1.0f + expf(-a)); break;
      case 2: C[i] = tanhf(a); break;
      case 3: { float t = tanhf(a); C[i] = 1.0f - t * t; } break;
      case 4: C[i] = expf(a); break;
      case 5: { float l = a < -10.0f ? -10.0f : (a > 10.0f ? 10.0f : a); C[i] = expf(0.5f * l); } break;
      case 6: C[i] = a / (1.0f + expf(-a)); break;
      default: C[i] = a;
    }
  }
}

/* Binary kernels:
 *  0 add (A:171-177)   1 sub (A:198-205)   2 mul (A:189-196)
 *  3 relugrad: Y>0 ? G : 0 (B:199-206)     4 sigmoidgrad: G*s*(1-s) (B:216-224)
 *  5 silugrad: G * s*(1 + z*(1-s)), s = sigmoid(z)                           */
ORC_API void orc_binary(int op, const float* A, const float* B, float* C, int n) {
  for (int i = 0; i < n; ++i) {
    float a = A[i], b = B[i];
    switch (op) {
      case 0: C[i] = a + b; break;
      case 1: C[i] = a - b; break;
      case 2: C[i] = a * b; break;
      case 3: C[i] = a > 0.0f ? b : 0.0f; break;
      case 4: { float s = 1.0f / (1.0f + expf(-a)); C[i] = b * s * (1.0f - s); } break;
      case 5: { float s = 1.0f / (1.0f + expf(-a)); C[i] = b * s * (1.0f + a * (1.0f - s)); } break;
      default: C[i] = a;
    }
  }
}

/* smul_kernel (A:207-214), addconst_kernel (B:281-289), fma_kernel (B:263-271). */
ORC_API void orc_smul(const float* A, float* C, float s, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] * s; }
ORC_API void orc_addconst(const float* A, float* C, float s, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] + s; }
ORC_API void orc_fma(const float* A, const float* B, const float* D, float* C, int n) {
  for (int i = 0; i < n; ++i) C[i] = A[i] + B[i] * D[i];
}

/* mse_reduce_kernel (B:236-258): sum of squared differences (double here, as
 * the reference's test compares it with a Double CPU sum, TestGroup2.swift:115-145). */
ORC_API double orc_mse_sum(const float* r, const float* t, int n) {
  double s = 0;
  for (int i = 0; i < n; ++i) { double d = (double)r[i] - t[i]; s += d * d; }
  return s;
}

/* kl_reduce_kernel (B:334-357): 0.5 * sum(mu^2 + exp(lv) - 1 - lv), lv clamped. */
ORC_API double orc_kl_sum(const float* mu, const float* lv, int n) {
  double s = 0;
  for (int i = 0; i < n; ++i) {
    float l = lv[i] < -10.0f ? -10.0f : (lv[i] > 10.0f ? 10.0f : lv[i]);
    s += 0.5 * ((double)mu[i] * mu[i] + exp((double)l) - 1.0 - l);
  }
  return s;
}

/* l1grad_kernel (B:453-461): sign(recon - target) * invN. */
ORC_API void orc_l1grad(const float* r, const float* t, float* out, float invN, int n) {
  for (int i = 0; i < n; ++i) {
    float d = r[i] - t[i];
    out[i] = (d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f)) * invN;
  }
}

/* vae_grad_kernel (B:365-380). */
ORC_API void orc_vae_grad(const float* dz, const float* mu, const float* lv,
                          const float* eps, float* dmu, float* dlv, float betaN,
                          float betaHalfN, int n) {
  for (int i = 0; i < n; ++i) {
    float l = lv[i] < -10.0f ? -10.0f : (lv[i] > 10.0f ? 10.0f : lv[i]);
    dmu[i] = dz[i] + betaN * mu[i];
    dlv[i] = dz[i] * eps[i] * 0.5f * expf(0.5f * l) + betaHalfN * (expf(l) - 1.0f);
  }
}

/* split2_kernel / merge2_kernel (B:302-331). */
ORC_API void orc_split2(const float* X, float* A, float* B, int c, int plane) {
  memcpy(A, X, sizeof(float) * (size_t)c * plane);
  memcpy(B, X + (size_t)c * plane, sizeof(float) * (size_t)c * plane);
}
ORC_API void orc_merge2(const float* A, const float* B, float* X, int c, int plane) {
  memcpy(X, A, sizeof(float) * (size_t)c * plane);
  memcpy(X + (size_t)c * plane, B, sizeof(float) * (size_t)c * plane);
}

/* yume_hash + randn_kernel (MetalKernelSourcesB.swift:385-402): counter-based
 * Box-Muller keyed by (seed, index); uint32 wrap-around arithmetic. */
static inline uint32_t yume_hash(uint32_t x) {
  x = ((x >> ((x >> 28u) + 4u)) ^ x) * 277803737u;
  return (x >> 22u) ^ x;
}
ORC_API void orc_randn(float* out, uint32_t seed, int n) {
  for (int i = 0; i < n; ++i) {
    uint32_t g = (uint32_t)i;
    uint32_t h1 = yume_hash(g * 747796405u + seed * 2891336453u + 1u);
    uint32_t h2 = yume_hash(g * 2654435761u + seed * 1013904223u + 0x9E3779B9u);
    float u1 = (float)(h1 >> 8) / 16777216.0f;
    if (u1 < 1e-7f) u1 = 1e-7f;
    float u2 = (float)(h2 >> 8) / 16777216.0f;
    out[i] = sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
  }
}
ORC_API uint32_t orc_yume_hash(uint32_t x) { return yume_hash(x); }

/* SplitMix64 (ConvVAEHelpers.swift:10-20). */
ORC_API uint64_t orc_splitmix64_next(uint64_t* state) {
  *state += 0x9E3779B97F4A7C15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* trainingNoiseSeed (ConvVAEHelpers.swift:33-37). */
ORC_API uint32_t orc_training_noise_seed(int64_t step, int64_t batch_index) {
  uint64_t a = (uint64_t)step * 0x9E3779B97F4A7C15ull;
  uint64_t b = (uint64_t)batch_index * 0xC2B2AE3D27D4EB4Full;
  return (uint32_t)((a ^ (b + 0x165667B19E3779F9ull)) >> 32);
}

/* adam_kernel (MetalKernelSourcesA.swift:271-287), t clamped to >= 1 as the
 * caller does (GpuSessionOps.swift:246-248).  b1/b2/eps are parameters here
 * (the reference hard-codes 0.9/0.999/1e-8, the defaults of the tests). */
ORC_API void orc_adam(float* p, const float* g, float* m, float* v, int n, int t,
                      float lr, float b1, float b2, float eps) {
  if (t < 1) t = 1;
  float c1 = 1.0f - powf(b1, (float)t), c2 = 1.0f - powf(b2, (float)t);
  for (int i = 0; i < n; ++i) {
    float gi = g[i];
    m[i] = b1 * m[i] + (1.0f - b1) * gi;
    v[i] = b2 * v[i] + (1.0f - b2) * gi * gi;
    float mh = m[i] / c1, vh = v[i] / c2;
    p[i] -= lr * mh / (sqrtf(vh) + eps);
  }
}

/* sanitizeGrads (GradSanitize.swift:18-101) on one flat buffer holding all
 * gradients: g *= preScale; NaN/Inf -> 0 (not counted in the norm); if the
 * global L2 norm exceeds maxNorm, scale everything by maxNorm/norm.  Returns
 * the pre-clip norm; *fixed receives the number of non-finite values. */
ORC_API float orc_sanitize_grads(float* g, long n, float maxNorm, float preScale, long* fixed) {
  float total = 0.0f;
  long nf = 0;
  for (long i = 0; i < n; ++i) {
    float v = g[i];
    if (preScale != 1.0f) v *= preScale;
    if (isnan(v) || isinf(v)) { v = 0.0f; nf++; } else total += v * v;
    g[i] = v;
  }
  float norm = sqrtf(total);
  if (norm > maxNorm) {
    float s = maxNorm / norm;
    for (long i = 0; i < n; ++i) g[i] *= s;
  }
  if (fixed) *fixed = nf;
  return norm;
}

/* motionTimeEmbedding (MotionPlanner.swift:155-165): t clamped to [0,1]
 * (non-finite -> 0); emb[i] = sin(t * 1000^(i/d)), emb[i+1] = cos(...) for
 * even i; computed in double, stored as float. */
ORC_API void orc_motion_time_embedding(double t, int dim, float* out) {
  double tt = isfinite(t) ? t : 0.0;
  if (tt < 0) tt = 0;
  if (tt > 1) tt = 1;
  for (int i = 0; i < dim; i += 2) {
    double w = pow(1000.0, (double)i / (double)dim);
    out[i] = (float)sin(tt * w);
    out[i + 1] = (float)cos(tt * w);
  }
}

/* timeEmbedding (DenoiserMLP.swift:7-17): integer t, base 10000, interleaved. */
ORC_API void orc_time_embedding_int(int t, int dim, float* out) {
  for (int i = 0; i < dim; i += 2) {
    double w = pow(10000.0, (double)i / (double)dim);
    out[i] = (float)sin((double)t / w);
    out[i + 1] = (float)cos((double)t / w);
  }
}

/* timestep_embedding (src/diffusion.py:6-10): [cos | sin] halves with
 * freqs = exp(-ln(max_period) * j / half), fp32 like the torch prototype. */
ORC_API void orc_timestep_embedding_torch(const float* t, int n, int dim, float max_period,
                                          float* out) {
  int half = dim / 2;
  for (int b = 0; b < n; ++b)
    for (int j = 0; j < half; ++j) {
      float f = expf(-logf(max_period) * (float)j / (float)half);
      float a = t[b] * f;
      out[(size_t)b * dim + j] = cosf(a);
      out[(size_t)b * dim + half + j] = sinf(a);
    }
}

/* ======================================================================= */
/* 2. Batched layer math (NCHW = per-image CHW stacked), composed from the  */
/*    reference kernels the way the reference's layers compose them.       */
/* ======================================================================= */

/* ConvLayerGPU.forward (ConvGPU.swift:57-64): per image, cols = im2col(x),
 * y = W * cols + b (biasRow).  Optional nearest-x2 upsample of the input
 * (the decoder's "up + conv", ConvGPU.swift:393 / Ops:336), cropped to
 * (ih, iw) when the upsampled size is odd-cropped; optional residual add and
 * per-(image, channel) bias (time-embedding projection).  The im2col + matmul
 * runs through the packed core above (same sums, tiled). */
ORC_API void orc_conv2d_fwd(const float* x, int N, int C, int H, int W,
                            const float* w, const float* b, int OC, int k, int stride,
                            int pad, int up, int Hin, int Win, const float* bias2d,
                            const float* residual, float* y) {
  /* up: x has spatial (Hs, Ws) = ceil(Hin/2), ceil(Win/2) and is viewed as the
   * (Hin, Win) nearest upsample; else (H, W) = (Hin, Win). */
  ConvGeom g;
  g.C = C; g.h = H; g.w = W; g.k = k; g.s = stride; g.pad = pad; g.up = up;
  g.ih = up ? Hin : H;
  g.iw = up ? Win : W;
  g.oh = (g.ih + 2 * pad - k) / stride + 1;
  g.ow = (g.iw + 2 * pad - k) / stride + 1;
  const size_t plane_out = (size_t)g.oh * g.ow;
  conv_core_fwd(x, N, &g, w, OC, y);
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; ++n)
    for (int o = 0; o < OC; ++o) {
      float bb = (b ? b[o] : 0.0f) + (bias2d ? bias2d[(size_t)n * OC + o] : 0.0f);
      float* row = y + ((size_t)n * OC + o) * plane_out;
      const float* res = residual ? residual + ((size_t)n * OC + o) * plane_out : NULL;
      for (size_t p = 0; p < plane_out; ++p) row[p] = row[p] + bb + (res ? res[p] : 0.0f);
    }
}

/* ConvLayerGPU.backward (ConvGPU.swift:66-81) summed over the batch the way
 * TrainContext.forwardBackward accumulates per-frame grads
 * (TrainConvVAE.swift:168-219): dW += gradW(dOut, cols), db += biasRowGrad,
 * dx = convBackInputS1 (stride 1) or col2im(W^T dOut) (stride 2) -- one
 * gather formula, MetalKernelSourcesB.swift:28-58 / 125-159.  With `up`, dx
 * is the downsample2x (2x2 sum, Ops:379) of the upsampled-input gradient,
 * restricted to the cropped size.  Any of dx/dw/db may be NULL.  dw and db
 * are overwritten; dbias2d (N, OC) receives per-image channel sums. */
ORC_API void orc_conv2d_bwd(const float* x, int N, int C, int H, int W,
                            const float* w, int OC, int k, int stride, int pad, int up,
                            int Hin, int Win, const float* dy, float* dx, float* dw,
                            float* db, float* dbias2d) {
  ConvGeom g;
  g.C = C; g.h = H; g.w = W; g.k = k; g.s = stride; g.pad = pad; g.up = up;
  g.ih = up ? Hin : H;
  g.iw = up ? Win : W;
  g.oh = (g.ih + 2 * pad - k) / stride + 1;
  g.ow = (g.iw + 2 * pad - k) / stride + 1;
  const size_t plane_in = (size_t)g.ih * g.iw, plane_out = (size_t)g.oh * g.ow;
  if (dw) {
    memset(dw, 0, sizeof(float) * (size_t)OC * C * k * k);
    conv_core_wgrad(x, dy, N, &g, OC, dw);
  }
  if (db) memset(db, 0, sizeof(float) * OC);
  if (db || dbias2d) {
    for (int n = 0; n < N; ++n) {
      const float* dyn = dy + (size_t)n * OC * plane_out;
      for (int o = 0; o < OC; ++o) {
        double s = 0;
        for (size_t p = 0; p < plane_out; ++p) s += dyn[(size_t)o * plane_out + p];
        if (db) db[o] += (float)s;
        if (dbias2d) dbias2d[(size_t)n * OC + o] = (float)s;
      }
    }
  }
  if (dx) {
    if (!up) {
      conv_core_dgrad(dy, N, &g, w, OC, dx);
    } else {
      float* dxin = (float*)malloc(sizeof(float) * (size_t)N * C * plane_in);
      conv_core_dgrad(dy, N, &g, w, OC, dxin);
#pragma omp parallel for collapse(2) schedule(static)
      for (int n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c) {
          float* dxc = dx + ((size_t)n * C + c) * H * W;
          const float* src = dxin + ((size_t)n * C + c) * plane_in;
          memset(dxc, 0, sizeof(float) * H * W);
          for (int yy = 0; yy < g.ih; ++yy)
            for (int xx = 0; xx < g.iw; ++xx)
              dxc[(size_t)(yy / 2) * W + xx / 2] += src[(size_t)yy * g.iw + xx];
        }
      free(dxin);
    }
  }
}

/* GroupNorm with affine gamma/beta and eps (torch.nn.GroupNorm semantics, the
 * workload op; affine-free clamp variant is orc_groupnorm_ref above), followed
 * by SiLU when silu != 0.  Per image; double statistics like groupNormCPU
 * (LossFunctions.swift:97-126).  mean/rstd (N*G) are optional outputs. */
ORC_API void orc_gn_silu_fwd(const float* x, int N, int C, int HW, int G, float eps,
                             const float* gamma, const float* beta, int silu, float* y,
                             float* mean_out, float* rstd_out) {
  int cg = C / G;
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; ++n)
    for (int g = 0; g < G; ++g) {
      const float* xn = x + (size_t)n * C * HW;
      double s = 0, q = 0, cnt = (double)cg * HW;
      for (int c = g * cg; c < (g + 1) * cg; ++c)
        for (int p = 0; p < HW; ++p) { double v = xn[(size_t)c * HW + p]; s += v; q += v * v; }
      double mean = s / cnt, var = q / cnt - mean * mean;
      if (var < 0) var = 0;
      double rstd = 1.0 / sqrt(var + eps);
      if (mean_out) mean_out[n * G + g] = (float)mean;
      if (rstd_out) rstd_out[n * G + g] = (float)rstd;
      for (int c = g * cg; c < (g + 1) * cg; ++c) {
        double ga = gamma ? gamma[c] : 1.0, be = beta ? beta[c] : 0.0;
        for (int p = 0; p < HW; ++p) {
          size_t idx = (size_t)n * C * HW + (size_t)c * HW + p;
          double a = (x[idx] - mean) * rstd * ga + be;
          if (silu) a = a / (1.0 + exp(-a));
          y[idx] = (float)a;
        }
      }
    }
}

/* Backward of orc_gn_silu_fwd.  dy is the gradient w.r.t. the SiLU output
 * (or the GN output when silu == 0).  dx = rstd*(dxh - mean(dxh) -
 * xh*mean(dxh*xh)) with dxh = da*gamma, the affine form of groupNormGradCPU
 * (LossFunctions.swift:132-176).  dgamma/dbeta are sums over (N, HW);
 * `addend` (optional) is added to dx (residual fan-in, Ops:453). */
ORC_API void orc_gn_silu_bwd(const float* x, const float* dy, int N, int C, int HW, int G,
                             float eps, const float* gamma, const float* beta, int silu,
                             const float* addend, float* dx, float* dgamma, float* dbeta) {
  int cg = C / G;
  double* dg = (double*)calloc((size_t)N * C, sizeof(double));
  double* dbt = (double*)calloc((size_t)N * C, sizeof(double));
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; ++n)
    for (int g = 0; g < G; ++g) {
      const float* xn = x + (size_t)n * C * HW;
      double s = 0, q = 0, cnt = (double)cg * HW;
      for (int c = g * cg; c < (g + 1) * cg; ++c)
        for (int p = 0; p < HW; ++p) { double v = xn[(size_t)c * HW + p]; s += v; q += v * v; }
      double mean = s / cnt, var = q / cnt - mean * mean;
      if (var < 0) var = 0;
      double rstd = 1.0 / sqrt(var + eps);
      double sd = 0, sdx = 0;
      for (int c = g * cg; c < (g + 1) * cg; ++c) {
        double ga = gamma ? gamma[c] : 1.0, be = beta ? beta[c] : 0.0;
        for (int p = 0; p < HW; ++p) {
          size_t idx = (size_t)n * C * HW + (size_t)c * HW + p;
          double xh = (x[idx] - mean) * rstd;
          double a = xh * ga + be, da = dy[idx];
          if (silu) { double sg = 1.0 / (1.0 + exp(-a)); da *= sg * (1.0 + a * (1.0 - sg)); }
          dg[(size_t)n * C + c] += da * xh;
          dbt[(size_t)n * C + c] += da;
          double dxh = da * ga;
          sd += dxh; sdx += dxh * xh;
        }
      }
      double md = sd / cnt, mdx = sdx / cnt;
      for (int c = g * cg; c < (g + 1) * cg; ++c) {
        double ga = gamma ? gamma[c] : 1.0, be = beta ? beta[c] : 0.0;
        for (int p = 0; p < HW; ++p) {
          size_t idx = (size_t)n * C * HW + (size_t)c * HW + p;
          double xh = (x[idx] - mean) * rstd;
          double a = xh * ga + be, da = dy[idx];
          if (silu) { double sg = 1.0 / (1.0 + exp(-a)); da *= sg * (1.0 + a * (1.0 - sg)); }
          double v = rstd * (da * ga - md - xh * mdx);
          if (addend) v += addend[idx];
          dx[idx] = (float)v;
        }
      }
    }
  for (int c = 0; c < C; ++c) {
    double a = 0, b = 0;
    for (int n = 0; n < N; ++n) { a += dg[(size_t)n * C + c]; b += dbt[(size_t)n * C + c]; }
    if (dgamma) dgamma[c] = (float)a;
    if (dbeta) dbeta[c] = (float)b;
  }
  free(dg);
  free(dbt);
}

/* LinearGPU.forward (DenoiserMLP.swift:51-54): Y = X * W^T + b, X (n, ic),
 * W (oc, ic); act 1 applies SiLU to the output. */
ORC_API void orc_linear_fwd(const float* X, const float* Wt, const float* b, float* Y, int n,
                            int ic, int oc, int act) {
  for (int r = 0; r < n; ++r)
    for (int o = 0; o < oc; ++o) {
      double s = b ? b[o] : 0.0;
      for (int i = 0; i < ic; ++i) s += (double)X[(size_t)r * ic + i] * Wt[(size_t)o * ic + i];
      float v = (float)s;
      if (act == 1) v = v / (1.0f + expf(-v));
      Y[(size_t)r * oc + o] = v;
    }
}

/* LinearGPU.backward (DenoiserMLP.swift:57-64): dX = dY * W, dW = dY^T * X,
 * db = sumCols(dY).  Any output may be NULL; dW/db are overwritten. */
ORC_API void orc_linear_bwd(const float* X, const float* Wt, const float* dY, float* dX,
                            float* dW, float* db, int n, int ic, int oc) {
  if (dX)
    for (int r = 0; r < n; ++r)
      for (int i = 0; i < ic; ++i) {
        double s = 0;
        for (int o = 0; o < oc; ++o) s += (double)dY[(size_t)r * oc + o] * Wt[(size_t)o * ic + i];
        dX[(size_t)r * ic + i] = (float)s;
      }
  if (dW)
    for (int o = 0; o < oc; ++o)
      for (int i = 0; i < ic; ++i) {
        double s = 0;
        for (int r = 0; r < n; ++r) s += (double)dY[(size_t)r * oc + o] * X[(size_t)r * ic + i];
        dW[(size_t)o * ic + i] = (float)s;
      }
  if (db)
    for (int o = 0; o < oc; ++o) {
      double s = 0;
      for (int r = 0; r < n; ++r) s += dY[(size_t)r * oc + o];
      db[o] = (float)s;
    }
}

/* VAE loss head (L1 reconstruction + beta * KL averaged per latent
 * element, the KL scaling of ConvVAEGPU.backward, ConvGPU.swift:435-438):
 * returns loss; writes dRecon = sign(r - t)/n_r (l1grad_kernel, B:453-461). */
ORC_API double orc_l1_kl_loss(const float* recon, const float* target, long nr,
                              const float* mu, const float* lv, long nl, float beta,
                              float* drecon) {
  double l1 = 0;
  float inv = (float)(1.0 / (double)nr);
  for (long i = 0; i < nr; ++i) {
    float d = recon[i] - target[i];
    l1 += fabs((double)d);
    if (drecon) drecon[i] = (d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f)) * inv;
  }
  double kl = orc_kl_sum(mu, lv, (int)nl);
  return l1 / (double)nr + (double)beta * kl / (double)nl;
}

/* ---- Sobel edge loss (LossFunctions.swift:29-66, 194-235), HWC images ---- */
static const double kSobelGx[9] = {-1, 0, 1, -2, 0, 2, -1, 0, 1};
static const double kSobelGy[9] = {-1, -2, -1, 0, 0, 0, 1, 2, 1};

static double orc_luma(const float* img, long i) {
  return 0.2126 * (double)img[i] + 0.7152 * (double)img[i + 1] + 0.0722 * (double)img[i + 2];
}

/* Sobel responses (sx, sy) of the luma at interior pixel (x, y). */
static void orc_sobel_at(const float* img, int w, int x, int y, double* sx, double* sy) {
  double ax = 0, ay = 0;
  int k = 0;
  for (int dy = -1; dy <= 1; ++dy)
    for (int dx = -1; dx <= 1; ++dx, ++k) {
      const double l = orc_luma(img, ((long)(y + dy) * w + (x + dx)) * 3);
      ax += kSobelGx[k] * l;
      ay += kSobelGy[k] * l;
    }
  *sx = ax;
  *sy = ay;
}

/* sobelLumaGradient: |grad luma| per pixel, border pixels 0. */
ORC_API void orc_sobel_luma(const float* img, int w, int h, float* out) {
  for (long i = 0; i < (long)w * h; ++i) out[i] = 0.f;
  for (int y = 1; y < h - 1; ++y)
    for (int x = 1; x < w - 1; ++x) {
      double sx, sy;
      orc_sobel_at(img, w, x, y, &sx, &sy);
      out[(long)y * w + x] = (float)sqrt(sx * sx + sy * sy);
    }
}

/* sobelEdgeLoss: mean over w*h of (|grad R| - |grad T|)^2 (the maps in float). */
ORC_API double orc_sobel_edge_loss(const float* recon, const float* target, int w, int h) {
  const long n = (long)w * h;
  float* er = (float*)malloc(n * sizeof(float));
  float* et = (float*)malloc(n * sizeof(float));
  orc_sobel_luma(recon, w, h, er);
  orc_sobel_luma(target, w, h, et);
  double s = 0;
  for (long i = 0; i < n; ++i) {
    const double d = (double)(er[i] - et[i]);
    s += d * d;
  }
  free(er);
  free(et);
  return s / (double)n;
}

/* sobelEdgeGradCPU: dLoss/drecon (HWC) with scale 2/(w*h), each interior
 * pixel q scattering its 3x3 window back onto the luma of the recon. */
ORC_API void orc_sobel_edge_grad(const float* recon, const float* target, int w, int h,
                                 float* grad) {
  const long n = (long)w * h;
  for (long i = 0; i < 3 * n; ++i) grad[i] = 0.f;
  const double scale = 2.0 / (double)n;
  for (int y = 1; y < h - 1; ++y)
    for (int x = 1; x < w - 1; ++x) {
      double sxr, syr, sxt, syt;
      orc_sobel_at(recon, w, x, y, &sxr, &syr);
      orc_sobel_at(target, w, x, y, &sxt, &syt);
      const double mr = sqrt(sxr * sxr + syr * syr), mt = sqrt(sxt * sxt + syt * syt);
      const double diff = mr - mt;
      if (diff == 0) continue;
      const double inv = mr > 1e-6 ? 1.0 / mr : 0.0;
      const double dX = diff * inv * scale * sxr, dY = diff * inv * scale * syr;
      int k = 0;
      for (int dy = -1; dy <= 1; ++dy)
        for (int dx = -1; dx <= 1; ++dx, ++k) {
          const double c = dX * kSobelGx[k] + dY * kSobelGy[k];
          const long li = ((long)(y + dy) * w + (x + dx)) * 3;
          grad[li] += (float)(c * 0.2126);
          grad[li + 1] += (float)(c * 0.7152);
          grad[li + 2] += (float)(c * 0.0722);
        }
    }
}

/* ---- Layered 8-channel loss (LayeredVAELoss.swift:95-196), CHW planes ----
 * recon / target: 8 planes of n pixels (bg RGB | obj RGB | mask | light);
 * comp: 3 planes (the composed frame). */

/* composeCHW (:95-110): clamp((bg*(1-m) + obj*m) * light, 0, 1), in float. */
ORC_API void orc_layered_compose(const float* recon, long long n, float* out) {
  for (long long i = 0; i < n; ++i) {
    const float m = recon[6 * n + i], l = recon[7 * n + i], im = 1.0f - m;
    for (int c = 0; c < 3; ++c) {
      const float v = (recon[c * n + i] * im + recon[(3 + c) * n + i] * m) * l;
      out[c * n + i] = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
    }
  }
}

/* layeredLoss (:129-149): wl * MSE over the 8 planes + wc * MSE of the composed
 * frame against comp, each mean over its own element count, sums in double. */
ORC_API double orc_layered_loss(const float* recon, const float* target, const float* comp,
                                long long n, float wl, float wc) {
  double layer = 0.0, compose = 0.0;
  for (long long i = 0; i < 8 * n; ++i) {
    const double d = (double)(recon[i] - target[i]);
    layer += d * d;
  }
  layer /= (double)(8 * n);
  float* y = (float*)malloc((size_t)(3 * n) * sizeof(float));
  orc_layered_compose(recon, n, y);
  for (long long i = 0; i < 3 * n; ++i) {
    const double d = (double)(y[i] - comp[i]);
    compose += d * d;
  }
  free(y);
  compose /= (double)(3 * n);
  return (double)wl * layer + (double)wc * compose;
}

/* layeredLossGradient (:158-196): dL/drecon for all 8 planes; the clamp passes
 * the gradient only strictly inside (0, 1); float composition, double chain. */
ORC_API void orc_layered_grad(const float* recon, const float* target, const float* comp,
                              long long n, float wl, float wc, float* g) {
  const double dl = 2.0 * (double)wl / (double)(8 * n);
  const double dc = 2.0 * (double)wc / (double)(3 * n);
  for (long long i = 0; i < n; ++i) {
    const float m = recon[6 * n + i], l = recon[7 * n + i], im = 1.0f - m;
    double dmask = 0.0, dlight = 0.0;
    for (int c = 0; c < 3; ++c) {
      const float bg = recon[c * n + i], ob = recon[(3 + c) * n + i];
      const float base = bg * im + ob * m;
      const float v = base * l;
      const float y = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
      const double e = (double)(y - comp[c * n + i]);
      const double gc = dc * e * ((v > 0.0f && v < 1.0f) ? 1.0 : 0.0);
      g[c * n + i] = (float)(dl * (double)(bg - target[c * n + i]) + gc * (double)(l * im));
      g[(3 + c) * n + i] =
          (float)(dl * (double)(ob - target[(3 + c) * n + i]) + gc * (double)(l * m));
      dmask += gc * (double)l * (double)(ob - bg);
      dlight += gc * (double)base;
    }
    g[6 * n + i] = (float)(dl * (double)(m - target[6 * n + i]) + dmask);
    g[7 * n + i] = (float)(dl * (double)(l - target[7 * n + i]) + dlight);
  }
}
