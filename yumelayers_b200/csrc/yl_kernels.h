// yl_kernels.h -- internal C++ launch API shared by the C-ABI entry points
// and the training executor.  All tensors are device pointers; activations
// are NHWC fp32 with a pixel stride (floats per pixel) that is a multiple
// of 4 so every 16-byte gather stays inside one pixel.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "yl_internal.h"

namespace yl {

// Implicit-GEMM operand gather over an NHWC source.  Rows of the GEMM are
// output pixels (img, oy, ox) of an oh x ow grid; the contraction index is
// k = tap * cin + ci with tap = ky * ksize + kx.
enum ConvMode : int { MODE_FPROP = 0, MODE_DGRAD = 1 };

struct ConvGather {
  const float* src = nullptr;
  long long img_stride = 0;  // floats per image of src
  int row_stride = 0;        // floats per source row
  int ps = 0;                // floats per source pixel (multiple of 4)
  int cin = 0;               // contraction channels per tap (multiple of 4, <= ps)
  int hv = 0, wv = 0;        // FPROP: virtual input extent; DGRAD: dy extent
  int up = 0;                // FPROP only: source is read at (iy >> 1, ix >> 1)
  int mode = MODE_FPROP;
  int ksize = 3, stride = 1, pad = 1;
  int oh = 0, ow = 0;        // output pixel grid
  int m_total = 0;           // images * oh * ow
  int k_total = 0;           // ksize * ksize * cin
};

struct ConvEpilogue {
  float* out = nullptr;
  int ldo = 0;               // floats per output pixel (multiple of 4)
  int n_total = 0;           // valid output channels
  const float* bias = nullptr;      // [n_total]
  const float* bias2d = nullptr;    // [img][n_total]: per-image channel bias
  const float* residual = nullptr;  // residual[m * ldr + n], may alias out
  int ldr = 0;
  int round_tf32 = 1;        // round outputs to tf32 (they feed another conv)
  // GroupNorm statistics of the output for the GroupNorm that reads it: when
  // gn_mean is set, conv_fprop also writes mean/rstd per (image, group) of the
  // stored values (torch semantics: biased variance + eps).  Needs
  // n_total = gn_groups * 2^k channels (k >= 2); otherwise YL_ERR_UNSUPPORTED.
  float* gn_mean = nullptr;
  float* gn_rstd = nullptr;
  int gn_groups = 0;
  float gn_eps = 1e-6f;
  // set by conv_fprop: per-tile partial sums (float2) and channels per group
  float2* gn_part = nullptr;
  int gn_cg = 0;
};

// True when conv_fprop can produce GroupNorm statistics for this epilogue.
bool conv_gn_stats_supported(int n_total, int groups);

// out = gather(A) x W^T (+ bias, bias2d, residual); W is [n_rows][k_total]
// row-major (n_rows >= n_total; rows past n_rows read as zero).
yl_status conv_fprop(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                     const ConvEpilogue& e);

// dX (n x sh x sw, into e) of a nearest-x2 upsample + 3x3 pad-1 conv from its
// output gradient dy (n x hv x wv x cout, pixel stride ldy; hv in {2sh - 1,
// 2sh}, wv in {2sw - 1, 2sw}: the x2 grid, possibly cut) and the dgrad
// weights wd [rows][9][cout].  YL_ERR_UNSUPPORTED (nothing launched) when the
// shapes do not fit the merged-tap path.
yl_status conv_dgrad_upsampled(yl_ctx* ctx, const float* dy, int ldy, int cout, int n, int sh,
                               int sw, int hv, int wv, const float* wd, int rows,
                               const ConvEpilogue& e);

// dW[co][k] (+)= sum_p dy[p][co] * gather(p, k), p over all m_total pixels,
// and, when db != nullptr, db[co] (+)= sum_p dy[p][co] from the same reads.
// dy is [m_total][ldy]; dw is [cout][k_total].  Uses ctx scratch for split-K.
yl_status conv_wgrad(yl_ctx* ctx, const float* dy, int ldy, int cout, const ConvGather& g,
                     float* dw, int accumulate, float* db = nullptr);
// Same contraction with an explicit split-K workspace and split count; the
// workspace must hold conv_wgrad_ws_floats(g, cout, dy, ldy, splits) floats.
yl_status conv_wgrad_ws(yl_ctx* ctx, const float* dy, int ldy, int cout, const ConvGather& g,
                        float* dw, int accumulate, float* workspace, int splits,
                        float* db = nullptr);
int conv_wgrad_pick_splits(yl_ctx* ctx, int cout, const ConvGather& g, const float* dy, int ldy);
size_t conv_wgrad_ws_floats(const ConvGather& g, int cout, const float* dy, int ldy, int splits);

// Column sums of dy [images * hw][ldy] over pixels: db[c] (and, when
// db_img != nullptr, db_img[img][c]).  Deterministic (fixed order).
yl_status channel_sums(yl_ctx* ctx, const float* dy, int images, long long hw, int ldy, int c,
                       float* db, float* db_img, int accumulate);

// out[o][t][i] = in[o*so + t*st + i*si] for i < i_src, 0 for i_src <= i < i_out.
// With transpose_oi the roles of o and i are swapped when reading
// (out[i][t][o] layout for dgrad weights).  Optional tf32 rounding.
yl_status weight_permute(yl_ctx* ctx, const float* in, float* out, int O, int T, int I_out,
                         int I_src, long long so, long long st, long long si, int round);

// A batch of weight_permute jobs run by one launch.  The job table is copied
// to the device on the first call and reused afterwards (the caller keeps the
// same jobs and buffers).
struct PermuteJob {
  const float* in;
  float* out;
  int O, T, I_out, I_src;
  long long so, st, si;
  int round;
};
struct PermuteBatchBuffers {
  PermuteJob* jobs = nullptr;
  long long* item_start = nullptr;
  int njobs = 0;
  long long items = 0;
  ~PermuteBatchBuffers();
};
yl_status weight_permute_batch(yl_ctx* ctx, const std::vector<PermuteJob>& jobs,
                               PermuteBatchBuffers* bufs);

// NCHW (c channels) <-> NHWC (pixel stride ps >= c, extra channels zero).
yl_status nchw_to_nhwc(yl_ctx* ctx, const float* in, float* out, int n, int c, long long hw,
                       int ps, int round);
yl_status nhwc_to_nchw(yl_ctx* ctx, const float* in, float* out, int n, int c, long long hw,
                       int ps);

// 3x3 patches of a 4-channel NHWC tensor (pixel stride ld) as 64-channel
// pixels [n*h*w][64]: out[p][t*4 + c] = src[p + sign*(ky-1, kx-1)][c].
yl_status rgb_patches(yl_ctx* ctx, const float* src, int ld, int n, int h, int w, int sign,
                      int round, float* out);
// y[p][0..3] = bias + sum over the 9 taps t of z[p + (ky-1, kx-1)][t*4 + 0..3]
// (z is [n*h*w][36]).
yl_status rgb_tap_sum(yl_ctx* ctx, const float* z, int n, int h, int w, const float* bias,
                      float* y, int ldy);

// dst[img][y][x][c] += / = sum of the 2x2 block of src (an up x2 grid of
// uh x uw, cropped) -- the adjoint of nearest upsampling into (h, w).
yl_status downsample_sum_nhwc(yl_ctx* ctx, const float* src, int uh, int uw, float* dst, int n,
                              int h, int w, int c, int ps_src, int ps_dst);

}  // namespace yl
