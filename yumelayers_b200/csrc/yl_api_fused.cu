// yl_api_fused.cu -- C-ABI entry points of the B200 operators on batched
// tensors (NCHW = the reference's per-image CHW stacked, or NHWC).  Each
// call converts to the internal NHWC layout (pixel stride rounded up to a
// multiple of 4, conv operands rounded to tf32) in scratch slot 1, runs the
// kernels, and converts back.  The training executor calls the kernels
// directly on NHWC buffers and never pays for these conversions.
#include <cmath>

#include "yl_kernels.h"
#include "yl_norm.h"
#include "yume_c.h"

using namespace yl;

namespace {

inline int round4(int c) { return (c + 3) & ~3; }

struct ConvShape {
  int ih, iw, oh, ow, cp, ocp;
};

yl_status conv_shape(const yl_conv_desc* d, ConvShape* s) {
  YL_CHECK(d, YL_ERR_INVALID, "conv: descriptor is NULL");
  YL_CHECK(d->n > 0 && d->c > 0 && d->h > 0 && d->w > 0 && d->oc > 0, YL_ERR_SHAPE,
           "conv: non-positive dimension");
  YL_CHECK(d->k >= 1 && d->stride >= 1 && d->pad >= 0, YL_ERR_SHAPE, "conv: bad kernel geometry");
  YL_CHECK(d->layout == YL_LAYOUT_NCHW || d->layout == YL_LAYOUT_NHWC, YL_ERR_INVALID,
           "conv: unknown layout %d", d->layout);
  s->ih = d->up ? d->up_h : d->h;
  s->iw = d->up ? d->up_w : d->w;
  if (d->up)
    YL_CHECK(d->up_h > 0 && d->up_w > 0 && d->up_h <= 2 * d->h && d->up_w <= 2 * d->w &&
                 (d->up_h + 1) / 2 == d->h && (d->up_w + 1) / 2 == d->w,
             YL_ERR_SHAPE, "conv: upsampled size %dx%d does not match source %dx%d", d->up_h,
             d->up_w, d->h, d->w);
  YL_CHECK(s->ih + 2 * d->pad >= d->k && s->iw + 2 * d->pad >= d->k, YL_ERR_SHAPE,
           "conv: kernel larger than padded input");
  s->oh = (s->ih + 2 * d->pad - d->k) / d->stride + 1;
  s->ow = (s->iw + 2 * d->pad - d->k) / d->stride + 1;
  s->cp = round4(d->c);
  s->ocp = round4(d->oc);
  return YL_OK;
}

// [n][hw][c] (pixel stride c) -> [n][hw][ps], padded with zeros.
__global__ void repack_kernel(const float* __restrict__ in, int cin_stride, int c,
                              float* __restrict__ out, int ps, long long pixels, int round) {
  const long long total = pixels * ps;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % ps);
    const long long p = i / ps;
    float v = k < c ? in[p * cin_stride + k] : 0.f;
    if (round) {
      unsigned r;
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
      v = __uint_as_float(r & 0xFFFFE000u);
    }
    out[i] = v;
  }
}

yl_status to_internal(yl_ctx* ctx, const float* x, int layout, int n, int c, long long hw, int ps,
                      int round, float* out) {
  if (layout == YL_LAYOUT_NCHW) return nchw_to_nhwc(ctx, x, out, n, c, hw, ps, round);
  long long pixels = (long long)n * hw;
  repack_kernel<<<grid_1d(pixels * ps, 256), 256, 0, ctx->stream>>>(x, c, c, out, ps, pixels,
                                                                    round);
  return check_launch("repack_kernel");
}

yl_status from_internal(yl_ctx* ctx, const float* in, int ps, int layout, int n, int c,
                        long long hw, float* out) {
  if (layout == YL_LAYOUT_NCHW) return nhwc_to_nchw(ctx, in, out, n, c, hw, ps);
  long long pixels = (long long)n * hw;
  repack_kernel<<<grid_1d(pixels * c, 256), 256, 0, ctx->stream>>>(in, ps, c, out, c, pixels, 0);
  return check_launch("repack_kernel");
}

ConvGather make_fprop_gather(const yl_conv_desc* d, const ConvShape& s, const float* xh) {
  ConvGather g;
  g.src = xh;
  g.img_stride = (long long)d->h * d->w * s.cp;
  g.row_stride = d->w * s.cp;
  g.ps = s.cp;
  g.cin = s.cp;
  g.hv = s.ih;
  g.wv = s.iw;
  g.up = d->up;
  g.mode = MODE_FPROP;
  g.ksize = d->k;
  g.stride = d->stride;
  g.pad = d->pad;
  g.oh = s.oh;
  g.ow = s.ow;
  g.m_total = d->n * s.oh * s.ow;
  g.k_total = d->k * d->k * s.cp;
  return g;
}

// Scratch layout helper for one C-ABI call (slot 1).
struct Pieces {
  ScratchCarver carve;
  size_t add(size_t floats) { return carve.take(floats * sizeof(float)); }
};

}  // namespace

extern "C" {

yl_status yl_conv2d_out_shape(const yl_conv_desc* d, int* oh, int* ow) {
  ConvShape s;
  YL_TRY(conv_shape(d, &s));
  if (oh) *oh = s.oh;
  if (ow) *ow = s.ow;
  return YL_OK;
}

yl_status yl_conv2d_fwd(yl_ctx* ctx, const yl_conv_desc* d, const float* x, const float* w,
                        const float* b, const float* residual, float* y) {
  YL_CHECK(ctx && x && w && y, YL_ERR_INVALID, "yl_conv2d_fwd: NULL argument");
  ConvShape s;
  YL_TRY(conv_shape(d, &s));
  const long long hw_in = (long long)d->h * d->w, hw_out = (long long)s.oh * s.ow;
  Pieces pc;
  size_t o_x = pc.add(d->n * hw_in * s.cp), o_w = pc.add((size_t)d->oc * d->k * d->k * s.cp),
         o_y = pc.add(d->n * hw_out * s.ocp), o_r = residual ? pc.add(d->n * hw_out * s.ocp) : 0;
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  char* sb = (char*)base;
  float *xh = (float*)(sb + o_x), *wt = (float*)(sb + o_w), *yh = (float*)(sb + o_y);
  float* rh = residual ? (float*)(sb + o_r) : nullptr;
  YL_TRY(to_internal(ctx, x, d->layout, d->n, d->c, hw_in, s.cp, 1, xh));
  YL_TRY(weight_permute(ctx, w, wt, d->oc, d->k * d->k, s.cp, d->c, (long long)d->c * d->k * d->k,
                        1, d->k * d->k, 1));
  if (residual) YL_TRY(to_internal(ctx, residual, d->layout, d->n, d->oc, hw_out, s.ocp, 0, rh));
  ConvGather g = make_fprop_gather(d, s, xh);
  ConvEpilogue e;
  e.out = yh;
  e.ldo = s.ocp;
  e.n_total = d->oc;
  e.bias = b;
  e.residual = rh;
  e.ldr = s.ocp;
  e.round_tf32 = 0;
  YL_TRY(conv_fprop(ctx, g, wt, d->oc, e));
  return from_internal(ctx, yh, s.ocp, d->layout, d->n, d->oc, hw_out, y);
}

yl_status yl_conv2d_bwd_data(yl_ctx* ctx, const yl_conv_desc* d, const float* dy, const float* w,
                             float* dx) {
  YL_CHECK(ctx && dy && w && dx, YL_ERR_INVALID, "yl_conv2d_bwd_data: NULL argument");
  ConvShape s;
  YL_TRY(conv_shape(d, &s));
  const long long hw_in = (long long)d->h * d->w, hw_v = (long long)s.ih * s.iw,
                  hw_out = (long long)s.oh * s.ow;
  Pieces pc;
  size_t o_dy = pc.add(d->n * hw_out * s.ocp), o_w = pc.add((size_t)d->c * d->k * d->k * s.ocp),
         o_dv = pc.add(d->n * hw_v * s.cp), o_dx = d->up ? pc.add(d->n * hw_in * s.cp) : 0;
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  char* sb = (char*)base;
  float *dyh = (float*)(sb + o_dy), *wd = (float*)(sb + o_w), *dvh = (float*)(sb + o_dv);
  float* dxh = d->up ? (float*)(sb + o_dx) : dvh;
  YL_TRY(to_internal(ctx, dy, d->layout, d->n, d->oc, hw_out, s.ocp, 1, dyh));
  // Wd[ci][tap][co] = W[co][ci][tap]
  YL_TRY(weight_permute(ctx, w, wd, d->c, d->k * d->k, s.ocp, d->oc, d->k * d->k, 1,
                        (long long)d->c * d->k * d->k, 1));
  ConvGather g;
  g.src = dyh;
  g.img_stride = hw_out * s.ocp;
  g.row_stride = s.ow * s.ocp;
  g.ps = s.ocp;
  g.cin = s.ocp;
  g.hv = s.oh;
  g.wv = s.ow;
  g.up = 0;
  g.mode = MODE_DGRAD;
  g.ksize = d->k;
  g.stride = d->stride;
  g.pad = d->pad;
  g.oh = s.ih;
  g.ow = s.iw;
  g.m_total = (int)(d->n * hw_v);
  g.k_total = d->k * d->k * s.ocp;
  ConvEpilogue e;
  e.out = dvh;
  e.ldo = s.cp;
  e.n_total = d->c;
  e.round_tf32 = 0;
  if (d->up && d->k == 3 && d->pad == 1 && d->stride == 1) {
    // upsample conv (the x2 grid, or one cut by a row / column): dX at the
    // source resolution through the merged phase taps
    ConvEpilogue eu = e;
    eu.out = dxh;
    const yl_status st = conv_dgrad_upsampled(ctx, dyh, s.ocp, s.ocp, d->n, d->h, d->w, s.ih,
                                              s.iw, wd, d->c, eu);
    if (st == YL_OK) return from_internal(ctx, dxh, s.cp, d->layout, d->n, d->c, hw_in, dx);
    if (st != YL_ERR_UNSUPPORTED) return st;
  }
  YL_TRY(conv_fprop(ctx, g, wd, d->c, e));
  if (d->up) YL_TRY(downsample_sum_nhwc(ctx, dvh, s.ih, s.iw, dxh, d->n, d->h, d->w, s.cp, s.cp, s.cp));
  return from_internal(ctx, dxh, s.cp, d->layout, d->n, d->c, hw_in, dx);
}

yl_status yl_conv2d_bwd_filter(yl_ctx* ctx, const yl_conv_desc* d, const float* x, const float* dy,
                               float* dw, float* db) {
  YL_CHECK(ctx && x && dy && (dw || db), YL_ERR_INVALID, "yl_conv2d_bwd_filter: NULL argument");
  ConvShape s;
  YL_TRY(conv_shape(d, &s));
  const long long hw_in = (long long)d->h * d->w, hw_out = (long long)s.oh * s.ow;
  const int kk = d->k * d->k;
  Pieces pc;
  size_t o_x = pc.add(d->n * hw_in * s.cp), o_dy = pc.add(d->n * hw_out * s.ocp),
         o_dw = pc.add((size_t)s.ocp * kk * s.cp);
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  char* sb = (char*)base;
  float *xh = (float*)(sb + o_x), *dyh = (float*)(sb + o_dy), *dwi = (float*)(sb + o_dw);
  if (db) {  // db sums the caller's fp32 dy (before the tf32 rounding of the GEMM operand)
    YL_TRY(to_internal(ctx, dy, d->layout, d->n, d->oc, hw_out, s.ocp, 0, dyh));
    YL_TRY(channel_sums(ctx, dyh, d->n, hw_out, s.ocp, d->oc, db, nullptr, 0));
  }
  if (dw) {
    YL_TRY(to_internal(ctx, dy, d->layout, d->n, d->oc, hw_out, s.ocp, 1, dyh));
    YL_TRY(to_internal(ctx, x, d->layout, d->n, d->c, hw_in, s.cp, 1, xh));
    ConvGather g = make_fprop_gather(d, s, xh);
    YL_TRY(conv_wgrad(ctx, dyh, s.ocp, s.ocp, g, dwi, 0));
    // dwi[o][tap][ci] -> dw[o][ci][tap]
    YL_TRY(weight_permute(ctx, dwi, dw, d->oc, d->c, kk, kk, (long long)kk * s.cp, 1, s.cp, 0));
  }
  return YL_OK;
}

yl_status yl_conv_transpose2d_fwd(yl_ctx* ctx, const yl_conv_desc* d, const float* x,
                                  const float* w, const float* b, float* y) {
  YL_CHECK(d && !d->up, YL_ERR_UNSUPPORTED, "transposed conv of an upsampled input is not defined");
  YL_TRY(yl_conv2d_bwd_data(ctx, d, x, w, y));
  if (!b) return YL_OK;
  // per-channel bias on the (n, c, h, w) result
  if (d->layout == YL_LAYOUT_NHWC) return yl_add_bias(ctx, y, b, y, d->n * d->h * d->w, d->c);
  const size_t plane = (size_t)d->h * d->w;
  for (int img = 0; img < d->n; ++img)
    YL_TRY(yl_bias_row(ctx, y + img * d->c * plane, b, y + img * d->c * plane, d->c, (int)plane));
  return YL_OK;
}

yl_status yl_conv_transpose2d_bwd_data(yl_ctx* ctx, const yl_conv_desc* d, const float* dy,
                                       const float* w, float* dx) {
  return yl_conv2d_fwd(ctx, d, dy, w, nullptr, nullptr, dx);
}

yl_status yl_conv_transpose2d_bwd_filter(yl_ctx* ctx, const yl_conv_desc* d, const float* x,
                                         const float* dy, float* dw, float* db) {
  YL_CHECK(ctx && d && x && dy, YL_ERR_INVALID, "yl_conv_transpose2d_bwd_filter: NULL argument");
  if (dw) YL_TRY(yl_conv2d_bwd_filter(ctx, d, dy, x, dw, nullptr));
  if (db) {
    // db sums dy (shaped like the conv's input) per channel.
    ConvShape s;
    YL_TRY(conv_shape(d, &s));
    const long long hw = (long long)d->h * d->w;
    void* base = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)d->n * hw * s.cp * sizeof(float), &base, 1));
    YL_TRY(to_internal(ctx, dy, d->layout, d->n, d->c, hw, s.cp, 0, (float*)base));
    YL_TRY(channel_sums(ctx, (float*)base, d->n, hw, s.cp, d->c, db, nullptr, 0));
  }
  return YL_OK;
}

yl_status yl_groupnorm_silu_fwd(yl_ctx* ctx, const float* x, int n, int c, int h, int w,
                                int layout, int groups, float eps, int mode, const float* gamma,
                                const float* beta, int apply_silu, float* y, float* mean_out,
                                float* rstd_out) {
  YL_CHECK(ctx && x && y, YL_ERR_INVALID, "yl_groupnorm_silu_fwd: NULL argument");
  YL_CHECK(layout == YL_LAYOUT_NCHW || layout == YL_LAYOUT_NHWC, YL_ERR_INVALID, "bad layout");
  const long long hw = (long long)h * w;
  const bool direct = layout == YL_LAYOUT_NHWC && c % 4 == 0;
  Pieces pc;  // staging copies only when the caller's layout is not the internal one
  size_t o_x = direct ? 0 : pc.add(n * hw * c), o_y = direct ? 0 : pc.add(n * hw * c);
  size_t o_s = pc.add(2 * (size_t)n * groups);
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  char* sb = (char*)base;
  float* xh = direct ? (float*)x : (float*)(sb + o_x);
  float* yh = direct ? y : (float*)(sb + o_y);
  float* mean = mean_out ? mean_out : (float*)(sb + o_s);
  float* rstd = rstd_out ? rstd_out : (float*)(sb + o_s) + (size_t)n * groups;
  if (xh != x) YL_TRY(to_internal(ctx, x, layout, n, c, hw, c, 0, xh));
  YL_TRY(gn_silu_forward(ctx, xh, n, c, groups, hw, c, eps, mode, gamma, beta, apply_silu, yh, c, 0,
                         mean, rstd));
  if (yh != y) YL_TRY(from_internal(ctx, yh, c, layout, n, c, hw, y));
  return YL_OK;
}

yl_status yl_groupnorm_silu_bwd(yl_ctx* ctx, const float* x, const float* dy, int n, int c, int h,
                                int w, int layout, int groups, float eps, int mode,
                                const float* gamma, const float* beta, int apply_silu,
                                const float* mean_in, const float* rstd_in, const float* addend,
                                float* dx, float* dgamma, float* dbeta) {
  YL_CHECK(ctx && x && dy && dx, YL_ERR_INVALID, "yl_groupnorm_silu_bwd: NULL argument");
  YL_CHECK(layout == YL_LAYOUT_NCHW || layout == YL_LAYOUT_NHWC, YL_ERR_INVALID, "bad layout");
  const long long hw = (long long)h * w;
  const bool direct = layout == YL_LAYOUT_NHWC && c % 4 == 0;
  Pieces pc;  // staging copies only when the caller's layout is not the internal one
  const size_t e = direct ? 0 : (size_t)(n * hw * c);
  size_t o_x = pc.add(e), o_dy = pc.add(e), o_a = pc.add(addend ? e : 0), o_dx = pc.add(e),
         o_s = pc.add(2 * (size_t)n * groups);
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  char* sb = (char*)base;
  const float* xh = direct ? x : (float*)(sb + o_x);
  const float* dyh = direct ? dy : (float*)(sb + o_dy);
  const float* ah = (!addend || direct) ? addend : (float*)(sb + o_a);
  float* dxh = direct ? dx : (float*)(sb + o_dx);
  if (!direct) {
    YL_TRY(to_internal(ctx, x, layout, n, c, hw, c, 0, (float*)xh));
    YL_TRY(to_internal(ctx, dy, layout, n, c, hw, c, 0, (float*)dyh));
    if (addend) YL_TRY(to_internal(ctx, addend, layout, n, c, hw, c, 0, (float*)ah));
  }
  const float* mean = mean_in;
  const float* rstd = rstd_in;
  if (!mean || !rstd) {
    float* ms = (float*)(sb + o_s);
    YL_TRY(gn_stats(ctx, xh, n, c, groups, hw, c, eps, mode, ms, ms + (size_t)n * groups));
    mean = ms;
    rstd = ms + (size_t)n * groups;
  }
  YL_TRY(gn_silu_backward(ctx, xh, dyh, c, n, c, groups, hw, c, mean, rstd, gamma, beta, apply_silu,
                          ah, c, dxh, c, 0, dgamma, dbeta, 0));
  if (!direct) YL_TRY(from_internal(ctx, dxh, c, layout, n, c, hw, dx));
  return YL_OK;
}

yl_status yl_linear_fwd(yl_ctx* ctx, const float* X, const float* W, const float* b, float* Y,
                        int n, int ic, int oc) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_linear_fwd: ctx is NULL");
  return linear_forward(ctx, X, W, b, Y, n, ic, oc);
}

yl_status yl_linear_bwd(yl_ctx* ctx, const float* X, const float* W, const float* dY, float* dX,
                        float* dW, float* db, int n, int ic, int oc) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_linear_bwd: ctx is NULL");
  return linear_backward(ctx, X, W, dY, dX, dW, db, n, ic, oc, 0);
}

yl_status yl_timestep_embedding(yl_ctx* ctx, const float* t, int n, int dim, int variant,
                                float* out) {
  YL_CHECK(ctx, YL_ERR_INVALID, "yl_timestep_embedding: ctx is NULL");
  return time_embedding(ctx, t, n, dim, variant, out);
}

yl_status yl_adam_multi(yl_ctx* ctx, const yl_adam_tensor* table, int count, float lr, float b1,
                        float b2, float eps, int t, float grad_scale, float clip_max_norm,
                        int sanitize, float* norm_out_dev) {
  YL_CHECK(ctx && (table || count == 0), YL_ERR_INVALID, "yl_adam_multi: NULL argument");
  static_assert(sizeof(yl_adam_tensor) == sizeof(AdamTensor), "table layout");
  return adam_multi(ctx, reinterpret_cast<const AdamTensor*>(table), count, lr, b1, b2, eps, t,
                    grad_scale, clip_max_norm, sanitize, norm_out_dev);
}

yl_status yl_vae_latent_head_fwd(yl_ctx* ctx, const float* e, int n, int c, int h, int w,
                                 int layout, int64_t step, float* z) {
  YL_CHECK(ctx && e && z, YL_ERR_INVALID, "yl_vae_latent_head_fwd: NULL argument");
  const long long hw = (long long)h * w;
  Pieces pc;
  size_t o_e = pc.add(n * hw * 2 * c), o_z = pc.add(n * hw * c);
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  float* eh = (float*)((char*)base + o_e);
  float* zh = (float*)((char*)base + o_z);
  YL_TRY(to_internal(ctx, e, layout, n, 2 * c, hw, 2 * c, 0, eh));
  YL_TRY(latent_head_forward(ctx, eh, 2 * c, n, hw, c, step, zh, c));
  return from_internal(ctx, zh, c, layout, n, c, hw, z);
}

yl_status yl_vae_latent_head_bwd(yl_ctx* ctx, const float* e, const float* dz, int n, int c, int h,
                                 int w, int layout, int64_t step, float beta, float* de) {
  YL_CHECK(ctx && e && dz && de, YL_ERR_INVALID, "yl_vae_latent_head_bwd: NULL argument");
  const long long hw = (long long)h * w;
  Pieces pc;
  size_t o_e = pc.add(n * hw * 2 * c), o_dz = pc.add(n * hw * c), o_de = pc.add(n * hw * 2 * c);
  void* base = nullptr;
  YL_TRY(scratch_get(ctx, pc.carve.offset, &base, 1));
  float* eh = (float*)((char*)base + o_e);
  float* dzh = (float*)((char*)base + o_dz);
  float* deh = (float*)((char*)base + o_de);
  YL_TRY(to_internal(ctx, e, layout, n, 2 * c, hw, 2 * c, 0, eh));
  YL_TRY(to_internal(ctx, dz, layout, n, c, hw, c, 0, dzh));
  const double M = (double)n * c * hw;  // KL averaged per latent element (ConvGPU.swift:435-438)
  YL_TRY(latent_head_backward(ctx, eh, 2 * c, dzh, c, n, hw, c, step, (float)(beta / M),
                              (float)(0.5 * beta / M), deh, 2 * c));
  return from_internal(ctx, deh, 2 * c, layout, n, 2 * c, hw, de);
}

yl_status yl_loss_l1_kl(yl_ctx* ctx, const float* recon, const float* target, size_t n_recon,
                        const float* mu_logvar, int n, int c_lat, int h_lat, int w_lat, int layout,
                        float beta, float* drecon, float* loss_dev) {
  YL_CHECK(ctx && recon && target, YL_ERR_INVALID, "yl_loss_l1_kl: NULL argument");
  const long long hw = (long long)h_lat * w_lat;
  float* eh = nullptr;
  if (mu_logvar) {
    void* base = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)n * hw * 2 * c_lat * sizeof(float), &base, 1));
    eh = (float*)base;
    YL_TRY(to_internal(ctx, mu_logvar, layout, n, 2 * c_lat, hw, 2 * c_lat, 0, eh));
  }
  // L1 and its gradient are layout-agnostic elementwise sums over the flat arrays.
  return l1_kl_head(ctx, recon, target, (long long)n_recon, 1, 1, eh, 2 * c_lat,
                    mu_logvar ? (long long)n * hw : 0, c_lat, beta, drecon, loss_dev);
}

}  // extern "C"
