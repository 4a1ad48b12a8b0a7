// yl_norm.h -- internal API of the fused GroupNorm+SiLU kernels and the
// small training ops (Adam, loss/latent heads, Linear, time embedding).
#pragma once
#include <cstdint>

#include "yl_internal.h"

namespace yl {

// NHWC GroupNorm statistics: mean/rstd per (image, group).  mode 0: torch
// semantics (biased var + eps); mode 1: the reference's clamp var >= 1e-5.
yl_status gn_stats(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                   float eps, int mode, float* mean, float* rstd);
// y = [silu](GN(x) * gamma + beta), written with pixel stride ldy.
yl_status gn_silu_forward(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                          float eps, int mode, const float* gamma, const float* beta, int silu,
                          float* y, int ldy, int round, float* mean, float* rstd);
// The forward's second pass alone, with mean/rstd already computed (by the
// convolution that produced x).
yl_status gn_silu_apply(yl_ctx* ctx, const float* x, int n, int c, int g, long long hw, int ps,
                        const float* mean, const float* rstd, const float* gamma,
                        const float* beta, int silu, float* y, int ldy, int round);
// dx = d/dx of the forward given dy (+ addend); dgamma/dbeta overwritten or
// accumulated.
yl_status gn_silu_backward(yl_ctx* ctx, const float* x, const float* dy, int lddy, int n, int c,
                           int g, long long hw, int ps, const float* mean, const float* rstd,
                           const float* gamma, const float* beta, int silu, const float* addend,
                           int ldadd, float* dx, int lddx, int round, float* dgamma, float* dbeta,
                           int accumulate_params);

struct AdamTensor {
  float* param;
  const float* grad;
  float* m;
  float* v;
  long long n;
};
// Multi-tensor Adam.  grads are multiplied by grad_scale, non-finite values
// are zeroed when sanitize != 0, and when clip_max_norm > 0 the global L2
// norm is clipped (GradSanitize.swift:18-101); norm_out (device, optional)
// receives the pre-clip norm.  Bias corrections use step t >= 1.
yl_status adam_multi(yl_ctx* ctx, const AdamTensor* tensors, int count, float lr, float b1,
                     float b2, float eps, int t, float grad_scale, float clip_max_norm,
                     int sanitize, float* norm_out);

// Linear: Y = X W^T + b (W is [oc][ic]); backward outputs optional; with
// accumulate != 0 all of dX, dW, db are added to.
yl_status linear_forward(yl_ctx* ctx, const float* X, const float* W, const float* b, float* Y,
                         int n, int ic, int oc);
yl_status linear_backward(yl_ctx* ctx, const float* X, const float* W, const float* dY, float* dX,
                          float* dW, float* db, int n, int ic, int oc, int accumulate);

// 128-d (any even dim) sinusoidal embedding of t[n] (device); variant 0:
// motionTimeEmbedding (interleaved, base 1000, t clamped to [0,1]);
// variant 1: the prototype's timestep_embedding ([cos | sin], base 10000).
yl_status time_embedding(yl_ctx* ctx, const float* t, int n, int dim, int variant, float* out);

// Elementwise SiLU / SiLU-gradient on flat arrays.
yl_status silu_forward(yl_ctx* ctx, const float* x, float* y, long long n);
yl_status silu_backward(yl_ctx* ctx, const float* x, const float* dy, float* dx, long long n,
                        int accumulate);

// VAE latent head (NHWC): e is [n][hw][lde] with mu = channels [0, c) and
// logvar = channels [c, 2c).  z = mu + exp(0.5*clamp(lv,-10,10)) * eps with
// eps[img][ch][p] = randn(seed_img, ch*hw + p), seed_img = trainingNoiseSeed(step, img).
yl_status latent_head_forward(yl_ctx* ctx, const float* e, int lde, int n, long long hw, int c,
                              int64_t step, float* z, int ldz);
// de (same layout as e) from dz: dmu = dz + betaN*mu; dlv = dz*eps*0.5*sigma + betaHalfN*(exp(lv)-1).
yl_status latent_head_backward(yl_ctx* ctx, const float* e, int lde, const float* dz, int lddz,
                               int n, long long hw, int c, int64_t step, float betaN,
                               float betaHalfN, float* de, int ldde);

// L1 + beta*KL loss head.  recon/target are [n_pix][ld] with `ch` valid
// channels; drecon = sign(r - t) / (n_pix*ch) (padded channels zero).  The
// loss value (mean L1 + beta * KL / n_lat) is written to loss_out (device).
yl_status l1_kl_head(yl_ctx* ctx, const float* recon, const float* target, long long n_pix, int ld,
                     int ch, const float* e, int lde, long long n_lat_pix, int c_lat, float beta,
                     float* drecon, float* loss_out);
// MSE head: loss = mean((p - t)^2) over n_pix*ch, dpred = 2 (p - t) / count.
yl_status mse_head(yl_ctx* ctx, const float* pred, const float* target, long long n_pix, int ld,
                   int ch, float* dpred, float* loss_out);

}  // namespace yl
