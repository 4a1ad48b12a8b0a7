/*
 * yume_c.h -- C ABI of the B200 backend for YumeLayersCore's operator layer.
 *
 * This is the drop-in boundary that replaces the reference's Metal-backed
 * `GpuSession` operator API (Sources/YumeLayersCore/GpuSessionOps.swift,
 * GpuSessionNormGrad.swift, GpuTraining.swift, GPUTensor.swift,
 * MetalEngine.swift).  Plain pointers and sizes only: every `float*` tensor
 * argument is a CUDA device pointer unless its name says `host`.  All calls
 * are asynchronous on the context's stream unless documented otherwise and
 * return a yl_status; none of them aborts or exits the process
 * (the reference calls precondition/fatalError/exit(70): GpuSessionOps.swift:112,
 * MetalEngine.swift:73-79, GpuTraining.swift:92-97).
 *
 * Layout conventions.  Reference tensors are per-image CHW, `rows` = channels
 * and `cols` = H*W (GPUTensor.swift:9-14); conv weights are (oc, ic*k*k)
 * (ConvGPU.swift:18); Linear weights are (oc, ic) with Y = X*W^T + b
 * (DenoiserMLP.swift:51-54).  Batched entry points take NCHW (the reference
 * layout with the host batch loop folded in) or NHWC via a yl_layout value.
 */
#ifndef YUME_C_H
#define YUME_C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum yl_status {
  YL_OK = 0,
  YL_ERR_SHAPE = 1,         /* precondition on shapes (reference: precondition crash) */
  YL_ERR_OOM = 2,           /* allocation failed (reference: fatalError) */
  YL_ERR_TIMEOUT = 3,       /* a wait hit its deadline (reference: exit(70)) */
  YL_ERR_CUDA = 4,          /* CUDA runtime/driver error */
  YL_ERR_NCCL = 5,          /* NCCL error */
  YL_ERR_DEVICE_ASSERT = 6, /* a kernel reported an error through its error word */
  YL_ERR_INVALID = 7,       /* bad argument (null pointer, unknown enum) */
  YL_ERR_UNSUPPORTED = 8    /* valid request this build does not handle */
} yl_status;

typedef enum yl_layout { YL_LAYOUT_NCHW = 0, YL_LAYOUT_NHWC = 1 } yl_layout;

typedef struct yl_ctx yl_ctx;
typedef struct yl_tensor yl_tensor;
typedef struct yl_comm yl_comm;
typedef struct yl_trainer yl_trainer;

/* Thread-local text of the last non-OK status returned on this thread. */
const char* yl_last_error_message(void);
const char* yl_version(void);
/* Number of kernels this library has launched in the process so far. */
unsigned long long yl_kernel_launch_count(void);

/* ------------------------------------------------------------------ runtime
 * Replaces MetalEngine (MetalEngine.swift:6-419: device, queue, pools) and
 * GpuSession recording (GpuTraining.swift:4-151).  One context per GPU per
 * host thread; context calls are not thread-safe (GpuTraining.swift:36-38). */
yl_status yl_ctx_create(int device, yl_ctx** out);
yl_status yl_ctx_destroy(yl_ctx* ctx);
/* Use an external cudaStream_t (NULL restores the context's own stream). */
yl_status yl_ctx_set_stream(yl_ctx* ctx, void* cuda_stream);
void* yl_ctx_get_stream(yl_ctx* ctx);
/* GpuSession.begin() (GpuTraining.swift:17-20): marks the start of a step. */
yl_status yl_session_begin(yl_ctx* ctx);
/* GpuSession.commit() (GpuTraining.swift:123-134): records completion, no wait. */
yl_status yl_session_commit(yl_ctx* ctx);
/* GpuSession.end() (GpuTraining.swift:140-145, wait :72-112): waits for the
 * session's work with a deadline; YL_ERR_TIMEOUT instead of exit(70).  gpu_ms
 * (may be NULL) gets the device time between begin and end, bounded by the
 * wall time the way boundedGpuMs does (GpuWaitPolicy.swift:75-87). */
yl_status yl_session_end(yl_ctx* ctx, double timeout_s, double* gpu_ms);
/* Reads and clears the context's device error word (kernels write it when a
 * bounded wait gives up or a device-side check fails): YL_ERR_TIMEOUT for a
 * wait that gave up (the reference's hang guard, GpuTraining.swift:92-97,
 * exits with 70 instead), YL_ERR_DEVICE_ASSERT for a failed device check. */
yl_status yl_ctx_check_device_errors(yl_ctx* ctx);
/* Bound of every device-side wait of this context's kernels, in SM clock
 * cycles (<= 0: the default 2e9, about 1 s).  The reference's wait policy
 * (GpuWaitPolicy.swift:54-61) bounds the host wait only; this also bounds
 * the kernels' pipeline waits.  Tests shorten it to drive the timeout path. */
yl_status yl_ctx_set_wait_limit(yl_ctx* ctx, long long cycles);
/* Name of the last conv kernel template this context launched: which = 0
 * forward / dX, 1 filter gradient ("" before any).  Diagnostics only; no
 * counterpart in the reference, whose conv is one im2col + matmul path. */
const char* yl_ctx_last_kernel(yl_ctx* ctx, int which);

/* --------------------------------------------------------------- GPUTensor
 * GPUTensor (GPUTensor.swift:9-143): rows x cols fp32, row-major, owned by
 * the context's caching pool (MetalEngine.swift:33-82); release returns the
 * block to the pool once the stream has passed it. */
yl_status yl_tensor_create(yl_ctx* ctx, int rows, int cols, const float* host_or_null,
                           yl_tensor** out);
yl_status yl_tensor_release(yl_tensor* t);
float* yl_tensor_data(yl_tensor* t);
int yl_tensor_rows(const yl_tensor* t);
int yl_tensor_cols(const yl_tensor* t);
/* setData / toArray (GPUTensor.swift:54-120): synchronous copies. */
yl_status yl_tensor_upload(yl_tensor* t, const float* host, size_t n);
yl_status yl_tensor_download(yl_tensor* t, float* host, size_t n);
/* getValue / setValue (GPUTensor.swift:122-142). */
yl_status yl_tensor_get_value(yl_tensor* t, size_t index, float* value);
yl_status yl_tensor_set_value(yl_tensor* t, size_t index, float value);
/* GpuSession.copy / zeroFill (GpuSessionOps.swift:257-276), stream-ordered. */
yl_status yl_copy(yl_ctx* ctx, float* dst, const float* src, size_t n);
yl_status yl_zero_fill(yl_ctx* ctx, float* dst, size_t n);
/* Host <-> device byte copies on the context's stream; both synchronize
 * (the staging-buffer upload / toArray paths, GpuSessionOps.swift:8-20). */
yl_status yl_memcpy_htod(yl_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
yl_status yl_memcpy_dtoh(yl_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);

/* ------------------------------------------------- reference-mode operators
 * One entry point per GpuSession method, same argument meaning, caller-owned
 * outputs.  These reproduce the reference kernels' semantics exactly and are
 * what the reference's own unit tests exercise (TestGroup3.swift:296-537). */

/* matmul(_:_:transA:transB:M:N:K:) (GpuSessionOps.swift:80-108). */
yl_status yl_matmul(yl_ctx* ctx, const float* A, const float* B, float* C, int M, int N,
                    int K, int transA, int transB);
/* im2col (GpuSessionOps.swift:281-300): X (ic, ih, iw) -> (ic*kh*kw, oh*ow). */
yl_status yl_im2col(yl_ctx* ctx, const float* X, float* cols, int ic, int ih, int iw, int kh,
                    int kw, int stride, int pad);
/* col2im (GpuSessionOps.swift:303-333). */
yl_status yl_col2im(yl_ctx* ctx, const float* cols, float* G, int ic, int ih, int iw, int kh,
                    int kw, int stride, int pad, int oh, int ow);
/* gradW(_:_:oc:kk:) (GpuSessionOps.swift:349-359): C = A * B^T, A (oc, K), B (kk, K). */
yl_status yl_grad_w(yl_ctx* ctx, const float* A, const float* B, float* C, int oc, int kk,
                    int K);
/* convBackInputS1 (GpuSessionOps.swift:362-376). */
yl_status yl_conv_back_input_s1(yl_ctx* ctx, const float* dOut, const float* W, float* dx,
                                int ic, int oc, int ih, int iw, int k, int pad);
/* biasRow (GpuSessionOps.swift:389-396): C[r,c] = A[r,c] + b[r]. */
yl_status yl_bias_row(yl_ctx* ctx, const float* A, const float* b, float* C, int rows, int cols);
/* biasRowGrad (GpuSessionOps.swift:398-417): out[r] = sum_c G[r,c]. */
yl_status yl_bias_row_grad(yl_ctx* ctx, const float* G, float* out, int rows, int cols);
/* addBias (GpuSessionOps.swift:146-153): C[i] = A[i] + bias[i % cols]. */
yl_status yl_add_bias(yl_ctx* ctx, const float* A, const float* bias, float* C, int rows,
                      int cols);
/* sumCols (GpuSessionOps.swift:205-217): C[j] = sum_i A[i,j]. */
yl_status yl_sum_cols(yl_ctx* ctx, const float* A, float* C, int rows, int cols);
/* groupNorm(_:groups:) (GpuSessionOps.swift:121-131): affine-free, var >= 1e-5. */
yl_status yl_group_norm(yl_ctx* ctx, const float* A, float* C, int rows, int cols, int groups);
/* encodeGroupNormGrad (GpuSessionNormGrad.swift:10-24). */
yl_status yl_group_norm_grad(yl_ctx* ctx, const float* x, const float* dy, float* out, int rows,
                             int cols, int groups);

typedef enum yl_unary_op {
  YL_RELU = 0, YL_SIGMOID = 1, YL_TANH = 2, YL_TANH_GRAD = 3, YL_EXP = 4, YL_EXP_HALF = 5,
  YL_SILU = 6
} yl_unary_op;
/* relu / sigmoid / tanh / tanhGrad / exp / expHalf (GpuSessionOps.swift:186-202,
 * 419-442, 463-478) and SiLU (src/vae.py:11). */
yl_status yl_unary(yl_ctx* ctx, int op, const float* A, float* C, size_t n);

typedef enum yl_binary_op {
  YL_ADD = 0, YL_SUB = 1, YL_MUL = 2, YL_RELU_GRAD = 3, YL_SIGMOID_GRAD = 4, YL_SILU_GRAD = 5
} yl_binary_op;
/* add / sub / mul / reluGrad / sigmoidGrad (GpuSessionOps.swift:111-172, 427-451)
 * and the SiLU derivative. */
yl_status yl_binary(yl_ctx* ctx, int op, const float* A, const float* B, float* C, size_t n);
/* smul / addConst / fma / addInPlace (GpuSessionOps.swift:176, 481, 492, 453). */
yl_status yl_smul(yl_ctx* ctx, float s, const float* A, float* C, size_t n);
yl_status yl_add_const(yl_ctx* ctx, const float* A, float s, float* C, size_t n);
yl_status yl_fma(yl_ctx* ctx, const float* A, const float* B, const float* D, float* C,
                 size_t n);
yl_status yl_add_in_place(yl_ctx* ctx, float* A, const float* B, size_t n);
/* upsample2x / downsample2x (GpuSessionOps.swift:336-387), (c,h,w) <-> (c,2h,2w). */
yl_status yl_upsample2x(yl_ctx* ctx, const float* X, float* Y, int c, int h, int w);
yl_status yl_downsample2x(yl_ctx* ctx, const float* X, float* Y, int c, int h, int w);
/* split2 / merge2 (GpuSessionOps.swift:502-524). */
yl_status yl_split2(yl_ctx* ctx, const float* X, float* mu, float* logvar, int c, int plane);
yl_status yl_merge2(yl_ctx* ctx, const float* mu, const float* logvar, float* X, int c,
                    int plane);
/* randn(seed:rows:cols:) (GpuSessionOps.swift:527-535), same (seed, index) hash. */
yl_status yl_randn(yl_ctx* ctx, float* out, uint32_t seed, size_t n);
/* encodeMSE (GpuSessionOps.swift:25-42) and kl (:538-547): the sum is written
 * to the device scalar out_dev (read it after yl_session_end). */
yl_status yl_mse_sum(yl_ctx* ctx, const float* recon, const float* target, size_t n,
                     float* out_dev);
yl_status yl_kl_sum(yl_ctx* ctx, const float* mu, const float* logvar, size_t n, float* out_dev);
/* encodeL1Grad (GpuSessionOps.swift:134-143): sign(r - t) / n. */
yl_status yl_l1_grad(yl_ctx* ctx, const float* recon, const float* target, float* out, size_t n);
/* vaeGrad (GpuSessionOps.swift:550-563). */
yl_status yl_vae_grad(yl_ctx* ctx, const float* dz, const float* mu, const float* logvar,
                      const float* eps, float* dmu, float* dlogvar, float betaN,
                      float betaHalfN, size_t n);
/* adamUpdate (GpuSessionOps.swift:242-252): b1 .9, b2 .999, eps 1e-8, t >= 1. */
yl_status yl_adam_update(yl_ctx* ctx, float* param, const float* grad, float* m, float* v,
                         size_t n, int t, float lr);

/* -------------------------------------------------- B200 batched operators
 * The same layer semantics on whole batches (the reference loops frames on
 * the host, TrainConvVAE.swift:168-219), fused the way the hardware wants:
 * tcgen05 implicit-GEMM convolutions (tf32 operands, fp32 accumulation),
 * GroupNorm+SiLU in two memory passes, multi-tensor Adam in one launch. */

/* Conv2d geometry.  The input is (n, c, h, w); with up = 1 it is the source
 * of a nearest x2 upsample cropped to (up_h, up_w) (the decoder's
 * "upsample2x + conv", ConvGPU.swift:380-399), read without materialising the
 * upsampled tensor; up_h is 2h or 2h - 1 and up_w is 2w or 2w - 1 (anything
 * else is YL_ERR_SHAPE).  Output size: (in + 2*pad - k)/stride + 1 per axis
 * (ConvGPU.swift:58-59).  Weights are (oc, c, k, k) = the reference's
 * (oc, ic*k*k) (ConvGPU.swift:18); bias has oc entries. */
typedef struct yl_conv_desc {
  int n, c, h, w;
  int oc, k, stride, pad;
  int up, up_h, up_w;
  int layout; /* yl_layout of every activation argument */
} yl_conv_desc;
yl_status yl_conv2d_out_shape(const yl_conv_desc* d, int* oh, int* ow);
/* ConvLayerGPU.forward (ConvGPU.swift:57-64): y = conv(x, w) + b (+ residual). */
yl_status yl_conv2d_fwd(yl_ctx* ctx, const yl_conv_desc* d, const float* x, const float* w,
                        const float* b, const float* residual, float* y);
/* ConvLayerGPU.backward dX (ConvGPU.swift:71-79): convBackInputS1 for stride
 * 1, matmul(W, dOut, transA) + col2im for stride 2; with up = 1 the result is
 * the downsample2x (2x2 sum) of the upsampled-input gradient. */
yl_status yl_conv2d_bwd_data(yl_ctx* ctx, const yl_conv_desc* d, const float* dy, const float* w,
                             float* dx);
/* ConvLayerGPU.backward dW/db (ConvGPU.swift:68-69): gradW + biasRowGrad,
 * summed over the batch.  dw or db may be NULL. */
yl_status yl_conv2d_bwd_filter(yl_ctx* ctx, const yl_conv_desc* d, const float* x, const float* dy,
                               float* dw, float* db);
/* Transposed convolution = the adjoint of the conv `d` describes: x has the
 * conv's output shape, y its input shape, b has c entries.  Its backward
 * passes are the conv's forward and its filter gradient with roles swapped
 * (the reference's stride-2 dX path, ConvGPU.swift:75-78). */
yl_status yl_conv_transpose2d_fwd(yl_ctx* ctx, const yl_conv_desc* d, const float* x,
                                  const float* w, const float* b, float* y);
yl_status yl_conv_transpose2d_bwd_data(yl_ctx* ctx, const yl_conv_desc* d, const float* dy,
                                       const float* w, float* dx);
yl_status yl_conv_transpose2d_bwd_filter(yl_ctx* ctx, const yl_conv_desc* d, const float* x,
                                         const float* dy, float* dw, float* db);

/* GroupNorm + optional SiLU (groupNorm, GpuSessionOps.swift:121-131, and the
 * activation that follows it).  mode 0: torch.nn.GroupNorm (biased variance
 * + eps, affine gamma/beta, either may be NULL); mode 1: the reference's rule
 * var = max(E[x^2] - E[x]^2, 1e-5), no eps (MetalKernelSourcesC.swift:35-38).
 * Channels per group must be a multiple of 4.  mean_out / rstd_out (n*groups,
 * optional) receive the statistics for the backward call. */
yl_status yl_groupnorm_silu_fwd(yl_ctx* ctx, const float* x, int n, int c, int h, int w,
                                int layout, int groups, float eps, int mode, const float* gamma,
                                const float* beta, int apply_silu, float* y, float* mean_out,
                                float* rstd_out);
/* yl_groupnorm_silu_fwd for callers that may not allocate device memory
 * during the call (a host whose allocator refuses growth after start-up, or
 * code that must not add allocations to work it is recording).  It has no
 * counterpart in the reference, whose every op allocates its output.
 * The statistics partials live in a fixed 1 MiB array inside the library
 * (n * chunks * 2 * groups doubles, chunks <= 592/n + 1); larger requests
 * return YL_ERR_SHAPE without launching.  NHWC layout only; mean_out and
 * rstd_out (n*groups) are required.  The first call on each device looks the
 * array up (cudaGetSymbolAddress) and must come before any stream capture;
 * the address is kept for the life of the process, so a cudaDeviceReset of
 * that device is not supported afterwards.  Nothing needs to start at zero.
 * Calls that overlap on one device share the array and race: serialise them. */
yl_status yl_groupnorm_silu_fwd_noalloc(yl_ctx* ctx, const float* x, int n, int c, int h, int w,
                                        int groups, float eps, int mode, const float* gamma,
                                        const float* beta, int apply_silu, float* y,
                                        float* mean_out, float* rstd_out);
/* encodeGroupNormGrad (GpuSessionNormGrad.swift:10-24) with the affine and
 * SiLU terms: dx (+= addend when not NULL), dgamma/dbeta summed over (n, h, w).
 * mean/rstd may be NULL (recomputed). */
yl_status yl_groupnorm_silu_bwd(yl_ctx* ctx, const float* x, const float* dy, int n, int c, int h,
                                int w, int layout, int groups, float eps, int mode,
                                const float* gamma, const float* beta, int apply_silu,
                                const float* mean, const float* rstd, const float* addend,
                                float* dx, float* dgamma, float* dbeta);

/* LinearGPU (DenoiserMLP.swift:20-71): Y = X W^T + b, X (n, ic), W (oc, ic);
 * backward dX = dY W, dW = dY^T X, db = sumCols(dY); outputs may be NULL. */
yl_status yl_linear_fwd(yl_ctx* ctx, const float* X, const float* W, const float* b, float* Y,
                        int n, int ic, int oc);
yl_status yl_linear_bwd(yl_ctx* ctx, const float* X, const float* W, const float* dY, float* dX,
                        float* dW, float* db, int n, int ic, int oc);

/* Sinusoidal embedding of t[n] (device).  variant 0: motionTimeEmbedding
 * (MotionPlanner.swift:155-165: interleaved sin/cos, base 1000, t clamped to
 * [0,1]); variant 1: timestep_embedding (src/diffusion.py:6-10: [cos | sin],
 * base 10000). */
yl_status yl_timestep_embedding(yl_ctx* ctx, const float* t, int n, int dim, int variant,
                                float* out);

/* Multi-tensor Adam in one launch (adamUpdate per tensor, ConvGPU.swift:83-86,
 * preceded by sanitizeGrads, GradSanitize.swift:18-101): g *= grad_scale;
 * sanitize != 0 zeroes NaN/Inf; clip_max_norm > 0 scales all gradients by
 * max_norm/norm when the global L2 norm exceeds it (norm_out_dev, optional,
 * receives the norm).  Bias correction uses t >= 1. */
typedef struct yl_adam_tensor {
  float* param;
  const float* grad;
  float* m;
  float* v;
  long long n;
} yl_adam_tensor;
yl_status yl_adam_multi(yl_ctx* ctx, const yl_adam_tensor* table, int count, float lr, float b1,
                        float b2, float eps, int t, float grad_scale, float clip_max_norm,
                        int sanitize, float* norm_out_dev);

/* VAE latent head (ConvVAEGPU encode tail, split2 + expHalf + randn + fma,
 * GpuSessionOps.swift:472-535): e is (n, 2c, h, w) = [mu | logvar];
 * z = mu + exp(0.5*clamp(logvar,-10,10)) * eps, eps[img][ch][p] =
 * randn(trainingNoiseSeed(step, img), ch*h*w + p) (ConvVAEHelpers.swift:33-37). */
yl_status yl_vae_latent_head_fwd(yl_ctx* ctx, const float* e, int n, int c, int h, int w,
                                 int layout, int64_t step, float* z);
/* vaeGrad + merge2 (GpuSessionOps.swift:502-563) with the KL averaged over the
 * n*c*h*w latent elements (ConvGPU.swift:435-438): de = [dmu | dlogvar]. */
yl_status yl_vae_latent_head_bwd(yl_ctx* ctx, const float* e, const float* dz, int n, int c, int h,
                                 int w, int layout, int64_t step, float beta, float* de);
/* L1 reconstruction + beta * mean KL: drecon = sign(recon - target)/n_recon
 * (encodeL1Grad, GpuSessionOps.swift:134-143); loss_dev (device scalar) =
 * mean|recon - target| + beta * KL_sum / (n*c_lat*h_lat*w_lat).  mu_logvar may
 * be NULL (pure L1). */
yl_status yl_loss_l1_kl(yl_ctx* ctx, const float* recon, const float* target, size_t n_recon,
                        const float* mu_logvar, int n, int c_lat, int h_lat, int w_lat, int layout,
                        float beta, float* drecon, float* loss_dev);
/* Sobel edge loss of each image (encodeSobelEdgeGrad, GpuSessionEdgeLoss.swift:
 * 10-41; sobelEdgeLoss / sobelEdgeGradCPU, LossFunctions.swift:29-66, 194-235):
 * loss[i] = mean over h*w of (|grad luma recon| - |grad luma target|)^2 with
 * 3x3 Sobel on the interior pixels (luma = 0.2126 R + 0.7152 G + 0.0722 B);
 * grad = dloss/drecon in the input layout (channels 0..2 written).  recon and
 * target are [n][3][h][w] (YL_LAYOUT_NCHW) or [n][h][w][ld] (YL_LAYOUT_NHWC,
 * ld >= 3).  grad or loss (device, n floats) may be NULL. */
yl_status yl_sobel_edge_loss(yl_ctx* ctx, const float* recon, const float* target, int n, int h,
                             int w, int layout, int ld, float* grad, float* loss);
/* Layered 8-channel loss of each image (layered_grad_kernel,
 * MetalKernelSourcesB.swift:414-449; layeredLoss / layeredLossGradient,
 * LayeredVAELoss.swift:129-196).  recon and target are [n][8][plane] CHW planes
 * (bg R G B | obj R G B | mask | light), comp is [n][3][plane] (the frame):
 * loss[i] = layer_weight * mean over 8*plane of (recon - target)^2
 *         + compose_weight * mean over 3*plane of
 *           (clamp((bg*(1-m) + obj*m) * light, 0, 1) - comp)^2,
 * grad = dloss/drecon, [n][8][plane] (the clamp passes the gradient only
 * strictly inside (0, 1)).  grad or loss (device, n floats) may be NULL. */
yl_status yl_layered_loss(yl_ctx* ctx, const float* recon, const float* target, const float* comp,
                          int n, long long plane, float layer_weight, float compose_weight,
                          float* grad, float* loss);
/* composeCHW (LayeredVAELoss.swift:95-110): out [n][3][plane] =
 * clamp((bg*(1-m) + obj*m) * light, 0, 1) per channel. */
yl_status yl_layered_compose(yl_ctx* ctx, const float* recon, int n, long long plane, float* out);

/* ------------------------------------------------ data-parallel communicator
 * NCCL over NVLink/NVSwitch, one rank per GPU.  Rank 0 creates the id; the
 * caller distributes its bytes (the reference has no multi-GPU path; its
 * closest relative is the per-frame gradient sum, TrainConvVAE.swift:177-217). */
#define YL_COMM_ID_BYTES 128
yl_status yl_comm_get_unique_id(uint8_t* out_id /* YL_COMM_ID_BYTES */);
/* The communicator is non-blocking: set-up and every collective that NCCL
 * finishes on its own threads are waited for with a deadline (300 s for
 * yl_comm_init; timeout_s for yl_comm_init_timeout), and a rank that never
 * joins makes the call return YL_ERR_TIMEOUT instead of blocking for good.
 * NCCL may use at most 8 CTAs per collective (YL_NCCL_MAX_CTAS in the
 * environment overrides it; 0 keeps NCCL's default). */
yl_status yl_comm_init(yl_ctx* ctx, const uint8_t* id, int rank, int world, yl_comm** out);
yl_status yl_comm_init_timeout(yl_ctx* ctx, const uint8_t* id, int rank, int world,
                               double timeout_s, yl_comm** out);
yl_status yl_comm_destroy(yl_comm* comm);
/* Aborts outstanding collectives (failure handling); destroy afterwards. */
yl_status yl_comm_abort(yl_comm* comm);
/* In-place sum over ranks, ordered on `stream` (NULL: the communicator's stream). */
yl_status yl_allreduce_sum(yl_comm* comm, float* buf, size_t n, void* stream);

/* ------------------------------------------------------- training step
 * The joint VAE + motion-net step (TrainContext.runStep,
 * TrainConvVAE.swift:327-362, and runMotionStepPixel, MotionTrainer.swift:
 * 214-260, re-expressed for the conv VAE and motion U-Net): encoder means of
 * frames 0 and 16 (no gradient), VAE forward/backward on frame k with
 * L1 + beta*KL, U-Net on [zA | zB | lerp(zA, zB, t)] predicting mu(frame k)
 * with MSE, gradient all-reduce overlapped with backward, Adam (0.9, 0.999,
 * 1e-8).  Nothing is allocated after the first step. */
typedef struct yl_trainer_config {
  int batch;            /* frame-pair samples per GPU */
  int height, width;    /* frame size, multiples of 8 (854 wide frames are padded to 856) */
  uint64_t seed;        /* parameter initialisation */
  float lr_vae, lr_motion;
  float beta_kl;        /* KL weight (1e-6), KL averaged per latent element */
  float clip_max_norm;  /* > 0: sanitizeGrads semantics (NaN->0 + global L2 clip); 0: off */
  int train_vae, train_motion;
  size_t bucket_bytes;  /* all-reduce bucket size; 0 = 25 MB */
  int profile;          /* time every conv / GroupNorm launch with CUDA events */
} yl_trainer_config;
yl_status yl_trainer_create(yl_ctx* ctx, const yl_trainer_config* cfg, yl_comm* comm_or_null,
                            yl_trainer** out);
/* A trainer borrows its communicator: destroy the trainer before the
 * communicator (yl_comm_abort may come first; yl_comm_destroy may not). */
yl_status yl_trainer_destroy(yl_trainer* tr);
/* frames: device, [3][batch][3][height][width] fp32 in [-1, 1] = frame 0,
 * frame 16 and frame k of every sample (NCHW); t: device [batch] (k/16);
 * losses_out (device [2], may be NULL): VAE loss, motion loss (rank mean). */
yl_status yl_trainer_step(yl_trainer* tr, const float* frames, const float* t, float* losses_out);
/* The same from host buffers (pinned memory makes the copies asynchronous):
 * copies in, runs the step, copies the two losses back and synchronizes. */
yl_status yl_trainer_step_host(yl_trainer* tr, const float* frames_host, const float* t_host,
                               float* losses_host);
/* Replace the runtime options (learning rates, which parts train, profiling);
 * batch and frame size must match creation. */
yl_status yl_trainer_set_config(yl_trainer* tr, const yl_trainer_config* cfg);
/* The inference path of Interpolation.swift:263-373 without the file and
 * video IO: frame_a, frame_b are device [3][height][width] frames (the
 * trainer's size), times[count] (host) the frame times in [0, 1].  Writes
 * count device frames to frames_out ([count][3][height][width]): the first and
 * last are copies of A and B; each interior frame decodes the motion net's
 * predicted latent for (encoder mean of A, encoder mean of B, t) (mode 0) or
 * the smoothstep lerp of the two means (mode 1, the reference's path without
 * a motion network, Interpolation.swift:340-343).  Interior frames are decoded
 * in groups of the trainer's batch.  Synchronous. */
yl_status yl_trainer_interpolate(yl_trainer* tr, const float* frame_a, const float* frame_b,
                                 const float* times, int count, int mode, float* frames_out);
/* interpolationFrameCount / interpolationTimes (Interpolation.swift:47-58):
 * *count_out = max(2, round(seconds * fps)) (2 for invalid arguments); when
 * times_out is not NULL it receives count evenly spaced times 0..1. */
yl_status yl_interpolation_plan(double seconds, int fps, int max_count, float* times_out,
                                int* count_out);
/* Steps taken so far (the Adam step counter t of the last step; the next step
 * uses t + 1).  Setting it restores a checkpoint's optimizerStep
 * (Train.swift:100-114: without it resumed training restarts Adam's bias
 * correction). */
yl_status yl_trainer_get_step(yl_trainer* tr, int64_t* step);
yl_status yl_trainer_set_step(yl_trainer* tr, int64_t step);
/* which: 0 = VAE, 1 = motion U-Net.  Flat fp32 buffers on the device;
 * kind: 0 parameters, 1 gradients, 2 Adam m, 3 Adam v. */
yl_status yl_trainer_param_count(yl_trainer* tr, int which, size_t* n);
yl_status yl_trainer_buffer(yl_trainer* tr, int which, int kind, float** dev_ptr);
/* Parameter table (for checkpoints and tests): conv weights are stored
 * [oc][k*k][ic rounded up to 4] at `offset` with shape4 = (oc, ic, k, k);
 * Linear weights [oc][ic] with shape4 = (oc, ic, 0, 0); vectors (n, 1, 1, 1). */
yl_status yl_trainer_param_entry(yl_trainer* tr, int which, int index, char* name,
                                 size_t name_len, size_t* offset, int* shape4);
/* Re-derive the tf32 weight copies after parameters were written externally. */
yl_status yl_trainer_prepare_weights(yl_trainer* tr);
/* conv fprop, conv dgrad, conv wgrad, GN+SiLU fwd, GN+SiLU bwd, and (also counted
 * in classes 0/1) the forward and dX passes of the stride-1 3x3 128->128 convs at
 * the frame resolution: the step's dominant launch type */
#define YL_KERNEL_CLASSES 6
typedef struct yl_kernel_stats {
  double ms[YL_KERNEL_CLASSES];
  double flops[YL_KERNEL_CLASSES];      /* algorithmic: 2*N*Cout*Cin*k*k*OH*OW */
  double bytes[YL_KERNEL_CLASSES];
  int launches[YL_KERNEL_CLASSES];
  double exec_flops[YL_KERNEL_CLASSES]; /* 2 x the MACs the conv kernels ran */
} yl_kernel_stats;
/* Accumulated CUDA-event times of the profiled steps (cfg.profile = 1). */
yl_status yl_trainer_kernel_stats(yl_trainer* tr, yl_kernel_stats* out, int reset);
/* The same profiled conv brackets per kernel template, as of the last
 * yl_trainer_kernel_stats call: flops = algorithmic 2*N*Cout*Cin*k*k*OH*OW,
 * exec_flops = 2 x the MACs the kernel ran (zero-padded channels counted;
 * the merged-tap upsample convs run 16/36 of the algorithmic MACs).  Writes
 * min(capacity, *count) entries; *count = number of templates.  No
 * counterpart in the reference (its profileConv, Diagnostics.swift:123-201,
 * times one im2col + matmul path). */
/* Profiled data-parallel steps: device time the compute stream waited, after
 * the last backward kernel, for the gradient and loss reductions (the
 * communication backward did not hide), summed over *steps steps.  No
 * counterpart in the reference (single device). */
yl_status yl_trainer_comm_stats(yl_trainer* tr, double* exposed_ms, int* steps, int reset);
typedef struct yl_template_stats {
  char name[96];
  double ms, flops, exec_flops;
  int launches;
} yl_template_stats;
yl_status yl_trainer_template_stats(yl_trainer* tr, yl_template_stats* out, int capacity,
                                    int* count);
yl_status yl_trainer_activation_bytes(yl_trainer* tr, size_t* bytes);

/* ---------------------------------------------------------------- diagnostics
 * profileConv / runGpuBench (Diagnostics.swift:83-201): device time per launch
 * of one conv shape's forward, dX and dW kernels on NHWC buffers the call
 * allocates and frees itself (input n x h x w x c, or its x2 upsample when
 * up = 1; k x k kernel, pad k/2). */
typedef struct yl_conv_profile {
  double fprop_ms, dgrad_ms, wgrad_ms;
  double flops; /* 2 * MACs of one pass */
  int wgrad_splits;
} yl_conv_profile;
yl_status yl_profile_conv(yl_ctx* ctx, int n, int c, int h, int w, int oc, int k, int stride,
                          int up, int reps, yl_conv_profile* out);
/* One multi-tensor Adam step over n parameters split into `tensors` (<= 48)
 * tensors; *ms = average device time of one step.  Diagnostic only. */
yl_status yl_profile_adam(yl_ctx* ctx, long long n, int tensors, int reps, double* ms);
/* GroupNorm(32)+SiLU forward (statistics + apply) and backward on an
 * n x h x w x c NHWC tensor; apply_ms (may be NULL) gets the apply pass alone,
 * the training step's forward when a conv supplied the statistics. */
yl_status yl_profile_groupnorm(yl_ctx* ctx, int n, int c, int h, int w, int reps, double* fwd_ms,
                               double* bwd_ms, double* apply_ms);
/* Layered 8-channel loss + gradient on n images of `plane` pixels (synthetic
 * planes); *ms = average device time of one yl_layered_loss call. */
yl_status yl_profile_layered(yl_ctx* ctx, int n, long long plane, int reps, double* ms);
/* Failure-path probes for the bounded waits (gpuWaitOutcome,
 * GpuWaitPolicy.swift:54-61, tested by TestGroup1.swift:129): the wait probe
 * queues one kernel whose single thread waits on an mbarrier nothing arrives
 * on; the wait gives up after the context's wait limit and the next
 * yl_ctx_check_device_errors / yl_session_end returns YL_ERR_TIMEOUT.  The
 * spin queues one kernel that stays busy for `seconds` (<= 10) and ends
 * normally, so a shorter yl_session_end deadline can run out on the host. */
yl_status yl_debug_wait_probe(yl_ctx* ctx);
yl_status yl_debug_spin(yl_ctx* ctx, double seconds);

#ifdef __cplusplus
}
#endif
#endif /* YUME_C_H */
