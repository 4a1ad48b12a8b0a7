// yl_trainer.cu -- the joint VAE + motion-net training step behind the C ABI,
// data-parallel over NCCL.
//
// One step on each rank of the joint frame-pair workload, per-rank batch B
// (TrainContext.runStep, TrainConvVAE.swift:327-362, and the motion step,
// MotionTrainer.swift:214-260 / 450-485, folded into one):
//   1. encoder forward (no gradient) on frames 0 and 16 -> zA, zB (latent means)
//   2. VAE forward + L1 + beta*KL loss + backward on frame k
//   3. U-Net forward on [zA | zB | lerp(zA, zB, t)] + MSE to mu(frame k) + backward
//   4. gradient all-reduce (sum; 1/world folded into Adam), overlapped with the
//      backward passes: fixed-size buckets of the flat gradient buffer are
//      launched on a communication stream as soon as the backward frontier
//      (the lowest parameter offset whose gradient is final) passes them
//   5. one multi-tensor Adam launch per model, then the tf32 weight copies.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "yl_nets.h"
#include "yl_norm.h"
#include "yume_c.h"

using namespace yl;

#define YL_NCCL(expr)                                                                  \
  do {                                                                                 \
    ncclResult_t r_ = (expr);                                                          \
    if (r_ != ncclSuccess)                                                             \
      return ::yl::set_error(YL_ERR_NCCL, "%s failed: %s", #expr, ncclGetErrorString(r_)); \
  } while (0)

struct yl_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  cudaStream_t stream = nullptr;
};

namespace {

// Communicators are created non-blocking: every NCCL call may return
// ncclInProgress while NCCL finishes it on its own threads (communicator
// set-up, the connections of a first collective).  The call's outcome is then
// polled from ncclCommGetAsyncError with a deadline, so a peer that never
// joins ends in a status instead of a host thread blocked for good.
constexpr double kNcclCallTimeoutS = 300.0;

ncclResult_t nccl_settle(ncclComm_t comm, ncclResult_t r, double timeout_s) {
  if (r != ncclInProgress) return r;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = ncclCommGetAsyncError(comm, &st);
    if (q != ncclSuccess) return q;
    if (st != ncclInProgress) return st;
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

ncclResult_t all_reduce_sum(yl_comm* c, float* buf, size_t n, cudaStream_t stream) {
  return nccl_settle(c->comm,
                     ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, c->comm, stream),
                     kNcclCallTimeoutS);
}

yl_status nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return YL_OK;
  if (r == ncclInProgress)
    return set_error(YL_ERR_TIMEOUT, "%s: NCCL still in progress after %.0f s", what,
                     kNcclCallTimeoutS);
  return set_error(YL_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

// CTAs NCCL may use per collective: the gradient all-reduce runs beside the
// persistent conv kernels (one CTA per SM) and is hidden behind backward, so
// a few CTAs carry its bytes in time while leaving the SMs to the convs.
// YL_NCCL_MAX_CTAS overrides it (0: NCCL's default).
int nccl_max_ctas() {
  const char* e = std::getenv("YL_NCCL_MAX_CTAS");
  if (e && *e) return std::max(0, std::atoi(e));
  return 8;
}

struct Bucket {
  size_t lo, hi;
  bool launched;
};

struct Overlap {
  yl_comm* comm = nullptr;
  yl_ctx* ctx = nullptr;
  std::vector<Bucket> buckets;  // descending lo (launch order)
  size_t next = 0;
  cudaEvent_t ready_ev = nullptr;
  yl_status status = YL_OK;

  void build(size_t count, size_t bucket_floats) {
    buckets.clear();
    size_t hi = count;
    while (hi > 0) {
      size_t lo = hi > bucket_floats ? hi - bucket_floats : 0;
      buckets.push_back({lo, hi, false});
      hi = lo;
    }
  }
  void reset() {
    next = 0;
    for (auto& b : buckets) b.launched = false;
  }
};

void launch_ready(Overlap* ov, Net* net, size_t lo) {
  if (!ov->comm || ov->status != YL_OK) return;
  while (ov->next < ov->buckets.size() && lo <= ov->buckets[ov->next].lo) {
    Bucket& b = ov->buckets[ov->next];
    // the comm stream waits for the backward work queued so far, then sums the bucket
    cudaError_t e = cudaEventRecord(ov->ready_ev, ov->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ov->comm->stream, ov->ready_ev, 0);
    if (e != cudaSuccess) {
      ov->status = set_error(YL_ERR_CUDA, "bucket event: %s", cudaGetErrorString(e));
      return;
    }
    const ncclResult_t r =
        all_reduce_sum(ov->comm, net->params.g + b.lo, b.hi - b.lo, ov->comm->stream);
    if (r != ncclSuccess) {
      ov->status = nccl_status(r, "gradient bucket all-reduce");
      return;
    }
    b.launched = true;
    ++ov->next;
  }
}

void hook_fn(void* arg, Net* net, size_t lo) { launch_ready((Overlap*)arg, net, lo); }

}  // namespace

struct yl_trainer {
  yl_ctx* ctx = nullptr;
  yl_comm* comm = nullptr;
  yl_trainer_config cfg{};
  std::unique_ptr<VAE> vae;
  std::unique_ptr<UNet> unet;
  Overlap ov_vae, ov_unet;
  float *frames = nullptr, *tdev = nullptr, *za = nullptr, *zb = nullptr, *losses = nullptr;
  float *ia = nullptr, *ib = nullptr;  // interpolation: latents of A and B, one copy per slot
  cudaEvent_t comm_done = nullptr;
  int64_t step = 0;
  double prof_ms[kProfClasses] = {}, prof_flops[kProfClasses] = {}, prof_bytes[kProfClasses] = {};
  int prof_launches[kProfClasses] = {};
  double prof_exec[kProfClasses] = {};
  std::map<std::string, TemplateStat> prof_templates;
  std::map<std::string, TemplateStat> last_templates;  // as of the last kernel_stats call
  // profiled steps of a data-parallel run: the compute stream's wait for the
  // gradient and loss reductions after the last backward kernel (exposed
  // communication), one event pair per step, read in yl_trainer_comm_stats
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> comm_wait_ev;
  double comm_exposed_ms = 0.0;
  int comm_steps = 0;
};

extern "C" {

yl_status yl_comm_get_unique_id(uint8_t* out) {
  YL_CHECK(out, YL_ERR_INVALID, "yl_comm_get_unique_id: out is NULL");
  ncclUniqueId id;
  YL_NCCL(ncclGetUniqueId(&id));
  static_assert(sizeof(id) == YL_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(out, &id, sizeof(id));
  return YL_OK;
}

yl_status yl_comm_init(yl_ctx* ctx, const uint8_t* id_bytes, int rank, int world, yl_comm** out) {
  return yl_comm_init_timeout(ctx, id_bytes, rank, world, kNcclCallTimeoutS, out);
}

yl_status yl_comm_init_timeout(yl_ctx* ctx, const uint8_t* id_bytes, int rank, int world,
                               double timeout_s, yl_comm** out) {
  YL_CHECK(ctx && id_bytes && out && timeout_s > 0, YL_ERR_INVALID,
           "yl_comm_init: NULL argument or non-positive timeout");
  YL_CHECK(world >= 1 && rank >= 0 && rank < world, YL_ERR_INVALID, "yl_comm_init: rank %d of %d",
           rank, world);
  YL_CUDA(cudaSetDevice(ctx->device));
  auto* c = new yl_comm();
  c->rank = rank;
  c->world = world;
  c->device = ctx->device;
  ncclUniqueId id;
  std::memcpy(&id, id_bytes, sizeof(id));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  const int max_ctas = nccl_max_ctas();
  if (max_ctas > 0) {
    config.minCTAs = 1;
    config.maxCTAs = max_ctas;
  }
  ncclResult_t r = ncclCommInitRankConfig(&c->comm, world, id, rank, &config);
  if (c->comm) r = nccl_settle(c->comm, r, timeout_s);
  if (r != ncclSuccess) {
    if (c->comm) ncclCommAbort(c->comm);  // also ends the set-up threads of a timed-out init
    delete c;
    if (r == ncclInProgress)
      return set_error(YL_ERR_TIMEOUT,
                       "ncclCommInitRankConfig: rank %d of %d: not every rank joined in %.1f s",
                       rank, world, timeout_s);
    return set_error(YL_ERR_NCCL, "ncclCommInitRankConfig: %s", ncclGetErrorString(r));
  }
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  // the communication stream gets the higher priority so bucket reductions are
  // not starved behind queued backward kernels
  YL_CUDA(cudaStreamCreateWithPriority(&c->stream, cudaStreamNonBlocking, hi));
  *out = c;
  return YL_OK;
}

yl_status yl_comm_destroy(yl_comm* c) {
  if (!c) return YL_OK;
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->comm) {
    // a non-blocking communicator: finalize (bounded), then free; abort if a
    // peer never finishes its side
    const ncclResult_t r = nccl_settle(c->comm, ncclCommFinalize(c->comm), kNcclCallTimeoutS);
    if (r == ncclSuccess) ncclCommDestroy(c->comm);
    else ncclCommAbort(c->comm);
  }
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return YL_OK;
}

yl_status yl_comm_abort(yl_comm* c) {
  if (!c) return YL_OK;
  if (c->comm) ncclCommAbort(c->comm);
  c->comm = nullptr;
  return YL_OK;
}

yl_status yl_allreduce_sum(yl_comm* c, float* buf, size_t n, void* stream) {
  YL_CHECK(c && buf, YL_ERR_INVALID, "yl_allreduce_sum: NULL argument");
  YL_CHECK(c->comm, YL_ERR_NCCL, "yl_allreduce_sum: communicator was aborted");
  YL_TRY(nccl_status(all_reduce_sum(c, buf, n, stream ? (cudaStream_t)stream : c->stream),
                     "yl_allreduce_sum"));
  return YL_OK;
}

yl_status yl_trainer_create(yl_ctx* ctx, const yl_trainer_config* cfg, yl_comm* comm,
                            yl_trainer** out) {
  YL_CHECK(ctx && cfg && out, YL_ERR_INVALID, "yl_trainer_create: NULL argument");
  YL_CHECK(cfg->batch >= 1 && cfg->height % 8 == 0 && cfg->width % 8 == 0 && cfg->height >= 16 &&
               cfg->width >= 16,
           YL_ERR_SHAPE, "yl_trainer_create: batch %d, frame %dx%d (multiples of 8 required)",
           cfg->batch, cfg->height, cfg->width);
  YL_CUDA(cudaSetDevice(ctx->device));
  auto tr = std::make_unique<yl_trainer>();
  tr->ctx = ctx;
  tr->comm = comm;
  tr->cfg = *cfg;
  const int B = cfg->batch;
  tr->vae = std::make_unique<VAE>();
  tr->vae->ctx = ctx;
  YL_TRY(tr->vae->build(ctx, B, cfg->height, cfg->width, cfg->seed));
  tr->vae->dom_pixels = (long long)cfg->height * cfg->width;
  tr->unet = std::make_unique<UNet>();
  tr->unet->ctx = ctx;
  YL_TRY(tr->unet->build(ctx, B, tr->vae->hl, tr->vae->wl, cfg->seed));
  const size_t frame = (size_t)3 * cfg->height * cfg->width;
  YL_TRY(tr->vae->arena.alloc(3 * B * frame, &tr->frames));
  YL_TRY(tr->vae->arena.alloc(64, &tr->tdev));
  YL_TRY(tr->vae->arena.alloc(64, &tr->losses));
  const size_t lat = (size_t)B * tr->vae->hl * tr->vae->wl * VAE::kLatent;
  YL_TRY(tr->vae->arena.alloc(lat, &tr->za));
  YL_TRY(tr->vae->arena.alloc(lat, &tr->zb));
  YL_TRY(tr->vae->arena.alloc(lat, &tr->ia));
  YL_TRY(tr->vae->arena.alloc(lat, &tr->ib));
  YL_CUDA(cudaEventCreateWithFlags(&tr->comm_done, cudaEventDisableTiming));
  const size_t bucket_floats = (cfg->bucket_bytes ? cfg->bucket_bytes : (25u << 20)) / 4;
  Overlap* ovs[2] = {&tr->ov_vae, &tr->ov_unet};
  Net* nets[2] = {tr->vae.get(), tr->unet.get()};
  for (int i = 0; i < 2; ++i) {
    ovs[i]->comm = comm && comm->world > 1 ? comm : nullptr;
    ovs[i]->ctx = ctx;
    ovs[i]->build(nets[i]->params.count, bucket_floats);
    YL_CUDA(cudaEventCreateWithFlags(&ovs[i]->ready_ev, cudaEventDisableTiming));
    nets[i]->hook = hook_fn;
    nets[i]->hook_arg = ovs[i];
  }
  YL_TRY(tr->vae->prepare_weights());
  YL_TRY(tr->unet->prepare_weights());
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  *out = tr.release();
  return YL_OK;
}

yl_status yl_trainer_destroy(yl_trainer* tr) {
  if (!tr) return YL_OK;
  cudaSetDevice(tr->ctx->device);
  cudaStreamSynchronize(tr->ctx->stream);
  if (tr->comm && tr->comm->stream) cudaStreamSynchronize(tr->comm->stream);
  cudaEventDestroy(tr->comm_done);
  cudaEventDestroy(tr->ov_vae.ready_ev);
  cudaEventDestroy(tr->ov_unet.ready_ev);
  delete tr;
  return YL_OK;
}

static yl_status adam_step(yl_trainer* tr, Net& net, float lr, float scale) {
  AdamTensor t{net.params.w, net.params.g, net.params.m, net.params.v,
               (long long)net.params.count};
  const float clip = tr->cfg.clip_max_norm;
  YL_TRY(adam_multi(tr->ctx, &t, 1, lr, 0.9f, 0.999f, 1e-8f, (int)tr->step, scale, clip,
                    clip > 0.f ? 1 : 0, nullptr));
  return net.prepare_weights();
}

yl_status yl_trainer_step(yl_trainer* tr, const float* frames, const float* t, float* losses_out) {
  YL_CHECK(tr && frames && t, YL_ERR_INVALID, "yl_trainer_step: NULL argument");
  yl_ctx* ctx = tr->ctx;
  VAE& vae = *tr->vae;
  UNet& unet = *tr->unet;
  const int B = tr->cfg.batch, H = tr->cfg.height, W = tr->cfg.width;
  const size_t set = (size_t)B * 3 * H * W;
  const bool train_vae = tr->cfg.train_vae != 0, train_motion = tr->cfg.train_motion != 0;
  tr->step += 1;
  tr->ov_vae.reset();
  tr->ov_unet.reset();
  vae.profiling = unet.profiling = tr->cfg.profile != 0;
  YL_CUDA(cudaMemsetAsync(tr->losses, 0, 2 * sizeof(float), ctx->stream));
  if (train_motion) {  // endpoints: encoder means of frames 0 and 16, no gradient
    YL_TRY(frames_to_nhwc4(ctx, frames, B, H, W, vae.x_in.p, 1));
    YL_TRY(vae.encode());
    YL_TRY(copy_mu(ctx, vae.e, tr->za, VAE::kLatent));
    YL_TRY(frames_to_nhwc4(ctx, frames + set, B, H, W, vae.x_in.p, 1));
    YL_TRY(vae.encode());
    YL_TRY(copy_mu(ctx, vae.e, tr->zb, VAE::kLatent));
  }
  // the motion net's forward + backward; its gradient buckets go to the
  // communication stream as its backward frontier passes them
  auto motion_step = [&]() -> yl_status {
    YL_TRY(unet.set_inputs(tr->za, tr->zb, VAE::kLatent, t));
    YL_TRY(unet.forward());
    YL_TRY(mse_head(ctx, unet.pred.p, unet.target.p, unet.pred.pixels(), unet.pred.ld,
                    UNet::kLat, unet.dpred.p, tr->losses + 1));
    YL_TRY(unet.backward());
    launch_ready(&tr->ov_unet, &unet, 0);
    return tr->ov_unet.status;
  };
  YL_TRY(frames_to_nhwc4(ctx, frames + 2 * set, B, H, W, vae.x_in.p, 1));
  if (train_vae) {
    // the reconstruction target keeps the frame's fp32 values
    YL_TRY(frames_to_nhwc4(ctx, frames + 2 * set, B, H, W, vae.x_tgt.p, 0));
    YL_TRY(vae.forward_train(tr->step));
    YL_TRY(l1_kl_head(ctx, vae.recon.p, vae.x_tgt.p, vae.recon.pixels(), 4, 3, vae.e.p, vae.e.ld,
                      vae.e.pixels(), VAE::kLatent, tr->cfg.beta_kl, vae.drecon.p, tr->losses));
    if (train_motion) {
      // the motion step needs only the encoder mean of frame k: it runs before
      // the VAE backward, so its whole gradient all-reduce hides behind that
      // backward and only the VAE's last bucket is left after the compute
      YL_TRY(copy_mu(ctx, vae.e, unet.target.p, VAE::kLatent));
      YL_TRY(motion_step());
    }
    YL_TRY(vae.backward(tr->step, tr->cfg.beta_kl));
    launch_ready(&tr->ov_vae, &vae, 0);
    YL_TRY(tr->ov_vae.status);
  } else if (train_motion) {
    YL_TRY(vae.encode());
    YL_TRY(copy_mu(ctx, vae.e, unet.target.p, VAE::kLatent));
    YL_TRY(motion_step());
  }
  float scale = 1.f;
  if (tr->comm && tr->comm->world > 1) {
    cudaEvent_t w0 = nullptr, w1 = nullptr;
    if (tr->cfg.profile) {
      YL_CUDA(cudaEventCreate(&w0));
      YL_CUDA(cudaEventCreate(&w1));
      YL_CUDA(cudaEventRecord(w0, ctx->stream));
    }
    // the step's loss values are averaged across ranks too (after all queued work)
    YL_CUDA(cudaEventRecord(tr->ov_vae.ready_ev, ctx->stream));
    YL_CUDA(cudaStreamWaitEvent(tr->comm->stream, tr->ov_vae.ready_ev, 0));
    YL_TRY(nccl_status(all_reduce_sum(tr->comm, tr->losses, 2, tr->comm->stream),
                       "loss all-reduce"));
    YL_CUDA(cudaEventRecord(tr->comm_done, tr->comm->stream));
    YL_CUDA(cudaStreamWaitEvent(ctx->stream, tr->comm_done, 0));
    if (w0) {
      YL_CUDA(cudaEventRecord(w1, ctx->stream));
      tr->comm_wait_ev.push_back({w0, w1});
    }
    scale = 1.f / (float)tr->comm->world;
  }
  if (train_vae) YL_TRY(adam_step(tr, vae, tr->cfg.lr_vae, scale));
  if (train_motion) YL_TRY(adam_step(tr, unet, tr->cfg.lr_motion, scale));
  if (losses_out) {
    if (scale != 1.f) YL_TRY(yl_smul(ctx, scale, tr->losses, losses_out, 2));
    else YL_CUDA(cudaMemcpyAsync(losses_out, tr->losses, 2 * sizeof(float),
                                 cudaMemcpyDeviceToDevice, ctx->stream));
  }
  return YL_OK;
}

yl_status yl_trainer_step_host(yl_trainer* tr, const float* frames_host, const float* t_host,
                               float* losses_host) {
  YL_CHECK(tr && frames_host && t_host, YL_ERR_INVALID, "yl_trainer_step_host: NULL argument");
  yl_ctx* ctx = tr->ctx;
  const size_t n = (size_t)3 * tr->cfg.batch * 3 * tr->cfg.height * tr->cfg.width;
  YL_CUDA(cudaMemcpyAsync(tr->frames, frames_host, n * sizeof(float), cudaMemcpyHostToDevice,
                          ctx->stream));
  YL_CUDA(cudaMemcpyAsync(tr->tdev, t_host, tr->cfg.batch * sizeof(float), cudaMemcpyHostToDevice,
                          ctx->stream));
  YL_TRY(yl_trainer_step(tr, tr->frames, tr->tdev, tr->losses + 8));
  if (losses_host) {
    YL_CUDA(cudaMemcpyAsync(losses_host, tr->losses + 8, 2 * sizeof(float), cudaMemcpyDeviceToHost,
                            ctx->stream));
  }
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  return yl_ctx_check_device_errors(ctx);
}

// ------------------------------------------------------------------ inference
// z[slot][i] = a[slot][i] + (b[slot][i] - a[slot][i]) * s[slot]
__global__ void latent_lerp_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                   const float* __restrict__ s, long long per, int n,
                                   float* __restrict__ z) {
  const long long total = per * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const float k = s[i / per];
    z[i] = a[i] + (b[i] - a[i]) * k;
  }
}

static double smoothstep_d(double t) {  // Interpolation.swift:64-69
  if (!std::isfinite(t)) return 0.0;
  const double x = std::min(std::max(t, 0.0), 1.0);
  return x * x * (3.0 - 2.0 * x);
}

yl_status yl_interpolation_plan(double seconds, int fps, int max_count, float* times_out,
                                int* count_out) {
  YL_CHECK(count_out, YL_ERR_INVALID, "yl_interpolation_plan: NULL count");
  int count = 2;  // interpolationFrameCount (Interpolation.swift:47-51)
  if (std::isfinite(seconds) && seconds > 0 && fps > 0)
    count = std::max(2, (int)std::lround(seconds * (double)fps));
  *count_out = count;
  if (!times_out) return YL_OK;
  YL_CHECK(max_count >= count, YL_ERR_SHAPE, "yl_interpolation_plan: %d frames, room for %d",
           count, max_count);
  for (int i = 0; i < count; ++i)  // interpolationTimes (Interpolation.swift:54-58)
    times_out[i] = (float)((double)i / (double)(count - 1));
  return YL_OK;
}

yl_status yl_trainer_interpolate(yl_trainer* tr, const float* frame_a, const float* frame_b,
                                 const float* times, int count, int mode, float* frames_out) {
  YL_CHECK(tr && frame_a && frame_b && times && frames_out, YL_ERR_INVALID,
           "yl_trainer_interpolate: NULL argument");
  YL_CHECK(count >= 2 && (mode == 0 || mode == 1), YL_ERR_INVALID,
           "yl_trainer_interpolate: count %d, mode %d", count, mode);
  yl_ctx* ctx = tr->ctx;
  VAE& vae = *tr->vae;
  UNet& unet = *tr->unet;
  vae.profiling = unet.profiling = false;
  const int B = tr->cfg.batch, H = tr->cfg.height, W = tr->cfg.width;
  const size_t F = (size_t)3 * H * W, px = (size_t)H * W;
  const size_t L = (size_t)vae.hl * vae.wl * VAE::kLatent;
  // latents of A and B: the encoder means, deterministic (encodeLatent,
  // Interpolation.swift:157-170); unused slots hold copies of A
  for (int b = 0; b < B; ++b)
    YL_TRY(frames_to_nhwc4(ctx, b == 1 ? frame_b : frame_a, 1, H, W, vae.x_in.p + b * px * 4, 1));
  YL_TRY(vae.encode());
  YL_TRY(copy_mu(ctx, vae.e, tr->za, VAE::kLatent));
  const float* mu_b = tr->za + L;
  if (B == 1) {
    YL_TRY(frames_to_nhwc4(ctx, frame_b, 1, H, W, vae.x_in.p, 1));
    YL_TRY(vae.encode());
    YL_TRY(copy_mu(ctx, vae.e, tr->zb, VAE::kLatent));
    mu_b = tr->zb;
  }
  for (int b = 0; b < B; ++b) {
    YL_CUDA(cudaMemcpyAsync(tr->ia + b * L, tr->za, L * sizeof(float), cudaMemcpyDeviceToDevice,
                            ctx->stream));
    YL_CUDA(cudaMemcpyAsync(tr->ib + b * L, mu_b, L * sizeof(float), cudaMemcpyDeviceToDevice,
                            ctx->stream));
  }
  // the first and last frames are the inputs themselves (Interpolation.swift:348-353)
  YL_CUDA(cudaMemcpyAsync(frames_out, frame_a, F * sizeof(float), cudaMemcpyDeviceToDevice,
                          ctx->stream));
  YL_CUDA(cudaMemcpyAsync(frames_out + (size_t)(count - 1) * F, frame_b, F * sizeof(float),
                          cudaMemcpyDeviceToDevice, ctx->stream));
  std::vector<float> tv(B);
  for (int i0 = 1; i0 < count - 1; i0 += B) {
    const int nv = std::min(B, count - 1 - i0);
    for (int b = 0; b < B; ++b) {
      const double t = times[i0 + std::min(b, nv - 1)];
      tv[b] = (float)(mode == 0 ? t : smoothstep_d(t));
    }
    YL_CUDA(cudaMemcpyAsync(tr->tdev, tv.data(), B * sizeof(float), cudaMemcpyHostToDevice,
                            ctx->stream));
    if (mode == 0) {  // the motion net's prediction (lerp + correction)
      YL_TRY(unet.set_inputs(tr->ia, tr->ib, VAE::kLatent, tr->tdev));
      YL_TRY(unet.forward());
      YL_CUDA(cudaMemcpyAsync(vae.z.p, unet.pred.p, B * L * sizeof(float),
                              cudaMemcpyDeviceToDevice, ctx->stream));
    } else {  // smoothstep lerp of the latents (Interpolation.swift:340-343)
      latent_lerp_kernel<<<grid_1d((long long)B * L, 256), 256, 0, ctx->stream>>>(
          tr->ia, tr->ib, tr->tdev, (long long)L, B, vae.z.p);
      YL_TRY(check_launch("latent_lerp_kernel"));
    }
    YL_TRY(vae.decode());
    YL_TRY(nhwc_to_nchw(ctx, vae.recon.p, frames_out + (size_t)i0 * F, nv, 3, (long long)px, 4));
    // tv is reused by the next chunk: the upload must have left the host buffer
    YL_CUDA(cudaStreamSynchronize(ctx->stream));
  }
  return yl_ctx_check_device_errors(ctx);
}

yl_status yl_trainer_get_step(yl_trainer* tr, int64_t* step) {
  YL_CHECK(tr && step, YL_ERR_INVALID, "yl_trainer_get_step: NULL argument");
  *step = tr->step;
  return YL_OK;
}

yl_status yl_trainer_set_step(yl_trainer* tr, int64_t step) {
  YL_CHECK(tr && step >= 0, YL_ERR_INVALID, "yl_trainer_set_step: bad argument");
  tr->step = step;
  return YL_OK;
}

yl_status yl_trainer_param_count(yl_trainer* tr, int which, size_t* n) {
  YL_CHECK(tr && n && (which == 0 || which == 1), YL_ERR_INVALID, "yl_trainer_param_count");
  *n = which == 0 ? tr->vae->params.count : tr->unet->params.count;
  return YL_OK;
}

yl_status yl_trainer_buffer(yl_trainer* tr, int which, int kind, float** dev_ptr) {
  YL_CHECK(tr && dev_ptr && (which == 0 || which == 1) && kind >= 0 && kind <= 3, YL_ERR_INVALID,
           "yl_trainer_buffer: bad argument");
  ParamSet& p = which == 0 ? tr->vae->params : tr->unet->params;
  float* b[4] = {p.w, p.g, p.m, p.v};
  *dev_ptr = b[kind];
  return YL_OK;
}

yl_status yl_trainer_param_entry(yl_trainer* tr, int which, int index, char* name,
                                 size_t name_len, size_t* offset, int* shape4) {
  YL_CHECK(tr && (which == 0 || which == 1), YL_ERR_INVALID, "yl_trainer_param_entry");
  Net& net = which == 0 ? (Net&)*tr->vae : (Net&)*tr->unet;
  if (index < 0 || index >= (int)net.param_table.size())
    return set_error(YL_ERR_INVALID, "parameter index %d out of range", index);
  const ParamEntry& e = net.param_table[index];
  if (name && name_len) {
    std::strncpy(name, e.name.c_str(), name_len - 1);
    name[name_len - 1] = 0;
  }
  if (offset) *offset = e.offset;
  if (shape4) {
    shape4[0] = e.d0;
    shape4[1] = e.d1;
    shape4[2] = e.d2;
    shape4[3] = e.d3;
  }
  return YL_OK;
}

yl_status yl_trainer_prepare_weights(yl_trainer* tr) {
  YL_CHECK(tr, YL_ERR_INVALID, "yl_trainer_prepare_weights: NULL");
  YL_TRY(tr->vae->prepare_weights());
  return tr->unet->prepare_weights();
}

yl_status yl_trainer_kernel_stats(yl_trainer* tr, yl_kernel_stats* out, int reset) {
  YL_CHECK(tr && out, YL_ERR_INVALID, "yl_trainer_kernel_stats: NULL argument");
  // events of the profiled steps are read here, after the fact, so profiling
  // adds no synchronisation inside a step
  YL_TRY(tr->vae->prof_collect(tr->prof_ms, tr->prof_flops, tr->prof_bytes, tr->prof_launches,
                               tr->prof_exec, &tr->prof_templates));
  YL_TRY(tr->unet->prof_collect(tr->prof_ms, tr->prof_flops, tr->prof_bytes, tr->prof_launches,
                                tr->prof_exec, &tr->prof_templates));
  for (int i = 0; i < kProfClasses && i < YL_KERNEL_CLASSES; ++i) {
    out->ms[i] = tr->prof_ms[i];
    out->flops[i] = tr->prof_flops[i];
    out->bytes[i] = tr->prof_bytes[i];
    out->launches[i] = tr->prof_launches[i];
    out->exec_flops[i] = tr->prof_exec[i];
  }
  if (reset) {
    std::memset(tr->prof_ms, 0, sizeof(tr->prof_ms));
    std::memset(tr->prof_flops, 0, sizeof(tr->prof_flops));
    std::memset(tr->prof_bytes, 0, sizeof(tr->prof_bytes));
    std::memset(tr->prof_launches, 0, sizeof(tr->prof_launches));
    std::memset(tr->prof_exec, 0, sizeof(tr->prof_exec));
    tr->last_templates = std::move(tr->prof_templates);
    tr->prof_templates.clear();
  } else {
    tr->last_templates = tr->prof_templates;
  }
  return YL_OK;
}

yl_status yl_trainer_comm_stats(yl_trainer* tr, double* exposed_ms, int* steps, int reset) {
  YL_CHECK(tr && exposed_ms && steps, YL_ERR_INVALID, "yl_trainer_comm_stats: NULL argument");
  if (!tr->comm_wait_ev.empty()) YL_CUDA(cudaStreamSynchronize(tr->ctx->stream));
  for (auto& e : tr->comm_wait_ev) {
    float t = 0.f;
    YL_CUDA(cudaEventElapsedTime(&t, e.first, e.second));
    tr->comm_exposed_ms += t;
    tr->comm_steps += 1;
    cudaEventDestroy(e.first);
    cudaEventDestroy(e.second);
  }
  tr->comm_wait_ev.clear();
  *exposed_ms = tr->comm_exposed_ms;
  *steps = tr->comm_steps;
  if (reset) {
    tr->comm_exposed_ms = 0.0;
    tr->comm_steps = 0;
  }
  return YL_OK;
}

yl_status yl_trainer_template_stats(yl_trainer* tr, yl_template_stats* out, int capacity,
                                    int* count) {
  YL_CHECK(tr && count, YL_ERR_INVALID, "yl_trainer_template_stats: NULL argument");
  *count = (int)tr->last_templates.size();
  int i = 0;
  for (const auto& kv : tr->last_templates) {
    if (!out || i >= capacity) break;
    yl_template_stats& o = out[i++];
    std::memset(o.name, 0, sizeof(o.name));
    std::strncpy(o.name, kv.first.c_str(), sizeof(o.name) - 1);
    o.ms = kv.second.ms;
    o.flops = kv.second.flops;
    o.exec_flops = kv.second.exec;
    o.launches = kv.second.launches;
  }
  return YL_OK;
}

yl_status yl_trainer_set_config(yl_trainer* tr, const yl_trainer_config* cfg) {
  YL_CHECK(tr && cfg, YL_ERR_INVALID, "yl_trainer_set_config: NULL argument");
  YL_CHECK(cfg->batch == tr->cfg.batch && cfg->height == tr->cfg.height &&
               cfg->width == tr->cfg.width,
           YL_ERR_SHAPE, "yl_trainer_set_config: batch and frame size are fixed at creation");
  tr->cfg = *cfg;
  return YL_OK;
}

yl_status yl_trainer_activation_bytes(yl_trainer* tr, size_t* bytes) {
  YL_CHECK(tr && bytes, YL_ERR_INVALID, "yl_trainer_activation_bytes: NULL argument");
  *bytes = tr->vae->arena.bytes + tr->unet->arena.bytes;
  return YL_OK;
}

}  // extern "C"
