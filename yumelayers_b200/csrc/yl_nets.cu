// yl_nets.cu -- the training executor: layers, the conv VAE, the motion
// U-Net and the joint data-parallel step, on NHWC activations and one flat
// parameter buffer per model.
//
// Layer semantics follow the reference's layers -- ConvLayerGPU
// (ConvGPU.swift:11-86), ResidualBlockGPU (ResidualBlock.swift:9-53),
// LinearGPU (DenoiserMLP.swift:20-71), ConvVAEGPU encode/decode/backward
// (ConvGPU.swift:301-462), the motion net's lerp + residual prediction
// (MotionMLP.swift:39-111) and TrainContext's step (TrainConvVAE.swift:
// 327-362) -- re-expressed for the target architectures (GroupNorm32+SiLU
// residual blocks, 128/256-channel VAE, 128/256/384-level U-Net).
//
// Per step nothing is allocated after the first step: activations are
// allocated at construction, gradient temporaries come from a pool that
// stops growing after step 1, and all parameters/gradients/Adam moments of a
// model are single contiguous buffers (one multi-tensor Adam launch, one
// contiguous range per all-reduce bucket).
#include <cuda.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "yl_kernels.h"
#include "yl_nets.h"
#include "yl_norm.h"
#include "yl_ptx.cuh"

namespace yl {

// ------------------------------------------------------------------ small kernels
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t i) {
  return (float)((mix64(seed * 0x9E3779B97F4A7C15ull + i + 1) >> 40) + 0.5) / 16777216.0f;
}

// value[o][t][i] = bound * U(-1,1) for o < o_real and i < i_real, else 0.
__global__ void init_uniform_kernel(float* p, int O, int T, int I, int o_real, int i_real,
                                   float bound, uint64_t seed) {
  const long long n = (long long)O * T * I;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % I);
    const int o = (int)(idx / ((long long)T * I));
    p[idx] = (o < o_real && i < i_real) ? bound * (2.f * hash_uniform(seed, idx) - 1.f) : 0.f;
  }
}
// value[i] = mean + std * N(0,1) (Box-Muller on two hashed uniforms).
__global__ void init_normal_kernel(float* p, long long n, float mean, float stdv, uint64_t seed) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float u1 = hash_uniform(seed, 2 * i), u2 = hash_uniform(seed, 2 * i + 1);
    p[i] = mean + stdv * sqrtf(-2.f * logf(u1)) * cosf(6.2831853f * u2);
  }
}

// dst[p][dc0 + k] = src[p][k] (+ dst when accumulate), k < c (channel-slice copy).
__global__ void slice_copy_kernel(const float* __restrict__ src, int lds, float* __restrict__ dst,
                                  int ldd, long long pixels, int c4, int accumulate) {
  const long long total = pixels * c4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i % c4);
    const long long p = i / c4;
    float4 v = *reinterpret_cast<const float4*>(src + p * lds + 4 * q);
    float4* d = reinterpret_cast<float4*>(dst + p * ldd + 4 * q);
    if (accumulate) {
      const float4 o = *d;
      v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
    }
    *d = v;
  }
}

// Motion-net input (MotionMLP.swift:39-55: concat [zA | zB] and lerp(zA, zB, t)):
// out[p] = [zA | zB | (1-t) zA + t zB], 32 channels each, t per image, rounded
// to tf32 for the first conv; lerp_out keeps the fp32 lerp the prediction adds.
__global__ void motion_input_kernel(const float* __restrict__ za, const float* __restrict__ zb,
                                   int ldz, const float* __restrict__ t, long long hw, int n,
                                   int c, float* __restrict__ out, float* __restrict__ lerp_out) {
  const long long total = (long long)n * hw * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % c);
    const long long p = i / c;
    const int img = (int)(p / hw);
    const float a = za[p * ldz + k], b = zb[p * ldz + k], tt = t[img];
    float* o = out + p * 3 * c;
    o[k] = round_tf32(a);
    o[c + k] = round_tf32(b);
    const float l = (1.f - tt) * a + tt * b;
    o[2 * c + k] = round_tf32(l);
    lerp_out[p * c + k] = l;
  }
}

static yl_status copy_slice(yl_ctx* ctx, const float* src, int lds, float* dst, int ldd,
                            long long pixels, int c, int accumulate) {
  YL_CHECK(c % 4 == 0 && lds % 4 == 0 && ldd % 4 == 0, YL_ERR_SHAPE, "copy_slice: alignment");
  slice_copy_kernel<<<grid_1d(pixels * (c / 4), 256), 256, 0, ctx->stream>>>(src, lds, dst, ldd,
                                                                            pixels, c / 4,
                                                                            accumulate);
  return check_launch("slice_copy_kernel");
}

// ------------------------------------------------------------------ memory
DeviceArena::~DeviceArena() {
  for (void* p : blocks) cudaFree(p);
}
yl_status DeviceArena::alloc(size_t floats, float** out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, std::max<size_t>(floats, 64) * sizeof(float));
  if (e != cudaSuccess)
    return set_error(YL_ERR_OOM, "activation allocation of %.2f GB failed: %s",
                     floats * 4.0 / 1e9, cudaGetErrorString(e));
  blocks.push_back(p);
  bytes += floats * sizeof(float);
  *out = (float*)p;
  return YL_OK;
}

yl_status GradPool::get(size_t floats, float** out) {
  int best = -1;
  for (int i = 0; i < (int)items.size(); ++i)
    if (!items[i].used && items[i].n >= floats && (best < 0 || items[i].n < items[best].n))
      best = i;
  if (best < 0) {
    float* p = nullptr;
    YL_TRY(arena->alloc(floats, &p));
    items.push_back({p, floats, false});
    best = (int)items.size() - 1;
  }
  items[best].used = true;
  *out = items[best].p;
  return YL_OK;
}
void GradPool::put(float* p) {
  for (auto& it : items)
    if (it.p == p) it.used = false;
}

yl_status Act::make(DeviceArena& a, int n_, int h_, int w_, int c_, int ld_) {
  n = n_; h = h_; w = w_; c = c_; ld = ld_ ? ld_ : c_;
  return a.alloc((size_t)n * h * w * ld, &p);
}

// ------------------------------------------------------------------ parameters
size_t ParamSet::reserve(size_t n) {
  size_t off = count;
  count += (n + 3) & ~size_t(3);  // keep every tensor 16-byte aligned
  return off;
}
yl_status ParamSet::allocate() {
  YL_CUDA(cudaMalloc(&w, count * sizeof(float)));
  YL_CUDA(cudaMalloc(&g, count * sizeof(float)));
  YL_CUDA(cudaMalloc(&m, count * sizeof(float)));
  YL_CUDA(cudaMalloc(&v, count * sizeof(float)));
  YL_CUDA(cudaMemset(w, 0, count * sizeof(float)));
  YL_CUDA(cudaMemset(g, 0, count * sizeof(float)));
  YL_CUDA(cudaMemset(m, 0, count * sizeof(float)));
  YL_CUDA(cudaMemset(v, 0, count * sizeof(float)));
  return YL_OK;
}
ParamSet::~ParamSet() {
  cudaFree(w);
  cudaFree(g);
  cudaFree(m);
  cudaFree(v);
}

// ------------------------------------------------------------------ layers
void ConvL::setup(Net& net, const char* nm, int cin_, int cout_, int k_, int stride_, int pad_) {
  name = nm;
  cin = cin_;
  cout = cout_;
  cin_p = (cin + 3) & ~3;
  cout_p = (cout + 3) & ~3;
  k = k_;
  stride = stride_;
  pad = pad_;
  rgb = (k == 3 && stride == 1 && pad == 1) ? (cin_p == 4 ? 1 : cout_p == 4 ? 2 : 0) : 0;
  off_w = net.params.reserve((size_t)cout_p * k * k * cin_p);
  off_b = net.params.reserve(cout_p);
  net.param_table.push_back({name + ".weight", off_w, cout, cin, k, k});
  net.param_table.push_back({name + ".bias", off_b, cout, 1, 1, 1});
  net.convs.push_back(this);
}
yl_status ConvL::bind(Net& net) {
  W = net.params.w + off_w;
  b = net.params.w + off_b;
  gW = net.params.g + off_w;
  gb = net.params.g + off_b;
  YL_TRY(net.arena.alloc((size_t)cout_p * k * k * cin_p, &Wr));
  YL_TRY(net.arena.alloc((size_t)cin_p * k * k * cout_p, &Wd));
  if (rgb == 2) {
    YL_TRY(net.arena.alloc((size_t)36 * cin_p, &Wx));
    YL_TRY(net.arena.alloc((size_t)cin_p * 64, &Wx2));
  }
  return YL_OK;
}
yl_status ConvL::init(yl_ctx* ctx, uint64_t seed, bool zero) {
  const float bound = zero ? 0.f : std::sqrt(6.0f / (float)(cin * k * k));  // Kaiming-uniform
  init_uniform_kernel<<<grid_1d((long long)cout_p * k * k * cin_p, 256), 256, 0, ctx->stream>>>(
      W, cout_p, k * k, cin_p, cout, cin, bound, seed);
  YL_TRY(check_launch("init_uniform_kernel"));
  YL_CUDA(cudaMemsetAsync(b, 0, cout_p * sizeof(float), ctx->stream));
  return YL_OK;
}
// tf32-rounded copies of the weights in the fprop layout [cout][tap][cin] and
// the dgrad layout [cin][tap][cout]; run once per step after the optimizer.
void ConvL::prepare_jobs(std::vector<PermuteJob>& first, std::vector<PermuteJob>& second) const {
  const int kk = k * k;
  first.push_back({W, Wr, cout_p, kk, cin_p, cin_p, (long long)kk * cin_p, cin_p, 1, 1});
  first.push_back({W, Wd, cin_p, kk, cout_p, cout_p, 1, cin_p, (long long)kk * cin_p, 1});
  if (rgb == 2) {
    // [t*4 + co][ci] = W[co][t][ci] and [ci][t*4 + co] (from the dgrad copy), padded
    second.push_back({Wr, Wx, 9, 4, cin_p, cin_p, cin_p, 9LL * cin_p, 1, 0});
    second.push_back({Wd, Wx2, cin_p, 1, 64, 36, 36, 0, 1, 0});
  }
}

yl_status ConvL::prepare(yl_ctx* ctx) {
  std::vector<PermuteJob> a, b;
  prepare_jobs(a, b);
  for (const auto& j : a)
    YL_TRY(weight_permute(ctx, j.in, j.out, j.O, j.T, j.I_out, j.I_src, j.so, j.st, j.si, j.round));
  for (const auto& j : b)
    YL_TRY(weight_permute(ctx, j.in, j.out, j.O, j.T, j.I_out, j.I_src, j.so, j.st, j.si, j.round));
  return YL_OK;
}

// A 1x1 gather over an NHWC tensor of ps floats per pixel (c channels).
static ConvGather pointwise(const float* src, int n, int h, int w, int ps, int c) {
  ConvGather g;
  g.src = src;
  g.img_stride = (long long)h * w * ps;
  g.row_stride = w * ps;
  g.ps = ps;
  g.cin = c;
  g.hv = h;
  g.wv = w;
  g.mode = MODE_FPROP;
  g.ksize = 1;
  g.stride = 1;
  g.pad = 0;
  g.oh = h;
  g.ow = w;
  g.m_total = n * h * w;
  g.k_total = c;
  return g;
}

ConvGather ConvL::gather(const Act& x, int oh, int ow, int up, int hv, int wv) const {
  ConvGather g;
  g.src = x.p;
  g.img_stride = (long long)x.h * x.w * x.ld;
  g.row_stride = x.w * x.ld;
  g.ps = x.ld;
  g.cin = cin_p;
  g.hv = up ? hv : x.h;
  g.wv = up ? wv : x.w;
  g.up = up;
  g.mode = MODE_FPROP;
  g.ksize = k;
  g.stride = stride;
  g.pad = pad;
  g.oh = oh;
  g.ow = ow;
  g.m_total = x.n * oh * ow;
  g.k_total = k * k * cin_p;
  return g;
}

// The step's dominant launch type for the kernel-class timing: a stride-1 3x3
// 128 -> 128 conv pass at the frame resolution.
bool ConvL::dominant(const Net& net, int h, int w, int up) const {
  return k == 3 && stride == 1 && !up && cin_p == 128 && cout_p == 128 && net.dom_pixels > 0 &&
         (long long)h * w == net.dom_pixels;
}

yl_status ConvL::forward(Net& net, const Act& x, const Act& y, const float* residual, int ldr,
                         const float* bias2d, int up, int hv, int wv, GNL* gn_next) {
  if (rgb == 2 && !residual && !bias2d && !up && !gn_next) {
    // 4 output channels: z[p][t*4 + co] = x[p] . W[co][t] as one 1x1 GEMM, then the tap sum
    float* z = nullptr;
    YL_TRY(net.pool.get((size_t)x.n * x.h * x.w * 36, &z));
    ConvEpilogue e;
    e.out = z;
    e.ldo = 36;
    e.n_total = 36;
    e.round_tf32 = 0;
    net.prof_begin(0);
    YL_TRY(conv_fprop(net.ctx, pointwise(x.p, x.n, x.h, x.w, x.ld, cin_p), Wx, 36, e));
    YL_TRY(rgb_tap_sum(net.ctx, z, x.n, x.h, x.w, b, y.p, y.ld));
    net.prof_end(0, 2.0 * x.pixels() * cout * cin * k * k);
    net.pool.put(z);
    return YL_OK;
  }
  // 4 input channels (the RGB frame) take the general path: the narrow TMA
  // plan loads one zero-filled 32-channel box per tap straight from the
  // 16-byte pixels (no patch tensor), through the halo-box kernel.  An
  // upsample conv (a cut x2 grid included) runs as merged phase taps.
  ConvGather g = gather(x, y.h, y.w, up, hv, wv);
  ConvEpilogue e;
  e.out = y.p;
  e.ldo = y.ld;
  e.n_total = cout_p;
  e.bias = b;
  e.bias2d = bias2d;
  e.residual = residual;
  e.ldr = ldr;
  e.round_tf32 = 1;
  const bool fuse_gn = gn_next && gn_next->c == cout_p && conv_gn_stats_supported(cout_p, gn_next->G);
  if (fuse_gn) {
    e.gn_mean = gn_next->mean;
    e.gn_rstd = gn_next->rstd;
    e.gn_groups = gn_next->G;
    e.gn_eps = 1e-6f;
  }
  net.prof_begin(0);
  if (dominant(net, y.h, y.w, up)) net.prof_mark_dominant();
  yl_status st = conv_fprop(net.ctx, g, Wr, cout_p, e);
  net.prof_end(0, 2.0 * g.m_total * cout * cin * k * k);
  if (st == YL_OK && fuse_gn) gn_next->stats_ready = true;
  return st;
}

yl_status ConvL::backward(Net& net, const Act& x, const Act& dy, const Act* dx,
                          const float* dx_addend, int ld_addend, float* dbias2d, int up, int hv,
                          int wv) {
  yl_ctx* ctx = net.ctx;
  if (rgb == 1 && !up && !dbias2d) {
    // dW[co][t*4 + ci] = sum_p dy[p][co] * patches(x)[p][t*4 + ci]; db fused
    float *xp = nullptr, *dw = nullptr;
    YL_TRY(net.pool.get((size_t)x.n * x.h * x.w * 64, &xp));
    YL_TRY(net.pool.get((size_t)cout_p * 64, &dw));
    net.prof_begin(2);
    YL_TRY(rgb_patches(ctx, x.p, x.ld, x.n, x.h, x.w, 1, 1, xp));
    YL_TRY(conv_wgrad(ctx, dy.p, dy.ld, cout_p, pointwise(xp, x.n, x.h, x.w, 64, 64), dw, 0, gb));
    net.prof_end(2, 2.0 * x.pixels() * cout * cin * k * k);
    YL_TRY(weight_permute(ctx, dw, gW, cout_p, 1, 36, 36, 64, 0, 1, 0));
    net.pool.put(xp);
    net.pool.put(dw);
    if (dx) return set_error(YL_ERR_UNSUPPORTED, "%s: dX of a 4-channel input", name.c_str());
    return YL_OK;
  }
  if (rgb == 2 && !up && !dbias2d && dx) {
    // d[p][t*4 + co] = dy[p - (ky-1, kx-1)][co]: dX = d . Wx2^T and
    // dW[t*4 + co][ci] = sum_p d[p][t*4 + co] x[p][ci], both 1x1 GEMMs
    float *d = nullptr, *dw = nullptr, *db = nullptr;
    YL_TRY(net.pool.get((size_t)x.n * x.h * x.w * 64, &d));
    YL_TRY(net.pool.get((size_t)64 * cin_p, &dw));
    YL_TRY(net.pool.get(64, &db));
    net.prof_begin(2);
    YL_TRY(rgb_patches(ctx, dy.p, dy.ld, x.n, x.h, x.w, -1, 1, d));
    YL_TRY(conv_wgrad(ctx, d, 64, 64, pointwise(x.p, x.n, x.h, x.w, x.ld, cin_p), dw, 0, db));
    net.prof_end(2, 2.0 * x.pixels() * cout * cin * k * k);
    YL_TRY(weight_permute(ctx, dw, gW, 4, 9, cin_p, cin_p, cin_p, 4LL * cin_p, 1, 0));
    // the bias gradient is the centre tap's column sums (t = 4: no shift)
    YL_CUDA(cudaMemcpyAsync(gb, db + 16, 4 * sizeof(float), cudaMemcpyDeviceToDevice,
                            ctx->stream));
    ConvEpilogue e;
    e.out = dx->p;
    e.ldo = dx->ld;
    e.n_total = cin_p;
    e.residual = dx_addend;
    e.ldr = ld_addend;
    e.round_tf32 = 1;
    net.prof_begin(1);
    YL_TRY(conv_fprop(ctx, pointwise(d, x.n, x.h, x.w, 64, 64), Wx2, cin_p, e));
    net.prof_end(1, 2.0 * x.pixels() * cout * cin * k * k);
    net.pool.put(d);
    net.pool.put(dw);
    net.pool.put(db);
    return YL_OK;
  }
  // dW (split-K tcgen05, MN-major operands) and db (fixed-order column sums)
  ConvGather g = gather(x, dy.h, dy.w, up, hv, wv);
  net.prof_begin(2);
  // db comes out of the filter-gradient pass unless per-image sums are needed
  YL_TRY(conv_wgrad(ctx, dy.p, dy.ld, cout_p, g, gW, 0, dbias2d ? nullptr : gb));
  net.prof_end(2, 2.0 * g.m_total * cout * cin * k * k);
  if (dbias2d)
    YL_TRY(channel_sums(ctx, dy.p, dy.n, (long long)dy.h * dy.w, dy.ld, cout_p, gb, dbias2d, 0));
  if (!dx) return YL_OK;
  if (up && !dx_addend && k == 3 && pad == 1 && stride == 1) {
    // dX at the source resolution through the 16 merged phase taps (a cut x2
    // grid included)
    ConvEpilogue e;
    e.out = dx->p;
    e.ldo = dx->ld;
    e.n_total = cin_p;
    e.round_tf32 = 1;
    net.prof_begin(1);
    const yl_status st =
        conv_dgrad_upsampled(ctx, dy.p, dy.ld, cout_p, x.n, x.h, x.w, hv, wv, Wd, cin_p, e);
    net.prof_end(1, 2.0 * (double)x.n * hv * wv * cout * cin * k * k);
    if (st == YL_OK) return YL_OK;
    if (st != YL_ERR_UNSUPPORTED) return st;
  }
  // dX: the same implicit GEMM over dy with the dgrad weights
  const int oh = up ? hv : x.h, ow = up ? wv : x.w;
  float* target = dx->p;
  int ldt = dx->ld;
  if (up) {
    YL_TRY(net.pool.get((size_t)x.n * oh * ow * cin_p, &target));
    ldt = cin_p;
  }
  ConvGather gd;
  gd.src = dy.p;
  gd.img_stride = (long long)dy.h * dy.w * dy.ld;
  gd.row_stride = dy.w * dy.ld;
  gd.ps = dy.ld;
  gd.cin = cout_p;
  gd.hv = dy.h;
  gd.wv = dy.w;
  gd.up = 0;
  gd.mode = MODE_DGRAD;
  gd.ksize = k;
  gd.stride = stride;
  gd.pad = pad;
  gd.oh = oh;
  gd.ow = ow;
  gd.m_total = x.n * oh * ow;
  gd.k_total = k * k * cout_p;
  ConvEpilogue e;
  e.out = target;
  e.ldo = ldt;
  e.n_total = cin_p;
  e.residual = up ? nullptr : dx_addend;
  e.ldr = ld_addend;
  e.round_tf32 = 1;
  net.prof_begin(1);
  if (dominant(net, x.h, x.w, up)) net.prof_mark_dominant();
  YL_TRY(conv_fprop(ctx, gd, Wd, cin_p, e));
  net.prof_end(1, 2.0 * gd.m_total * cout * cin * k * k);
  if (up) {
    YL_CHECK(!dx_addend, YL_ERR_UNSUPPORTED, "upsampled conv backward with an addend");
    YL_TRY(downsample_sum_nhwc(ctx, target, oh, ow, dx->p, x.n, x.h, x.w, cin_p, cin_p, dx->ld));
    net.pool.put(target);
  }
  return YL_OK;
}

void GNL::setup(Net& net, const char* nm, int c_) {
  name = nm;
  c = c_;
  G = 32;
  off_g = net.params.reserve(c);
  off_b = net.params.reserve(c);
  net.param_table.push_back({name + ".gamma", off_g, c, 1, 1, 1});
  net.param_table.push_back({name + ".beta", off_b, c, 1, 1, 1});
}
yl_status GNL::bind(Net& net, int n) {
  gamma = net.params.w + off_g;
  beta = net.params.w + off_b;
  ggamma = net.params.g + off_g;
  gbeta = net.params.g + off_b;
  YL_TRY(net.arena.alloc((size_t)n * G, &mean));
  return net.arena.alloc((size_t)n * G, &rstd);
}
yl_status GNL::init(yl_ctx* ctx, uint64_t seed) {
  // workload init: gamma = 1 + 0.02 N(0,1), beta = 0.02 N(0,1)
  init_normal_kernel<<<grid_1d(c, 256), 256, 0, ctx->stream>>>(gamma, c, 1.f, 0.02f, seed);
  YL_TRY(check_launch("init_normal_kernel"));
  init_normal_kernel<<<grid_1d(c, 256), 256, 0, ctx->stream>>>(beta, c, 0.f, 0.02f, seed ^ 0x5bd1e995);
  return check_launch("init_normal_kernel");
}
yl_status GNL::forward(Net& net, const Act& x, const Act& y) {
  net.prof_begin(3);
  const double e4 = 4.0 * x.n * x.h * x.w * c;
  yl_status st;
  if (stats_ready) {  // the producing conv wrote mean/rstd: one read + one write
    st = gn_silu_apply(net.ctx, x.p, x.n, c, G, (long long)x.h * x.w, x.ld, mean, rstd, gamma,
                       beta, 1, y.p, y.ld, 1);
    net.prof_end(3, 0.0, 2.0 * e4);
  } else {
    st = gn_silu_forward(net.ctx, x.p, x.n, c, G, (long long)x.h * x.w, x.ld, 1e-6f, 0, gamma,
                         beta, 1, y.p, y.ld, 1, mean, rstd);
    net.prof_end(3, 0.0, 3.0 * e4);
  }
  stats_ready = false;
  return st;
}
yl_status GNL::backward(Net& net, const Act& x, const Act& dy, const Act& dx, const float* addend,
                        int ldadd) {
  net.prof_begin(4);
  yl_status st = gn_silu_backward(net.ctx, x.p, dy.p, dy.ld, x.n, c, G, (long long)x.h * x.w, x.ld,
                                  mean, rstd, gamma, beta, 1, addend, ldadd, dx.p, dx.ld, 1, ggamma,
                                  gbeta, 0);
  const double e = (double)x.n * x.h * x.w * c;
  net.prof_end(4, 0.0, 4.0 * (4 * e + (addend ? e : 0) + e));
  return st;
}

void LinL::setup(Net& net, const char* nm, int ic_, int oc_) {
  name = nm;
  ic = ic_;
  oc = oc_;
  off_w = net.params.reserve((size_t)oc * ic);
  off_b = net.params.reserve(oc);
  net.param_table.push_back({name + ".weight", off_w, oc, ic, 0, 0});  // 0: no spatial kernel
  net.param_table.push_back({name + ".bias", off_b, oc, 1, 1, 1});
}
void LinL::bind(Net& net) {
  W = net.params.w + off_w;
  b = net.params.w + off_b;
  gW = net.params.g + off_w;
  gb = net.params.g + off_b;
}
yl_status LinL::init(yl_ctx* ctx, uint64_t seed) {
  // LinearGPU init (DenoiserMLP.swift:33-40): U(-1/sqrt(ic), 1/sqrt(ic)), zero bias
  init_uniform_kernel<<<grid_1d((long long)oc * ic, 256), 256, 0, ctx->stream>>>(
      W, oc, 1, ic, oc, ic, 1.f / std::sqrt((float)ic), seed);
  YL_TRY(check_launch("init_uniform_kernel"));
  YL_CUDA(cudaMemsetAsync(b, 0, oc * sizeof(float), ctx->stream));
  return YL_OK;
}

// ------------------------------------------------------------------ residual block
void RB::setup(Net& net, const std::string& nm, int cin_, int cout_, bool temb) {
  name = nm;
  cin = cin_;
  cout = cout_;
  has_temb = temb;
  gn1.setup(net, (nm + ".norm1").c_str(), cin);
  c1.setup(net, (nm + ".conv1").c_str(), cin, cout, 3, 1, 1);
  gn2.setup(net, (nm + ".norm2").c_str(), cout);
  c2.setup(net, (nm + ".conv2").c_str(), cout, cout, 3, 1, 1);
  has_skip = cin != cout;
  if (has_skip) skip.setup(net, (nm + ".skip").c_str(), cin, cout, 1, 1, 0);
  param_lo = gn1.off_g;
}
yl_status RB::bind(Net& net, int n, int h, int w) {
  YL_TRY(gn1.bind(net, n));
  YL_TRY(c1.bind(net));
  YL_TRY(gn2.bind(net, n));
  YL_TRY(c2.bind(net));
  if (has_skip) YL_TRY(skip.bind(net));
  YL_TRY(h1.make(net.arena, n, h, w, cin));
  YL_TRY(c1o.make(net.arena, n, h, w, cout));
  YL_TRY(h2.make(net.arena, n, h, w, cout));
  YL_TRY(y.make(net.arena, n, h, w, cout));
  if (has_temb) YL_TRY(net.arena.alloc((size_t)n * cout, &dproj));
  return YL_OK;
}
yl_status RB::init(yl_ctx* ctx, uint64_t seed) {
  YL_TRY(gn1.init(ctx, seed + 1));
  YL_TRY(c1.init(ctx, seed + 2));
  YL_TRY(gn2.init(ctx, seed + 3));
  YL_TRY(c2.init(ctx, seed + 4));
  if (has_skip) YL_TRY(skip.init(ctx, seed + 5));
  return YL_OK;
}
yl_status RB::forward(Net& net, const Act& x, const float* proj, GNL* gn_next) {
  YL_TRY(gn1.forward(net, x, h1));
  YL_TRY(c1.forward(net, h1, c1o, nullptr, 0, proj, 0, 0, 0, &gn2));
  YL_TRY(gn2.forward(net, c1o, h2));
  if (has_skip) {
    YL_TRY(skip.forward(net, x, y));
    return c2.forward(net, h2, y, y.p, y.ld, nullptr, 0, 0, 0, gn_next);
  }
  return c2.forward(net, h2, y, x.p, x.ld, nullptr, 0, 0, 0, gn_next);
}
yl_status RB::backward(Net& net, const Act& x, const Act& dy, const Act& dx) {
  Act dh2 = h2, dc1 = c1o, dh1 = h1;
  YL_TRY(net.pool.get(h2.elems(), &dh2.p));
  YL_TRY(net.pool.get(c1o.elems(), &dc1.p));
  YL_TRY(net.pool.get(h1.elems(), &dh1.p));
  dh2.ld = h2.c;
  dc1.ld = c1o.c;
  dh1.ld = h1.c;
  YL_TRY(c2.backward(net, h2, dy, &dh2));
  YL_TRY(gn2.backward(net, c1o, dh2, dc1));
  YL_TRY(c1.backward(net, h1, dc1, &dh1, nullptr, 0, has_temb ? dproj : nullptr));
  if (has_skip) {
    Act dxs = x;
    YL_TRY(net.pool.get(x.elems(), &dxs.p));
    dxs.ld = x.c;
    YL_TRY(skip.backward(net, x, dy, &dxs));
    YL_TRY(gn1.backward(net, x, dh1, dx, dxs.p, dxs.ld));
    net.pool.put(dxs.p);
  } else {
    YL_TRY(gn1.backward(net, x, dh1, dx, dy.p, dy.ld));
  }
  net.pool.put(dh2.p);
  net.pool.put(dc1.p);
  net.pool.put(dh1.p);
  net.grads_ready(param_lo);
  return YL_OK;
}

// ------------------------------------------------------------------ Net
Net::~Net() {
  for (auto& e : prof_ev) {
    cudaEventDestroy(e.first);
    cudaEventDestroy(e.second);
  }
}
void Net::prof_begin(int cls) {
  if (!profiling) return;
  ProfEvent pe;
  cudaEventCreate(&pe.a);
  cudaEventCreate(&pe.b);
  cudaEventRecord(pe.a, ctx->stream);
  pe.cls = cls;
  pending.push_back(pe);
}
void Net::prof_end(int cls, double flops, double bytes) {
  if (!profiling || pending.empty()) return;
  ProfEvent& pe = pending.back();
  cudaEventRecord(pe.b, ctx->stream);
  pe.flops = flops;
  pe.bytes = bytes;
  if (cls <= 2) {  // a conv class: the template the bracket launched (2: filter gradient)
    const int which = cls == 2 ? 1 : 0;
    std::memcpy(pe.kname, ctx->last_kernel[which], sizeof(pe.kname));
    pe.exec = ctx->last_exec_flops[which];
  }
  done.push_back(pe);
  pending.pop_back();
}
void Net::prof_mark_dominant() {
  if (profiling && !pending.empty()) pending.back().cls2 = kProfDominant;
}
yl_status Net::prof_collect(double* ms, double* flops, double* bytes, int* launches,
                            double* exec, std::map<std::string, TemplateStat>* templates) {
  if (done.empty()) return YL_OK;
  YL_CUDA(cudaStreamSynchronize(ctx->stream));
  for (auto& pe : done) {
    float t = 0.f;
    YL_CUDA(cudaEventElapsedTime(&t, pe.a, pe.b));
    if (templates && pe.kname[0]) {
      TemplateStat& ts = (*templates)[pe.kname];
      ts.ms += t;
      ts.flops += pe.flops;
      ts.exec += pe.exec;
      ts.launches += 1;
    }
    ms[pe.cls] += t;
    flops[pe.cls] += pe.flops;
    bytes[pe.cls] += pe.bytes;
    launches[pe.cls] += 1;
    exec[pe.cls] += pe.exec;
    if (pe.cls2 >= 0) {
      ms[pe.cls2] += t;
      flops[pe.cls2] += pe.flops;
      bytes[pe.cls2] += pe.bytes;
      launches[pe.cls2] += 1;
      exec[pe.cls2] += pe.exec;
    }
    cudaEventDestroy(pe.a);
    cudaEventDestroy(pe.b);
  }
  done.clear();
  return YL_OK;
}
void Net::grads_ready(size_t lo) {
  if (hook) hook(hook_arg, this, lo);
}
// The tf32 weight copies of every conv after each optimizer step: two launches
// (copies of W, then the copies derived from those).
yl_status Net::prepare_weights() {
  if (perm_first.empty())
    for (ConvL* c : convs) c->prepare_jobs(perm_first, perm_second);
  YL_TRY(weight_permute_batch(ctx, perm_first, &perm_buf_first));
  return weight_permute_batch(ctx, perm_second, &perm_buf_second);
}

// ------------------------------------------------------------------ VAE
yl_status VAE::build(yl_ctx* c, int n, int h, int w, uint64_t seed) {
  ctx = c;
  N = n;
  H = h;
  W = w;
  YL_CHECK(h % 8 == 0 && w % 8 == 0, YL_ERR_SHAPE, "VAE: frame %dx%d must be a multiple of 8", h,
           w);
  const int h2 = h / 2, w2 = w / 2, h4 = h / 4, w4 = w / 4;
  hl = h / 8;
  wl = w / 8;
  // encoder (frozen layer table: conv-in, 3 stride-2 stages with 2 RBs each, conv-out)
  conv_in.setup(*this, "enc.conv_in", 3, 128, 3, 1, 1);
  e1a.setup(*this, "enc.rb1a", 128, 128);
  e1b.setup(*this, "enc.rb1b", 128, 128);
  down1.setup(*this, "enc.down1", 128, 128, 3, 2, 1);
  e2a.setup(*this, "enc.rb2a", 128, 256);
  e2b.setup(*this, "enc.rb2b", 256, 256);
  down2.setup(*this, "enc.down2", 256, 256, 3, 2, 1);
  e3a.setup(*this, "enc.rb3a", 256, 256);
  e3b.setup(*this, "enc.rb3b", 256, 256);
  down3.setup(*this, "enc.down3", 256, 256, 3, 2, 1);
  gn_eo.setup(*this, "enc.norm_out", 256);
  conv_eo.setup(*this, "enc.conv_out", 256, 2 * kLatent, 3, 1, 1);
  // decoder (mirrored, nearest-up + conv)
  conv_z.setup(*this, "dec.conv_in", kLatent, 256, 3, 1, 1);
  up1.setup(*this, "dec.up1", 256, 256, 3, 1, 1);
  d1a.setup(*this, "dec.rb1a", 256, 256);
  d1b.setup(*this, "dec.rb1b", 256, 256);
  up2.setup(*this, "dec.up2", 256, 256, 3, 1, 1);
  d2a.setup(*this, "dec.rb2a", 256, 256);
  d2b.setup(*this, "dec.rb2b", 256, 256);
  up3.setup(*this, "dec.up3", 256, 128, 3, 1, 1);
  d3a.setup(*this, "dec.rb3a", 128, 128);
  d3b.setup(*this, "dec.rb3b", 128, 128);
  gn_do.setup(*this, "dec.norm_out", 128);
  conv_do.setup(*this, "dec.conv_out", 128, 3, 3, 1, 1);
  YL_TRY(params.allocate());
  // activations
  YL_TRY(x_in.make(arena, n, h, w, 4));
  YL_TRY(x_tgt.make(arena, n, h, w, 4));
  YL_TRY(conv_in.bind(*this));
  YL_TRY(a0.make(arena, n, h, w, 128));
  YL_TRY(e1a.bind(*this, n, h, w));
  YL_TRY(e1b.bind(*this, n, h, w));
  YL_TRY(down1.bind(*this));
  YL_TRY(a1.make(arena, n, h2, w2, 128));
  YL_TRY(e2a.bind(*this, n, h2, w2));
  YL_TRY(e2b.bind(*this, n, h2, w2));
  YL_TRY(down2.bind(*this));
  YL_TRY(a2.make(arena, n, h4, w4, 256));
  YL_TRY(e3a.bind(*this, n, h4, w4));
  YL_TRY(e3b.bind(*this, n, h4, w4));
  YL_TRY(down3.bind(*this));
  YL_TRY(a3.make(arena, n, hl, wl, 256));
  YL_TRY(gn_eo.bind(*this, n));
  YL_TRY(hg.make(arena, n, hl, wl, 256));
  YL_TRY(conv_eo.bind(*this));
  YL_TRY(e.make(arena, n, hl, wl, 2 * kLatent));
  YL_TRY(z.make(arena, n, hl, wl, kLatent));
  YL_TRY(conv_z.bind(*this));
  YL_TRY(b0.make(arena, n, hl, wl, 256));
  YL_TRY(up1.bind(*this));
  YL_TRY(b1.make(arena, n, h4, w4, 256));
  YL_TRY(d1a.bind(*this, n, h4, w4));
  YL_TRY(d1b.bind(*this, n, h4, w4));
  YL_TRY(up2.bind(*this));
  YL_TRY(b2.make(arena, n, h2, w2, 256));
  YL_TRY(d2a.bind(*this, n, h2, w2));
  YL_TRY(d2b.bind(*this, n, h2, w2));
  YL_TRY(up3.bind(*this));
  YL_TRY(b3.make(arena, n, h, w, 128));
  YL_TRY(d3a.bind(*this, n, h, w));
  YL_TRY(d3b.bind(*this, n, h, w));
  YL_TRY(gn_do.bind(*this, n));
  YL_TRY(hd.make(arena, n, h, w, 128));
  YL_TRY(conv_do.bind(*this));
  YL_TRY(recon.make(arena, n, h, w, 4));
  YL_TRY(drecon.make(arena, n, h, w, 4));
  // init (seeded)
  uint64_t s = seed * 1000003ull;
  for (ConvL* cv : convs) YL_TRY(cv->init(ctx, ++s));
  RB* rbs[] = {&e1a, &e1b, &e2a, &e2b, &e3a, &e3b, &d1a, &d1b, &d2a, &d2b, &d3a, &d3b};
  for (RB* rb : rbs) YL_TRY(rb->init(ctx, (s += 16)));
  YL_TRY(gn_eo.init(ctx, ++s));
  YL_TRY(gn_do.init(ctx, ++s));
  return YL_OK;
}

yl_status VAE::encode() {
  YL_TRY(conv_in.forward(*this, x_in, a0, nullptr, 0, nullptr, 0, 0, 0, &e1a.gn1));
  YL_TRY(e1a.forward(*this, a0, nullptr, &e1b.gn1));
  YL_TRY(e1b.forward(*this, e1a.y));
  YL_TRY(down1.forward(*this, e1b.y, a1, nullptr, 0, nullptr, 0, 0, 0, &e2a.gn1));
  YL_TRY(e2a.forward(*this, a1, nullptr, &e2b.gn1));
  YL_TRY(e2b.forward(*this, e2a.y));
  YL_TRY(down2.forward(*this, e2b.y, a2, nullptr, 0, nullptr, 0, 0, 0, &e3a.gn1));
  YL_TRY(e3a.forward(*this, a2, nullptr, &e3b.gn1));
  YL_TRY(e3b.forward(*this, e3a.y));
  YL_TRY(down3.forward(*this, e3b.y, a3, nullptr, 0, nullptr, 0, 0, 0, &gn_eo));
  YL_TRY(gn_eo.forward(*this, a3, hg));
  return conv_eo.forward(*this, hg, e);
}

yl_status VAE::decode() {
  YL_TRY(conv_z.forward(*this, z, b0));
  YL_TRY(up1.forward(*this, b0, b1, nullptr, 0, nullptr, 1, b1.h, b1.w, &d1a.gn1));
  YL_TRY(d1a.forward(*this, b1, nullptr, &d1b.gn1));
  YL_TRY(d1b.forward(*this, d1a.y));
  YL_TRY(up2.forward(*this, d1b.y, b2, nullptr, 0, nullptr, 1, b2.h, b2.w, &d2a.gn1));
  YL_TRY(d2a.forward(*this, b2, nullptr, &d2b.gn1));
  YL_TRY(d2b.forward(*this, d2a.y));
  YL_TRY(up3.forward(*this, d2b.y, b3, nullptr, 0, nullptr, 1, b3.h, b3.w, &d3a.gn1));
  YL_TRY(d3a.forward(*this, b3, nullptr, &d3b.gn1));
  YL_TRY(d3b.forward(*this, d3a.y, nullptr, &gn_do));
  YL_TRY(gn_do.forward(*this, d3b.y, hd));
  return conv_do.forward(*this, hd, recon);
}

yl_status VAE::forward_train(int64_t step) {
  YL_TRY(encode());
  YL_TRY(latent_head_forward(ctx, e.p, e.ld, N, (long long)hl * wl, kLatent, step, z.p, z.ld));
  return decode();
}

// Gradient of a block output: a temporary sized like `like` (pixel stride = channels).
static yl_status grad_like(Net& net, const Act& like, Act* out) {
  *out = like;
  out->ld = like.c;
  return net.pool.get(like.elems(), &out->p);
}

yl_status VAE::backward(int64_t step, float beta) {
  Act g0, g1;
  // decoder tail
  YL_TRY(grad_like(*this, hd, &g0));
  YL_TRY(conv_do.backward(*this, hd, drecon, &g0));
  grads_ready(conv_do.off_w);
  YL_TRY(grad_like(*this, d3b.y, &g1));
  YL_TRY(gn_do.backward(*this, d3b.y, g0, g1));
  grads_ready(gn_do.off_g);
  pool.put(g0.p);
  // decoder blocks, last to first
  struct Step { RB* rb; const Act* in; };
  auto rb_back = [&](RB& rb, const Act& in, Act& dy) -> yl_status {
    Act dx;
    YL_TRY(grad_like(*this, in, &dx));
    YL_TRY(rb.backward(*this, in, dy, dx));
    pool.put(dy.p);
    dy = dx;
    return YL_OK;
  };
  auto up_back = [&](ConvL& cv, const Act& src, const Act& out, Act& dy) -> yl_status {
    Act dx;
    YL_TRY(grad_like(*this, src, &dx));
    YL_TRY(cv.backward(*this, src, dy, &dx, nullptr, 0, nullptr, 1, out.h, out.w));
    grads_ready(cv.off_w);
    pool.put(dy.p);
    dy = dx;
    return YL_OK;
  };
  auto conv_back = [&](ConvL& cv, const Act& src, Act& dy) -> yl_status {
    Act dx;
    YL_TRY(grad_like(*this, src, &dx));
    YL_TRY(cv.backward(*this, src, dy, &dx));
    grads_ready(cv.off_w);
    pool.put(dy.p);
    dy = dx;
    return YL_OK;
  };
  YL_TRY(rb_back(d3b, d3a.y, g1));
  YL_TRY(rb_back(d3a, b3, g1));
  YL_TRY(up_back(up3, d2b.y, b3, g1));
  YL_TRY(rb_back(d2b, d2a.y, g1));
  YL_TRY(rb_back(d2a, b2, g1));
  YL_TRY(up_back(up2, d1b.y, b2, g1));
  YL_TRY(rb_back(d1b, d1a.y, g1));
  YL_TRY(rb_back(d1a, b1, g1));
  YL_TRY(up_back(up1, b0, b1, g1));
  YL_TRY(conv_back(conv_z, z, g1));  // g1 = dz
  // latent head: de = [dmu | dlogvar] with the KL averaged per latent element
  Act de;
  YL_TRY(grad_like(*this, e, &de));
  const double M = (double)N * kLatent * hl * wl;
  YL_TRY(latent_head_backward(ctx, e.p, e.ld, g1.p, g1.ld, N, (long long)hl * wl, kLatent, step,
                              (float)(beta / M), (float)(0.5 * beta / M), de.p, de.ld));
  pool.put(g1.p);
  g1 = de;
  YL_TRY(conv_back(conv_eo, hg, g1));
  Act ga;
  YL_TRY(grad_like(*this, a3, &ga));
  YL_TRY(gn_eo.backward(*this, a3, g1, ga));
  grads_ready(gn_eo.off_g);
  pool.put(g1.p);
  g1 = ga;
  YL_TRY(conv_back(down3, e3b.y, g1));
  YL_TRY(rb_back(e3b, e3a.y, g1));
  YL_TRY(rb_back(e3a, a2, g1));
  YL_TRY(conv_back(down2, e2b.y, g1));
  YL_TRY(rb_back(e2b, e2a.y, g1));
  YL_TRY(rb_back(e2a, a1, g1));
  YL_TRY(conv_back(down1, e1b.y, g1));
  YL_TRY(rb_back(e1b, e1a.y, g1));
  YL_TRY(rb_back(e1a, a0, g1));
  // conv-in: the input frames need no gradient
  YL_TRY(conv_in.backward(*this, x_in, g1, nullptr));
  grads_ready(conv_in.off_w);
  pool.put(g1.p);
  return YL_OK;
}

// ------------------------------------------------------------------ motion U-Net
yl_status UNet::build(yl_ctx* c, int n, int h, int w, uint64_t seed) {
  ctx = c;
  N = n;
  H = h;
  W = w;
  const int h2 = (h + 1) / 2, w2 = (w + 1) / 2, h3 = (h2 + 1) / 2, w3 = (w2 + 1) / 2;
  // time conditioning: emb128 -> Linear 512 -> SiLU -> Linear 512, per-block
  // projections.  Registered first: their gradients are the last ones the
  // backward pass completes, and the all-reduce frontier walks offsets down.
  static const int kCouts[kBlocks] = {128, 128, 256, 256, 384, 384, 256, 256, 128, 128};
  static const char* kNames[kBlocks] = {"down1.rb_a", "down1.rb_b", "down2.rb_a", "down2.rb_b",
                                        "mid.rb_a",   "mid.rb_b",   "up1.rb_a",   "up1.rb_b",
                                        "up2.rb_a",   "up2.rb_b"};
  t_l1.setup(*this, "time.fc1", kEmb, kTime);
  t_l2.setup(*this, "time.fc2", kTime, kTime);
  for (int i = 0; i < kBlocks; ++i)
    proj[i].setup(*this, (std::string(kNames[i]) + ".temb_proj").c_str(), kTime, kCouts[i]);
  conv_in.setup(*this, "conv_in", 3 * kLat, 128, 3, 1, 1);
  r1a.setup(*this, "down1.rb_a", 128, 128, true);
  r1b.setup(*this, "down1.rb_b", 128, 128, true);
  dn1.setup(*this, "down1.conv", 128, 128, 3, 2, 1);
  r2a.setup(*this, "down2.rb_a", 128, 256, true);
  r2b.setup(*this, "down2.rb_b", 256, 256, true);
  dn2.setup(*this, "down2.conv", 256, 256, 3, 2, 1);
  r3a.setup(*this, "mid.rb_a", 256, 384, true);
  r3b.setup(*this, "mid.rb_b", 384, 384, true);
  upc1.setup(*this, "up1.conv", 384, 256, 3, 1, 1);
  r4a.setup(*this, "up1.rb_a", 512, 256, true);
  r4b.setup(*this, "up1.rb_b", 256, 256, true);
  upc2.setup(*this, "up2.conv", 256, 128, 3, 1, 1);
  r5a.setup(*this, "up2.rb_a", 256, 128, true);
  r5b.setup(*this, "up2.rb_b", 128, 128, true);
  gn_o.setup(*this, "norm_out", 128);
  conv_o.setup(*this, "conv_out", 128, kLat, 3, 1, 1);
  RB* rbs[kBlocks] = {&r1a, &r1b, &r2a, &r2b, &r3a, &r3b, &r4a, &r4b, &r5a, &r5b};
  for (int i = 0; i < kBlocks; ++i) {
    blocks[i] = rbs[i];
    YL_CHECK(rbs[i]->cout == kCouts[i], YL_ERR_INVALID, "U-Net block table mismatch");
  }
  YL_TRY(params.allocate());
  t_l1.bind(*this);
  t_l2.bind(*this);
  for (int i = 0; i < kBlocks; ++i) proj[i].bind(*this);
  YL_TRY(arena.alloc((size_t)n, &t));
  YL_TRY(arena.alloc((size_t)n * kEmb, &emb));
  YL_TRY(arena.alloc((size_t)n * kTime, &th));
  YL_TRY(arena.alloc((size_t)n * kTime, &ta));
  YL_TRY(arena.alloc((size_t)n * kTime, &temb));
  YL_TRY(arena.alloc((size_t)n * kTime, &ts));
  YL_TRY(arena.alloc((size_t)n * kTime, &dts));
  YL_TRY(arena.alloc((size_t)n * kTime, &dtmp));
  YL_TRY(arena.alloc((size_t)n * kTime, &dtmp2));
  for (int i = 0; i < kBlocks; ++i) YL_TRY(arena.alloc((size_t)n * rbs[i]->cout, &pj[i]));
  YL_TRY(inp.make(arena, n, h, w, 3 * kLat));
  YL_TRY(lerp.make(arena, n, h, w, kLat));
  YL_TRY(conv_in.bind(*this));
  YL_TRY(h0.make(arena, n, h, w, 128));
  YL_TRY(r1a.bind(*this, n, h, w));
  YL_TRY(r1b.bind(*this, n, h, w));
  YL_TRY(dn1.bind(*this));
  YL_TRY(p1.make(arena, n, h2, w2, 128));
  YL_TRY(r2a.bind(*this, n, h2, w2));
  YL_TRY(r2b.bind(*this, n, h2, w2));
  YL_TRY(dn2.bind(*this));
  YL_TRY(p2.make(arena, n, h3, w3, 256));
  YL_TRY(r3a.bind(*this, n, h3, w3));
  YL_TRY(r3b.bind(*this, n, h3, w3));
  YL_TRY(upc1.bind(*this));
  YL_TRY(cat1.make(arena, n, h2, w2, 512));
  YL_TRY(r4a.bind(*this, n, h2, w2));
  YL_TRY(r4b.bind(*this, n, h2, w2));
  YL_TRY(upc2.bind(*this));
  YL_TRY(cat2.make(arena, n, h, w, 256));
  YL_TRY(r5a.bind(*this, n, h, w));
  YL_TRY(r5b.bind(*this, n, h, w));
  YL_TRY(gn_o.bind(*this, n));
  YL_TRY(ho.make(arena, n, h, w, 128));
  YL_TRY(conv_o.bind(*this));
  YL_TRY(pred.make(arena, n, h, w, kLat));
  YL_TRY(dpred.make(arena, n, h, w, kLat));
  YL_TRY(target.make(arena, n, h, w, kLat));
  uint64_t s = seed * 7919ull + 17;
  YL_TRY(t_l1.init(ctx, ++s));
  YL_TRY(t_l2.init(ctx, ++s));
  for (int i = 0; i < kBlocks; ++i) YL_TRY(proj[i].init(ctx, ++s));
  for (ConvL* cv : convs) YL_TRY(cv->init(ctx, ++s, cv == &conv_o));  // zero-init output conv
  for (int i = 0; i < kBlocks; ++i) YL_TRY(blocks[i]->init(ctx, (s += 16)));
  YL_TRY(gn_o.init(ctx, ++s));
  return YL_OK;
}

yl_status UNet::forward() {
  // time MLP
  YL_TRY(time_embedding(ctx, t, N, kEmb, 0, emb));
  YL_TRY(linear_forward(ctx, emb, t_l1.W, t_l1.b, th, N, kEmb, kTime));
  YL_TRY(silu_forward(ctx, th, ta, (long long)N * kTime));
  YL_TRY(linear_forward(ctx, ta, t_l2.W, t_l2.b, temb, N, kTime, kTime));
  YL_TRY(silu_forward(ctx, temb, ts, (long long)N * kTime));
  for (int i = 0; i < kBlocks; ++i)
    YL_TRY(linear_forward(ctx, ts, proj[i].W, proj[i].b, pj[i], N, kTime, blocks[i]->cout));
  // down path
  YL_TRY(conv_in.forward(*this, inp, h0, nullptr, 0, nullptr, 0, 0, 0, &r1a.gn1));
  YL_TRY(r1a.forward(*this, h0, pj[0], &r1b.gn1));
  YL_TRY(r1b.forward(*this, r1a.y, pj[1]));
  YL_TRY(dn1.forward(*this, r1b.y, p1, nullptr, 0, nullptr, 0, 0, 0, &r2a.gn1));
  YL_TRY(r2a.forward(*this, p1, pj[2], &r2b.gn1));
  YL_TRY(r2b.forward(*this, r2a.y, pj[3]));
  YL_TRY(dn2.forward(*this, r2b.y, p2, nullptr, 0, nullptr, 0, 0, 0, &r3a.gn1));
  YL_TRY(r3a.forward(*this, p2, pj[4], &r3b.gn1));
  YL_TRY(r3b.forward(*this, r3a.y, pj[5]));
  // up path: up + conv written into the first half of the concat buffer, skip copied after it
  Act c1lo = cat1;
  c1lo.c = 256;
  YL_TRY(upc1.forward(*this, r3b.y, c1lo, nullptr, 0, nullptr, 1, cat1.h, cat1.w));
  YL_TRY(copy_slice(ctx, r2b.y.p, r2b.y.ld, cat1.p + 256, cat1.ld, cat1.pixels(), 256, 0));
  YL_TRY(r4a.forward(*this, cat1, pj[6], &r4b.gn1));
  YL_TRY(r4b.forward(*this, r4a.y, pj[7]));
  Act c2lo = cat2;
  c2lo.c = 128;
  YL_TRY(upc2.forward(*this, r4b.y, c2lo, nullptr, 0, nullptr, 1, cat2.h, cat2.w));
  YL_TRY(copy_slice(ctx, r1b.y.p, r1b.y.ld, cat2.p + 128, cat2.ld, cat2.pixels(), 128, 0));
  YL_TRY(r5a.forward(*this, cat2, pj[8], &r5b.gn1));
  YL_TRY(r5b.forward(*this, r5a.y, pj[9], &gn_o));
  YL_TRY(gn_o.forward(*this, r5b.y, ho));
  // prediction = lerp(zA, zB, t) + net output (MotionMLP.swift:39-55), the fp32
  // lerp added in the epilogue
  return conv_o.forward(*this, ho, pred, lerp.p, lerp.ld);
}

yl_status UNet::backward() {
  Act g, gx;
  YL_TRY(grad_like(*this, ho, &g));
  YL_TRY(conv_o.backward(*this, ho, dpred, &g));
  grads_ready(conv_o.off_w);
  YL_TRY(grad_like(*this, r5b.y, &gx));
  YL_TRY(gn_o.backward(*this, r5b.y, g, gx));
  grads_ready(gn_o.off_g);
  pool.put(g.p);
  g = gx;
  auto rb_back = [&](RB& rb, const Act& in, Act& dy) -> yl_status {
    Act dx;
    YL_TRY(grad_like(*this, in, &dx));
    YL_TRY(rb.backward(*this, in, dy, dx));
    pool.put(dy.p);
    dy = dx;
    return YL_OK;
  };
  YL_TRY(rb_back(r5b, r5a.y, g));
  YL_TRY(rb_back(r5a, cat2, g));  // g = d(cat2): [d up2-out | d skip1]
  Act dcat2 = g;
  Act dlo = dcat2;
  dlo.c = 128;
  Act gu;
  YL_TRY(grad_like(*this, r4b.y, &gu));
  YL_TRY(upc2.backward(*this, r4b.y, dlo, &gu, nullptr, 0, nullptr, 1, cat2.h, cat2.w));
  grads_ready(upc2.off_w);
  g = gu;
  YL_TRY(rb_back(r4b, r4a.y, g));
  YL_TRY(rb_back(r4a, cat1, g));  // g = d(cat1)
  Act dcat1 = g;
  Act dlo1 = dcat1;
  dlo1.c = 256;
  YL_TRY(grad_like(*this, r3b.y, &gu));
  YL_TRY(upc1.backward(*this, r3b.y, dlo1, &gu, nullptr, 0, nullptr, 1, cat1.h, cat1.w));
  grads_ready(upc1.off_w);
  g = gu;
  YL_TRY(rb_back(r3b, r3a.y, g));
  YL_TRY(rb_back(r3a, p2, g));
  // dn2 backward: d(r2b.y) = dgrad + skip gradient from cat1[:, 256:]
  YL_TRY(grad_like(*this, r2b.y, &gu));
  YL_TRY(dn2.backward(*this, r2b.y, g, &gu, dcat1.p + 256, dcat1.ld));
  grads_ready(dn2.off_w);
  pool.put(g.p);
  pool.put(dcat1.p);
  g = gu;
  YL_TRY(rb_back(r2b, r2a.y, g));
  YL_TRY(rb_back(r2a, p1, g));
  YL_TRY(grad_like(*this, r1b.y, &gu));
  YL_TRY(dn1.backward(*this, r1b.y, g, &gu, dcat2.p + 128, dcat2.ld));
  grads_ready(dn1.off_w);
  pool.put(g.p);
  pool.put(dcat2.p);
  g = gu;
  YL_TRY(rb_back(r1b, r1a.y, g));
  YL_TRY(rb_back(r1a, h0, g));
  YL_TRY(conv_in.backward(*this, inp, g, nullptr));
  grads_ready(conv_in.off_w);
  pool.put(g.p);
  // time MLP: the per-block projections' gradients come from each block's conv1 bias sums
  YL_CUDA(cudaMemsetAsync(dts, 0, (size_t)N * kTime * sizeof(float), ctx->stream));
  for (int i = 0; i < kBlocks; ++i) {
    const int co = blocks[i]->cout;
    YL_TRY(linear_backward(ctx, ts, proj[i].W, blocks[i]->dproj, dts, nullptr, nullptr, N, kTime,
                           co, 1));
    YL_TRY(linear_backward(ctx, ts, proj[i].W, blocks[i]->dproj, nullptr, proj[i].gW, proj[i].gb,
                           N, kTime, co, 0));
  }
  YL_TRY(silu_backward(ctx, temb, dts, dtmp, (long long)N * kTime, 0));
  YL_TRY(linear_backward(ctx, ta, t_l2.W, dtmp, dtmp2, t_l2.gW, t_l2.gb, N, kTime, kTime, 0));
  YL_TRY(silu_backward(ctx, th, dtmp2, dtmp, (long long)N * kTime, 0));
  YL_TRY(linear_backward(ctx, emb, t_l1.W, dtmp, nullptr, t_l1.gW, t_l1.gb, N, kEmb, kTime, 0));
  grads_ready(0);
  return YL_OK;
}

yl_status UNet::set_inputs(const float* za, const float* zb, int ldz, const float* tdev) {
  YL_CUDA(cudaMemcpyAsync(t, tdev, N * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
  motion_input_kernel<<<grid_1d((long long)N * H * W * kLat, 256), 256, 0, ctx->stream>>>(
      za, zb, ldz, t, (long long)H * W, N, kLat, inp.p, lerp.p);
  return check_launch("motion_input_kernel");
}

// ------------------------------------------------------------------ frames
// One thread per pixel: three coalesced plane reads, one 16-byte write.
__global__ void frames_to_nhwc4_kernel(const float* __restrict__ in, long long hw, long long total,
                                       int round, float* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / hw, p = i - img * hw;
    const float* src = in + img * 3 * hw + p;
    float r = __ldg(src), g = __ldg(src + hw), b = __ldg(src + 2 * hw);
    if (round) {
      r = round_tf32(r);
      g = round_tf32(g);
      b = round_tf32(b);
    }
    reinterpret_cast<float4*>(out)[i] = make_float4(r, g, b, 0.f);
  }
}

yl_status frames_to_nhwc4(yl_ctx* ctx, const float* nchw3, int n, int h, int w, float* out,
                          int round) {
  const long long hw = (long long)h * w, total = (long long)n * hw;
  frames_to_nhwc4_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(nchw3, hw, total, round,
                                                                       out);
  return check_launch("frames_to_nhwc4_kernel");
}

yl_status copy_mu(yl_ctx* ctx, const Act& e, float* dst, int c) {
  return copy_slice(ctx, e.p, e.ld, dst, c, e.pixels(), c, 0);
}

}  // namespace yl
