// yl_nets.h -- layer and model classes of the training executor.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "yl_kernels.h"

namespace yl {

// Persistent device allocations of one model (freed with the model).
struct DeviceArena {
  std::vector<void*> blocks;
  size_t bytes = 0;
  ~DeviceArena();
  yl_status alloc(size_t floats, float** out);
};

// Reusable gradient temporaries; grows only during the first step.
struct GradPool {
  struct Item {
    float* p;
    size_t n;
    bool used;
  };
  DeviceArena* arena = nullptr;
  std::vector<Item> items;
  yl_status get(size_t floats, float** out);
  void put(float* p);
};

// NHWC activation view: n x h x w pixels, c valid channels, pixel stride ld.
struct Act {
  float* p = nullptr;
  int n = 0, h = 0, w = 0, c = 0, ld = 0;
  long long pixels() const { return (long long)n * h * w; }
  size_t elems() const { return (size_t)n * h * w * c; }
  yl_status make(DeviceArena& a, int n, int h, int w, int c, int ld = 0);
};

// One contiguous buffer each for parameters, gradients and Adam moments.
struct ParamSet {
  size_t count = 0;
  float *w = nullptr, *g = nullptr, *m = nullptr, *v = nullptr;
  size_t reserve(size_t n);
  yl_status allocate();
  ~ParamSet();
};

struct ParamEntry {
  std::string name;
  size_t offset;
  int d0, d1, d2, d3;  // logical shape (conv weights: oc, ic, k, k; stored [oc][k*k][ic_padded])
};

struct Net;

// Profiled time and work of one conv kernel template over the profiled steps.
struct TemplateStat {
  double ms = 0.0, flops = 0.0, exec = 0.0;
  int launches = 0;
};

struct ConvL {
  std::string name;
  int cin = 0, cout = 0, cin_p = 0, cout_p = 0, k = 3, stride = 1, pad = 1;
  size_t off_w = 0, off_b = 0;
  float *W = nullptr, *b = nullptr, *gW = nullptr, *gb = nullptr;
  float *Wr = nullptr, *Wd = nullptr;  // tf32 copies: fprop [cout][tap][cin], dgrad [cin][tap][cout]
  // 3x3 convs with a 4-channel (RGB) side run as 1x1 GEMMs over 3x3 patches:
  // rgb 1 = 4-channel input (its filter gradient runs over 64-channel 3x3
  // patches); rgb 2 = 4-channel output (Wx: [9*4][cin] tap weights,
  // Wx2: [cin][64] dX patch weights)
  int rgb = 0;
  float *Wx = nullptr, *Wx2 = nullptr;
  void setup(Net& net, const char* name, int cin, int cout, int k, int stride, int pad);
  yl_status bind(Net& net);
  yl_status init(yl_ctx* ctx, uint64_t seed, bool zero = false);
  yl_status prepare(yl_ctx* ctx);
  // the weight copies prepare() makes, as permute jobs: `first` read W, `second`
  // read copies made by `first`
  void prepare_jobs(std::vector<PermuteJob>& first, std::vector<PermuteJob>& second) const;
  ConvGather gather(const Act& x, int oh, int ow, int up, int hv, int wv) const;
  // gn_next: the GroupNorm that reads y; its statistics come out of this
  // conv's epilogue when the channel grouping allows it
  yl_status forward(Net& net, const Act& x, const Act& y, const float* residual = nullptr,
                    int ldr = 0, const float* bias2d = nullptr, int up = 0, int hv = 0,
                    int wv = 0, struct GNL* gn_next = nullptr);
  yl_status backward(Net& net, const Act& x, const Act& dy, const Act* dx,
                     const float* dx_addend = nullptr, int ld_addend = 0,
                     float* dbias2d = nullptr, int up = 0, int hv = 0, int wv = 0);
  bool dominant(const struct Net& net, int h, int w, int up) const;
};

struct GNL {
  std::string name;
  int c = 0, G = 32;
  size_t off_g = 0, off_b = 0;
  float *gamma = nullptr, *beta = nullptr, *ggamma = nullptr, *gbeta = nullptr;
  float *mean = nullptr, *rstd = nullptr;
  bool stats_ready = false;  // mean/rstd already written by the producing conv
  void setup(Net& net, const char* name, int c);
  yl_status bind(Net& net, int n);
  yl_status init(yl_ctx* ctx, uint64_t seed);
  yl_status forward(Net& net, const Act& x, const Act& y);
  yl_status backward(Net& net, const Act& x, const Act& dy, const Act& dx,
                     const float* addend = nullptr, int ldadd = 0);
};

struct LinL {
  std::string name;
  int ic = 0, oc = 0;
  size_t off_w = 0, off_b = 0;
  float *W = nullptr, *b = nullptr, *gW = nullptr, *gb = nullptr;
  void setup(Net& net, const char* name, int ic, int oc);
  void bind(Net& net);
  yl_status init(yl_ctx* ctx, uint64_t seed);
};

// GroupNorm32 -> SiLU -> conv3x3 -> (+ per-image bias) -> GroupNorm32 -> SiLU
// -> conv3x3, plus the identity or a 1x1 conv skip.
struct RB {
  std::string name;
  int cin = 0, cout = 0;
  bool has_skip = false, has_temb = false;
  GNL gn1, gn2;
  ConvL c1, c2, skip;
  Act h1, c1o, h2, y;
  float* dproj = nullptr;  // per-image channel sums of conv1's output gradient
  size_t param_lo = 0;
  void setup(Net& net, const std::string& name, int cin, int cout, bool temb = false);
  yl_status bind(Net& net, int n, int h, int w);
  yl_status init(yl_ctx* ctx, uint64_t seed);
  // gn_next: the GroupNorm that reads this block's output (statistics fused)
  yl_status forward(Net& net, const Act& x, const float* proj = nullptr,
                    GNL* gn_next = nullptr);
  yl_status backward(Net& net, const Act& x, const Act& dy, const Act& dx);
};

// Kernel-class timing used by the bench (classes: 0 conv fprop, 1 conv
// dgrad, 2 conv wgrad, 3 GN+SiLU forward, 4 GN+SiLU backward; 5 counts again
// the fprop and dX launches of stride-1 3x3 128->128 convs at dom_pixels
// pixels per image, the step's dominant launch type).
constexpr int kProfClasses = 6;
constexpr int kProfDominant = 5;

struct Net {
  yl_ctx* ctx = nullptr;
  DeviceArena arena;
  GradPool pool;
  ParamSet params;
  std::vector<ParamEntry> param_table;
  std::vector<ConvL*> convs;
  // called with the lowest parameter offset whose gradient is complete
  void (*hook)(void* arg, Net* net, size_t lo) = nullptr;
  void* hook_arg = nullptr;
  bool profiling = false;
  long long dom_pixels = 0;  // output pixels per image of the dominant launch type
  struct ProfEvent {
    cudaEvent_t a, b;
    int cls, cls2 = -1;  // cls2: a second class the launch also counts in
    double flops, bytes;
    double exec = 0.0;      // FLOPs the conv kernel executed (conv classes)
    char kname[96] = {0};  // the conv kernel template the bracket launched
  };
  std::vector<ProfEvent> pending, done;
  std::vector<PermuteJob> perm_first, perm_second;
  PermuteBatchBuffers perm_buf_first, perm_buf_second;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> prof_ev;

  Net() { pool.arena = &arena; }
  virtual ~Net();
  void prof_begin(int cls);
  void prof_end(int cls, double flops, double bytes = 0.0);
  // the open event also counts in class 5 (call between prof_begin and prof_end)
  void prof_mark_dominant();
  yl_status prof_collect(double* ms, double* flops, double* bytes, int* launches, double* exec,
                         std::map<std::string, TemplateStat>* templates = nullptr);
  void grads_ready(size_t lo);
  yl_status prepare_weights();
};

// Conv VAE of the 854x480 frame workload: frames padded to 856, 32-channel
// latent at 1/8 resolution.
struct VAE : Net {
  static constexpr int kLatent = 32;
  int N = 0, H = 0, W = 0, hl = 0, wl = 0;
  ConvL conv_in, down1, down2, down3, conv_eo, conv_z, up1, up2, up3, conv_do;
  RB e1a, e1b, e2a, e2b, e3a, e3b, d1a, d1b, d2a, d2b, d3a, d3b;
  GNL gn_eo, gn_do;
  Act x_in, x_tgt, a0, a1, a2, a3, hg, e, z, b0, b1, b2, b3, hd, recon, drecon;
  yl_status build(yl_ctx* ctx, int n, int h, int w, uint64_t seed);
  yl_status encode();                 // x_in -> e = [mu | logvar]
  yl_status decode();                 // z -> recon
  yl_status forward_train(int64_t step);
  yl_status backward(int64_t step, float beta);  // from drecon
};

// Motion U-Net (levels 128/256/384) in the 32-channel latent space.
struct UNet : Net {
  static constexpr int kLat = 32, kEmb = 128, kTime = 512, kBlocks = 10;
  int N = 0, H = 0, W = 0;
  LinL t_l1, t_l2, proj[kBlocks];
  ConvL conv_in, dn1, dn2, upc1, upc2, conv_o;
  RB r1a, r1b, r2a, r2b, r3a, r3b, r4a, r4b, r5a, r5b;
  RB* blocks[kBlocks] = {};
  GNL gn_o;
  float *t = nullptr, *emb = nullptr, *th = nullptr, *ta = nullptr, *temb = nullptr, *ts = nullptr;
  float *dts = nullptr, *dtmp = nullptr, *dtmp2 = nullptr;
  float* pj[kBlocks] = {};
  Act inp, lerp, h0, p1, p2, cat1, cat2, ho, pred, dpred, target;
  yl_status build(yl_ctx* ctx, int n, int h, int w, uint64_t seed);
  yl_status set_inputs(const float* za, const float* zb, int ldz, const float* t_dev);
  yl_status forward();
  yl_status backward();  // from dpred
};

yl_status frames_to_nhwc4(yl_ctx* ctx, const float* nchw3, int n, int h, int w, float* out,
                          int round);
yl_status copy_mu(yl_ctx* ctx, const Act& e, float* dst, int c);

}  // namespace yl
