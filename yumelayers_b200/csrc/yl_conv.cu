// yl_conv.cu -- implicit-GEMM convolution on the 5th-generation tensor cores.
//
// Replaces the reference's im2col + tiled fp32 matmul (ConvLayerGPU.forward,
// ConvGPU.swift:57-64 -> im2col3d_kernel MetalKernelSourcesA.swift:325-352 ->
// matmul_tiled_kernel A:34-94 -> biasrow3d_kernel B:112-121), its dW path
// (gradw_plain_kernel A:122-137, biasrowgrad B:162-189) and its dX paths
// (conv_back_input_s1_kernel B:125-159; matmul(transA) + col2im B:28-58).
// Nothing is materialised: each CTA gathers its im2col tile straight into
// shared memory in the tcgen05 SWIZZLE_128B layout.
//
// fprop / dgrad kernel (one 128 x BN output tile per CTA, 6 warps):
//   warps 0-3  gather the A tile (128 output pixels x 32 k) with 16-byte
//              cp.async, zero-filling padding, stride-2 holes and tails;
//              afterwards they run the epilogue (TMEM -> registers -> bias,
//              per-image bias, residual, tf32 rounding -> global).
//   warp 4     TMA-loads the weight tile (BN rows x 32 k, SWIZZLE_128B).
//   warp 5     allocates TMEM and issues tcgen05.mma kind::tf32 (M=128,
//              N=BN, K=8 per instruction) from one thread, releasing each
//              stage with tcgen05.commit.
// wgrad kernel: both operands gathered MN-major (pixels are the contraction
// dimension), deterministic split-K over pixels into a workspace that a
// fixed-order reduction sums.
//
// Operands are tf32 (fp32 storage, 10-bit mantissa, fp32 accumulation): a
// bf16 operand's rounding alone puts relative L2 error near 3e-3, above the
// 1e-3 per-op tolerance; tf32 rounding-to-nearest stays near 4e-4.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include "yl_conv_common.cuh"

namespace yl {

// ------------------------------------------------------------------ fprop / dgrad
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    conv_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, ConvGather g, ConvEpilogue e,
                     int* err) {
  using Cfg = TileCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
  const int nk = (g.k_total + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 128 + 1);  // 128 gather threads + the TMA arrive.expect_tx
      mbar_init(&empty[s], 1);       // one tcgen05.commit
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) tma_prefetch_desc(&tmap_w);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const long long lim = wait_limit(err);

  if (warp < 4) {
    // ---------------- A-operand gather (implicit im2col) ----------------
    const int t = threadIdx.x;
    const int j = t & 7;       // 16-byte chunk of the 128-byte row
    const int rb = t >> 3;     // rows rb + 16 i, i = 0..7
    const int ohw = g.oh * g.ow;
    int row_img[8], row_y[8], row_x[8];
    bool row_ok[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int m = m0 + rb + 16 * i;
      row_ok[i] = m < g.m_total;
      int mm = row_ok[i] ? m : 0;
      int img = mm / ohw;
      int rem = mm - img * ohw;
      row_img[i] = img;
      row_y[i] = rem / g.ow;
      row_x[i] = rem - row_y[i] * g.ow;
    }
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S;
      if (kb >= S && !mbar_wait(&empty[s], ((kb / S) - 1) & 1, lim)) {
        ok = false;
        break;
      }
      const uint32_t a_base = smem_u32(smem + s * Cfg::kStageBytes);
      const int k = kb * kBK + 4 * j;
      const bool kval = k < g.k_total;
      const int tap = kval ? k / g.cin : 0;
      const int ci = k - tap * g.cin;
      const int ky = tap / g.ksize, kx = tap - (tap / g.ksize) * g.ksize;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = rb + 16 * i;
        bool v = kval && row_ok[i];
        int iy, ix;
        if (g.mode == MODE_FPROP) {
          iy = row_y[i] * g.stride + ky - g.pad;
          ix = row_x[i] * g.stride + kx - g.pad;
          v = v && iy >= 0 && iy < g.hv && ix >= 0 && ix < g.wv;
          if (g.up) {
            iy >>= 1;
            ix >>= 1;
          }
        } else {
          const int ty = row_y[i] + g.pad - ky, tx = row_x[i] + g.pad - kx;
          v = v && ty >= 0 && tx >= 0 && (ty % g.stride) == 0 && (tx % g.stride) == 0;
          iy = ty / g.stride;
          ix = tx / g.stride;
          v = v && iy < g.hv && ix < g.wv;
        }
        const float* p = g.src;
        if (v) p = g.src + (long long)row_img[i] * g.img_stride + (long long)iy * g.row_stride +
                   (long long)ix * g.ps + ci;
        cp_async_16(a_base + r * 128 + ((j ^ (r & 7)) << 4), p, v);
      }
      cp_async_arrive_noinc(&full[s]);
    }
    cp_async_wait_all();
    if (!ok) report_error(err, YL_DEVERR_TIMEOUT);
  } else if (warp == 4) {
    // ---------------- B-operand (weights) via TMA ----------------
    if (lane == 0) {
      uint32_t issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (kb >= S && !mbar_wait(&empty[s], ((kb / S) - 1) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        mbar_arrive_expect_tx(&full[s], Cfg::kBTileBytes);
        tma_load_2d(smem_u32(smem + s * Cfg::kStageBytes + kATileBytes), &tmap_w, &full[s],
                    kb * kBK, n0);
        ++issued;
      }
      // no copy may still be landing in shared memory when the CTA exits (the
      // gather threads' cp.async arrivals complete the same phases)
      drain_ring(full, S, issued);
    }
  } else {
    // ---------------- MMA issue (single thread) ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, BN, 0, 0);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&full[s], (kb / S) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t a_addr = smem_u32(smem + s * Cfg::kStageBytes);
        const uint32_t b_addr = a_addr + kATileBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint64_t ad = sw128_desc(a_addr + kk * 32, 16, 1024);
          const uint64_t bd = sw128_desc(b_addr + kk * 32, 16, 1024);
          umma_tf32(tmem, ad, bd, idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
      // every MMA this thread issued has completed before TMEM is released
      mbar_wait(accum, 0);
    }
  }

  // ---------------- epilogue: TMEM -> registers -> global ----------------
  if (warp < 4) {
    const bool got = mbar_wait(accum, 0, lim);
    if (!got) report_error(err, YL_DEVERR_TIMEOUT);
    tc_fence_after();
    const int row = warp * 32 + lane;
    const int m = m0 + row;
    const bool mval = got && m < g.m_total;
    const int img = mval ? m / (g.oh * g.ow) : 0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (n0 + c0 >= e.n_total) break;  // warp-uniform
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
      if (!mval) continue;
      const int nb = n0 + c0;
      float v[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
      if (e.bias) {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (nb + q < e.n_total) v[q] += __ldg(e.bias + nb + q);
      }
      if (e.bias2d) {
        const float* b2 = e.bias2d + (long long)img * e.n_total + nb;
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (nb + q < e.n_total) v[q] += __ldg(b2 + q);
      }
      const bool full32 = (nb + 32 <= e.n_total);
      if (e.residual) {
        const float* rp = e.residual + (long long)m * e.ldr + nb;
        if (full32 && (e.ldr & 3) == 0) {
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            float4 rv = *reinterpret_cast<const float4*>(rp + q);
            v[q] += rv.x; v[q + 1] += rv.y; v[q + 2] += rv.z; v[q + 3] += rv.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q)
            if (nb + q < e.n_total) v[q] += rp[q];
        }
      }
      if (e.round_tf32) {
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] = round_tf32(v[q]);
      }
      float* op = e.out + (long long)m * e.ldo + nb;
      if (full32 && (e.ldo & 3) == 0) {
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(op + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (nb + q < e.n_total) op[q] = v[q];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ wgrad
struct WgradArgs {
  const float* dy;
  int ldy;
  int cout;
  ConvGather g;         // the conv's input gather (FPROP coordinates); g.m_total = pixels
  int n_total;          // ksize^2 * cin
  int p_per_split;      // multiple of kBK
  float* ws;            // [split][cout][n_total]
  long long ws_split_stride;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) conv_wgrad_kernel(WgradArgs w, int* err) {
  using Cfg = TileCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
  const ConvGather& g = w.g;
  const int p_begin = blockIdx.z * w.p_per_split;
  const int p_end = min(g.m_total, p_begin + w.p_per_split);
  const int nk = p_end > p_begin ? (p_end - p_begin + kBK - 1) / kBK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const long long lim = wait_limit(err);

  if (warp < 4) {
    const int t = threadIdx.x;
    const int j = t & 7;
    const int r0 = t >> 3;  // this thread's rows: r0 and r0 + 16
    const int ohw = g.oh * g.ow;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S;
      if (kb >= S && !mbar_wait(&empty[s], ((kb / S) - 1) & 1, lim)) {
        ok = false;
        break;
      }
      const uint32_t a_base = smem_u32(smem + s * Cfg::kStageBytes);
      const uint32_t b_base = a_base + kATileBytes;
      // pixel decomposition of this thread's two rows
      int pimg[2], py[2], px[2];
      bool pval[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int p = p_begin + kb * kBK + r0 + 16 * h;
        pval[h] = p < p_end;
        const int pp = pval[h] ? p : 0;
        pimg[h] = pp / ohw;
        const int rem = pp - pimg[h] * ohw;
        py[h] = rem / g.ow;
        px[h] = rem - py[h] * g.ow;
      }
      // A = dy^T: 4 atoms of 32 output channels x 32 pixel rows
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int h = i & 1, a = i >> 1;
        const int r = r0 + 16 * h;
        const int co = m0 + 32 * a + 4 * j;
        const bool v = pval[h] && co < w.cout;
        const float* p = w.dy;
        if (v) p = w.dy + (long long)(p_begin + kb * kBK + r) * w.ldy + co;
        cp_async_16(a_base + a * 4096 + b32_swizzle(r, j), p, v);
      }
      // B = im2col(x)^T: BN/32 atoms of 32 (tap, ci) columns x 32 pixel rows
#pragma unroll
      for (int i = 0; i < BN / 16; ++i) {
        const int h = i & 1, a = i >> 1;
        const int r = r0 + 16 * h;
        const int n = n0 + 32 * a + 4 * j;
        bool v = pval[h] && n < w.n_total;
        const int tap = v ? n / g.cin : 0;
        const int ci = n - tap * g.cin;
        const int ky = tap / g.ksize, kx = tap - (tap / g.ksize) * g.ksize;
        int iy = py[h] * g.stride + ky - g.pad;
        int ix = px[h] * g.stride + kx - g.pad;
        v = v && iy >= 0 && iy < g.hv && ix >= 0 && ix < g.wv;
        if (g.up) {
          iy >>= 1;
          ix >>= 1;
        }
        const float* p = g.src;
        if (v) p = g.src + (long long)pimg[h] * g.img_stride + (long long)iy * g.row_stride +
                   (long long)ix * g.ps + ci;
        cp_async_16(b_base + a * 4096 + b32_swizzle(r, j), p, v);
      }
      cp_async_arrive_noinc(&full[s]);
    }
    cp_async_wait_all();
    if (!ok) report_error(err, YL_DEVERR_TIMEOUT);
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, BN, 1, 1);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&full[s], (kb / S) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        fence_proxy_async_smem();
        const uint32_t a_addr = smem_u32(smem + s * Cfg::kStageBytes);
        const uint32_t b_addr = a_addr + kATileBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          // MN-major tf32 needs SWIZZLE_128B_BASE32B: LBO = stride between
          // 32-element MN atoms (4096 B), SBO = stride between 4-row k groups
          // (512 B); one K=8 instruction covers 8 rows = 1024 B.
          const uint64_t ad = sw128b32_desc(a_addr + kk * 1024, 4096, 512);
          const uint64_t bd = sw128b32_desc(b_addr + kk * 1024, 4096, 512);
          umma_tf32(tmem, ad, bd, idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
      // every MMA this thread issued has completed before TMEM is released
      mbar_wait(accum, 0);
    }
  }

  if (warp < 4) {
    const bool got = mbar_wait(accum, 0, lim);
    if (!got) report_error(err, YL_DEVERR_TIMEOUT);
    tc_fence_after();
    const int co = m0 + warp * 32 + lane;
    const bool rval = got && co < w.cout;
    float* dst = w.ws + (long long)blockIdx.z * w.ws_split_stride + (long long)co * w.n_total;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (n0 + c0 >= w.n_total) break;
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
      if (!rval) continue;
      const int nb = n0 + c0;
      if (nk == 0) {
#pragma unroll
        for (int q = 0; q < 32; ++q) r[q] = 0u;
      }
      if (nb + 32 <= w.n_total && (w.n_total & 3) == 0) {
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(dst + nb + q) =
              make_float4(__uint_as_float(r[q]), __uint_as_float(r[q + 1]),
                          __uint_as_float(r[q + 2]), __uint_as_float(r[q + 3]));
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (nb + q < w.n_total) dst[nb + q] = __uint_as_float(r[q]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
static yl_status validate_gather(const ConvGather& g) {
  YL_CHECK(g.src != nullptr, YL_ERR_INVALID, "conv: source is NULL");
  YL_CHECK(g.ps % 4 == 0 && g.cin % 4 == 0 && g.cin <= g.ps, YL_ERR_SHAPE,
           "conv: pixel stride %d / channels %d must be multiples of 4", g.ps, g.cin);
  YL_CHECK(((uintptr_t)g.src & 15) == 0, YL_ERR_INVALID, "conv: source not 16-byte aligned");
  YL_CHECK(g.row_stride % 4 == 0 && g.img_stride % 4 == 0, YL_ERR_SHAPE,
           "conv: source strides must be multiples of 4 floats");
  YL_CHECK(g.ksize >= 1 && g.stride >= 1 && g.pad >= 0, YL_ERR_SHAPE, "conv: bad kernel geometry");
  YL_CHECK(g.k_total == g.ksize * g.ksize * g.cin, YL_ERR_SHAPE, "conv: k_total mismatch");
  YL_CHECK(g.m_total >= 0 && g.oh > 0 && g.ow > 0, YL_ERR_SHAPE, "conv: bad output grid");
  return YL_OK;
}

template <int BN>
static yl_status launch_gemm(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                             const ConvEpilogue& e) {
  using Cfg = TileCfg<BN>;
  CUtensorMap tm;
  YL_TRY(make_weight_tmap(&tm, w, n_rows, g.k_total, BN));
  YL_CUDA(cudaFuncSetAttribute(conv_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg::kSmemBytes));
  dim3 grid((g.m_total + kBM - 1) / kBM, (e.n_total + BN - 1) / BN);
  snprintf(ctx->last_kernel[0], sizeof(ctx->last_kernel[0]), "conv_gemm_kernel<%d>", BN);
  ctx->last_exec_flops[0] = 2.0 * g.m_total * (double)g.k_total * e.n_total;
  conv_gemm_kernel<BN><<<grid, kThreads, Cfg::kSmemBytes, ctx->stream>>>(tm, g, e, ctx->dev_err);
  return check_launch("conv_gemm_kernel");
}

yl_status conv_fprop_gather(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                            const ConvEpilogue& e) {
  YL_TRY(validate_gather(g));
  YL_CHECK(e.out && e.n_total > 0 && e.ldo >= e.n_total, YL_ERR_SHAPE, "conv: bad output");
  YL_CHECK(n_rows >= 1, YL_ERR_SHAPE, "conv: no weight rows");
  if (g.m_total == 0) return YL_OK;
  if (e.n_total <= 32) return launch_gemm<32>(ctx, g, w, n_rows, e);
  if (e.n_total <= 64) return launch_gemm<64>(ctx, g, w, n_rows, e);
  if (e.n_total <= 128 || e.n_total % 256 != 0) return launch_gemm<128>(ctx, g, w, n_rows, e);
  return launch_gemm<256>(ctx, g, w, n_rows, e);
}

yl_status conv_wgrad_gather(yl_ctx* ctx, const float* dy, int ldy, int cout,
                            const ConvGather& g, float* dw, int accumulate, float* ws,
                            int splits) {
  YL_TRY(validate_gather(g));
  YL_CHECK(dy && dw && ws, YL_ERR_INVALID, "wgrad: NULL argument");
  YL_CHECK(ldy % 4 == 0 && cout % 4 == 0 && ldy >= cout, YL_ERR_SHAPE,
           "wgrad: dy stride %d / channels %d must be multiples of 4", ldy, cout);
  YL_CHECK(((uintptr_t)dy & 15) == 0, YL_ERR_INVALID, "wgrad: dy not 16-byte aligned");
  YL_CHECK(splits >= 1, YL_ERR_INVALID, "wgrad: splits < 1");
  constexpr int BN = 128;
  using Cfg = TileCfg<BN>;
  const int n_total = g.k_total;
  long long kblocks = (g.m_total + kBK - 1) / kBK;
  long long per = (kblocks + splits - 1) / splits;
  WgradArgs a;
  a.dy = dy;
  a.ldy = ldy;
  a.cout = cout;
  a.g = g;
  a.n_total = n_total;
  a.p_per_split = (int)(per * kBK);
  a.ws = ws;
  a.ws_split_stride = (long long)cout * n_total;
  YL_CUDA(cudaFuncSetAttribute(conv_wgrad_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg::kSmemBytes));
  dim3 grid((cout + kBM - 1) / kBM, (n_total + BN - 1) / BN, splits);
  snprintf(ctx->last_kernel[1], sizeof(ctx->last_kernel[1]), "conv_wgrad_kernel<%d>", BN);
  ctx->last_exec_flops[1] = 2.0 * a.g.m_total * (double)a.g.k_total * a.cout;
  conv_wgrad_kernel<BN><<<grid, kThreads, Cfg::kSmemBytes, ctx->stream>>>(a, ctx->dev_err);
  YL_TRY(check_launch("conv_wgrad_kernel"));
  long long n = (long long)cout * n_total;
  splitk_reduce_kernel<<<grid_1d(n / 4 + 1, 256), 256, 0, ctx->stream>>>(ws, splits, n, dw, n,
                                                                         accumulate);
  return check_launch("splitk_reduce_kernel");
}

yl_status conv_wgrad(yl_ctx* ctx, const float* dy, int ldy, int cout, const ConvGather& g,
                     float* dw, int accumulate, float* db) {
  const int splits = conv_wgrad_pick_splits(ctx, cout, g, dy, ldy);
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, conv_wgrad_ws_floats(g, cout, dy, ldy, splits) * sizeof(float), &ws));
  return conv_wgrad_ws(ctx, dy, ldy, cout, g, dw, accumulate, (float*)ws, splits, db);
}

// ------------------------------------------------------------------ reductions / layouts
// Per-(image, chunk) partial column sums of dy, then a fixed-order total.
__global__ void channel_partial_kernel(const float* __restrict__ dy, long long hw, int ldy, int c,
                                       int chunks, float* __restrict__ part) {
  const int img = blockIdx.x / chunks, chunk = blockIdx.x % chunks;
  const int col = blockIdx.y * 32 + threadIdx.x;
  const long long per = (hw + chunks - 1) / chunks;
  const long long p0 = chunk * per, p1 = min(hw, p0 + per);
  float s = 0.f;
  if (col < c) {
    const float* base = dy + (long long)img * hw * ldy + col;
    for (long long p = p0 + threadIdx.y; p < p1; p += blockDim.y) s += base[p * ldy];
  }
  __shared__ float red[8][33];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && col < c) {
    float t = 0.f;
    for (int y = 0; y < (int)blockDim.y; ++y) t += red[y][threadIdx.x];
    part[(long long)blockIdx.x * c + col] = t;
  }
}

__global__ void channel_final_kernel(const float* __restrict__ part, int images, int chunks, int c,
                                     float* db, float* db_img, int accumulate) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= c) return;
  float total = 0.f;
  for (int img = 0; img < images; ++img) {
    float s = 0.f;
    for (int k = 0; k < chunks; ++k) s += part[((long long)img * chunks + k) * c + col];
    if (db_img) db_img[(long long)img * c + col] = s;
    total += s;
  }
  if (db) db[col] = accumulate ? db[col] + total : total;
}

yl_status channel_sums(yl_ctx* ctx, const float* dy, int images, long long hw, int ldy, int c,
                       float* db, float* db_img, int accumulate) {
  if (!db && !db_img) return YL_OK;
  int chunks = (int)std::max(1LL, std::min(64LL, hw / 2048));
  while ((long long)images * chunks > 4096 && chunks > 1) chunks /= 2;
  void* ws = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)images * chunks * c * sizeof(float), &ws));
  dim3 grid(images * chunks, (c + 31) / 32);
  channel_partial_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(dy, hw, ldy, c, chunks,
                                                                (float*)ws);
  YL_TRY(check_launch("channel_partial_kernel"));
  channel_final_kernel<<<(c + 127) / 128, 128, 0, ctx->stream>>>((float*)ws, images, chunks, c, db,
                                                                 db_img, accumulate);
  return check_launch("channel_final_kernel");
}

__global__ void weight_permute_kernel(const float* __restrict__ in, float* __restrict__ out, int O,
                                      int T, int I_out, int I_src, long long so, long long st,
                                      long long si, int round) {
  const long long n = (long long)O * T * I_out;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % I_out);
    const long long r = idx / I_out;
    const int t = (int)(r % T);
    const int o = (int)(r / T);
    float v = i < I_src ? in[o * so + t * st + i * si] : 0.f;
    out[idx] = round ? round_tf32(v) : v;
  }
}

yl_status weight_permute(yl_ctx* ctx, const float* in, float* out, int O, int T, int I_out,
                         int I_src, long long so, long long st, long long si, int round) {
  long long n = (long long)O * T * I_out;
  weight_permute_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(in, out, O, T, I_out, I_src, so,
                                                                  st, si, round);
  return check_launch("weight_permute_kernel");
}

// 3x3 neighbourhoods of a 4-channel NHWC tensor as 64-channel pixels:
// out[p][t * 4 + c] = src[p + sign * (ky - 1, kx - 1)][c] for tap t = ky * 3 + kx
// (zero outside the image), channels 36..63 zero.  With sign +1 a 3x3 conv of
// src becomes a 1x1 conv of out; with sign -1 (src = an output gradient) the
// same patches give the conv's dX and dW as 1x1 GEMMs.
__global__ void rgb_patches_kernel(const float* __restrict__ src, int ld, int n, int h, int w,
                                   int sign, int round, float* __restrict__ out) {
  const long long total = (long long)n * h * w * 16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i & 15);
    const long long pix = i >> 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < 9) {
      const int x = (int)(pix % w);
      const long long r = pix / w;
      const int y = (int)(r % h);
      const long long img = r / h;
      const int yy = y + sign * (t / 3 - 1), xx = x + sign * (t % 3 - 1);
      if (yy >= 0 && yy < h && xx >= 0 && xx < w) {
        v = __ldg(reinterpret_cast<const float4*>(src + ((img * h + yy) * w + xx) * ld));
        if (round) v = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
      }
    }
    reinterpret_cast<float4*>(out)[i] = v;
  }
}

yl_status rgb_patches(yl_ctx* ctx, const float* src, int ld, int n, int h, int w, int sign,
                      int round, float* out) {
  YL_CHECK(ld % 4 == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)out & 15) == 0, YL_ERR_SHAPE,
           "rgb_patches: 16-byte pixels required");
  rgb_patches_kernel<<<grid_1d((long long)n * h * w * 16, 256), 256, 0, ctx->stream>>>(
      src, ld, n, h, w, sign, round, out);
  return check_launch("rgb_patches_kernel");
}

// y[p][c] = bias[c] + sum_t z[p + (ky - 1, kx - 1)][t * 4 + c]: the tap sum
// that turns the 36-channel 1x1 product z = x * W[t][c] into the 3x3 conv
// with 4 output channels.
__global__ void rgb_tap_sum_kernel(const float* __restrict__ z, int n, int h, int w,
                                   const float* __restrict__ bias, float* __restrict__ y,
                                   int ldy) {
  const long long total = (long long)n * h * w;
  for (long long pix = blockIdx.x * (long long)blockDim.x + threadIdx.x; pix < total;
       pix += (long long)gridDim.x * blockDim.x) {
    const int x = (int)(pix % w);
    const long long r = pix / w;
    const int yv = (int)(r % h);
    const long long img = r / h;
    float4 acc = bias ? make_float4(bias[0], bias[1], bias[2], bias[3])
                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const int yy = yv + t / 3 - 1, xx = x + t % 3 - 1;
      if (yy < 0 || yy >= h || xx < 0 || xx >= w) continue;
      const float4 v = __ldg(reinterpret_cast<const float4*>(z + ((img * h + yy) * w + xx) * 36) + t);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    *reinterpret_cast<float4*>(y + pix * ldy) = acc;
  }
}

yl_status rgb_tap_sum(yl_ctx* ctx, const float* z, int n, int h, int w, const float* bias,
                      float* y, int ldy) {
  YL_CHECK(ldy % 4 == 0 && ((uintptr_t)z & 15) == 0 && ((uintptr_t)y & 15) == 0, YL_ERR_SHAPE,
           "rgb_tap_sum: 16-byte pixels required");
  rgb_tap_sum_kernel<<<grid_1d((long long)n * h * w, 256), 256, 0, ctx->stream>>>(z, n, h, w, bias,
                                                                                 y, ldy);
  return check_launch("rgb_tap_sum_kernel");
}

// Many weight_permute jobs in one launch: each block takes 4096-element items
// of one job (found by binary search on the item prefix sums).
constexpr long long kPermItem = 4096;

__global__ void weight_permute_batch_kernel(const PermuteJob* __restrict__ jobs, int njobs,
                                            const long long* __restrict__ item_start) {
  const long long items = item_start[njobs];
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    int lo = 0, hi = njobs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (item_start[mid] <= it) lo = mid;
      else hi = mid - 1;
    }
    const PermuteJob& j = jobs[lo];
    const long long n = (long long)j.O * j.T * j.I_out;
    const long long base = (it - item_start[lo]) * kPermItem;
    const long long end = min(n, base + kPermItem);
    for (long long idx = base + threadIdx.x; idx < end; idx += blockDim.x) {
      const int i = (int)(idx % j.I_out);
      const long long r = idx / j.I_out;
      const int t = (int)(r % j.T);
      const int o = (int)(r / j.T);
      const float v = i < j.I_src ? j.in[o * j.so + t * j.st + i * j.si] : 0.f;
      j.out[idx] = j.round ? round_tf32(v) : v;
    }
  }
}

yl_status weight_permute_batch(yl_ctx* ctx, const std::vector<PermuteJob>& jobs,
                               PermuteBatchBuffers* bufs) {
  if (jobs.empty()) return YL_OK;
  if (!bufs->jobs) {
    // the table lives on the device for the owner's lifetime (pointers are fixed)
    std::vector<long long> start(jobs.size() + 1, 0);
    for (size_t k = 0; k < jobs.size(); ++k) {
      const long long n = (long long)jobs[k].O * jobs[k].T * jobs[k].I_out;
      start[k + 1] = start[k] + (n + kPermItem - 1) / kPermItem;
    }
    YL_CUDA(cudaMalloc(&bufs->jobs, jobs.size() * sizeof(PermuteJob)));
    YL_CUDA(cudaMalloc(&bufs->item_start, start.size() * sizeof(long long)));
    YL_CUDA(cudaMemcpyAsync(bufs->jobs, jobs.data(), jobs.size() * sizeof(PermuteJob),
                            cudaMemcpyHostToDevice, ctx->stream));
    YL_CUDA(cudaMemcpyAsync(bufs->item_start, start.data(), start.size() * sizeof(long long),
                            cudaMemcpyHostToDevice, ctx->stream));
    YL_CUDA(cudaStreamSynchronize(ctx->stream));  // host vectors go out of scope
    bufs->njobs = (int)jobs.size();
    bufs->items = start.back();
  }
  const int grid = (int)std::min<long long>(bufs->items, (long long)ctx->num_sms * 8);
  weight_permute_batch_kernel<<<grid, 256, 0, ctx->stream>>>(bufs->jobs, bufs->njobs,
                                                             bufs->item_start);
  return check_launch("weight_permute_batch_kernel");
}

PermuteBatchBuffers::~PermuteBatchBuffers() {
  if (jobs) cudaFree(jobs);
  if (item_start) cudaFree(item_start);
}

// 32 x 32 tiled transposes between [n][c][hw] and [n][hw][ps].
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ in, float* __restrict__ out, int c,
                                    long long hw, int ps, int round) {
  __shared__ float tile[32][33];
  const int img = blockIdx.z;
  const long long p0 = (long long)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int ch = c0 + k;
    const long long p = p0 + threadIdx.x;
    tile[k][threadIdx.x] = (ch < c && p < hw) ? in[((long long)img * c + ch) * hw + p] : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const long long p = p0 + k;
    const int ch = c0 + threadIdx.x;
    if (p < hw && ch < ps) {
      float v = tile[threadIdx.x][k];
      out[((long long)img * hw + p) * ps + ch] = round ? round_tf32(v) : v;
    }
  }
}

__global__ void nhwc_to_nchw_kernel(const float* __restrict__ in, float* __restrict__ out, int c,
                                    long long hw, int ps) {
  __shared__ float tile[32][33];
  const int img = blockIdx.z;
  const long long p0 = (long long)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const long long p = p0 + k;
    const int ch = c0 + threadIdx.x;
    tile[k][threadIdx.x] = (p < hw && ch < c) ? in[((long long)img * hw + p) * ps + ch] : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int ch = c0 + k;
    const long long p = p0 + threadIdx.x;
    if (ch < c && p < hw) out[((long long)img * c + ch) * hw + p] = tile[threadIdx.x][k];
  }
}

yl_status nchw_to_nhwc(yl_ctx* ctx, const float* in, float* out, int n, int c, long long hw, int ps,
                       int round) {
  YL_CHECK(ps >= c, YL_ERR_SHAPE, "nchw_to_nhwc: pixel stride %d < channels %d", ps, c);
  dim3 grid((unsigned)((hw + 31) / 32), (ps + 31) / 32, n);
  nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(in, out, c, hw, ps, round);
  return check_launch("nchw_to_nhwc_kernel");
}

yl_status nhwc_to_nchw(yl_ctx* ctx, const float* in, float* out, int n, int c, long long hw,
                       int ps) {
  dim3 grid((unsigned)((hw + 31) / 32), (c + 31) / 32, n);
  nhwc_to_nchw_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(in, out, c, hw, ps);
  return check_launch("nhwc_to_nchw_kernel");
}

// Sum of the (up to) 2x2 block of the cropped up-grid (uh x uw) that maps to
// each source pixel: the adjoint of the nearest upsample the decoder's
// "up + conv" reads (downsample2x_kernel, MetalKernelSourcesA.swift:440).
__global__ void downsample_sum_nhwc_kernel(const float* __restrict__ src, int uh, int uw,
                                           float* __restrict__ dst, int n, int h, int w, int c4,
                                           int ps_src, int ps_dst) {
  const long long total = (long long)n * h * w * c4;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int cq = (int)(idx % c4);
    long long r = idx / c4;
    const int x = (int)(r % w);
    r /= w;
    const int y = (int)(r % h);
    const int img = (int)(r / h);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int dy2 = 0; dy2 < 2; ++dy2)
#pragma unroll
      for (int dx2 = 0; dx2 < 2; ++dx2) {
        const int yy = 2 * y + dy2, xx = 2 * x + dx2;
        if (yy < uh && xx < uw) {
          float4 v = *reinterpret_cast<const float4*>(
              src + (((long long)img * uh + yy) * uw + xx) * ps_src + 4 * cq);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
      }
    *reinterpret_cast<float4*>(dst + (((long long)img * h + y) * w + x) * ps_dst + 4 * cq) = acc;
  }
}

yl_status downsample_sum_nhwc(yl_ctx* ctx, const float* src, int uh, int uw, float* dst, int n,
                              int h, int w, int c, int ps_src, int ps_dst) {
  YL_CHECK(c % 4 == 0 && ps_src % 4 == 0 && ps_dst % 4 == 0, YL_ERR_SHAPE,
           "downsample_sum_nhwc: channels must be multiples of 4");
  long long total = (long long)n * h * w * (c / 4);
  downsample_sum_nhwc_kernel<<<grid_1d(total, 256), 256, 0, ctx->stream>>>(src, uh, uw, dst, n, h,
                                                                           w, c / 4, ps_src, ps_dst);
  return check_launch("downsample_sum_nhwc_kernel");
}

}  // namespace yl
