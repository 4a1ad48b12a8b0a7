// yl_conv_tma.cu -- convolution through TMA boxes: every operand tile of the
// implicit GEMM is a rectangular box of an NHWC tensor or of one of its 2x2
// "phase views" (the sub-lattice of pixels (2i+a, 2j+b), itself a strided
// 4-D tensor), loaded by one thread with out-of-range reads as zero (= the
// convolution padding).  A small tap table says which view and which offset
// each tap reads, so one kernel covers:
//   * stride-1 conv forward and its dX (the flipped taps),
//   * stride-2 conv forward (each tap reads one input phase view),
//   * nearest-x2 upsample + 3x3 conv forward as four output phases, each a
//     2x2 conv on the source with merged weights (16 MACs per output instead
//     of 36, no upsampled tensor) -- the decoder's "up + conv",
//   * stride-2 dX as four output phases with 1, 2, 2 and 4 taps,
// and one wgrad kernel covers stride-1, stride-2 (input phase views) and
// upsample-conv (output-gradient phase views) filter gradients.
// Shapes the tap tables do not cover fall back to the cp.async gathers of
// yl_conv.cu.
#include <cstdio>

#include "yl_conv_common.cuh"
#include "yl_norm.h"

namespace yl {

yl_status conv_fprop_gather(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                            const ConvEpilogue& e);
yl_status conv_wgrad_gather(yl_ctx* ctx, const float* dy, int ldy, int cout,
                            const ConvGather& g, float* dw, int accumulate, float* ws,
                            int splits);

constexpr int kMaxTaps = 16;

struct TapPhase {
  int ntaps, w_row0, ya, xa;
  int8_t map[kMaxTaps], dy[kMaxTaps], dx[kMaxTaps];
};

struct ConvPlan {
  int cpt;             // 32-channel chunks per tap
  int gh, gw;          // tile grid extent (the output phase lattice)
  int n_img, tiles_x, tiles_y;
  int out_h, out_w;    // output tensor extent
  int ys, xs;          // output pixel = (oy * ys + ya, ox * xs + xa)
  int n_nblk;          // BN-wide blocks of output channels
  int pix_tiles;       // tiles_x * tiles_y * n_img
  int n_tiles;         // pix_tiles * n_nblk * phases
  int tma_out;         // non-transposed epilogue: stage rows in shared memory, TMA store
  int* sched;          // [0] tiles handed out past the first wave, [1] CTAs done; both
                       // zero at launch and reset by the last CTA (nullptr: static order)
  TapPhase ph[4];      // indexed by the tile's phase
};

// Tiles reach the MMA and epilogue warps through a small shared-memory ring
// written by the producer warp, which takes each CTA's first tile by its block
// index and every later one from the launch's atomic counter: a CTA that
// starts late or runs slower (an SM shared with another kernel) simply takes
// fewer tiles instead of holding up the launch with a fixed share.
constexpr int kTileRing = 8;
constexpr int kRingTimeout = -2;

__device__ __forceinline__ int next_tile(const ConvPlan& p, uint32_t k) {
  if (k == 0) return blockIdx.x;
  if (p.sched) return (int)gridDim.x + atomicAdd(p.sched, 1);
  return (int)(blockIdx.x + k * gridDim.x);
}
// Producer: publish the CTA's k-th tile (>= n_tiles: no more tiles).
__device__ __forceinline__ bool ring_put(uint64_t* tfull, uint64_t* tempty, volatile int* ring,
                                         uint32_t k, int tile, long long lim) {
  const uint32_t s = k % kTileRing;
  if (k >= kTileRing && !mbar_wait(&tempty[s], ((k / kTileRing) - 1) & 1, lim)) return false;
  ring[s] = tile;
  mbar_arrive(&tfull[s]);  // release: the consumers' wait acquires the store
  return true;
}
// MMA thread: the CTA's k-th tile (kRingTimeout when the wait gave up).
__device__ __forceinline__ int ring_take(uint64_t* tfull, uint64_t* tempty,
                                         const volatile int* ring, uint32_t k, long long lim) {
  const uint32_t s = k % kTileRing;
  if (!mbar_wait(&tfull[s], (k / kTileRing) & 1, lim)) return kRingTimeout;
  const int t = ring[s];
  mbar_arrive(&tempty[s]);
  return t;
}
// Epilogue warp: every lane reads the tile, lane 0 releases the slot.
__device__ __forceinline__ int ring_take_warp(uint64_t* tfull, uint64_t* tempty,
                                              const volatile int* ring, uint32_t k,
                                              long long lim, int lane) {
  const uint32_t s = k % kTileRing;
  const bool ok = mbar_wait(&tfull[s], (k / kTileRing) & 1, lim);
  const int t = ok ? ring[s] : kRingTimeout;
  __syncwarp();
  if (ok && lane == 0) mbar_arrive(&tempty[s]);
  return __shfl_sync(0xffffffffu, t, 0);
}

// A tile is MT x 128 GEMM rows (MT*4 lattice rows x 32 lattice columns) by BN
// output channels.  MT = 2 gives two M=128 accumulators that share every B
// (weight) tile, which halves the weight bytes per MMA for cout <= 128.
template <int BN, int MT>
struct FpropCfg {
  static constexpr int kATile = MT * kATileBytes;
  static constexpr int kBTile = BN * 128;
  static constexpr int kStage = kATile + kBTile;
  // output staging of the non-transposed epilogue: 2 buffers of one lattice
  // row (32 pixels x 32 channels, 4 KB) per epilogue warp
  static constexpr int kOut = 4 * 2 * 4096;
  static constexpr int kFit = (227 * 1024 - kOut - 2048) / kStage;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kAccCols = MT * BN < 32 ? 32 : MT * BN;
  static constexpr int kTmemCols = 2 * kAccCols;  // two accumulator buffers
  static constexpr int kSmemBytes =
      kStages * kStage + kOut + (2 * kStages + 5 + 2 * 8) * 8 + 4 * 8 + 16 + 1024;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
  static_assert(kSmemBytes <= 227 * 1024, "stages exceed shared memory");
};

// HALO (transposed 128 x 256 tile of a stride-1 3x3 conv): the three taps of
// one kernel column (same dx, dy = d, d+1, d+2) read one box of 8 + 2 lattice
// rows, and tap j's 256-pixel operand starts j image rows (4 KB, a whole
// number of 1024-byte swizzle atoms) into it.  The boxes and the weight tiles
// stream through two rings so each box is fetched once per three MMAs: 40 KB
// of pixels per 3 taps instead of 96 KB.
struct HaloCfg {
  static constexpr int kBoxRows = 10;
  static constexpr int kABox = 32 * kBoxRows * 128;  // 40 KB
  static constexpr int kWTile = 128 * 128;           // 16 KB
  static constexpr int kAS = 2, kWS = 6;
  static constexpr int kOut = 4 * 2 * 4096;  // epilogue staging, as FpropCfg::kOut
  static constexpr int kRing = kAS * kABox + kWS * kWTile + kOut;
  static constexpr int kSmemBytes = kRing + (2 * (kAS + kWS) + 5 + 2 * 8) * 8 + 4 * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "halo rings exceed shared memory");
};

struct FpropTile {
  int nb, z, img, ty, tx;
};

__device__ __forceinline__ FpropTile fprop_tile(const ConvPlan& p, int t) {
  FpropTile c;
  c.nb = t % p.n_nblk;
  t /= p.n_nblk;
  const int pix = t % p.pix_tiles;
  c.z = t / p.pix_tiles;
  c.tx = pix % p.tiles_x;
  const int r = pix / p.tiles_x;
  c.ty = r % p.tiles_y;
  c.img = r / p.tiles_y;
  return c;
}

// GroupNorm statistics from the conv epilogue.  Partial (sum, sum of squares)
// per (tile, slot, group of the tile's channel block) go to e.gn_part; a
// slot is one epilogue warp's share of the tile (one warp per lattice row
// and subtile without TR, the whole tile with TR).
template <int CG>
__device__ __forceinline__ void gn_chunk_partials(const float (&v)[32], bool valid,
                                                  float2* part_row, int g0, int lane) {
  // per-lane (sum, sumsq) of each of the chunk's 32/CG groups, then a
  // transposing butterfly: every exchange halves the values a lane keeps until
  // one group is left, then plain xor steps finish that group's sum
  constexpr int NG = 32 / CG;
  float val[2 * NG];
#pragma unroll
  for (int k = 0; k < NG; ++k) {
    float s = 0.f, ss = 0.f;
    if (valid) {
#pragma unroll
      for (int i = 0; i < CG; ++i) {
        const float x = v[k * CG + i];
        s += x;
        ss += x * x;
      }
    }
    val[2 * k] = s;
    val[2 * k + 1] = ss;
  }
  int grp = 0;
#pragma unroll
  for (int o = 16, n = 2 * NG; o >= 1; o >>= 1) {
    if (n > 2) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = upper ? val[i] : val[i + n / 2];
        const float keep = upper ? val[i + n / 2] : val[i];
        val[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
      grp = grp * 2 + (upper ? 1 : 0);
      n /= 2;
    } else {
      val[0] += __shfl_xor_sync(0xffffffffu, val[0], o);
      val[1] += __shfl_xor_sync(0xffffffffu, val[1], o);
    }
  }
  // lanes that differ only in the plain-reduction bits hold the same group
  constexpr int kSplitBits = NG == 8 ? 3 : NG == 4 ? 2 : NG == 2 ? 1 : 0;
  if ((lane & ((1 << (5 - kSplitBits)) - 1)) == 0) part_row[g0 + grp] = make_float2(val[0], val[1]);
}

__device__ __forceinline__ void gn_chunk_partials_any(int cg, const float (&v)[32], bool valid,
                                                      float2* part_row, int g0, int lane) {
  switch (cg) {
    case 4: gn_chunk_partials<4>(v, valid, part_row, g0, lane); break;
    case 8: gn_chunk_partials<8>(v, valid, part_row, g0, lane); break;
    case 16: gn_chunk_partials<16>(v, valid, part_row, g0, lane); break;
    default: gn_chunk_partials<32>(v, valid, part_row, g0, lane); break;
  }
}

// Persistent: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// Warp 4 streams A/B k-blocks through the shared-memory ring across tile
// boundaries, warp 5 issues the MMAs into one of two TMEM accumulator
// buffers, warps 0-3 drain the other buffer (epilogue) meanwhile.
//
// TR (transposed accumulator, BN = 128, MT = 2): the weight tile is the MMA's
// A operand (M = 128 output channels) and the 256-pixel tile its B operand
// (N = 256), one M=128 x N=256 MMA per K step instead of two 128 x 128 ones.
// TMEM then holds [channel][pixel]: epilogue thread = one output channel,
// and each store instruction of a warp writes 32 consecutive channels of one
// pixel.
template <int BN, int MT, bool TR = false, bool HALO = false>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tma_fprop_kernel(const __grid_constant__ CUtensorMap ta0,
                          const __grid_constant__ CUtensorMap ta1,
                          const __grid_constant__ CUtensorMap ta2,
                          const __grid_constant__ CUtensorMap ta3,
                          const __grid_constant__ CUtensorMap tw,
                          const __grid_constant__ CUtensorMap to0,
                          const __grid_constant__ CUtensorMap to1,
                          const __grid_constant__ CUtensorMap to2,
                          const __grid_constant__ CUtensorMap to3, ConvPlan p, ConvEpilogue e,
                          int* err) {
  static_assert(!HALO || (TR && BN == 128 && MT == 2), "halo boxes feed the transposed tile");
  using Cfg = FpropCfg<BN, MT>;
  constexpr int S = Cfg::kStages;
  constexpr int kRows = 4 * MT;  // lattice rows per tile
  constexpr int kRing = HALO ? HaloCfg::kRing : S * Cfg::kStage + Cfg::kOut;
  // epilogue staging: 2 buffers of 4 KB per epilogue warp after the operand rings
  constexpr int kOutOff = HALO ? kRing - HaloCfg::kOut : S * Cfg::kStage;
  constexpr int kRingBars = HALO ? 2 * (HaloCfg::kAS + HaloCfg::kWS) : 2 * S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  // plain: full[S], empty[S]; halo: box full/empty [kAS], weight full/empty [kWS]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRing);
  uint64_t* empty = full + S;
  uint64_t* acc_full = full + kRingBars;  // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;     // [2]: epilogue (128 threads) -> MMA
  uint64_t* drain = acc_empty + 2;        // MMA thread: all of its MMAs completed
  uint64_t* tfull = drain + 1;            // [kTileRing]: producer -> MMA + epilogue
  uint64_t* tempty = tfull + kTileRing;   // [kTileRing]: MMA + 4 epilogue warps -> producer
  int* tring = reinterpret_cast<int*>(tempty + kTileRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tring + kTileRing);
  static_assert(kTileRing == 8, "the shared-memory budgets above reserve 8 ring slots");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long lim = wait_limit(err);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRingBars; ++s) mbar_init(&full[s], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    for (int r = 0; r < kTileRing; ++r) {
      mbar_init(&tfull[r], 1);
      mbar_init(&tempty[r], 1 + 4);
    }
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&ta0);
    tma_prefetch_desc(&tw);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (HALO && warp == 4) {
    if (lane == 0) {
      // per tile: kernel column g (taps g, g+3, g+6), 32-channel chunk c:
      // one 10-row pixel box, then the three taps' weight tiles
      constexpr int AS = HaloCfg::kAS, WS = HaloCfg::kWS;
      uint64_t* afull = full;
      uint64_t* aempty = full + AS;
      uint64_t* wfull = full + 2 * AS;
      uint64_t* wempty = wfull + WS;
      uint32_t ia = 0, iw = 0;  // box / weight fills issued
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int tile = next_tile(p, k);
        if (!ring_put(tfull, tempty, tring, k, tile, lim)) {
          ok = false;
          break;
        }
        if (tile >= p.n_tiles) break;
        const FpropTile c = fprop_tile(p, tile);
        const TapPhase& ph = p.ph[0];
        const int ox0 = c.tx * 32, oy0 = c.ty * kRows, n0 = c.nb * BN;
        for (int g = 0; ok && g < 3; ++g) {
          const int dy0 = min(ph.dy[g], min(ph.dy[g + 3], ph.dy[g + 6]));
          for (int ch = 0; ok && ch < p.cpt; ++ch) {
            const int sa = ia % AS;
            if (ia >= AS && !mbar_wait(&aempty[sa], ((ia / AS) - 1) & 1, lim)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&afull[sa], HaloCfg::kABox);
            tma_load_4d(smem_u32(smem + sa * HaloCfg::kABox), &ta0, &afull[sa], ch * 32,
                        ox0 + ph.dx[g], oy0 + dy0, c.img);
            ++ia;
            for (int j = 0; j < 3; ++j) {
              const int sw = iw % WS;
              if (iw >= WS && !mbar_wait(&wempty[sw], ((iw / WS) - 1) & 1, lim)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&wfull[sw], HaloCfg::kWTile);
              tma_load_2d(smem_u32(smem + AS * HaloCfg::kABox + sw * HaloCfg::kWTile), &tw,
                          &wfull[sw], ((g + 3 * j) * p.cpt + ch) * kBK, ph.w_row0 + n0);
              ++iw;
            }
          }
        }
      }
      if (!ok) report_error(err, YL_DEVERR_TIMEOUT);
      // no copy may still be landing in shared memory when the CTA exits
      drain_ring(afull, AS, ia);
      drain_ring(wfull, WS, iw);
    }
  } else if (HALO && warp == 5) {
    if (lane == 0) {
      constexpr int AS = HaloCfg::kAS, WS = HaloCfg::kWS;
      uint64_t* afull = full;
      uint64_t* aempty = full + AS;
      uint64_t* wfull = full + 2 * AS;
      uint64_t* wempty = wfull + WS;
      constexpr uint32_t idesc = idesc_tf32(BN, MT * kBM, 0, 0);
      uint32_t ia = 0, iw = 0;
      int tc = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k, ++tc) {
        const int tile = ring_take(tfull, tempty, tring, k, lim);
        if (tile == kRingTimeout) {
          ok = false;
          break;
        }
        if (tile >= p.n_tiles) break;
        const int buf = tc & 1, use = tc >> 1;
        if (tc >= 2 && !mbar_wait(&acc_empty[buf], (use - 1) & 1, lim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const TapPhase& ph = p.ph[0];
        const uint32_t dacc = tmem + (uint32_t)(buf * Cfg::kAccCols);
        for (int g = 0; ok && g < 3; ++g) {
          const int dy0 = min(ph.dy[g], min(ph.dy[g + 3], ph.dy[g + 6]));
          for (int ch = 0; ch < p.cpt; ++ch, ++ia) {
            const int sa = ia % AS;
            if (!mbar_wait(&afull[sa], (ia / AS) & 1, lim)) {
              ok = false;
              break;
            }
            const uint32_t box = smem_u32(smem + sa * HaloCfg::kABox);
            for (int j = 0; j < 3; ++j, ++iw) {
              const int sw = iw % WS;
              if (!mbar_wait(&wfull[sw], (iw / WS) & 1, lim)) {
                ok = false;
                break;
              }
              tc_fence_after();
              // tap j's pixels: image row (dy - dy0) of the box, 32 px x 128 B per row
              const uint32_t px = box + (uint32_t)((ph.dy[g + 3 * j] - dy0) * 32 * 128);
              const uint32_t wt = smem_u32(smem + AS * HaloCfg::kABox + sw * HaloCfg::kWTile);
#pragma unroll
              for (int kk = 0; kk < kBK / 8; ++kk)
                umma_tf32(dacc, sw128_desc(wt + kk * 32, 16, 1024),
                          sw128_desc(px + kk * 32, 16, 1024), idesc, (g | ch | j | kk) != 0);
              umma_commit(&wempty[sw]);
            }
            if (!ok) break;
            umma_commit(&aempty[sa]);
          }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      if (!ok) report_error(err, YL_DEVERR_TIMEOUT);
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp == 4) {
    if (lane == 0) {
      const CUtensorMap* maps[4] = {&ta0, &ta1, &ta2, &ta3};
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int tile = next_tile(p, k);
        if (!ring_put(tfull, tempty, tring, k, tile, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        if (tile >= p.n_tiles) break;
        const FpropTile c = fprop_tile(p, tile);
        const TapPhase& ph = p.ph[c.z];
        const int nk = ph.ntaps * p.cpt;
        const int ox0 = c.tx * 32, oy0 = c.ty * kRows, n0 = c.nb * BN;
        int t = 0, chunk = 0;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1, lim)) {
            report_error(err, YL_DEVERR_TIMEOUT);
            ok = false;
            break;
          }
          const uint32_t a_dst = smem_u32(smem + s * Cfg::kStage);
          mbar_arrive_expect_tx(&full[s], Cfg::kStage);
          tma_load_4d(a_dst, maps[ph.map[t]], &full[s], chunk * 32, ox0 + ph.dx[t],
                      oy0 + ph.dy[t], c.img);
          tma_load_2d(a_dst + Cfg::kATile, &tw, &full[s], kb * kBK, ph.w_row0 + n0);
          if (++chunk == p.cpt) {
            chunk = 0;
            ++t;
          }
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      drain_ring(full, S, it);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = TR ? idesc_tf32(BN, MT * kBM, 0, 0) : idesc_tf32(kBM, BN, 0, 0);
      uint32_t it = 0;
      int tc = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k, ++tc) {
        const int tile = ring_take(tfull, tempty, tring, k, lim);
        if (tile == kRingTimeout) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        if (tile >= p.n_tiles) break;
        const int buf = tc & 1, use = tc >> 1;
        if (tc >= 2 && !mbar_wait(&acc_empty[buf], (use - 1) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const FpropTile c = fprop_tile(p, tile);
        const int nk = p.ph[c.z].ntaps * p.cpt;
        const uint32_t dacc = tmem + (uint32_t)(buf * Cfg::kAccCols);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, lim)) {
            report_error(err, YL_DEVERR_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * Cfg::kStage);
          const uint32_t b_addr = a_addr + Cfg::kATile;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint64_t bdesc = sw128_desc(b_addr + kk * 32, 16, 1024);
            if constexpr (TR) {
              umma_tf32(dacc, bdesc, sw128_desc(a_addr + kk * 32, 16, 1024), idesc,
                        (kb | kk) != 0);
            } else {
#pragma unroll
              for (int m = 0; m < MT; ++m)
                umma_tf32(dacc + (uint32_t)(m * BN),
                          sw128_desc(a_addr + m * kATileBytes + kk * 32, 16, 1024), bdesc, idesc,
                          (kb | kk) != 0);
            }
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else {
    // epilogue: warp w owns TMEM lanes 32w..32w+31 = lattice row 4m + w of subtile m
    int tc = 0;
    uint32_t ost = 0;  // TMA-stored row chunks of this warp (staging buffer = ost & 1)
    for (uint32_t k = 0;; ++k, ++tc) {
      const int tile = ring_take_warp(tfull, tempty, tring, k, lim, lane);
      if (tile == kRingTimeout) {
        report_error(err, YL_DEVERR_TIMEOUT);
        break;
      }
      if (tile >= p.n_tiles) break;
      const int buf = tc & 1, use = tc >> 1;
      const FpropTile c = fprop_tile(p, tile);
      const TapPhase& ph = p.ph[c.z];
      const int n0 = c.nb * BN;
      if constexpr (TR) {
        // while the accumulator is still being computed: pull this tile's
        // residual into L2, one 128-byte line of 32 channels per thread and
        // lattice row
        const int t = warp * 32 + lane, q = t >> 2, ch = n0 + (t & 3) * 32;
        const int gx = c.tx * 32 + q, X = gx * p.xs + ph.xa;
        if (e.residual && ch < e.n_total && gx < p.gw && X < p.out_w) {
#pragma unroll 1
          for (int j = 0; j < kRows; ++j) {
            const int gy = c.ty * kRows + j, Y = gy * p.ys + ph.ya;
            if (gy >= p.gh || Y >= p.out_h) break;
            const long long pix = ((long long)c.img * p.out_h + Y) * p.out_w + X;
            prefetch_l2(e.residual + pix * e.ldr + ch);
          }
        }
      }
      if (!mbar_wait(&acc_full[buf], use & 1, lim)) {
        report_error(err, YL_DEVERR_TIMEOUT);
        break;
      }
      tc_fence_after();
      if constexpr (TR) {
        // lane row = output channel, column = pixel (lattice row j of the tile, column q)
        const int co = n0 + warp * 32 + lane;
        const bool cval = co < e.n_total;
        float badd = 0.f;
        if (cval && e.bias) badd += __ldg(e.bias + co);
        if (cval && e.bias2d) badd += __ldg(e.bias2d + (long long)c.img * e.n_total + co);
        const uint32_t tbase =
            tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * Cfg::kAccCols);
        float gs = 0.f, gss = 0.f;  // GroupNorm partials of this channel
#pragma unroll 1
        for (int j = 0; j < kRows; ++j) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + (uint32_t)(j * 32), r);
          tmem_ld_wait();
          const int gy = c.ty * kRows + j;
          const int Y = gy * p.ys + ph.ya;
          if (gy >= p.gh || Y >= p.out_h) continue;
          const long long rowp = ((long long)c.img * p.out_h + Y) * p.out_w;
          // columns q < qn are inside the lattice and the image (both bounds
          // are monotone in q); addresses advance by a fixed 32-bit stride
          const int X0 = c.tx * 32 * p.xs + ph.xa;
          int qn = p.gw - c.tx * 32;
          if (qn > 32) qn = 32;
          const int qx = X0 < p.out_w ? (p.out_w - X0 + p.xs - 1) / p.xs : 0;
          if (qx < qn) qn = qx;
          // all residual loads first: out may alias nothing, but the compiler
          // cannot know that and would otherwise wait on each load in turn
          float v[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]) + badd;
          if (e.residual) {
            const float* rrow = e.residual + (rowp + X0) * e.ldr + (cval ? co : 0);
            const int sr = p.xs * e.ldr;
            float rv[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) rv[q] = cval && q < qn ? rrow[q * sr] : 0.f;
#pragma unroll
            for (int q = 0; q < 32; ++q) v[q] += rv[q];
          }
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            if (e.round_tf32) v[q] = round_tf32(v[q]);
            if (cval && q < qn) {
              gs += v[q];
              gss += v[q] * v[q];
            }
          }
          if (p.tma_out) {
            // staging row q = pixel q, this lane's channel at 4-byte column
            // `lane` of the 128-byte row (16-byte chunks swizzled by q), then
            // one TMA store of the warp's 32 pixels x 32 channels
            uint8_t* ob = smem + kOutOff + (warp * 2 + (ost & 1)) * 4096;
            if (ost >= 2) {
              if (lane == 0) bulk_wait_group_read<1>();
              __syncwarp();
            }
            const uint32_t col = (uint32_t)(lane & 3) << 2;
#pragma unroll
            for (int q = 0; q < 32; ++q)
              *reinterpret_cast<float*>(ob + q * 128 + ((((lane >> 2) ^ (q & 7)) << 4) | col)) =
                  v[q];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const CUtensorMap* om = c.z == 0 ? &to0 : c.z == 1 ? &to1 : c.z == 2 ? &to2 : &to3;
              tma_store_4d(om, smem_u32(ob), n0 + warp * 32, c.tx * 32, gy, c.img);
              bulk_commit_group();
            }
            ++ost;
          } else if (cval) {
            float* orow = e.out + (rowp + X0) * e.ldo + co;
            const int so = p.xs * e.ldo;
#pragma unroll
            for (int q = 0; q < 32; ++q)
              if (q < qn) orow[q * so] = v[q];
          }
        }
        if (e.gn_part) {
          // the cg lanes of a group are consecutive: butterfly over them
          for (int o = 1; o < e.gn_cg; o <<= 1) {
            gs += __shfl_xor_sync(0xffffffffu, gs, o);
            gss += __shfl_xor_sync(0xffffffffu, gss, o);
          }
          const int gpb = BN / e.gn_cg;
          if ((lane & (e.gn_cg - 1)) == 0)
            e.gn_part[(long long)tile * gpb + (warp * 32 + lane) / e.gn_cg] = make_float2(gs, gss);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
#pragma unroll 1
      for (int m = 0; m < MT; ++m) {
        const int gy = c.ty * kRows + m * 4 + warp, gx = c.tx * 32 + lane;
        const int Y = gy * p.ys + ph.ya, X = gx * p.xs + ph.xa;
        const bool mval = gy < p.gh && gx < p.gw && Y < p.out_h && X < p.out_w;
        const long long mrow = ((long long)c.img * p.out_h + Y) * p.out_w + X;
        const uint32_t tbase = tmem + ((uint32_t)(warp * 32) << 16) +
                               (uint32_t)(buf * Cfg::kAccCols + m * BN);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          if (n0 + c0 >= e.n_total) break;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + (uint32_t)c0, r);
          tmem_ld_wait();
          const int nb = n0 + c0;
          float v[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
          if (mval) {
            if (e.bias) {
#pragma unroll
              for (int q = 0; q < 32; ++q)
                if (nb + q < e.n_total) v[q] += __ldg(e.bias + nb + q);
            }
            if (e.bias2d) {
              const float* b2 = e.bias2d + (long long)c.img * e.n_total + nb;
#pragma unroll
              for (int q = 0; q < 32; ++q)
                if (nb + q < e.n_total) v[q] += __ldg(b2 + q);
            }
            const bool full32 = (nb + 32 <= e.n_total);
            if (e.residual) {
              const float* rp = e.residual + mrow * e.ldr + nb;
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
            if (!p.tma_out) {
              float* op = e.out + mrow * e.ldo + nb;
              if (full32 && (e.ldo & 3) == 0) {
#pragma unroll
                for (int q = 0; q < 32; q += 4)
                  *reinterpret_cast<float4*>(op + q) =
                      make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
              } else {
#pragma unroll
                for (int q = 0; q < 32; ++q)
                  if (nb + q < e.n_total) op[q] = v[q];
              }
            }
          }
          if (p.tma_out) {
            // the warp's lattice row (32 pixels x these 32 channels) through a
            // 128-byte-swizzled staging buffer and one TMA store: whole lines
            // per request instead of 16-byte pieces of 32 pixels' lines
            uint8_t* ob = smem + kOutOff + (warp * 2 + (ost & 1)) * 4096;
            if (ost >= 2) {
              if (lane == 0) bulk_wait_group_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(ob + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && gy < p.gh) {
              const CUtensorMap* om = c.z == 0 ? &to0 : c.z == 1 ? &to1 : c.z == 2 ? &to2 : &to3;
              tma_store_4d(om, smem_u32(ob), nb, c.tx * 32, gy, c.img);
              bulk_commit_group();
            }
            ++ost;
          }
          if (e.gn_part) {
            const int gpb = BN / e.gn_cg;
            float2* row = e.gn_part + ((long long)tile * (MT * 4) + m * 4 + warp) * gpb;
            gn_chunk_partials_any(e.gn_cg, v, mval, row, c0 / e.gn_cg, lane);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    if (p.tma_out && lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  // the last CTA to finish returns the launch's tile counter to zero (this
  // CTA's producer took its last tile before the barrier above)
  if (threadIdx.x == 0 && p.sched) {
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
      __threadfence();
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

// ------------------------------------------------------------------ wgrad
// WG_UP: the filter gradient of a nearest-x2 upsample + 3x3 conv as four
// independent GEMMs, one per output phase (a, b): the merged 2x2 taps of that
// phase against the phase view of dy, at the source resolution (16 merged
// taps instead of 9 taps at the output resolution); a final pass sums the
// merged gradients back onto the 9 kernel taps.
enum WgradMode : int { WG_PLAIN = 0, WG_STRIDE2 = 1, WG_UP = 2 };

struct WgradPlan {
  int mode;
  int nblk_ph;            // WG_UP: column blocks per output phase
  int gh, gw, xblocks;    // k-block lattice (WG_UP: the source resolution)
  int n_img;
  long long blocks, per_split;
  int ksize, pad, cin, cout, n_total;
  int ga, gb;             // 32-channel atoms per A (dy) / B (input) TMA box
  float* ws;
  long long ws_split_stride;
  // optional bias gradient: the first column block of each (phase, split)
  // also sums its dy tiles per channel into db_ws[phase * splits + split][cout]
  float* db_ws;
};

// dW tile: MT x 128 output channels (rows) by NSUB x NW columns of
// [tap][cin]; k-blocks are BKP lattice columns of one lattice row.  A = dy
// (MT*4 atoms of 32 output channels), B = the input pixels each column's tap
// reads (NSUB*NW/32 atoms of 32 input channels, a tile may span several
// taps); both MN-major in SWIZZLE_128B_ATOM_32B.  MT = 2 shares every B atom
// between two M=128 accumulators, NSUB = 2 shares every A atom between two
// MMAs: both raise the MMA work per byte brought in from L2.
template <int MT, int NSUB, int NW, int BKP>
struct WgradCfg {
  static constexpr int kAtomBytes = BKP * 128;
  static constexpr int kBN = NSUB * NW;
  static constexpr int kAAtoms = MT * 4;
  static constexpr int kBAtoms = kBN / 32;
  static constexpr int kATile = kAAtoms * kAtomBytes;
  static constexpr int kStage = kATile + kBAtoms * kAtomBytes;
  static constexpr int kStages = (200 * 1024) / kStage > 8 ? 8 : (200 * 1024) / kStage;
  static constexpr int kCols = MT * kBN;
  static constexpr int kTmemCols =
      kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  static constexpr int kSmemBytes = kStages * kStage + (2 * kStages + 2) * 8 + 16 + 1024;
  static_assert(NW % 32 == 0 && NW >= 32 && NW <= 256, "MMA N");
  static_assert(kCols <= 512, "accumulators exceed TMEM");
  static_assert(BKP % 8 == 0, "k-block is whole K=8 MMA steps");
};

// Where B atom j of a tile reads: which input view and the lattice offset of
// its tap (for an upsample conv the offset also depends on the dy phase kp).
struct WgAtom {
  int8_t map, by, bx;
  int ci;
};

__device__ __forceinline__ WgAtom wgrad_atom(const WgradPlan& w, int n, int kp) {
  WgAtom a;
  const int tap = n / w.cin;
  a.ci = n - tap * w.cin;
  const int kw = w.mode == WG_UP ? 2 : w.ksize;  // merged taps form a 2x2 grid
  const int ky = tap / kw, kx = tap - (tap / kw) * kw;
  if (w.mode == WG_PLAIN) {
    a.map = 0;
    a.by = (int8_t)(ky - w.pad);
    a.bx = (int8_t)(kx - w.pad);
  } else if (w.mode == WG_STRIDE2) {
    const int ry = ky - w.pad, rx = kx - w.pad;
    a.map = (int8_t)(((ry & 1) << 1) | (rx & 1));
    a.by = (int8_t)(ry >> 1);
    a.bx = (int8_t)(rx >> 1);
  } else {  // WG_UP: column n of phase kp = (pa, pb) is merged tap (ty, tx) = (ky, kx) < 2
    const int pa = kp >> 1, pb = kp & 1;
    a.map = 0;
    a.by = (int8_t)(ky + pa - 1);
    a.bx = (int8_t)(kx + pb - 1);
  }
  return a;
}

template <int MT, int NSUB, int NW, int BKP>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tma_wgrad_kernel(const __grid_constant__ CUtensorMap ta0,
                          const __grid_constant__ CUtensorMap ta1,
                          const __grid_constant__ CUtensorMap ta2,
                          const __grid_constant__ CUtensorMap ta3,
                          const __grid_constant__ CUtensorMap tb0,
                          const __grid_constant__ CUtensorMap tb1,
                          const __grid_constant__ CUtensorMap tb2,
                          const __grid_constant__ CUtensorMap tb3, WgradPlan w, int* err) {
  using Cfg = WgradCfg<MT, NSUB, NW, BKP>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStage);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * (MT * kBM);
  // WG_UP: blockIdx.y = (output phase, column block within the phase)
  const int phase = w.mode == WG_UP ? (int)blockIdx.y / w.nblk_ph : 0;
  const int n0 = (w.mode == WG_UP ? (int)blockIdx.y % w.nblk_ph : (int)blockIdx.y) * Cfg::kBN;
  const int col0 = w.mode == WG_UP ? phase * 4 * w.cin + n0 : n0;
  const long long b_begin = blockIdx.z * w.per_split;
  const long long b_end = min(w.blocks, b_begin + w.per_split);
  const int nk = b_end > b_begin ? (int)(b_end - b_begin) : 0;
  // the epilogue warps read every dy stage for the bias gradient and release
  // it together with the MMA warp
  const bool with_db = w.db_ws != nullptr && n0 == 0;
  const long long lim = wait_limit(err);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], with_db ? 1 + 128 : 1);
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

  if (warp == 4) {
    if (lane == 0 && nk > 0) {
      const CUtensorMap* amaps[4] = {&ta0, &ta1, &ta2, &ta3};
      const CUtensorMap* bmaps[4] = {&tb0, &tb1, &tb2, &tb3};
      // k-blocks walk each image in column strips of BKP lattice columns, down
      // the rows of a strip: the rows a tap row reads again one or two
      // k-blocks later (and the other column tiles of this pixel range read at
      // the same time) are still in L2, so every input byte comes from DRAM
      // about once
      long long r = b_begin;
      int gy = (int)(r % w.gh);
      r /= w.gh;
      int xb = (int)(r % w.xblocks);
      int im = (int)(r / w.xblocks);
      const CUtensorMap* amap = amaps[phase];
      WgAtom at[Cfg::kBAtoms];
#pragma unroll
      for (int j = 0; j < Cfg::kBAtoms; ++j) at[j] = wgrad_atom(w, n0 + 32 * j, phase);
      uint32_t issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (kb >= S && !mbar_wait(&empty[s], ((kb / S) - 1) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        const uint32_t a_dst = smem_u32(smem + s * Cfg::kStage);
        const uint32_t b_dst = a_dst + Cfg::kATile;
        const int gx0 = xb * BKP;
        mbar_arrive_expect_tx(&full[s], Cfg::kStage);
        for (int a = 0; a < Cfg::kAAtoms; a += w.ga)
          tma_load_5d(a_dst + a * Cfg::kAtomBytes, amap, &full[s], 0, gx0, gy, m0 / 32 + a, im);
        // the atom table stays in registers: both loops have constant trip counts
        if (w.gb == 4) {
#pragma unroll
          for (int j = 0; j < Cfg::kBAtoms; j += 4)
            tma_load_5d(b_dst + j * Cfg::kAtomBytes, bmaps[at[j].map], &full[s], 0,
                        gx0 + at[j].bx, gy + at[j].by, at[j].ci / 32, im);
        } else {
#pragma unroll
          for (int j = 0; j < Cfg::kBAtoms; ++j)
            tma_load_5d(b_dst + j * Cfg::kAtomBytes, bmaps[at[j].map], &full[s], 0,
                        gx0 + at[j].bx, gy + at[j].by, at[j].ci / 32, im);
        }
        ++issued;
        if (++gy == w.gh) {
          gy = 0;
          if (++xb == w.xblocks) {
            xb = 0;
            if (++im == w.n_img) im = 0;
          }
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      drain_ring(full, S, issued);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, NW, 1, 1);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&full[s], (kb / S) & 1, lim)) {
          report_error(err, YL_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * Cfg::kStage);
        const uint32_t b_addr = a_addr + Cfg::kATile;
#pragma unroll
        for (int kk = 0; kk < BKP / 8; ++kk) {
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint64_t adesc =
                sw128b32_desc(a_addr + m * 4 * Cfg::kAtomBytes + kk * 1024, Cfg::kAtomBytes, 512);
#pragma unroll
            for (int j = 0; j < NSUB; ++j)
              umma_tf32(tmem + (uint32_t)(m * Cfg::kBN + j * NW), adesc,
                        sw128b32_desc(b_addr + j * (NW / 32) * Cfg::kAtomBytes + kk * 1024,
                                      Cfg::kAtomBytes, 512),
                        idesc, (kb | kk) != 0);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
      // every MMA this thread issued has completed before TMEM is released
      mbar_wait(accum, 0);
    }
  }

  if (warp < 4 && with_db) {
    // thread t sums channels m0 + t (+ 128) over the pixel rows of every stage;
    // channel c sits in atom c / 32, 16-byte chunk (c % 32) / 4 of each row
    const int t = threadIdx.x;
    float sum[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sum[m] = 0.f;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&full[s], (kb / S) & 1, lim)) {
        report_error(err, YL_DEVERR_TIMEOUT);
        break;
      }
      const uint8_t* a_tile = smem + s * Cfg::kStage;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const int c = m * kBM + t;
        const uint8_t* atom = a_tile + (c >> 5) * Cfg::kAtomBytes + ((c & 3) << 2);
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < BKP; ++r)
          acc += *reinterpret_cast<const float*>(atom + b32_swizzle(r, (c & 31) >> 2));
        sum[m] += acc;
      }
      mbar_arrive(&empty[s]);
    }
    const long long row = (long long)(phase * gridDim.z + blockIdx.z) * w.cout;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const int co = m0 + m * kBM + t;
      if (co < w.cout) w.db_ws[row + co] = sum[m];
    }
  }

  if (warp < 4) {
    const bool got = mbar_wait(accum, 0, lim);
    if (!got) report_error(err, YL_DEVERR_TIMEOUT);
    tc_fence_after();
#pragma unroll 1
    for (int m = 0; m < MT; ++m) {
      const int co = m0 + m * kBM + warp * 32 + lane;
      const bool rval = got && co < w.cout;
      float* dst =
          w.ws + (long long)blockIdx.z * w.ws_split_stride + (long long)co * w.n_total + col0 - n0;
#pragma unroll 1
      for (int c0 = 0; c0 < Cfg::kBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(m * Cfg::kBN + c0),
                           r);
        tmem_ld_wait();
        if (!rval) continue;
        if (nk == 0) {
#pragma unroll
          for (int q = 0; q < 32; ++q) r[q] = 0u;
        }
        const int nb = n0 + c0;
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(dst + nb + q) =
              make_float4(__uint_as_float(r[q]), __uint_as_float(r[q + 1]),
                          __uint_as_float(r[q + 2]), __uint_as_float(r[q + 3]));
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

// ------------------------------------------------------------------ weight transforms
// Row taps of output phase a for nearest-x2 upsample + 3x3 conv (pad 1):
// phase a = 0 reads source rows i-1 (kernel row 0) and i (rows 1, 2);
// phase a = 1 reads rows i (kernel rows 0, 1) and i+1 (row 2).
__device__ __forceinline__ bool up_row_in(int a, int t, int k) {
  return a == 0 ? (t == 0 ? k == 0 : k >= 1) : (t == 0 ? k <= 1 : k == 2);
}
// out[ph][co][t][ci] = sum of w[co][ky*3+kx][ci] over the kernel taps phase
// ph = (a, b) merges into its tap t = (ty, tx); rounded to tf32.
__global__ void up_merge_weights_kernel(const float* __restrict__ w, float* __restrict__ out,
                                        int rows, int cin) {
  const long long n = 4LL * rows * 4 * cin;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ci = (int)(i % cin);
    long long r = i / cin;
    const int t = (int)(r % 4);
    r /= 4;
    const int co = (int)(r % rows);
    const int ph = (int)(r / rows);
    const int a = ph >> 1, b = ph & 1, ty = t >> 1, tx = t & 1;
    float s = 0.f;
    for (int ky = 0; ky < 3; ++ky) {
      if (!up_row_in(a, ty, ky)) continue;
      for (int kx = 0; kx < 3; ++kx)
        if (up_row_in(b, tx, kx)) s += w[((long long)co * 9 + ky * 3 + kx) * cin + ci];
    }
    out[i] = round_tf32(s);
  }
}

// Stride-2 (pad 1) dX, output phase a: kernel rows with (a + 1 - ky) even.
// a = 0: {ky 1 (dy row offset 0)}; a = 1: {ky 0 (offset +1), ky 2 (offset 0)}.
__device__ __forceinline__ int s2_rows(int a, int* ks, int* offs) {
  if (a == 0) {
    ks[0] = 1;
    offs[0] = 0;
    return 1;
  }
  ks[0] = 0;
  offs[0] = 1;
  ks[1] = 2;
  offs[1] = 0;
  return 2;
}
// out[ci][ph * 4 + t][co] = sum of wd[ci][ky*3+kx][co] over the kernel taps
// that output phase ph = (a, b) merges into its source tap t = (ty, tx) (wd
// is the dgrad weight [ci][9][co]); rounded to tf32.  The dX of an upsample
// conv reads the four phase views of dy through these 16 merged taps.
__global__ void up_merge_dgrad_weights_kernel(const float* __restrict__ wd,
                                              float* __restrict__ out, int rows, int cout) {
  const long long n = 16LL * rows * cout;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(i % cout);
    long long r = i / cout;
    const int pt = (int)(r % 16);
    const int ci = (int)(r / 16);
    const int ph = pt >> 2, t = pt & 3;
    const int a = ph >> 1, b = ph & 1, ty = t >> 1, tx = t & 1;
    float s = 0.f;
    for (int ky = 0; ky < 3; ++ky) {
      if (!up_row_in(a, ty, ky)) continue;
      for (int kx = 0; kx < 3; ++kx)
        if (up_row_in(b, tx, kx)) s += wd[((long long)ci * 9 + ky * 3 + kx) * cout + co];
    }
    out[i] = round_tf32(s);
  }
}

// out[ph][ci][t][co] = wd[ci][tap(ph, t)][co] (wd is the dgrad weight [ci][9][co]).
__global__ void s2_phase_weights_kernel(const float* __restrict__ wd, float* __restrict__ out,
                                        int rows, int cout) {
  const long long n = 4LL * rows * 4 * cout;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(i % cout);
    long long r = i / cout;
    const int t = (int)(r % 4);
    r /= 4;
    const int ci = (int)(r % rows);
    const int ph = (int)(r / rows);
    int kr[2], orr[2], kc[2], oc[2];
    const int nr = s2_rows(ph >> 1, kr, orr), nc = s2_rows(ph & 1, kc, oc);
    float v = 0.f;
    if (t < nr * nc) {
      const int ky = kr[t / nc], kx = kc[t % nc];
      v = wd[((long long)ci * 9 + ky * 3 + kx) * cout + co];
    }
    out[i] = v;
  }
}

// ------------------------------------------------------------------ cropped x2 grids
// A nearest-x2 upsample cut to hv x wv (hv in {2sh - 1, 2sh}, wv in {2sw - 1,
// 2sw}) runs through the merged phase taps of the whole 2sh x 2sw grid U,
// whose phase outputs the tensor maps clip to the cut grid u.  The merged
// taps then still read U's pixels outside u -- the last upsampled column
// (X' = wv when wv < 2sw) and row (Y' = hv when hv < 2sh), which u's zero
// padding replaces -- and only the outputs next to the cut see them.  These
// kernels subtract exactly those terms: a few border pixels' worth of work.

// Border pixel b of a cut grid of ext_h x ext_w: the last column (when col)
// for rows [0, ext_h), then the last row for the columns the column did not
// already cover (crop_border_count counts both).
__device__ __forceinline__ void crop_border_pixel(int b, bool col, int ext_h, int ext_w, int* y,
                                                  int* x) {
  const int ncol = col ? ext_h : 0;
  if (b < ncol) {
    *y = b;
    *x = ext_w - 1;
  } else {
    *y = ext_h - 1;
    *x = b - ncol;
  }
}
__host__ __device__ __forceinline__ int crop_border_count(bool col, bool row, int ext_h,
                                                           int ext_w) {
  return (col ? ext_h : 0) + (row ? ext_w - (col ? 1 : 0) : 0);
}

// Taps that can reach outside u: kernel column 2 (a cut column) or row 2 (a
// cut row) -- taps 2, 5, 8 and 6, 7 of the 3x3 kernel.
__device__ __forceinline__ int cut_tap(int t5) { return t5 < 2 ? 2 + 3 * t5 : t5 + 4; }

// The three fixes are small gathered GEMMs, C[m][n] -= sum_k A[m][k] B[k][n],
// whose missing terms read as zero.  One 256-thread block per 32 x 32 tile
// of C: k streams through shared memory in 128-deep stages, each thread
// holding 4 outputs, and the gather offsets are worked out once per tap group
// (rows) or per stage (columns) into shared memory.  Fixed summation order:
// the results are deterministic.
constexpr int kCutKS = 128;

__device__ __forceinline__ void cut_fix_stage_fma(const float (&As)[kCutKS][33],
                                                  const float (&Bs)[kCutKS][33], int tx, int ty,
                                                  float (&acc)[4]) {
#pragma unroll 8
  for (int kk = 0; kk < kCutKS; ++kk) {
    const float bv = Bs[kk][tx];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = fmaf(As[kk][ty + 8 * j], bv, acc[j]);
  }
}

// Row gathers: C[m][n] -= sum over groups g and c < gk of
// A[arow(m, g) + c] * B[brow(n, g) + c] (an offset of -1 is a missing row).
template <class Op>
__global__ void __launch_bounds__(256) cut_fix_rows_kernel(Op op) {
  __shared__ float As[kCutKS][33], Bs[kCutKS][33];
  __shared__ long long ao[32], bo[32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int n0 = blockIdx.x * 32, m0 = blockIdx.y * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int g = 0; g < op.groups; ++g) {
    if (threadIdx.x < 32) ao[threadIdx.x] = op.arow(m0 + (int)threadIdx.x, g);
    else if (threadIdx.x < 64) bo[threadIdx.x - 32] = op.brow(n0 + (int)threadIdx.x - 32, g);
    // a group no row of this tile uses is skipped (the barrier publishes ao / bo)
    if (!__syncthreads_or(threadIdx.x < 32 && ao[threadIdx.x] >= 0)) continue;
    for (int c0 = 0; c0 < op.gk; c0 += kCutKS) {
#pragma unroll 4
      for (int i = 0; i < kCutKS * 32 / 256; ++i) {
        const int e = threadIdx.x + 256 * i, kk = e % kCutKS, r = e / kCutKS;
        const bool in = c0 + kk < op.gk;
        As[kk][r] = in && ao[r] >= 0 ? op.A[ao[r] + c0 + kk] : 0.f;
        Bs[kk][r] = in && bo[r] >= 0 ? op.B[bo[r] + c0 + kk] : 0.f;
      }
      __syncthreads();
      cut_fix_stage_fma(As, Bs, tx, ty, acc);
      __syncthreads();
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) op.store(m0 + ty + 8 * j, n0 + tx, acc[j]);
}

// Column gathers (one GEMM per tap, blockIdx.z): C[m][n] -= sum over k < gk
// of A[acol(k) + m] * B[bcol(k) + n] (-1: the term does not exist).
template <class Op>
__global__ void __launch_bounds__(256) cut_fix_cols_kernel(Op op) {
  __shared__ float As[kCutKS][33], Bs[kCutKS][33];
  __shared__ long long ao[kCutKS], bo[kCutKS];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int n0 = blockIdx.x * 32, m0 = blockIdx.y * 32, z = blockIdx.z;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < op.gk; k0 += kCutKS) {
    if (threadIdx.x < kCutKS) {
      long long a = -1, b = -1;
      op.cols(z, k0 + (int)threadIdx.x, &a, &b);
      ao[threadIdx.x] = a;
      bo[threadIdx.x] = b;
    }
    if (!__syncthreads_or(threadIdx.x < kCutKS && ao[threadIdx.x] >= 0)) continue;
#pragma unroll 4
    for (int i = 0; i < kCutKS * 32 / 256; ++i) {
      const int e = threadIdx.x + 256 * i, r = e % 32, kk = e / 32;
      As[kk][r] = ao[kk] >= 0 && m0 + r < op.M ? op.A[ao[kk] + m0 + r] : 0.f;
      Bs[kk][r] = bo[kk] >= 0 && n0 + r < op.N ? op.B[bo[kk] + n0 + r] : 0.f;
    }
    __syncthreads();
    cut_fix_stage_fma(As, Bs, tx, ty, acc);
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) op.store(z, m0 + ty + 8 * j, n0 + tx, acc[j]);
}

// Forward: out[img][Y][X][co] -= sum over taps (ky, kx) whose source pixel
// (Y', X') = (Y + ky - 1, X + kx - 1) lies in U but not in u of
// w[co][ky*3+kx][:] . x[img][Y'/2][X'/2][:], for the output pixels on the
// cut row / column.  m = (image, border pixel), n = co, groups = taps,
// c = ci.  A = x, B = w [cout][9][cin].
struct CutFixFprop {
  const float* A;
  const float* B;
  float* out;
  int ps, sh, sw, cin, cout, hv, wv, ldo, round, nb, M;
  bool col;
  int groups, gk;
  __device__ long long arow(int m, int g) const {
    if (m >= M) return -1;
    const int img = m / nb;
    int Y, X;
    crop_border_pixel(m - img * nb, col, hv, wv, &Y, &X);
    const int tap = cut_tap(g), yy = Y + tap / 3 - 1, xx = X + tap % 3 - 1;
    if (yy < 0 || yy >= 2 * sh || xx < 0 || xx >= 2 * sw || (yy < hv && xx < wv)) return -1;
    return (((long long)img * sh + (yy >> 1)) * sw + (xx >> 1)) * ps;
  }
  __device__ long long brow(int n, int g) const {
    return n < cout ? ((long long)n * 9 + cut_tap(g)) * cin : -1;
  }
  __device__ void store(int m, int n, float v) const {
    if (m >= M || n >= cout) return;
    const int img = m / nb;
    int Y, X;
    crop_border_pixel(m - img * nb, col, hv, wv, &Y, &X);
    float* op = out + (((long long)img * hv + Y) * wv + X) * ldo + n;
    const float r = *op - v;
    *op = round ? round_tf32(r) : r;
  }
};

// dX at the source resolution: dx[img][i][j][ci] -= the part of the merged
// sum that comes from the upsampled pixels of U outside u, du[Y'][X'] =
// sum_taps wd[ci][ky*3+kx][:] . dy[img][Y' - ky + 1][X' - kx + 1][:] (dy is
// hv x wv), over (Y', X') in {2i, 2i+1} x {2j, 2j+1} with Y' >= hv or X' >= wv.
// m = (image, border source pixel), n = ci, groups = (pixel of the 2x2
// block, tap), c = co.  A = dy, B = wd [cin][9][cout].
struct CutFixDgrad {
  const float* A;
  const float* B;
  float* dx;
  int ldy, cout, sh, sw, hv, wv, cin, ldo, round, nb, M;
  bool col;
  int groups, gk;
  __device__ long long arow(int m, int g) const {
    if (m >= M) return -1;
    const int img = m / nb;
    int i, j;
    crop_border_pixel(m - img * nb, col, sh, sw, &i, &j);
    const int v4 = g / 5, tap = cut_tap(g - 5 * v4);
    const int vy = 2 * i + (v4 >> 1), vx = 2 * j + (v4 & 1);
    if (vy < hv && vx < wv) return -1;  // a pixel of u: no excess
    const int yy = vy - tap / 3 + 1, xx = vx - tap % 3 + 1;
    if (yy < 0 || yy >= hv || xx < 0 || xx >= wv) return -1;
    return (((long long)img * hv + yy) * wv + xx) * ldy;
  }
  __device__ long long brow(int n, int g) const {
    return n < cin ? ((long long)n * 9 + cut_tap(g % 5)) * cout : -1;
  }
  __device__ void store(int m, int n, float v) const {
    if (m >= M || n >= cin) return;
    const int img = m / nb;
    int i, j;
    crop_border_pixel(m - img * nb, col, sh, sw, &i, &j);
    float* op = dx + (((long long)img * sh + i) * sw + j) * ldo + n;
    const float r = *op - v;
    *op = round ? round_tf32(r) : r;
  }
};

// Filter gradient: dw[co][ky*3+kx][ci] -= sum over images and the output
// pixels (Y, X) on the cut row / column whose tap source (Y', X') lies in U
// but not in u of dy[img][Y][X][co] * x[img][Y'/2][X'/2][ci].  One GEMM per
// tap that can reach outside u (blockIdx.z): m = co, n = ci, k = (image,
// border pixel).  A = dy, B = x.
struct CutFixWgrad {
  const float* A;
  const float* B;
  float* dw;
  int ldy, M, ps, N, sh, sw, hv, wv, nb;  // M = cout, N = cin
  bool col;
  int gk;  // n_img * nb
  __device__ void cols(int z, int k, long long* ao, long long* bo) const {
    if (k >= gk) return;
    const int img = k / nb;
    int Y, X;
    crop_border_pixel(k - img * nb, col, hv, wv, &Y, &X);
    const int tap = cut_tap(z), yy = Y + tap / 3 - 1, xx = X + tap % 3 - 1;
    if (yy < 0 || yy >= 2 * sh || xx < 0 || xx >= 2 * sw || (yy < hv && xx < wv)) return;
    *ao = (((long long)img * hv + Y) * wv + X) * ldy;
    *bo = (((long long)img * sh + (yy >> 1)) * sw + (xx >> 1)) * ps;
  }
  __device__ void store(int z, int m, int n, float v) const {
    if (m < M && n < N) dw[((long long)m * 9 + cut_tap(z)) * N + n] -= v;
  }
};

// ------------------------------------------------------------------ host side
struct View {
  const float* base;
  int c, w, h, n;
  long long sx, sy, sn;  // strides in floats
};

static View plain_view(const float* p, int c, int w, int h, int n, int ps) {
  return View{p, c, w, h, n, ps, (long long)w * ps, (long long)h * w * ps};
}
// Pixels (2i + a, 2j + b) of a w x h NHWC tensor as their own tensor.
static View phase_view(const float* p, int c, int w, int h, int n, int ps, int a, int b) {
  return View{p + ((long long)a * w + b) * ps, c, (w - b + 1) / 2, (h - a + 1) / 2, n,
              2LL * ps, 2LL * w * ps, (long long)h * w * ps};
}

// 4-D map {c, w, h, n} of a view with a box of box_c x box_w x box_h x 1.
// Returns false (and records nothing) when the view cannot be described:
// unaligned base or pixel stride, an empty extent, or an encode failure.
static bool encode_view_tmap(CUtensorMap* tm, const View& v, int box_c, int box_h,
                             CUtensorMapSwizzle swz, int box_w, int* cu_err) {
  *cu_err = 0;
  auto fn = get_encode_fn();
  if (!fn || ((uintptr_t)v.base & 15) != 0 || v.sx % 4 != 0 || v.w < 1 || v.h < 1) return false;
  cuuint64_t dims[4] = {(cuuint64_t)v.c, (cuuint64_t)v.w, (cuuint64_t)v.h, (cuuint64_t)v.n};
  cuuint64_t strides[3] = {(cuuint64_t)v.sx * 4, (cuuint64_t)v.sy * 4, (cuuint64_t)v.sn * 4};
  cuuint32_t box[4] = {(cuuint32_t)box_c, (cuuint32_t)box_w, (cuuint32_t)box_h, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(v.base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *cu_err = (int)r;
  return r == CUDA_SUCCESS;
}

static yl_status make_view_tmap(CUtensorMap* tm, const View& v, int box_c, int box_h,
                                CUtensorMapSwizzle swz, int box_w = 32) {
  YL_CHECK(get_encode_fn(), YL_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  int cu_err = 0;
  YL_CHECK(encode_view_tmap(tm, v, box_c, box_h, swz, box_w, &cu_err),
           cu_err ? YL_ERR_CUDA : YL_ERR_INVALID, "view tensor map: %s (%d)",
           cu_err ? "cuTensorMapEncodeTiled failed" : "alignment / extent", cu_err);
  return YL_OK;
}

// 5-D map of a view split into 32-channel atoms {32, w, h, atoms, n}; a box
// is `atoms` whole atoms of box_w pixels of one row, stored atom after atom
// (the MN-major operand layout).  A view with fewer than 32 channels is one
// partial atom (the rest of the box reads as zero); otherwise the channel
// count must be a multiple of 32.
static yl_status make_atom_tmap(CUtensorMap* tm, const View& v, int box_w, int atoms,
                                CUtensorMapSwizzle swz) {
  auto fn = get_encode_fn();
  YL_CHECK(fn, YL_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  YL_CHECK(((uintptr_t)v.base & 15) == 0 && v.sx % 4 == 0 && v.w >= 1 && v.h >= 1 &&
               (v.c <= 32 || v.c % 32 == 0) && v.c % 4 == 0,
           YL_ERR_INVALID, "atom tensor map: alignment / extent");
  const int c0 = v.c < 32 ? v.c : 32;
  cuuint64_t dims[5] = {(cuuint64_t)c0, (cuuint64_t)v.w, (cuuint64_t)v.h,
                        (cuuint64_t)((v.c + 31) / 32), (cuuint64_t)v.n};
  cuuint64_t strides[4] = {(cuuint64_t)v.sx * 4, (cuuint64_t)v.sy * 4, 128,
                           (cuuint64_t)v.sn * 4};
  cuuint32_t box[5] = {32, (cuuint32_t)box_w, 1, (cuuint32_t)atoms, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(v.base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  YL_CHECK(r == CUDA_SUCCESS, YL_ERR_CUDA, "cuTensorMapEncodeTiled (atoms) failed (%d)", (int)r);
  return YL_OK;
}

bool conv_gn_stats_supported(int n_total, int groups) {
  if (groups <= 0 || n_total % groups) return false;
  const int cg = n_total / groups;
  return cg == 4 || cg == 8 || cg == 16 || cg == 32;
}

// mean/rstd per (image, group) from the per-tile partials: one 128-thread
// block per (image, group); each thread sums a fixed strided subset of the
// image's (tile, slot) entries in double, then a fixed shared-memory tree.
__global__ void __launch_bounds__(128) gn_tile_stats_kernel(
    const float2* __restrict__ part, ConvPlan p, int nphase, int slots, int gpb, int groups,
    int cg, float eps, float* __restrict__ mean, float* __restrict__ rstd) {
  __shared__ double sh[2][128];
  const int idx = blockIdx.x;  // img * groups + g
  const int img = idx / groups, g = idx % groups;
  const int nb = g / gpb, gb = g % gpb;
  const int tpi = p.tiles_x * p.tiles_y;
  const long long items = (long long)nphase * tpi * slots;
  double s = 0.0, ss = 0.0;
  for (long long i = threadIdx.x; i < items; i += blockDim.x) {
    const int z = (int)(i / ((long long)tpi * slots));
    const long long rem = i - (long long)z * tpi * slots;
    const int pix = img * tpi + (int)(rem / slots), slot = (int)(rem % slots);
    const long long tile = ((long long)z * p.pix_tiles + pix) * p.n_nblk + nb;
    const float2 v = part[(tile * slots + slot) * gpb + gb];
    s += v.x;
    ss += v.y;
  }
  sh[0][threadIdx.x] = s;
  sh[1][threadIdx.x] = ss;
  __syncthreads();
  for (int o = 64; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      sh[0][threadIdx.x] += sh[0][threadIdx.x + o];
      sh[1][threadIdx.x] += sh[1][threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x) return;
  const double cnt = (double)p.out_h * p.out_w * cg;
  const double m = sh[0][0] / cnt;
  double var = sh[1][0] / cnt - m * m;
  if (var < 0) var = 0;
  mean[idx] = (float)m;
  rstd[idx] = (float)(1.0 / sqrt(var + (double)eps));
}

template <int BN, int MT, bool TR = false, bool HALO = false>
static yl_status launch_plan(yl_ctx* ctx, const View* views, int nviews, const float* w, int w_rows,
                             int w_cols, ConvPlan& p, int nphase, const ConvEpilogue& e) {
  using Cfg = FpropCfg<BN, MT>;
  constexpr int kSmem = HALO ? HaloCfg::kSmemBytes : Cfg::kSmemBytes;
  CUtensorMap ta[4], tw;
  for (int i = 0; i < 4; ++i)
    YL_TRY(make_view_tmap(&ta[i], views[i < nviews ? i : 0], 32,
                          HALO ? HaloCfg::kBoxRows : 4 * MT, CU_TENSOR_MAP_SWIZZLE_128B));
  YL_TRY(make_weight_tmap(&tw, w, w_rows, w_cols, BN));
  // output of each phase as a strided view of the lattice (the epilogue stores
  // 32-pixel x 32-channel pieces of lattice rows through these)
  CUtensorMap to[4];
  // (an output the maps cannot describe -- unaligned, or a phase with no
  // pixels -- keeps the per-thread stores)
  p.tma_out = (e.ldo & 3) == 0 && ((uintptr_t)e.out & 15) == 0;
  for (int z = 0; z < 4 && p.tma_out; ++z) {
    const TapPhase& ph = p.ph[z < nphase ? z : 0];
    View ov{e.out + ((long long)ph.ya * p.out_w + ph.xa) * e.ldo, e.n_total,
            std::min(p.gw, (p.out_w - ph.xa + p.xs - 1) / p.xs),
            std::min(p.gh, (p.out_h - ph.ya + p.ys - 1) / p.ys), p.n_img,
            (long long)p.xs * e.ldo, (long long)p.ys * p.out_w * e.ldo,
            (long long)p.out_h * p.out_w * e.ldo};
    int cu_err = 0;  // a map that cannot be built is not an error: per-thread stores
    if (!encode_view_tmap(&to[z], ov, 32, 1, CU_TENSOR_MAP_SWIZZLE_128B, 32, &cu_err))
      p.tma_out = 0;
  }
  if (!p.tma_out)
    for (int z = 0; z < 4; ++z) to[z] = tw;  // unused by the per-thread stores
  p.tiles_x = (p.gw + 31) / 32;
  p.tiles_y = (p.gh + 4 * MT - 1) / (4 * MT);
  p.n_nblk = (e.n_total + BN - 1) / BN;
  p.pix_tiles = p.tiles_x * p.tiles_y * p.n_img;
  const long long tiles = (long long)p.pix_tiles * p.n_nblk * nphase;
  YL_CHECK(tiles > 0 && tiles < (1LL << 31), YL_ERR_SHAPE, "conv: %lld tiles", tiles);
  p.n_tiles = (int)tiles;
  ConvEpilogue ek = e;
  const int slots = TR ? 1 : MT * 4;
  int gpb = 0;
  if (e.gn_mean) {
    YL_CHECK(conv_gn_stats_supported(e.n_total, e.gn_groups) && BN % (e.n_total / e.gn_groups) == 0,
             YL_ERR_UNSUPPORTED, "conv: GroupNorm statistics for %d channels in %d groups",
             e.n_total, e.gn_groups);
    ek.gn_cg = e.n_total / e.gn_groups;
    gpb = BN / ek.gn_cg;
    void* part = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)p.n_tiles * slots * gpb * sizeof(float2), &part, 2));
    ek.gn_part = (float2*)part;
  }
  YL_CUDA(cudaFuncSetAttribute(conv_tma_fprop_kernel<BN, MT, TR, HALO>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  const int grid = p.n_tiles < ctx->num_sms ? p.n_tiles : ctx->num_sms;
  p.sched = ctx->sched ? ctx->sched + 2 * (ctx->sched_next++ % kSchedSlots) : nullptr;
  snprintf(ctx->last_kernel[0], sizeof(ctx->last_kernel[0]), "conv_tma_fprop_kernel<%d, %d, %d, %d>",
           BN, MT, (int)TR, (int)HALO);
  double macs = 0.0;  // as run: every phase's output pixels x its taps x 32-channel chunks
  for (int z = 0; z < nphase; ++z) {
    const TapPhase& ph = p.ph[z];
    const long long rows = std::min(p.gh, (p.out_h - ph.ya + p.ys - 1) / p.ys);
    const long long cols = std::min(p.gw, (p.out_w - ph.xa + p.xs - 1) / p.xs);
    if (rows > 0 && cols > 0)
      macs += (double)p.n_img * rows * cols * ph.ntaps * p.cpt * 32.0 * e.n_total;
  }
  ctx->last_exec_flops[0] = 2.0 * macs;
  conv_tma_fprop_kernel<BN, MT, TR, HALO><<<grid, kThreads, kSmem, ctx->stream>>>(
      ta[0], ta[1], ta[2], ta[3], tw, to[0], to[1], to[2], to[3], p, ek, ctx->dev_err);
  YL_TRY(check_launch("conv_tma_fprop_kernel"));
  if (!e.gn_mean) return YL_OK;
  gn_tile_stats_kernel<<<p.n_img * e.gn_groups, 128, 0, ctx->stream>>>(
      ek.gn_part, p, nphase, slots, gpb, e.gn_groups, ek.gn_cg, e.gn_eps, e.gn_mean, e.gn_rstd);
  return check_launch("gn_tile_stats_kernel");
}

// The halo path's tap structure: one phase over one view, 9 taps whose
// kernel columns g (taps g, g+3, g+6) share a dx and span at most 3 rows.
static bool halo_taps(const ConvPlan& p, int nphase, int nviews) {
  if (nphase != 1 || nviews != 1 || p.ph[0].ntaps != 9) return false;
  const TapPhase& ph = p.ph[0];
  for (int g = 0; g < 3; ++g) {
    int lo = 127, hi = -128;
    for (int j = 0; j < 3; ++j) {
      const int t = g + 3 * j;
      if (ph.map[t] != 0 || ph.dx[t] != ph.dx[g]) return false;
      lo = std::min(lo, (int)ph.dy[t]);
      hi = std::max(hi, (int)ph.dy[t]);
    }
    if (hi - lo > HaloCfg::kBoxRows - 8) return false;
  }
  return true;
}

// Tile choice: BN covers the output channels in as few blocks as possible;
// two M subtiles (or, for cout <= 128 and long k loops, the transposed
// 128 x 256 accumulator) when the lattice is tall enough that 8-row tiles
// waste little of the last tile row.
static yl_status run_plan(yl_ctx* ctx, const View* views, int nviews, const float* w, int w_rows,
                          int w_cols, ConvPlan& p, int nphase, const ConvEpilogue& e) {
  // 8-row tiles when the last tile row wastes little: none (a multiple of 8
  // rows), a tall lattice, or at most 1/16 of the rows while the 8-row tiles
  // still fill the SMs
  const int t8 = (p.gh + 7) / 8;
  const long long tiles8 = (long long)t8 * ((p.gw + 31) / 32) * p.n_img * nphase *
                           ((e.n_total + 127) / 128);
  const bool tall = p.gh % 8 == 0 || p.gh >= 64 ||
                    ((t8 * 8 - p.gh) * 16 <= t8 * 8 && tiles8 >= ctx->num_sms);
  // the transposed epilogue costs more instructions per tile: only worth it
  // when every tile has a long k loop
  int min_nk = 1 << 30;
  for (int z = 0; z < nphase; ++z) min_nk = std::min(min_nk, p.ph[z].ntaps * p.cpt);
  if (e.n_total <= 32) return launch_plan<32, 1>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
  if (e.n_total <= 64) {
    if (tall) return launch_plan<64, 2>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
    return launch_plan<64, 1>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
  }
  if (tall && e.n_total % 128 == 0 && min_nk >= 9) {
    if (halo_taps(p, nphase, nviews))
      return launch_plan<128, 2, true, true>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
    return launch_plan<128, 2, true>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
  }
  if (e.n_total <= 128 || e.n_total % 256 != 0) {
    if (tall && e.n_total <= 128 && min_nk >= 9)
      return launch_plan<128, 2, true>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
    if (tall) return launch_plan<128, 2>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
    return launch_plan<128, 1>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
  }
  return launch_plan<256, 1>(ctx, views, nviews, w, w_rows, w_cols, p, nphase, e);
}

// Source extent of a gather (the physical tensor the gather reads).
static bool source_dims(const ConvGather& g, int* sw, int* sh) {
  if (g.ps <= 0 || g.row_stride % g.ps != 0 || g.row_stride == 0) return false;
  *sw = g.row_stride / g.ps;
  if (g.img_stride % g.row_stride != 0) return false;
  *sh = (int)(g.img_stride / g.row_stride);
  return true;
}

// The cp.async gather path, plus a separate statistics pass when the caller
// asked for the output's GroupNorm statistics.
static yl_status gather_fprop(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                              const ConvEpilogue& e) {
  YL_TRY(conv_fprop_gather(ctx, g, w, n_rows, e));
  if (!e.gn_mean) return YL_OK;
  const int n_img = g.m_total / (g.oh * g.ow);
  return gn_stats(ctx, e.out, n_img, e.n_total, e.gn_groups, (long long)g.oh * g.ow, e.ldo,
                  e.gn_eps, 0, e.gn_mean, e.gn_rstd);
}

yl_status conv_fprop(yl_ctx* ctx, const ConvGather& g, const float* w, int n_rows,
                     const ConvEpilogue& e) {
  int sw = 0, sh = 0;
  // fewer than 32 channels (RGB frames, the RGB head's dy): each tap reads one
  // 32-channel box of which the channels past cin read as zero, against
  // weights padded to 32 channels per tap
  const bool narrow = g.cin < 32 && 32 % g.cin == 0;
  const bool tma_ok = (g.cin % 32 == 0 || narrow) && g.m_total > 0 &&
                      g.m_total % (g.oh * g.ow) == 0 && ((uintptr_t)g.src & 15) == 0 &&
                      g.ps % 4 == 0 && source_dims(g, &sw, &sh) && e.n_total > 0 &&
                      e.ldo >= e.n_total;
  if (!tma_ok) return gather_fprop(ctx, g, w, n_rows, e);
  const int n_img = g.m_total / (g.oh * g.ow);
  ConvPlan p{};
  p.cpt = narrow ? 1 : g.cin / 32;
  p.n_img = n_img;
  const bool k3p1 = g.ksize == 3 && g.pad == 1;
  const int taps = g.ksize * g.ksize;
  const bool plain_s1 = g.stride == 1 && sw == g.wv && sh == g.hv && (g.mode == MODE_DGRAD || !g.up);
  if (narrow) {
    if (!plain_s1) return gather_fprop(ctx, g, w, n_rows, e);
    void* wsb = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)n_rows * taps * 32 * sizeof(float), &wsb));
    YL_TRY(weight_permute(ctx, w, (float*)wsb, n_rows, taps, 32, g.cin, (long long)taps * g.cin,
                          g.cin, 1, 0));
    w = (const float*)wsb;
  }
  const int kcols = taps * (narrow ? 32 : g.cin);
  if (g.mode == MODE_FPROP && g.stride == 1 && !g.up && sw == g.wv && sh == g.hv) {
    // plain stride-1 conv: tap (ky, kx) reads offset (ky - pad, kx - pad)
    View v = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    p.gh = g.oh; p.gw = g.ow; p.out_h = g.oh; p.out_w = g.ow; p.ys = p.xs = 1;
    TapPhase& ph = p.ph[0];
    ph.ntaps = taps;
    for (int t = 0; t < ph.ntaps; ++t) {
      ph.map[t] = 0;
      ph.dy[t] = (int8_t)(t / g.ksize - g.pad);
      ph.dx[t] = (int8_t)(t % g.ksize - g.pad);
    }
    return run_plan(ctx, &v, 1, w, n_rows, kcols, p, 1, e);
  }
  if (g.mode == MODE_DGRAD && g.stride == 1 && sw == g.wv && sh == g.hv) {
    // stride-1 dX: the flipped taps over dy
    View v = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    p.gh = g.oh; p.gw = g.ow; p.out_h = g.oh; p.out_w = g.ow; p.ys = p.xs = 1;
    TapPhase& ph = p.ph[0];
    ph.ntaps = taps;
    for (int t = 0; t < ph.ntaps; ++t) {
      ph.map[t] = 0;
      ph.dy[t] = (int8_t)(g.pad - t / g.ksize);
      ph.dx[t] = (int8_t)(g.pad - t % g.ksize);
    }
    return run_plan(ctx, &v, 1, w, n_rows, kcols, p, 1, e);
  }
  if (g.mode == MODE_FPROP && g.stride == 2 && !g.up && k3p1 && sw == g.wv && sh == g.hv &&
      sw >= 2 && sh >= 2) {
    // stride-2 conv: tap offset r = k - pad lands in input phase (r & 1) at lattice offset r >> 1
    View v[4];
    for (int a = 0; a < 2; ++a)
      for (int b = 0; b < 2; ++b) v[a * 2 + b] = phase_view(g.src, g.cin, sw, sh, n_img, g.ps, a, b);
    p.gh = g.oh; p.gw = g.ow; p.out_h = g.oh; p.out_w = g.ow; p.ys = p.xs = 1;
    TapPhase& ph = p.ph[0];
    ph.ntaps = 9;
    for (int t = 0; t < 9; ++t) {
      const int ry = t / 3 - 1, rx = t % 3 - 1;
      ph.map[t] = (int8_t)(((ry & 1) << 1) | (rx & 1));
      ph.dy[t] = (int8_t)(ry >> 1);
      ph.dx[t] = (int8_t)(rx >> 1);
    }
    return run_plan(ctx, v, 4, w, n_rows, g.k_total, p, 1, e);
  }
  if (g.mode == MODE_FPROP && g.up && g.stride == 1 && k3p1 && (g.hv + 1) / 2 == sh &&
      (g.wv + 1) / 2 == sw && g.hv <= 2 * sh && g.wv <= 2 * sw && g.oh == g.hv &&
      g.ow == g.wv) {
    // nearest-x2 upsample + conv: four output phases, each a 2x2 conv on the
    // source; a cut grid (hv or wv odd) clips the phase outputs, and the
    // terms of the cut pixels are subtracted afterwards
    const bool cut = g.hv != 2 * sh || g.wv != 2 * sw;
    void* wsb = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)4 * n_rows * 4 * g.cin * sizeof(float), &wsb));
    float* wm = (float*)wsb;
    up_merge_weights_kernel<<<grid_1d(16LL * n_rows * g.cin, 256), 256, 0, ctx->stream>>>(
        w, wm, n_rows, g.cin);
    YL_TRY(check_launch("up_merge_weights_kernel"));
    View v = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    p.gh = sh; p.gw = sw; p.out_h = g.oh; p.out_w = g.ow; p.ys = p.xs = 2;
    for (int ph = 0; ph < 4; ++ph) {
      const int a = ph >> 1, b = ph & 1;
      TapPhase& tp = p.ph[ph];
      tp.ntaps = 4;
      tp.w_row0 = ph * n_rows;
      tp.ya = a;
      tp.xa = b;
      for (int t = 0; t < 4; ++t) {
        tp.map[t] = 0;
        tp.dy[t] = (int8_t)((t >> 1) + a - 1);
        tp.dx[t] = (int8_t)((t & 1) + b - 1);
      }
    }
    if (!cut) return run_plan(ctx, &v, 1, wm, 4 * n_rows, 4 * g.cin, p, 4, e);
    // GroupNorm statistics must see the corrected border: a separate pass
    ConvEpilogue ec = e;
    ec.gn_mean = ec.gn_rstd = nullptr;
    YL_TRY(run_plan(ctx, &v, 1, wm, 4 * n_rows, 4 * g.cin, p, 4, ec));
    CutFixFprop f{};
    f.A = g.src;
    f.B = w;
    f.out = e.out;
    f.ps = g.ps;
    f.sh = sh;
    f.sw = sw;
    f.cin = g.cin;
    f.cout = e.n_total;
    f.hv = g.hv;
    f.wv = g.wv;
    f.ldo = e.ldo;
    f.round = e.round_tf32;
    f.col = g.wv < 2 * sw;
    f.nb = crop_border_count(f.col, g.hv < 2 * sh, g.hv, g.wv);
    f.M = n_img * f.nb;
    f.groups = 5;
    f.gk = g.cin;
    cut_fix_rows_kernel<<<dim3((f.cout + 31) / 32, (f.M + 31) / 32), 256, 0, ctx->stream>>>(f);
    YL_TRY(check_launch("cut_fix_rows_kernel<CutFixFprop>"));
    if (!e.gn_mean) return YL_OK;
    return gn_stats(ctx, e.out, n_img, e.n_total, e.gn_groups, (long long)g.oh * g.ow, e.ldo,
                    e.gn_eps, 0, e.gn_mean, e.gn_rstd);
  }
  if (g.mode == MODE_DGRAD && g.stride == 2 && k3p1 && sw == g.wv && sh == g.hv) {
    // stride-2 dX: output phase (a, b) gathers the dy taps whose parity matches
    void* wsb = nullptr;
    YL_TRY(scratch_get(ctx, (size_t)4 * n_rows * 4 * g.cin * sizeof(float), &wsb));
    float* wp = (float*)wsb;
    s2_phase_weights_kernel<<<grid_1d(16LL * n_rows * g.cin, 256), 256, 0, ctx->stream>>>(
        w, wp, n_rows, g.cin);
    YL_TRY(check_launch("s2_phase_weights_kernel"));
    View v = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    p.gh = (g.oh + 1) / 2; p.gw = (g.ow + 1) / 2; p.out_h = g.oh; p.out_w = g.ow;
    p.ys = p.xs = 2;
    for (int ph = 0; ph < 4; ++ph) {
      const int a = ph >> 1, b = ph & 1;
      const int nr = a == 0 ? 1 : 2, nc = b == 0 ? 1 : 2;
      const int ro[2] = {a == 0 ? 0 : 1, 0}, co[2] = {b == 0 ? 0 : 1, 0};
      TapPhase& tp = p.ph[ph];
      tp.ntaps = nr * nc;
      tp.w_row0 = ph * n_rows;
      tp.ya = a;
      tp.xa = b;
      for (int t = 0; t < tp.ntaps; ++t) {
        tp.map[t] = 0;
        tp.dy[t] = (int8_t)ro[t / nc];
        tp.dx[t] = (int8_t)co[t % nc];
      }
    }
    return run_plan(ctx, &v, 1, wp, 4 * n_rows, 4 * g.cin, p, 4, e);
  }
  return gather_fprop(ctx, g, w, n_rows, e);
}

// dX of a nearest-x2 upsample + 3x3 conv (pad 1) at the source resolution
// sh x sw: dX[u][v] = sum over the four output phases (a, b) and their 2x2
// merged taps of Wm[ph][t]^T dy_ph[u + 1 - a - ty][v + 1 - b - tx], with
// dy_ph the phase views of dy (hv x wv, the x2 grid, possibly cut by one row
// and / or column; the views read zero past the cut).  16 taps at the source
// resolution instead of 9 at the output resolution plus a 2x2 sum; a cut
// grid then has the terms of its cut pixels subtracted on the border.
yl_status conv_dgrad_upsampled(yl_ctx* ctx, const float* dy, int ldy, int cout, int n, int sh,
                               int sw, int hv, int wv, const float* wd, int rows,
                               const ConvEpilogue& e) {
  if (cout % 32 != 0 || ldy % 4 != 0 || ((uintptr_t)dy & 15) != 0 || sh < 1 || sw < 1 ||
      e.n_total <= 0 || e.ldo < e.n_total || (hv + 1) / 2 != sh || (wv + 1) / 2 != sw ||
      hv > 2 * sh || wv > 2 * sw || (e.gn_mean && (hv != 2 * sh || wv != 2 * sw)))
    return YL_ERR_UNSUPPORTED;
  void* wsb = nullptr;
  YL_TRY(scratch_get(ctx, (size_t)rows * 16 * cout * sizeof(float), &wsb));
  float* wm = (float*)wsb;
  up_merge_dgrad_weights_kernel<<<grid_1d(16LL * rows * cout, 256), 256, 0, ctx->stream>>>(
      wd, wm, rows, cout);
  YL_TRY(check_launch("up_merge_dgrad_weights_kernel"));
  View v[4];
  for (int ph = 0; ph < 4; ++ph) v[ph] = phase_view(dy, cout, wv, hv, n, ldy, ph >> 1, ph & 1);
  // a one-pixel dy has empty phase views: the plain path covers it
  for (int ph = 0; ph < 4; ++ph)
    if (v[ph].w < 1 || v[ph].h < 1) return YL_ERR_UNSUPPORTED;
  ConvPlan p{};
  p.cpt = cout / 32;
  p.n_img = n;
  p.gh = sh; p.gw = sw; p.out_h = sh; p.out_w = sw; p.ys = p.xs = 1;
  TapPhase& tp = p.ph[0];
  tp.ntaps = 16;
  for (int pt = 0; pt < 16; ++pt) {
    const int ph = pt >> 2, t = pt & 3;
    tp.map[pt] = (int8_t)ph;
    tp.dy[pt] = (int8_t)(1 - (ph >> 1) - (t >> 1));
    tp.dx[pt] = (int8_t)(1 - (ph & 1) - (t & 1));
  }
  YL_TRY(run_plan(ctx, v, 4, wm, rows, 16 * cout, p, 1, e));
  if (hv == 2 * sh && wv == 2 * sw) return YL_OK;
  CutFixDgrad f{};
  f.A = dy;
  f.B = wd;
  f.dx = e.out;
  f.ldy = ldy;
  f.cout = cout;
  f.sh = sh;
  f.sw = sw;
  f.hv = hv;
  f.wv = wv;
  f.cin = e.n_total;
  f.ldo = e.ldo;
  f.round = e.round_tf32;
  f.col = wv < 2 * sw;
  f.nb = crop_border_count(f.col, hv < 2 * sh, sh, sw);
  f.M = n * f.nb;
  f.groups = 20;  // 4 pixels of the 2x2 block x 5 taps
  f.gk = cout;
  cut_fix_rows_kernel<<<dim3((f.cin + 31) / 32, (f.M + 31) / 32), 256, 0, ctx->stream>>>(f);
  return check_launch("cut_fix_rows_kernel<CutFixDgrad>");
}

// Tile shape of the TMA wgrad for a cout x n_total filter gradient
// (n_total = taps * cin); mt = 0 means no TMA tile divides n_total.
struct WgTile {
  int mt, nsub, nw, bkp;
  int bn() const { return nsub * nw; }
};

static WgTile wgrad_tile(int cout, int n_total) {
  if (n_total == 288) return {1, 3, 96, 16};  // 9 taps of one (padded) 32-channel atom
  if (n_total == 64) return {1, 1, 64, 32};   // 1x1 over 64-channel patches
  if (cout % 256 == 0 && n_total % 256 == 0) return {2, 1, 256, 32};
  if (cout <= 128 && n_total % 512 == 0) return {1, 2, 256, 16};
  if (n_total % 384 == 0) return {1, 2, 192, 32};
  if (n_total % 256 == 0) return {1, 1, 256, 32};
  if (n_total % 128 == 0) return {1, 1, 128, 32};
  if (n_total % 288 == 0) return {1, 3, 96, 16};  // e.g. 3x3 over 96 channels
  return {0, 0, 0, 0};
}

// How a filter gradient runs: mode (-1: the cp.async gather kernel), the tile,
// the GEMM width per column group (WG_UP: 4 merged taps per output phase),
// the workspace row length and the number of output tiles.
struct WgShape {
  int mode = -1;
  bool narrow = false;  // cin < 32: one zero-padded 32-channel atom per tap
  WgTile tile{0, 0, 0, 0};
  int sw = 0, sh = 0;
  long long gemm_n = 0, ws_cols = 0, tiles = 0, kblocks = 0;
};

static WgShape wgrad_shape(const ConvGather& g, int cout, const float* dy, int ldy) {
  WgShape r;
  const bool k3p1 = g.ksize == 3 && g.pad == 1;
  const bool narrow = g.cin < 32 && 32 % g.cin == 0;
  if (!((g.cin % 32 == 0 || narrow) && (cout <= 32 || cout % 32 == 0) && cout % 4 == 0 &&
        g.m_total > 0 &&
        g.oh > 0 && g.ow > 0 && g.m_total % (g.oh * g.ow) == 0 && ((uintptr_t)g.src & 15) == 0 &&
        ((uintptr_t)dy & 15) == 0 && g.ps % 4 == 0 && ldy % 4 == 0 &&
        source_dims(g, &r.sw, &r.sh)))
    return r;
  int mode = -1;
  if (g.stride == 1 && !g.up && r.sw == g.wv && r.sh == g.hv) mode = WG_PLAIN;
  else if (g.stride == 2 && !g.up && k3p1 && r.sw == g.wv && r.sh == g.hv && r.sw >= 2 &&
           r.sh >= 2)
    mode = WG_STRIDE2;
  else if (g.stride == 1 && g.up && k3p1 && (g.hv + 1) / 2 == r.sh && (g.wv + 1) / 2 == r.sw &&
           g.hv <= 2 * r.sh && g.wv <= 2 * r.sw && g.hv >= 2 && g.wv >= 2 && g.oh == g.hv &&
           g.ow == g.wv)
    mode = WG_UP;  // the x2 grid, or one cut by a row and / or column (every phase non-empty)
  if (mode < 0 || (narrow && (mode != WG_PLAIN || g.ksize != 3))) return r;
  r.narrow = narrow;
  r.gemm_n = narrow ? 9 * 32 : mode == WG_UP ? 4LL * g.cin : g.k_total;
  r.tile = wgrad_tile(cout, (int)r.gemm_n);
  if (!r.tile.mt) return r;
  r.mode = mode;
  r.ws_cols = mode == WG_UP ? 16LL * g.cin : r.gemm_n;
  const long long mblk = (cout + r.tile.mt * kBM - 1) / (r.tile.mt * kBM);
  r.tiles = mblk * (r.ws_cols / r.tile.bn());
  const int gw = mode == WG_UP ? r.sw : g.ow, gh = mode == WG_UP ? r.sh : g.oh;
  r.kblocks = (long long)(g.m_total / (g.oh * g.ow)) * gh * ((gw + r.tile.bkp - 1) / r.tile.bkp);
  return r;
}

// Split-K factor: one wave of CTAs (tiles * splits <= SM count), at least
// four k-blocks per split.
int conv_wgrad_pick_splits(yl_ctx* ctx, int cout, const ConvGather& g, const float* dy, int ldy) {
  WgShape sh = wgrad_shape(g, cout, dy, ldy);
  long long tiles = sh.tiles, kblocks = sh.kblocks;
  if (sh.mode < 0) {  // gather kernel: 128 x 128 tiles, 32-pixel k-blocks
    tiles = (long long)((cout + kBM - 1) / kBM) * ((g.k_total + 127) / 128);
    kblocks = ((long long)g.m_total + kBK - 1) / kBK;
  }
  long long splits = std::max(1LL, ctx->num_sms / std::max(1LL, tiles));
  splits = std::min(splits, std::max(1LL, kblocks / 4));
  return (int)std::min(splits, 512LL);
}

size_t conv_wgrad_ws_floats(const ConvGather& g, int cout, const float* dy, int ldy, int splits) {
  WgShape sh = wgrad_shape(g, cout, dy, ldy);
  const long long cols = sh.mode < 0 ? g.k_total : sh.ws_cols;
  // + the bias-gradient partials (up to four phases per split), 64-float aligned
  const size_t main = ((size_t)splits * cout * cols + 63) & ~size_t(63);
  return main + (size_t)4 * splits * cout;
}

// db[c] (+)= sum over rows of part[rows][c], fixed order.
__global__ void db_reduce_kernel(const float* __restrict__ part, int rows, int c,
                                 float* __restrict__ db, int accumulate) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= c) return;
  float s = 0.f;
  for (int r = 0; r < rows; ++r) s += part[(long long)r * c + i];
  db[i] = accumulate ? db[i] + s : s;
}

template <int MT, int NSUB, int NW, int BKP>
static yl_status launch_wgrad(yl_ctx* ctx, const View* av, int nav, const View* bv, int nbv,
                              WgradPlan& w, int splits, int col_blocks) {
  using Cfg = WgradCfg<MT, NSUB, NW, BKP>;
  // A box: all of the tile's dy atoms at once when cout is whole atoms; B box:
  // four atoms (128 input channels of one tap) when the taps allow it
  w.ga = w.cout % 32 == 0 ? Cfg::kAAtoms : 1;
  w.gb = (w.cin / 32) % 4 == 0 && Cfg::kBAtoms % 4 == 0 ? 4 : 1;
  CUtensorMap ta[4], tb[4];
  for (int i = 0; i < 4; ++i) {
    YL_TRY(make_atom_tmap(&ta[i], av[i < nav ? i : 0], BKP, w.ga,
                          CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    YL_TRY(make_atom_tmap(&tb[i], bv[i < nbv ? i : 0], BKP, w.gb,
                          CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  }
  w.xblocks = (w.gw + BKP - 1) / BKP;
  w.blocks = (long long)w.n_img * w.gh * w.xblocks;
  w.per_split = (w.blocks + splits - 1) / splits;
  YL_CUDA(cudaFuncSetAttribute(conv_tma_wgrad_kernel<MT, NSUB, NW, BKP>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  dim3 grid((w.cout + MT * kBM - 1) / (MT * kBM), col_blocks, splits);
  snprintf(ctx->last_kernel[1], sizeof(ctx->last_kernel[1]), "conv_tma_wgrad_kernel<%d, %d, %d, %d>",
           MT, NSUB, NW, BKP);
  // as run: every lattice pixel against every workspace column (an upsample
  // conv's four phase GEMMs of 4 merged taps each make 16 taps of columns)
  ctx->last_exec_flops[1] = 2.0 * w.n_img * w.gh * w.gw * (double)w.cout * w.n_total;
  conv_tma_wgrad_kernel<MT, NSUB, NW, BKP><<<grid, kThreads, Cfg::kSmemBytes, ctx->stream>>>(
      ta[0], ta[1], ta[2], ta[3], tb[0], tb[1], tb[2], tb[3], w, ctx->dev_err);
  return check_launch("conv_tma_wgrad_kernel");
}

// dw[co][ky*3+kx][ci] (+)= sum over splits and output phases (a, b) of the
// merged gradient of the 2x2 tap (ty, tx) that kernel tap (ky, kx) belongs to
// in that phase (the adjoint of up_merge_weights_kernel), fixed order.
__global__ void wgrad_unmerge_kernel(const float* __restrict__ ws, int splits, long long stride,
                                     int cout, int cin, float* __restrict__ dw, int accumulate) {
  const long long n = (long long)cout * 9 * cin;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ci = (int)(i % cin);
    const long long r = i / cin;
    const int tap = (int)(r % 9), co = (int)(r / 9);
    const int ky = tap / 3, kx = tap % 3;
    const float* row = ws + (long long)co * 16 * cin + ci;
    float s = 0.f;
    for (int a = 0; a < 2; ++a) {
      const int ty = up_row_in(a, 0, ky) ? 0 : 1;
      for (int b = 0; b < 2; ++b) {
        const int tx = up_row_in(b, 0, kx) ? 0 : 1;
        const long long col = (long long)(((a * 2 + b) * 4 + ty * 2 + tx) * cin);
        for (int sp = 0; sp < splits; ++sp) s += row[sp * stride + col];
      }
    }
    dw[i] = accumulate ? dw[i] + s : s;
  }
}

// dw[co][t][ci] (+)= sum over splits of ws[split][co][t * 32 + ci] (the
// narrow-input layout with one zero-padded 32-channel atom per tap).
__global__ void wgrad_unpad_kernel(const float* __restrict__ ws, int splits, long long stride,
                                   int cout, int cin, float* __restrict__ dw, int accumulate) {
  const long long n = (long long)cout * 9 * cin;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ci = (int)(i % cin);
    const long long r = i / cin;
    const int t = (int)(r % 9), co = (int)(r / 9);
    const float* src = ws + (long long)co * 288 + t * 32 + ci;
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += src[sp * stride];
    dw[i] = accumulate ? dw[i] + s : s;
  }
}

yl_status conv_wgrad_ws(yl_ctx* ctx, const float* dy, int ldy, int cout, const ConvGather& g,
                        float* dw, int accumulate, float* ws, int splits, float* db) {
  const WgShape shp = wgrad_shape(g, cout, dy, ldy);
  if (shp.mode < 0 || splits < 1) {
    YL_TRY(conv_wgrad_gather(ctx, dy, ldy, cout, g, dw, accumulate, ws, splits));
    if (!db) return YL_OK;
    return channel_sums(ctx, dy, 1, g.m_total, ldy, cout, db, nullptr, accumulate);
  }
  const int mode = shp.mode, sw = shp.sw, sh = shp.sh;
  const WgTile tile = shp.tile;
  const int n_img = g.m_total / (g.oh * g.ow);
  View av[4], bv[4];
  int nav = 1, nbv = 1;
  WgradPlan w{};
  w.mode = mode;
  w.ksize = g.ksize;
  w.pad = g.pad;
  w.cin = shp.narrow ? 32 : g.cin;  // the column layout's channels per tap
  w.cout = cout;
  w.n_total = (int)shp.ws_cols;
  w.n_img = n_img;
  int col_blocks = (int)(shp.ws_cols / tile.bn());
  if (mode == WG_UP) {
    for (int ph = 0; ph < 4; ++ph)
      av[ph] = phase_view(dy, cout, g.ow, g.oh, n_img, ldy, ph >> 1, ph & 1);
    nav = 4;
    bv[0] = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    w.nblk_ph = (int)(shp.gemm_n / tile.bn());
    w.gh = sh;
    w.gw = sw;
  } else {
    av[0] = plain_view(dy, cout, g.ow, g.oh, n_img, ldy);
    if (mode == WG_STRIDE2) {
      for (int a = 0; a < 2; ++a)
        for (int b = 0; b < 2; ++b)
          bv[a * 2 + b] = phase_view(g.src, g.cin, sw, sh, n_img, g.ps, a, b);
      nbv = 4;
    } else {
      bv[0] = plain_view(g.src, g.cin, sw, sh, n_img, g.ps);
    }
    w.nblk_ph = col_blocks;
    w.gh = g.oh;
    w.gw = g.ow;
  }
  w.ws = ws;
  w.ws_split_stride = (long long)cout * shp.ws_cols;
  const size_t db_off = ((size_t)splits * cout * shp.ws_cols + 63) & ~size_t(63);
  w.db_ws = db ? ws + db_off : nullptr;
  if (tile.nsub == 3)
    YL_TRY((launch_wgrad<1, 3, 96, 16>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else if (tile.nw == 64)
    YL_TRY((launch_wgrad<1, 1, 64, 32>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else if (tile.mt == 2)
    YL_TRY((launch_wgrad<2, 1, 256, 32>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else if (tile.nsub == 2 && tile.nw == 256)
    YL_TRY((launch_wgrad<1, 2, 256, 16>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else if (tile.nsub == 2)
    YL_TRY((launch_wgrad<1, 2, 192, 32>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else if (tile.nw == 256)
    YL_TRY((launch_wgrad<1, 1, 256, 32>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  else
    YL_TRY((launch_wgrad<1, 1, 128, 32>(ctx, av, nav, bv, nbv, w, splits, col_blocks)));
  if (db) {
    const int rows = (mode == WG_UP ? 4 : 1) * splits;
    db_reduce_kernel<<<(cout + 127) / 128, 128, 0, ctx->stream>>>(w.db_ws, rows, cout, db,
                                                                 accumulate);
    YL_TRY(check_launch("db_reduce_kernel"));
  }
  if (shp.narrow) {
    const long long n = (long long)cout * 9 * g.cin;
    wgrad_unpad_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(ws, splits, w.ws_split_stride,
                                                                 cout, g.cin, dw, accumulate);
    return check_launch("wgrad_unpad_kernel");
  }
  if (mode == WG_UP) {
    const long long n = (long long)cout * 9 * g.cin;
    wgrad_unmerge_kernel<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(ws, splits, w.ws_split_stride,
                                                                   cout, g.cin, dw, accumulate);
    YL_TRY(check_launch("wgrad_unmerge_kernel"));
    if (g.hv == 2 * sh && g.wv == 2 * sw) return YL_OK;
    CutFixWgrad f{};
    f.A = dy;
    f.B = g.src;
    f.dw = dw;
    f.ldy = ldy;
    f.M = cout;
    f.ps = g.ps;
    f.N = g.cin;
    f.sh = sh;
    f.sw = sw;
    f.hv = g.hv;
    f.wv = g.wv;
    f.col = g.wv < 2 * sw;
    f.nb = crop_border_count(f.col, g.hv < 2 * sh, g.hv, g.wv);
    f.gk = n_img * f.nb;
    cut_fix_cols_kernel<<<dim3((g.cin + 31) / 32, (cout + 31) / 32, 5), 256, 0, ctx->stream>>>(f);
    return check_launch("cut_fix_cols_kernel<CutFixWgrad>");
  }
  const long long n = (long long)cout * g.k_total;
  splitk_reduce_kernel<<<grid_1d(n / 4 + 1, 256), 256, 0, ctx->stream>>>(ws, splits, n, dw, n,
                                                                         accumulate);
  return check_launch("splitk_reduce_kernel");
}

}  // namespace yl
