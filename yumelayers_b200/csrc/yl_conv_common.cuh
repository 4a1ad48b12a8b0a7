// yl_conv_common.cuh -- tile configuration and host helpers shared by the
// two implicit-GEMM convolution paths (yl_conv.cu: cp.async gathers;
// yl_conv_tma.cu: TMA boxes over NHWC tensors and their phase views).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "yl_kernels.h"
#include "yl_ptx.cuh"

namespace yl {

constexpr int kBM = 128;         // GEMM rows per CTA (UMMA M)
constexpr int kBK = 32;          // k per stage: 32 fp32 = one 128-byte swizzle row
constexpr int kThreads = 192;    // 4 gather/epilogue warps + TMA warp + MMA warp
constexpr int kATileBytes = kBM * 128;

template <int BN>
struct TileCfg {
  static constexpr int kBTileBytes = BN * 128;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kStages = (196 * 1024) / kStageBytes > 8 ? 8 : (196 * 1024) / kStageBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + (2 * kStages + 2) * 8 + 1024;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Fixed-order split-K reduction and tensor-map helpers
// Fixed-order sum of split-K partials: out[i] (+)= sum_s ws[s][i].
static __global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, long long stride,
                                     float* __restrict__ out, long long n, int accumulate) {
  const long long n4 = n >> 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(ws)[i];
    for (int s = 1; s < splits; ++s) {
      float4 v = reinterpret_cast<const float4*>(ws + s * stride)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (accumulate) {
      float4 o = reinterpret_cast<float4*>(out)[i];
      acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
  for (long long i = (n4 << 2) + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = ws[i];
    for (int s = 1; s < splits; ++s) acc += ws[s * stride + i];
    out[i] = accumulate ? out[i] + acc : acc;
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map over a row-major fp32 matrix [rows][cols]; box = {32, box_rows},
// SWIZZLE_128B, out-of-range elements read as zero.
static yl_status make_weight_tmap(CUtensorMap* tm, const float* w, int rows, int cols,
                                  int box_rows) {
  auto fn = get_encode_fn();
  YL_CHECK(fn, YL_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  YL_CHECK((cols & 3) == 0, YL_ERR_SHAPE, "weight row length %d is not a multiple of 4", cols);
  YL_CHECK(((uintptr_t)w & 15) == 0, YL_ERR_INVALID, "weight pointer not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(w), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  YL_CHECK(r == CUDA_SUCCESS, YL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return YL_OK;
}

}  // namespace yl
