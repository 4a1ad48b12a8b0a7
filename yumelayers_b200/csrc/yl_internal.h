// yl_internal.h -- shared host-side plumbing of the backend: status/error
// reporting, the context object, stream-ordered scratch memory.
#pragma once
#include <cuda_runtime.h>

#include <chrono>
#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "yume_c.h"

namespace yl {

// Records `msg` as this thread's last error and returns `st`.
yl_status set_error(yl_status st, const char* fmt, ...);

#define YL_CUDA(expr)                                                                      \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return ::yl::set_error(YL_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                  \
                             cudaGetErrorString(e_), __FILE__, __LINE__);                  \
  } while (0)

#define YL_CHECK(cond, st, ...)                         \
  do {                                                  \
    if (!(cond)) return ::yl::set_error(st, __VA_ARGS__); \
  } while (0)

#define YL_TRY(expr)               \
  do {                             \
    yl_status s_ = (expr);         \
    if (s_ != YL_OK) return s_;    \
  } while (0)

// Checks the launch that was just queued.
yl_status check_launch(const char* what);

inline unsigned grid_1d(size_t n, int block, int max_blocks = 148 * 32) {
  size_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > (size_t)max_blocks) g = max_blocks;
  return (unsigned)g;
}

}  // namespace yl

// The context: one device, one stream, a device error word, and a
// stream-ordered scratch buffer that ops carve their temporaries from.
struct yl_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_begin = nullptr;
  cudaEvent_t ev_end = nullptr;
  bool session_open = false;
  std::chrono::steady_clock::time_point wall_begin;
  // device control block (16 bytes): int error word at [0] (zeroed at
  // creation), long long bounded-wait limit in SM cycles at byte 8 (0 = the
  // kernels' default)
  int* dev_err = nullptr;
  // names of the last conv kernel templates launched on this context:
  // [0] forward / dX, [1] filter gradient (diagnostics, yl_ctx_last_kernel)
  char last_kernel[2][96] = {{0}, {0}};
  // FLOPs (2 x MACs) those launches executed, padding and merged taps as run
  double last_exec_flops[2] = {0.0, 0.0};
  // tile counters of the persistent conv kernels: kSchedSlots pairs (tiles
  // handed out, CTAs done), zero between launches; consecutive launches take
  // consecutive pairs so launches in flight together never share one
  int* sched = nullptr;
  unsigned sched_next = 0;
  // Scratch slots: 0 = temporaries of one internal kernel sequence (split-K
  // partials, reduction partials); 1 = layout conversions of a C-ABI call.
  // slot 0: operator temporaries; 1: NCHW<->NHWC staging of the batched
  // C-ABI entry points; 2: GroupNorm statistics partials written by a conv
  void* scratch[3] = {nullptr, nullptr, nullptr};
  size_t scratch_bytes[3] = {0, 0, 0};
};

namespace yl {
constexpr int kSchedSlots = 64;

// Returns a device buffer of at least `bytes` from scratch slot `slot`,
// valid for work queued on ctx->stream until the next call on the same slot.
// Grows with cudaMallocAsync/cudaFreeAsync (stream-ordered, so a buffer
// still in use by queued work is never reused early).
yl_status scratch_get(yl_ctx* ctx, size_t bytes, void** out, int slot = 0);

// Bump allocator over one scratch buffer (256-byte aligned pieces).
struct ScratchCarver {
  size_t offset = 0;
  size_t take(size_t bytes) {
    size_t o = offset;
    offset += (bytes + 255) & ~size_t(255);
    return o;
  }
};
}  // namespace yl
