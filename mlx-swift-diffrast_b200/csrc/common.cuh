// common.cuh — shared internals of libdiffrast (context, workspace, launch
// accounting, device helpers).  Not part of the public ABI (include/diffrast.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "diffrast.h"

// Device-side error bits, OR-ed into ctx->d_err by kernels that meet inputs they
// cannot honour; dr_ctx_sync() turns them into DR_EDEVICE.
enum : unsigned {
  DR_DEVERR_VERTEX = 1u,    // a triangle names a vertex outside [0, V)
  DR_DEVERR_TRI_ID = 2u,    // a rast pixel names a triangle outside [0, T)
  DR_DEVERR_CAPACITY = 4u,  // a fixed-capacity buffer would have overflowed
};

// Workspace slots: each is an independent grow-only device buffer.
enum WsSlot {
  WS_RASTER_REC = 0,   // per-(view, triangle) setup records
  WS_TILE_COUNT,       // per-(view, tile) candidate counts / cursors / offsets
  WS_TILE_LIST,        // concatenated per-tile candidate lists
  WS_SCAN_TMP,         // scan block sums
  WS_MIP,              // internally built mip pyramid
  WS_DMIP,             // pyramid gradients before the fold into level 0
  WS_HASH,             // topology hash table
  WS_AA,               // antialias scratch
  WS_NUM_SLOTS
};

struct dr_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  uint64_t launches = 0;
  void* ws[WS_NUM_SLOTS] = {};
  size_t ws_bytes[WS_NUM_SLOTS] = {};
  unsigned* d_err = nullptr;      // device error word
  int* h_pinned = nullptr;        // pinned host scratch for small readbacks
  int num_sms = 148;
  // Per-launch CUDA-event timing (dr_ctx_set_timing): events recorded on the
  // launching stream around every kernel, summed per kernel name on report.
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_next = 0;
  long pending_start = -1;
  std::vector<std::pair<const char*, size_t>> trecs;
};

namespace dr {

// Record a status + printf-style message on the context; returns the status.
dr_status fail(dr_ctx* ctx, dr_status st, const char* fmt, ...);
// Check the last CUDA error after a launch (and count the launch).
dr_status after_launch(dr_ctx* ctx, const char* what);
// Start-of-launch hook: records the timing start event when timing is on.
void timing_begin(dr_ctx* ctx);
// Make ctx current on the calling thread.
dr_status enter(dr_ctx* ctx);
// Grow-only workspace slot of at least `bytes`; nullptr on failure (status set).
void* ws_get(dr_ctx* ctx, int slot, size_t bytes);
// Exclusive scan of n uint32 counts (device) into offsets (device); writes the
// total into *total_dev (device, may alias nothing else).  Launch-only.
dr_status scan_u32(dr_ctx* ctx, const uint32_t* in, uint32_t* out, int64_t n,
                   uint32_t* total_dev);

inline unsigned grid_for(int64_t n, int block) {
  return (unsigned)((n + block - 1) / block);
}

}  // namespace dr

#define DR_ENTER(ctx)                                   \
  do {                                                  \
    if (!(ctx)) return DR_EINVAL;                       \
    dr_status _st = dr::enter(ctx);                     \
    if (_st != DR_OK) return _st;                       \
  } while (0)

#define DR_REQUIRE(ctx, cond, ...)                      \
  do {                                                  \
    if (!(cond)) return dr::fail((ctx), DR_EINVAL, __VA_ARGS__); \
  } while (0)

#define DR_TB(ctx) dr::timing_begin(ctx)

// Check a CUDA runtime call (memset / memcpy / sync); non-success -> DR_ECUDA.
#define DR_CUDA(ctx, call, what)                                        \
  do {                                                                  \
    cudaError_t _e = (call);                                            \
    if (_e != cudaSuccess) {                                            \
      cudaGetLastError();                                               \
      return dr::fail((ctx), DR_ECUDA, "%s: %s", (what), cudaGetErrorString(_e)); \
    }                                                                   \
  } while (0)

#define DR_LAUNCHED(ctx, what)                          \
  do {                                                  \
    dr_status _st = dr::after_launch((ctx), (what));    \
    if (_st != DR_OK) return _st;                       \
  } while (0)

// ---------------------------------------------------------------------------
// device helpers

__device__ __forceinline__ void dr_flag(unsigned* err, unsigned bit) {
  if (err) atomicOr(err, bit);
}

// Float -> int of floor(x), saturating, NaN -> 0 (the GPU conversion rule;
// the CPU oracle restates the same rule so out-of-range inputs agree).
__device__ __forceinline__ int dr_floor_i(float x) { return __float2int_rd(x); }

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
