// common.cuh — shared internals of libdiffrast (context, workspace, launch
// accounting, device helpers).  Not part of the public ABI (include/diffrast.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
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

// Minimum resident 256-thread blocks per SM requested from the compiler for
// the register-heavy per-pixel kernels (caps them at 65536 / (256 * n)
// registers): the raster and antialias VJPs at five (faster than the
// uncapped build on cfg4), the fused raster + interpolate VJP at four (64
// registers, no spills; at five it spills and measured no faster).  The
// antialias edge pass is held at four in its own declaration; the other
// per-pixel kernels measured fastest with no bound.
#ifndef DR_MINB_RASTER_BWD
#define DR_MINB_RASTER_BWD 5
#endif
#ifndef DR_MINB_AA_BWD
#define DR_MINB_AA_BWD 5
#endif
#ifndef DR_MINB_INTERP_RASTER_BWD
#define DR_MINB_INTERP_RASTER_BWD 4
#endif
// Texture VJPs (scatter-bound: latency of the float atomics) and the mipmap
// forwards (dependent gathers): four resident CTAs (64 registers) measured
// faster than three without spills, and than five or six with more spills
// (cfg3 / cfg5).  A bound of one CTA lets the compiler take more registers
// and is slower still.
#ifndef DR_MINB_TEX_BWD
#define DR_MINB_TEX_BWD 4
#endif
#ifndef DR_MINB_TEX_FWD
#define DR_MINB_TEX_FWD 4
#endif

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
  WS_LOSS,             // partial sums of a fused loss
  WS_ORDER,            // tile-order construction (box, bin counts, offsets)
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
  unsigned* d_overflow = nullptr; // tiles that took the full-scan path (fixed list capacity)
  int* h_pinned = nullptr;        // pinned host scratch for small readbacks
  // Fixed tile-list capacity in (tile, triangle) pairs (dr_ctx_set_raster_list_capacity);
  // 0 = size the list exactly from one readback per rasterize call.
  int64_t list_cap = 0;
  int num_sms = 148;
  // Per-launch CUDA-event timing (dr_ctx_set_timing): events recorded on the
  // launching stream around every kernel, summed per kernel name on report.
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_next = 0;
  long pending_start = -1;
  std::vector<std::pair<const char*, size_t>> trecs;
  // Tile order of the per-pixel kernels (dr_ctx_set_tile_order) for batches of
  // exactly order_n x order_h x order_w pixels; nullptr = image order.
  const int32_t* tile_order = nullptr;
  int order_n = 0, order_h = 0, order_w = 0;
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

// Pixel order of a per-pixel kernel launched with 256-thread blocks: image
// order (order == nullptr: pixel = block * 256 + thread), or one
// kOrderTileW x kOrderTileH tile per block, tile order[block] (tile = view *
// tiles per view + tile row * tiles per row + tile column; pixels past the
// image's edge are idle).  Wide tiles keep each block's reads of the per-pixel
// streams in long contiguous rows.
constexpr int kOrderTileW = 32, kOrderTileH = 8;
static_assert(kOrderTileW * kOrderTileH == 256, "one 256-thread block per tile");
struct PixOrder {
  const int32_t* order = nullptr;
  int H = 0, W = 0, ntx = 0, ntiles = 0;  // ntiles: tiles per view
  int64_t n_tiles = 0;
};

// The PixOrder and grid of a launch over an N x H x W batch: tiles when the
// context's tile order was set for exactly these sizes, else image order.
PixOrder pix_order(const dr_ctx* ctx, int N, int H, int W, unsigned& grid);

__device__ __forceinline__ int64_t pix_of(const PixOrder& o, int64_t P, bool& in) {
  if (!o.order) {
    const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    in = pix < P;
    return pix;
  }
  const int tile = __ldg(o.order + blockIdx.x);
  if (tile < 0 || (int64_t)tile >= o.n_tiles) {  // not an order from dr_tile_order: touch nothing
    in = false;
    return 0;
  }
  const int n = tile / o.ntiles, t = tile - n * o.ntiles;
  const int ty = t / o.ntx, tx = t - ty * o.ntx;
  const int px = tx * kOrderTileW + (int)(threadIdx.x % kOrderTileW);
  const int py = ty * kOrderTileH + (int)(threadIdx.x / kOrderTileW);
  in = px < o.W && py < o.H;
  return ((int64_t)n * o.H + py) * o.W + px;
}

// View n, row y and column x of pixel pix (0 <= pix < P) of an N x H x W
// batch of P pixels.  Divides in 32 bits when P allows (P is uniform over a
// launch, so the branch is too): a 64-bit division is a long instruction
// sequence, and the per-pixel kernels run it for every pixel.
__device__ __forceinline__ void pix_nyx(int64_t pix, int64_t P, int H, int W, int& n, int& y, int& x) {
  if (P <= 0xFFFFFFFFll) {
    const unsigned p = (unsigned)pix, hw = (unsigned)H * (unsigned)W;
    const unsigned nn = p / hw, q = p - nn * hw, yy = q / (unsigned)W;
    n = (int)nn;
    y = (int)yy;
    x = (int)(q - yy * (unsigned)W);
  } else {
    const int64_t hw = (int64_t)H * W;
    n = (int)(pix / hw);
    const int64_t q = pix - (int64_t)n * hw;
    y = (int)(q / W);
    x = (int)(q - (int64_t)y * W);
  }
}

// The view pix / HW of a pixel, in 32 bits when both fit.
__device__ __forceinline__ int view_of(int64_t pix, int64_t HW) {
  return ((unsigned long long)(pix | HW) >> 32) == 0ull ? (int)((unsigned)pix / (unsigned)HW) : (int)(pix / HW);
}

// pix_of, also giving the pixel's view n, row y and column x of the N x H x W
// batch (all 0 when !in): the tile order has them already.
__device__ __forceinline__ int64_t pix_of_nyx(const PixOrder& o, int64_t P, int H, int W, bool& in, int& n, int& y,
                                              int& x) {
  n = y = x = 0;
  if (!o.order) {
    const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    in = pix < P;
    if (in) pix_nyx(pix, P, H, W, n, y, x);
    return pix;
  }
  const int tile = __ldg(o.order + blockIdx.x);
  if (tile < 0 || (int64_t)tile >= o.n_tiles) {  // not an order from dr_tile_order: touch nothing
    in = false;
    return 0;
  }
  const int nn = tile / o.ntiles, t = tile - nn * o.ntiles;
  const int ty = t / o.ntx, tx = t - ty * o.ntx;
  const int px = tx * kOrderTileW + (int)(threadIdx.x % kOrderTileW);
  const int py = ty * kOrderTileH + (int)(threadIdx.x / kOrderTileW);
  in = px < o.W && py < o.H;
  if (in) {
    n = nn;
    y = py;
    x = px;
  }
  return ((int64_t)nn * o.H + py) * o.W + px;
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

// Per-pixel streams read or written once (rast, cotangents, outputs) use the
// streaming cache operator (evict first), so they pass through L2 without
// evicting the small tables the same kernel gathers from (attribute rows,
// vertices, texels) — a per-instruction hint, not a device setting.
__device__ __forceinline__ float4 ldcs4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void stcs4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

// Per-view vertex transform (the "xf" entry points): clip position of vertex v
// in view n is M_n v with M_n a row-major 4x4, evaluated in this fixed order
// (each product and sum rounded separately):
//   out_r = ((M[r][0] vx + M[r][1] vy) + M[r][2] vz) + M[r][3] vw
struct Mat4 {
  float4 r0, r1, r2, r3;
};

__device__ __forceinline__ Mat4 load_mat4(const float* m) {
  Mat4 M;
  M.r0 = ldg4(m); M.r1 = ldg4(m + 4); M.r2 = ldg4(m + 8); M.r3 = ldg4(m + 12);
  return M;
}

__device__ __forceinline__ float dot4_ordered(float4 a, float4 v) {
  return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a.x, v.x), __fmul_rn(a.y, v.y)), __fmul_rn(a.z, v.z)),
                   __fmul_rn(a.w, v.w));
}

__device__ __forceinline__ float4 mat4_apply(const Mat4& M, float4 v) {
  return make_float4(dot4_ordered(M.r0, v), dot4_ordered(M.r1, v), dot4_ordered(M.r2, v), dot4_ordered(M.r3, v));
}

// M^T g: the gradient of M v with respect to v.
__device__ __forceinline__ float4 mat4_apply_t(const Mat4& M, float4 g) {
  return make_float4(M.r0.x * g.x + M.r1.x * g.y + M.r2.x * g.z + M.r3.x * g.w,
                     M.r0.y * g.x + M.r1.y * g.y + M.r2.y * g.z + M.r3.y * g.w,
                     M.r0.z * g.x + M.r1.z * g.y + M.r2.z * g.z + M.r3.z * g.w,
                     M.r0.w * g.x + M.r1.w * g.y + M.r2.w * g.z + M.r3.w * g.w);
}

// Warp-level segmented suffix sum over runs of equal keys: after the call the
// first lane of each run holds the run's total.  seg_end is one past the
// caller's run; span (warp-uniform) bounds the longest run in the warp, so
// only ceil(log2(span)) shuffle steps run.  All 32 lanes must call it.
__device__ __forceinline__ float warp_seg_sum(float v, int lane, int seg_end, int span = 32) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    if (o >= span) break;
    const float y = __shfl_down_sync(0xffffffffu, v, o);
    if (lane + o < seg_end) v += y;
  }
  return v;
}

// warp_seg_sum of N values at once: one step loop (and one span check per
// step) for all of them; each value sees the same shuffles and additions in
// the same order as warp_seg_sum alone.
template <int N>
__device__ __forceinline__ void warp_seg_sum_n(float (&v)[N], int lane, int seg_end, int span) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    if (o >= span) break;
    const bool take = lane + o < seg_end;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float y = __shfl_down_sync(0xffffffffu, v[i], o);
      if (take) v[i] += y;
    }
  }
}

// Run structure of a per-lane key in a warp: returns seg_end and whether this
// lane is the run's head.
__device__ __forceinline__ int warp_runs(long long key, int lane, bool& head) {
  const long long key_up = __shfl_up_sync(0xffffffffu, key, 1);
  const unsigned heads = __ballot_sync(0xffffffffu, lane == 0 || key != key_up);
  const unsigned after = lane == 31 ? 0u : (heads >> (lane + 1));
  head = (heads >> lane) & 1u;
  return after ? lane + __ffs(after) : 32;
}

// Length of the longest run in the warp (warp-uniform), the span bound of
// warp_seg_sum.
__device__ __forceinline__ int warp_max_run(int lane, int seg_end, bool head) {
  return (int)__reduce_max_sync(0xffffffffu, head ? (unsigned)(seg_end - lane) : 0u);
}

// ---------------------------------------------------------------------------
// Fused mean-squared-error loss (the *_mse entry points).
//
// Cotangent of an op's output: the given tensor d, or, when the output feeds
// only a fused loss scale * sum((pred - target)^2), that loss's gradient
// (2 * scale * (pred - target)) * d_loss formed where it is read, with the
// arithmetic of the stand-alone MSE VJP (so the two agree bit for bit).
struct Cot {
  const float* d;       // given cotangent, or nullptr for the fused loss
  const float* pred;    // the forward output
  const float* target;
  float s2;             // 2 * scale
  const float* d_loss;  // device scalar: the loss's cotangent
};

// Per-thread factor of the fused form: *d_loss (1 when d is given).
__device__ __forceinline__ float cot_g(const Cot& c) { return c.d ? 1.0f : __ldg(c.d_loss); }

// STREAM: a per-pixel stream read once (the streaming cache operator);
// otherwise a read that neighbouring pixels repeat.
template <bool STREAM = false>
__device__ __forceinline__ float cot_at(const Cot& c, float g, int64_t i) {
  if (c.d) return STREAM ? __ldcs(c.d + i) : __ldg(c.d + i);
  const float r = STREAM ? __ldcs(c.pred + i) - __ldcs(c.target + i) : __ldg(c.pred + i) - __ldg(c.target + i);
  return (c.s2 * r) * g;
}

// Four consecutive elements from a 16-byte aligned index.
template <bool STREAM = false>
__device__ __forceinline__ float4 cot_at4(const Cot& c, float g, int64_t i) {
  if (c.d) return STREAM ? ldcs4(c.d + i) : ldg4(c.d + i);
  const float4 p = STREAM ? ldcs4(c.pred + i) : ldg4(c.pred + i), t = STREAM ? ldcs4(c.target + i) : ldg4(c.target + i);
  return make_float4((c.s2 * (p.x - t.x)) * g, (c.s2 * (p.y - t.y)) * g, (c.s2 * (p.z - t.z)) * g,
                     (c.s2 * (p.w - t.w)) * g);
}

// Sum of squared differences of four elements (the fused loss's terms).
__device__ __forceinline__ float sq_diff4(float4 a, float4 b) {
  const float x = a.x - b.x, y = a.y - b.y, z = a.z - b.z, w = a.w - b.w;
  return x * x + y * y + z * z + w * w;
}

// The forward's loss is summed per block and added to one of kLossSlots
// partial sums (spreading the atomics over several addresses); dr::loss_end
// writes their total to the caller's loss.
constexpr int kLossSlots = 32;

// Adds v summed over the block, times scale, to part[blockIdx.x % kLossSlots].
// Every thread of the block must call it (it synchronises the block).
__device__ __forceinline__ void block_loss_add(float v, float scale, float* part) {
  __shared__ float s_warp[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) s_warp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    float w = lane < nw ? s_warp[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) atomicAdd(part + (blockIdx.x % kLossSlots), scale * w);
  }
}

namespace dr {
// Zeroed partial sums for a fused loss (a workspace slot), and their total
// written to the caller's device scalar `loss` (one small launch).
dr_status loss_begin(dr_ctx* ctx, float** part);
dr_status loss_end(dr_ctx* ctx, const float* part, float* loss);
}  // namespace dr
