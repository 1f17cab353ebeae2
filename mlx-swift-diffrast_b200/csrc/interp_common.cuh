// interp_common.cuh — helpers shared by the interpolate forward (interp.cu),
// its VJP (interp_bwd.cu) and the rasterizer's interpolation epilogue
// (raster.cu).  Not part of the public ABI.
#pragma once

#include "common.cuh"

using dr::PixOrder;
using dr::pix_of;
using dr::pix_of_nyx;
using dr::view_of;
using dr::pix_nyx;
using dr::pix_order;

namespace {

struct DiffIdx {
  int k[DR_MAX_DIFF_ATTRS];
};

__device__ __forceinline__ bool tri_verts(const int32_t* __restrict__ tri, int t, int V, int& i0,
                                          int& i1, int& i2) {
  i0 = __ldg(tri + 3 * t);
  i1 = __ldg(tri + 3 * t + 1);
  i2 = __ldg(tri + 3 * t + 2);
  return !(i0 < 0 || i0 >= V || i1 < 0 || i1 >= V || i2 < 0 || i2 >= V);
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// One pixel's interpolation for A % 4 == 0 with 16-byte aligned rows and all
// pixel derivatives (.all): out (A floats) and out_da (2A floats, (d/dx, d/dy)
// per attribute) from the three vertex rows, barycentrics (bw, u, v) and the
// pixel's rast_db.  With a target (a fused loss) it adds sum((out - target)^2)
// to lsum.  The interpolate forward and the rasterizer's interpolation
// epilogue both run this, so their outputs agree bit for bit.  UNROLL
// channel groups' gathers are in flight together (two in the interpolate
// kernel; one in the rasterizer, whose registers are scarcer).
template <int UNROLL = 2>
__device__ __forceinline__ void interp_row4_da(const float* __restrict__ a0p, const float* __restrict__ a1p,
                                               const float* __restrict__ a2p, int A, float bw, float u, float v,
                                               float4 db, float* __restrict__ o, float* __restrict__ od,
                                               const float* __restrict__ tp, float& lsum) {
  // out_da rows are 2A floats, so every store is a float4.
#pragma unroll UNROLL
  for (int a = 0; a < A; a += 4) {
    const float4 x0 = ldg4(a0p + a), x1 = ldg4(a1p + a), x2 = ldg4(a2p + a);
    float4 y;
    y.x = bw * x0.x + u * x1.x + v * x2.x;
    y.y = bw * x0.y + u * x1.y + v * x2.y;
    y.z = bw * x0.z + u * x1.z + v * x2.z;
    y.w = bw * x0.w + u * x1.w + v * x2.w;
    stcs4(o + a, y);
    if (tp) lsum += sq_diff4(y, ldcs4(tp + a));
    const float4 d01 = make_float4(x1.x - x0.x, x1.y - x0.y, x1.z - x0.z, x1.w - x0.w);
    const float4 d02 = make_float4(x2.x - x0.x, x2.y - x0.y, x2.z - x0.z, x2.w - x0.w);
    stcs4(od + 2 * a, make_float4(d01.x * db.x + d02.x * db.z, d01.x * db.y + d02.x * db.w,
                                  d01.y * db.x + d02.y * db.z, d01.y * db.y + d02.y * db.w));
    stcs4(od + 2 * a + 4, make_float4(d01.z * db.x + d02.z * db.z, d01.z * db.y + d02.z * db.w,
                                      d01.w * db.x + d02.w * db.z, d01.w * db.y + d02.w * db.w));
  }
}

// The same row for a pixel that shows no triangle: zeros (and the loss of a
// zero prediction).
__device__ __forceinline__ void interp_row4_da_miss(int A, float* __restrict__ o, float* __restrict__ od,
                                                    const float* __restrict__ tp, float& lsum) {
  for (int a = 0; a < A; a += 4) {
    stcs4(o + a, make_float4(0.f, 0.f, 0.f, 0.f));
    if (tp) lsum += sq_diff4(make_float4(0.f, 0.f, 0.f, 0.f), ldcs4(tp + a));
  }
  for (int k = 0; k < 2 * A; k += 4) stcs4(od + k, make_float4(0.f, 0.f, 0.f, 0.f));
}

dr_status check_common(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                       const float* rast, int N, int H, int W, const int32_t* tri, int T,
                       const float* rast_db, const int32_t* diff_idx, int K, DiffIdx& idx) {
  DR_REQUIRE(ctx, attr && rast && (tri || T == 0), "interpolate: attr, rast and tri are required");
  DR_REQUIRE(ctx, N > 0 && H > 0 && W > 0 && V > 0 && A > 0 && T >= 0,
             "interpolate: bad sizes N=%d H=%d W=%d V=%d A=%d T=%d", N, H, W, V, A, T);
  DR_REQUIRE(ctx, attr_batch == 1 || attr_batch == N,
             "interpolate: attr batch dim %d incompatible with rast batch %d", attr_batch, N);
  DR_REQUIRE(ctx, aligned16(rast) && (!rast_db || aligned16(rast_db)),
             "interpolate: rast / rast_db must be 16-byte aligned");
  DR_REQUIRE(ctx, K >= 0, "interpolate: K < 0");
  if (K > 0) {
    DR_REQUIRE(ctx, rast_db != nullptr, "interpolate: rastDB is required when diffAttrs is set");
    if (diff_idx) {
      DR_REQUIRE(ctx, K <= DR_MAX_DIFF_ATTRS, "interpolate: at most %d diffAttrs indices", DR_MAX_DIFF_ATTRS);
      for (int k = 0; k < K; ++k) {
        DR_REQUIRE(ctx, diff_idx[k] >= 0 && diff_idx[k] < A,
                   "interpolate: diffAttrs.indices values must be in [0, A) (A=%d)", A);
        idx.k[k] = diff_idx[k];
      }
    } else {
      DR_REQUIRE(ctx, K == A, "interpolate: diff_idx == NULL (.all) requires K == A");
    }
  }
  return DR_OK;
}

}  // namespace

#define DR_INTERP_DISPATCH(KERNEL, ...)                                                  \
  do {                                                                                   \
    if (vec) {                                                                           \
      if (K == 0) KERNEL<true, false, false><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__); \
      else if (use_idx) KERNEL<true, true, true><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__); \
      else KERNEL<true, true, false><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__);        \
    } else {                                                                             \
      if (K == 0) KERNEL<false, false, false><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__); \
      else if (use_idx) KERNEL<false, true, true><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__); \
      else KERNEL<false, true, false><<<grid, 256, 0, ctx->stream>>>(__VA_ARGS__);       \
    }                                                                                    \
  } while (0)

