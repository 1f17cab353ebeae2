// interp_common.cuh — helpers shared by the interpolate forward (interp.cu) and
// its VJP (interp_bwd.cu).  Not part of the public ABI.
#pragma once

#include "common.cuh"

using dr::PixOrder;
using dr::pix_of;
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

