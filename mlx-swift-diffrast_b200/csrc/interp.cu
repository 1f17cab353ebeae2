// interp.cu — interpolate forward (with the pixel-derivative "DA" path) and
// its fused backward.
//
// Reference: Sources/MLXDiffRast/Interpolate.swift.  Forward = kernels
// diffrast_interp_fwd / _fwd_da (Interpolate.swift:137-228) in one kernel; the
// four VJP kernels _grad_attr, _grad_attr_da, _grad_rast, _grad_rast_db
// (Interpolate.swift:231-417) are one fused pass here, so rast / attr are read
// once.  attr_batch == 1 (the reference's broadcast of [V,A] / [1,V,A]) reads and
// accumulates one shared attribute table: the reference materialises N copies
// and lets MLX sum their gradients (Interpolate.swift:67-73).
#include "common.cuh"

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

// One thread per pixel.  VEC4: A % 4 == 0 and 16-byte aligned attr/out, so the
// vertex gathers and the output row are float4.
template <bool VEC4, bool DA, bool IDX>
__global__ void k_interp_fwd(const float* __restrict__ attr, bool attr_shared, int V, int A,
                             const float4* __restrict__ rast, int64_t P, int64_t HW,
                             const int32_t* __restrict__ tri, int T,
                             const float4* __restrict__ rast_db, const DiffIdx idx, int K,
                             float* __restrict__ out, float* __restrict__ out_da, unsigned* err) {
  int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= P) return;
  const float4 r = __ldg(rast + pix);
  // rast_db is independent of the triangle gathers: issue it with rast.
  float4 db = make_float4(0.f, 0.f, 0.f, 0.f);
  if (DA) db = __ldg(rast_db + pix);
  int t = (int)r.w - 1;
  float* o = out + pix * A;
  float* od = DA ? out_da + pix * 2 * K : nullptr;
  int i0, i1, i2;
  bool hit = t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  if (hit && !tri_verts(tri, t, V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  if (!hit) {
    if (VEC4) {
      for (int a = 0; a < A; a += 4) *reinterpret_cast<float4*>(o + a) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int a = 0; a < A; ++a) o[a] = 0.0f;
    }
    if (DA) {
      if (VEC4 && !IDX) {
        for (int k = 0; k < 2 * K; k += 4) *reinterpret_cast<float4*>(od + k) = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        for (int k = 0; k < 2 * K; ++k) od[k] = 0.0f;
      }
    }
    return;
  }
  const float u = r.x, v = r.y;
  const float bw = 1.0f - u - v;
  const int n = (int)(pix / HW);
  const float* an = attr + (attr_shared ? 0 : (int64_t)n * V * A);
  const float* a0p = an + (int64_t)i0 * A;
  const float* a1p = an + (int64_t)i1 * A;
  const float* a2p = an + (int64_t)i2 * A;
  if (VEC4 && DA && !IDX) {
    // .all with A % 4 == 0: out and out_da from the same float4 gathers;
    // out_da rows are 2A floats, so every store is a float4.  Unrolled by two
    // so the gathers of consecutive channel groups are in flight together.
#pragma unroll 2
    for (int a = 0; a < A; a += 4) {
      const float4 x0 = ldg4(a0p + a), x1 = ldg4(a1p + a), x2 = ldg4(a2p + a);
      float4 y;
      y.x = bw * x0.x + u * x1.x + v * x2.x;
      y.y = bw * x0.y + u * x1.y + v * x2.y;
      y.z = bw * x0.z + u * x1.z + v * x2.z;
      y.w = bw * x0.w + u * x1.w + v * x2.w;
      *reinterpret_cast<float4*>(o + a) = y;
      const float4 d01 = make_float4(x1.x - x0.x, x1.y - x0.y, x1.z - x0.z, x1.w - x0.w);
      const float4 d02 = make_float4(x2.x - x0.x, x2.y - x0.y, x2.z - x0.z, x2.w - x0.w);
      *reinterpret_cast<float4*>(od + 2 * a) =
          make_float4(d01.x * db.x + d02.x * db.z, d01.x * db.y + d02.x * db.w,
                      d01.y * db.x + d02.y * db.z, d01.y * db.y + d02.y * db.w);
      *reinterpret_cast<float4*>(od + 2 * a + 4) =
          make_float4(d01.z * db.x + d02.z * db.z, d01.z * db.y + d02.z * db.w,
                      d01.w * db.x + d02.w * db.z, d01.w * db.y + d02.w * db.w);
    }
    return;
  }
  if (VEC4) {
#pragma unroll 2
    for (int a = 0; a < A; a += 4) {
      const float4 x0 = ldg4(a0p + a), x1 = ldg4(a1p + a), x2 = ldg4(a2p + a);
      float4 y;
      y.x = bw * x0.x + u * x1.x + v * x2.x;
      y.y = bw * x0.y + u * x1.y + v * x2.y;
      y.z = bw * x0.z + u * x1.z + v * x2.z;
      y.w = bw * x0.w + u * x1.w + v * x2.w;
      *reinterpret_cast<float4*>(o + a) = y;
    }
  } else {
    for (int a = 0; a < A; ++a) o[a] = bw * __ldg(a0p + a) + u * __ldg(a1p + a) + v * __ldg(a2p + a);
  }
  if (DA) {
    for (int k = 0; k < K; ++k) {
      const int a = IDX ? idx.k[k] : k;
      const float x0 = __ldg(a0p + a), x1 = __ldg(a1p + a), x2 = __ldg(a2p + a);
      const float d01 = x1 - x0, d02 = x2 - x0;
      od[2 * k + 0] = d01 * db.x + d02 * db.z;
      od[2 * k + 1] = d01 * db.y + d02 * db.w;
    }
  }
}

// Fused VJP: d_attr, d_rast, d_rast_db in one pass.  Pixels of a warp that hit
// the same triangle (runs along the row) first sum their d_attr contributions
// with warp shuffles, so each run issues one set of atomics instead of one per
// pixel.  Channels go in groups of four (float4 atomics when VEC4).
template <bool VEC4, bool DA, bool IDX>
__global__ void k_interp_bwd(const float* __restrict__ attr, bool attr_shared, int V, int A,
                             const float4* __restrict__ rast, int64_t P, int64_t HW,
                             const int32_t* __restrict__ tri, int T,
                             const float4* __restrict__ rast_db, const DiffIdx idx, int K,
                             const float* __restrict__ d_out, const float* __restrict__ d_out_da,
                             float* __restrict__ d_attr, float4* __restrict__ d_rast,
                             float4* __restrict__ d_rast_db, unsigned* err) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool in = pix < P;
  float4 r = make_float4(0.f, 0.f, 0.f, -1.f);
  if (in) r = __ldg(rast + pix);
  int t = (int)r.w - 1;
  int i0 = 0, i1 = 0, i2 = 0;
  bool hit = in && t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  if (hit && !tri_verts(tri, t, V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  const int n = in ? (int)(pix / HW) : 0;
  // Run key: the triangle, and the view when every view has its own attributes.
  const long long key = hit ? ((attr_shared ? 0ll : (long long)n * T) + t) : -1ll - (long long)lane;
  bool head;
  const int seg_end = warp_runs(key, lane, head);
  const int span = warp_max_run(lane, seg_end, head);

  const float u = r.x, v = r.y;
  const float bw = 1.0f - u - v;
  const int64_t nb = attr_shared ? 0 : (int64_t)n * V * A;
  const float* a0p = attr + nb + (int64_t)i0 * A;
  const float* a1p = attr + nb + (int64_t)i1 * A;
  const float* a2p = attr + nb + (int64_t)i2 * A;
  float* g0p = d_attr + nb + (int64_t)i0 * A;
  float* g1p = d_attr + nb + (int64_t)i1 * A;
  float* g2p = d_attr + nb + (int64_t)i2 * A;
  const float* g = d_out + pix * A;
  const float* gd = DA ? d_out_da + pix * 2 * K : nullptr;
  float4 db = make_float4(0.f, 0.f, 0.f, 0.f);
  if (DA && hit) db = __ldg(rast_db + pix);
  float du = 0.0f, dv = 0.0f;
  float d_udx = 0.0f, d_udy = 0.0f, d_vdx = 0.0f, d_vdy = 0.0f;
  for (int a = 0; a < A; a += 4) {
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
    if (hit) {
      float ga[4], x0[4], x1[4], x2[4];
      if (VEC4) {
        const float4 q = ldg4(g + a), p0 = ldg4(a0p + a), p1 = ldg4(a1p + a), p2 = ldg4(a2p + a);
        ga[0] = q.x; ga[1] = q.y; ga[2] = q.z; ga[3] = q.w;
        x0[0] = p0.x; x0[1] = p0.y; x0[2] = p0.z; x0[3] = p0.w;
        x1[0] = p1.x; x1[1] = p1.y; x1[2] = p1.z; x1[3] = p1.w;
        x2[0] = p2.x; x2[1] = p2.y; x2[2] = p2.z; x2[3] = p2.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool ok = a + j < A;
          ga[j] = ok ? __ldg(g + a + j) : 0.f;
          x0[j] = ok ? __ldg(a0p + a + j) : 0.f;
          x1[j] = ok ? __ldg(a1p + a + j) : 0.f;
          x2[j] = ok ? __ldg(a2p + a + j) : 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c0[j] = bw * ga[j];
        c1[j] = u * ga[j];
        c2[j] = v * ga[j];
        du += (x1[j] - x0[j]) * ga[j];
        dv += (x2[j] - x0[j]) * ga[j];
      }
      if (DA && !IDX) {
        // .all: channel a + j has its (d/dx, d/dy) cotangent at 2(a + j).
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (!VEC4 && a + j >= A) break;
          const float gx = __ldg(gd + 2 * (a + j)), gy = __ldg(gd + 2 * (a + j) + 1);
          const float u_term = gx * db.x + gy * db.y;
          const float v_term = gx * db.z + gy * db.w;
          c0[j] += -u_term - v_term;
          c1[j] += u_term;
          c2[j] += v_term;
          const float d01 = x1[j] - x0[j], d02 = x2[j] - x0[j];
          d_udx += d01 * gx;
          d_udy += d01 * gy;
          d_vdx += d02 * gx;
          d_vdy += d02 * gy;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c0[j] = warp_seg_sum(c0[j], lane, seg_end, span);
      c1[j] = warp_seg_sum(c1[j], lane, seg_end, span);
      c2[j] = warp_seg_sum(c2[j], lane, seg_end, span);
    }
    if (hit && head) {
      if (VEC4) {
        atomicAdd(reinterpret_cast<float4*>(g0p + a), make_float4(c0[0], c0[1], c0[2], c0[3]));
        atomicAdd(reinterpret_cast<float4*>(g1p + a), make_float4(c1[0], c1[1], c1[2], c1[3]));
        atomicAdd(reinterpret_cast<float4*>(g2p + a), make_float4(c2[0], c2[1], c2[2], c2[3]));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (a + j >= A) break;
          atomicAdd(g0p + a + j, c0[j]);
          atomicAdd(g1p + a + j, c1[j]);
          atomicAdd(g2p + a + j, c2[j]);
        }
      }
    }
  }
  if (!in) return;
  if (!hit) {
    d_rast[pix] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (DA) d_rast_db[pix] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  d_rast[pix] = make_float4(du, dv, 0.0f, 0.0f);
  if (DA) {
    if (IDX) {
      // .indices: arbitrary (possibly repeated) attribute indices.
      for (int k = 0; k < K; ++k) {
        const int a = idx.k[k];
        const float gx = __ldg(gd + 2 * k), gy = __ldg(gd + 2 * k + 1);
        const float u_term = gx * db.x + gy * db.y;
        const float v_term = gx * db.z + gy * db.w;
        atomicAdd(g0p + a, -u_term - v_term);
        atomicAdd(g1p + a, u_term);
        atomicAdd(g2p + a, v_term);
        const float x0 = __ldg(a0p + a), x1 = __ldg(a1p + a), x2 = __ldg(a2p + a);
        const float d01 = x1 - x0, d02 = x2 - x0;
        d_udx += d01 * gx;
        d_udy += d01 * gy;
        d_vdx += d02 * gx;
        d_vdy += d02 * gy;
      }
    }
    d_rast_db[pix] = make_float4(d_udx, d_udy, d_vdx, d_vdy);
  }
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

using namespace dr;

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

extern "C" dr_status dr_interpolate_fwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                        const float* rast, int N, int H, int W, const int32_t* tri,
                                        int T, const float* rast_db, const int32_t* diff_idx, int K,
                                        float* out, float* out_da) {
  DR_ENTER(ctx);
  DiffIdx idx;
  dr_status st = check_common(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, idx);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, out && (K == 0 || out_da), "interpolate: out / out_da required");
  const int64_t P = (int64_t)N * H * W;
  const bool vec = (A % 4 == 0) && aligned16(attr) && aligned16(out);
  const bool use_idx = diff_idx != nullptr;
  const unsigned grid = grid_for(P, 256);
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* db4 = reinterpret_cast<const float4*>(rast_db);
  DR_TB(ctx);
  DR_INTERP_DISPATCH(k_interp_fwd, attr, attr_batch == 1, V, A, r4, P, (int64_t)H * W, tri, T, db4, idx, K, out,
                     out_da, ctx->d_err);
  DR_LAUNCHED(ctx, "interp_fwd");
  return DR_OK;
}

extern "C" dr_status dr_interpolate_bwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                        const float* rast, int N, int H, int W, const int32_t* tri,
                                        int T, const float* rast_db, const int32_t* diff_idx, int K,
                                        const float* d_out, const float* d_out_da, float* d_attr,
                                        float* d_rast, float* d_rast_db) {
  DR_ENTER(ctx);
  DiffIdx idx;
  dr_status st = check_common(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, idx);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, d_out && d_attr && d_rast && (K == 0 || (d_out_da && d_rast_db)),
             "interpolate_bwd: d_out, d_attr, d_rast (and d_out_da, d_rast_db with diffAttrs) required");
  DR_REQUIRE(ctx, aligned16(d_rast) && (K == 0 || aligned16(d_rast_db)),
             "interpolate_bwd: d_rast / d_rast_db must be 16-byte aligned");
  DR_CUDA(ctx, cudaMemsetAsync(d_attr, 0, sizeof(float) * (size_t)attr_batch * V * A, ctx->stream),
          "interpolate_bwd memset");
  const int64_t P = (int64_t)N * H * W;
  const bool vec = (A % 4 == 0) && aligned16(attr) && aligned16(d_out) && aligned16(d_attr);
  const bool use_idx = diff_idx != nullptr;
  const unsigned grid = grid_for(P, 256);
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* db4 = reinterpret_cast<const float4*>(rast_db);
  float4* dr4 = reinterpret_cast<float4*>(d_rast);
  float4* ddb4 = reinterpret_cast<float4*>(d_rast_db);
  DR_TB(ctx);
  DR_INTERP_DISPATCH(k_interp_bwd, attr, attr_batch == 1, V, A, r4, P, (int64_t)H * W, tri, T, db4, idx, K, d_out,
                     d_out_da, d_attr, dr4, ddb4, ctx->d_err);
  DR_LAUNCHED(ctx, "interp_bwd");
  return DR_OK;
}
