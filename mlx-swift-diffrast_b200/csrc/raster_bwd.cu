// raster_bwd.cu — rasterize backward (d_pos), Rasterize.swift:637-812, and
// the one-pass VJP of the fused two-layer raster + interpolate forward
// (interpolate's VJP, Interpolate.swift:231-417, feeding the rasterize VJP in
// registers).
//
// The gradients are compared with the CPU oracle within a relative L2
// tolerance, not bit for bit, so this translation unit is built with FMA
// contraction (the forward, raster.cu, keeps every operation separately
// rounded).
#include "interp_common.cuh"

namespace {

// Clip-space gradients g0..g2 of a pixel's three triangle vertices (clip
// positions q0..q2, already transformed in the per-view transform mode) from
// the pixel's rast cotangent (d_u, d_v, d_z) and, with DB, its rast_db
// cotangent gd: the per-pixel body of Rasterize.swift:637-812.
template <bool DB>
__device__ __forceinline__ void raster_vjp_px(int pw, int ph, int H, int W, float u_val, float v_val, float d_u,
                                              float d_v, float d_z, float4 gd, float4 q0, float4 q1, float4 q2,
                                              float4& g0, float4& g1, float4& g2) {
  const float bw_val = 1.0f - u_val - v_val;
  const float d_db0 = gd.x, d_db1 = gd.y, d_db2 = gd.z, d_db3 = gd.w;
  const float Px = __fdividef(2.0f * ((float)pw + 0.5f), (float)W) - 1.0f;
  const float Py = 1.0f - __fdividef(2.0f * ((float)ph + 0.5f), (float)H);
  // Gradient-only arithmetic (compared within tolerance, not bit for bit):
  // one fast reciprocal per w instead of IEEE divisions.
  const float inv_w0 = __fdividef(1.0f, q0.w), inv_w1 = __fdividef(1.0f, q1.w), inv_w2 = __fdividef(1.0f, q2.w);
  const float sx0 = q0.x * inv_w0, sy0 = q0.y * inv_w0, sz0 = q0.z * inv_w0;
  const float sx1 = q1.x * inv_w1, sy1 = q1.y * inv_w1, sz1 = q1.z * inv_w1;
  const float sx2 = q2.x * inv_w2, sy2 = q2.y * inv_w2, sz2 = q2.z * inv_w2;
  const float area = (sx1 - sx0) * (sy2 - sy0) - (sx2 - sx0) * (sy1 - sy0);
  const float inv_area = __fdividef(1.0f, area);
  const float dadsx0 = sy1 - sy2, dadsx1 = sy2 - sy0, dadsx2 = sy0 - sy1;
  const float dadsy0 = sx2 - sx1, dadsy1 = sx0 - sx2, dadsy2 = sx1 - sx0;
  const float de1dsx0 = Py - sy2, de1dsx2 = sy0 - Py, de1dsy0 = sx2 - Px, de1dsy2 = Px - sx0;
  const float de2dsx0 = sy1 - Py, de2dsx1 = Py - sy0, de2dsy0 = Px - sx1, de2dsy1 = sx0 - Px;
  const float dudsx0 = (de1dsx0 - u_val * dadsx0) * inv_area;
  const float dudsx1 = (0.0f - u_val * dadsx1) * inv_area;
  const float dudsx2 = (de1dsx2 - u_val * dadsx2) * inv_area;
  const float dudsy0 = (de1dsy0 - u_val * dadsy0) * inv_area;
  const float dudsy1 = (0.0f - u_val * dadsy1) * inv_area;
  const float dudsy2 = (de1dsy2 - u_val * dadsy2) * inv_area;
  const float dvdsx0 = (de2dsx0 - v_val * dadsx0) * inv_area;
  const float dvdsx1 = (de2dsx1 - v_val * dadsx1) * inv_area;
  const float dvdsx2 = (0.0f - v_val * dadsx2) * inv_area;
  const float dvdsy0 = (de2dsy0 - v_val * dadsy0) * inv_area;
  const float dvdsy1 = (de2dsy1 - v_val * dadsy1) * inv_area;
  const float dvdsy2 = (0.0f - v_val * dadsy2) * inv_area;
  const float dsz10 = sz1 - sz0, dsz20 = sz2 - sz0;
  float dsx0 = d_u * dudsx0 + d_v * dvdsx0 + d_z * (dudsx0 * dsz10 + dvdsx0 * dsz20);
  float dsx1 = d_u * dudsx1 + d_v * dvdsx1 + d_z * (dudsx1 * dsz10 + dvdsx1 * dsz20);
  float dsx2 = d_u * dudsx2 + d_v * dvdsx2 + d_z * (dudsx2 * dsz10 + dvdsx2 * dsz20);
  float dsy0 = d_u * dudsy0 + d_v * dvdsy0 + d_z * (dudsy0 * dsz10 + dvdsy0 * dsz20);
  float dsy1 = d_u * dudsy1 + d_v * dvdsy1 + d_z * (dudsy1 * dsz10 + dvdsy1 * dsz20);
  float dsy2 = d_u * dudsy2 + d_v * dvdsy2 + d_z * (dudsy2 * dsz10 + dvdsy2 * dsz20);
  const float dsz0_s = d_z * bw_val, dsz1_s = d_z * u_val, dsz2_s = d_z * v_val;
  if (DB) {
    const float Kx = 2.0f / (float)W, Ky = -2.0f / (float)H;
    const float rdb0 = (sy2 - sy0) * Kx * inv_area;
    const float rdb1 = (sx0 - sx2) * Ky * inv_area;
    const float rdb2 = (sy0 - sy1) * Kx * inv_area;
    const float rdb3 = (sx1 - sx0) * Ky * inv_area;
    const float s = d_db0 * rdb0 + d_db1 * rdb1 + d_db2 * rdb2 + d_db3 * rdb3;
    dsx0 += (-s * dadsx0) * inv_area;
    dsx1 += (-s * dadsx1) * inv_area;
    dsx2 += (-s * dadsx2) * inv_area;
    dsy0 += (-s * dadsy0) * inv_area;
    dsy1 += (-s * dadsy1) * inv_area;
    dsy2 += (-s * dadsy2) * inv_area;
    dsy0 += d_db0 * (-Kx) * inv_area;
    dsy2 += d_db0 * (Kx) * inv_area;
    dsx0 += d_db1 * (Ky) * inv_area;
    dsx2 += d_db1 * (-Ky) * inv_area;
    dsy0 += d_db2 * (Kx) * inv_area;
    dsy1 += d_db2 * (-Kx) * inv_area;
    dsx0 += d_db3 * (-Ky) * inv_area;
    dsx1 += d_db3 * (Ky) * inv_area;
  }
  g0 = make_float4(dsx0 * inv_w0, dsy0 * inv_w0, dsz0_s * inv_w0, -(sx0 * dsx0 + sy0 * dsy0 + sz0 * dsz0_s) * inv_w0);
  g1 = make_float4(dsx1 * inv_w1, dsy1 * inv_w1, dsz1_s * inv_w1, -(sx1 * dsx1 + sy1 * dsy1 + sz1 * dsz1_s) * inv_w1);
  g2 = make_float4(dsx2 * inv_w2, dsy2 * inv_w2, dsz2_s * inv_w2, -(sx2 * dsx2 + sy2 * dsy2 + sz2 * dsz2_s) * inv_w2);
}

// d_pos: Rasterize.swift:637-812, one thread per pixel.  Pixels of a warp that
// hit the same (view, triangle) first sum their 12 vertex gradients with warp
// shuffles; the first pixel of each run issues the float4 atomics.  With a
// per-view transform (XF) the clip-space gradient g of vertex v is mapped to
// the shared vertex buffer as M_n^T g.
template <bool DB, bool VEC, bool XF>
__global__ void __launch_bounds__(256, DR_MINB_RASTER_BWD) k_raster_bwd(const float* __restrict__ pos, const float* __restrict__ xform, int V,
                             const int32_t* __restrict__ tri, int T, bool shared_pos, int N, int H, int W,
                             const float4* __restrict__ rast, const float4* __restrict__ d_rast,
                             const float4* __restrict__ d_rast_db, float* __restrict__ d_pos,
                             unsigned* err) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int64_t P = (int64_t)N * H * W;
  const bool in = pix < P;
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (in) r = __ldcs(rast + pix);
  const int t = (int)r.w - 1;
  bool hit = in && t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  int i0 = 0, i1 = 0, i2 = 0;
  if (hit) {
    i0 = __ldg(tri + 3 * t); i1 = __ldg(tri + 3 * t + 1); i2 = __ldg(tri + 3 * t + 2);
    if (i0 < 0 || i0 >= V || i1 < 0 || i1 >= V || i2 < 0 || i2 >= V) {
      dr_flag(err, DR_DEVERR_VERTEX);
      hit = false;
    }
  }
  int pn = 0, ph = 0, pw = 0;
  if (in) pix_nyx(pix, P, H, W, pn, ph, pw);
  const int64_t pos_n_base = (shared_pos || XF) ? 0 : (int64_t)pn * V * 4;
  float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0, g2 = g0;
  Mat4 M;
  if (XF && hit) M = load_mat4(xform + (int64_t)pn * 16);
  if (hit) {
    const float4 g = __ldcs(d_rast + pix);
    const float4 gd = DB ? __ldcs(d_rast_db + pix) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 q0 = ldg4(pos + pos_n_base + (int64_t)i0 * 4);
    float4 q1 = ldg4(pos + pos_n_base + (int64_t)i1 * 4);
    float4 q2 = ldg4(pos + pos_n_base + (int64_t)i2 * 4);
    if (XF) {
      q0 = mat4_apply(M, q0);
      q1 = mat4_apply(M, q1);
      q2 = mat4_apply(M, q2);
    }
    raster_vjp_px<DB>(pw, ph, H, W, r.x, r.y, g.x, g.y, g.z, gd, q0, q1, q2, g0, g1, g2);
  }
  bool head;
  const long long key = hit ? (long long)pn * T + t : -1ll - (long long)lane;
  const int seg_end = warp_runs(key, lane, head);
  const int span = warp_max_run(lane, seg_end, head);
  {
    float gv[12] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w, g2.x, g2.y, g2.z, g2.w};
    warp_seg_sum_n<12>(gv, lane, seg_end, span);
    g0 = make_float4(gv[0], gv[1], gv[2], gv[3]);
    g1 = make_float4(gv[4], gv[5], gv[6], gv[7]);
    g2 = make_float4(gv[8], gv[9], gv[10], gv[11]);
  }
  if (!(hit && head)) return;
  if (XF) {
    g0 = mat4_apply_t(M, g0);
    g1 = mat4_apply_t(M, g1);
    g2 = mat4_apply_t(M, g2);
  }
  float* b0 = d_pos + pos_n_base + (int64_t)i0 * 4;
  float* b1 = d_pos + pos_n_base + (int64_t)i1 * 4;
  float* b2 = d_pos + pos_n_base + (int64_t)i2 * 4;
  if (VEC) {
    atomicAdd(reinterpret_cast<float4*>(b0), g0);
    atomicAdd(reinterpret_cast<float4*>(b1), g1);
    atomicAdd(reinterpret_cast<float4*>(b2), g2);
  } else {
    atomicAdd(b0 + 0, g0.x); atomicAdd(b0 + 1, g0.y); atomicAdd(b0 + 2, g0.z); atomicAdd(b0 + 3, g0.w);
    atomicAdd(b1 + 0, g1.x); atomicAdd(b1 + 1, g1.y); atomicAdd(b1 + 2, g1.z); atomicAdd(b1 + 3, g1.w);
    atomicAdd(b2 + 0, g2.x); atomicAdd(b2 + 1, g2.y); atomicAdd(b2 + 2, g2.z); atomicAdd(b2 + 3, g2.w);
  }
}

// The layers of the fused forward (dr_rasterize_xf_interp_fwd) whose out has a
// cotangent: each layer's rast and out's cotangent (given, or its fused
// loss's).
struct InterpRasterLayers {
  const float4* rast[2];
  Cot cot[2];
};

// The interpolate and rasterize VJPs of the fused forward in one pass, for the
// case where out_da, rast and rast_db take no cotangent of their own: the pixel's
// rast cotangent is then exactly the (d_u, d_v, 0) that the interpolate VJP
// forms, so it feeds the rasterize VJP in registers instead of a d_rast
// round trip through memory.  The pixel's rast, triangle and warp runs serve
// both scatters.  blockIdx.y is the layer; the pixels follow the context's
// tile order (so the attribute rows and vertices of a region stay in L2 while
// its views pass).  Per pixel: interpolate's VJP as k_interp_bwd with float4
// rows and no pixel derivatives, then k_raster_bwd's in per-view transform
// mode.
__global__ void __launch_bounds__(256, DR_MINB_INTERP_RASTER_BWD)
    k_interp_raster_bwd(const float* __restrict__ verts, const float* __restrict__ xform, int V,
                        const int32_t* __restrict__ tri, int T, int H, int W, int64_t P,
                        const float* __restrict__ attr, bool attr_shared, int A, const InterpRasterLayers layers,
                        float* __restrict__ d_attr, float* __restrict__ d_verts, const PixOrder po, unsigned* err) {
  // Constant indices (a select, not an index into the parameter block, which
  // would copy it to local memory).
  const bool second = blockIdx.y != 0;
  const float4* __restrict__ rast = second ? layers.rast[1] : layers.rast[0];
  const Cot cot = second ? layers.cot[1] : layers.cot[0];
  bool in;
  int n, ph, pw;
  const int64_t pix = pix_of_nyx(po, P, H, W, in, n, ph, pw);
  const int lane = threadIdx.x & 31;
  float4 r = make_float4(0.f, 0.f, 0.f, -1.f);
  if (in) r = __ldcs(rast + pix);
  const int t = (int)r.w - 1;
  int i0 = 0, i1 = 0, i2 = 0;
  bool hit = in && t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  if (hit && !tri_verts(tri, t, V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  // One run key for both scatters: the (view, triangle), since each view's
  // vertex gradient is mapped through its own transform.
  const long long key = hit ? (long long)n * T + t : -1ll - (long long)lane;
  bool head;
  const int seg_end = warp_runs(key, lane, head);
  const int span = warp_max_run(lane, seg_end, head);
  const float u = r.x, v = r.y;
  // Interpolate VJP: d_attr, and the pixel's d_u, d_v.
  float du = 0.0f, dv = 0.0f;
  {
    const float bw = 1.0f - u - v;
    const int64_t nb = attr_shared ? 0 : (int64_t)n * V * A;
    const float* a0p = attr + nb + (int64_t)i0 * A;
    const float* a1p = attr + nb + (int64_t)i1 * A;
    const float* a2p = attr + nb + (int64_t)i2 * A;
    float* g0p = d_attr + nb + (int64_t)i0 * A;
    float* g1p = d_attr + nb + (int64_t)i1 * A;
    float* g2p = d_attr + nb + (int64_t)i2 * A;
    const float gl = cot_g(cot);
    for (int a = 0; a < A; a += 4) {
      float cv[12] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (hit) {
        const float4 q = cot_at4<true>(cot, gl, pix * A + a), x0 = ldg4(a0p + a), x1 = ldg4(a1p + a),
                     x2 = ldg4(a2p + a);
        const float ga[4] = {q.x, q.y, q.z, q.w};
        const float d01[4] = {x1.x - x0.x, x1.y - x0.y, x1.z - x0.z, x1.w - x0.w};
        const float d02[4] = {x2.x - x0.x, x2.y - x0.y, x2.z - x0.z, x2.w - x0.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          cv[j] = bw * ga[j];
          cv[4 + j] = u * ga[j];
          cv[8 + j] = v * ga[j];
          du += d01[j] * ga[j];
          dv += d02[j] * ga[j];
        }
      }
      warp_seg_sum_n<12>(cv, lane, seg_end, span);
      if (hit && head) {
        atomicAdd(reinterpret_cast<float4*>(g0p + a), make_float4(cv[0], cv[1], cv[2], cv[3]));
        atomicAdd(reinterpret_cast<float4*>(g1p + a), make_float4(cv[4], cv[5], cv[6], cv[7]));
        atomicAdd(reinterpret_cast<float4*>(g2p + a), make_float4(cv[8], cv[9], cv[10], cv[11]));
      }
    }
  }
  // Rasterize VJP with the rast cotangent (du, dv, 0): d_verts.
  float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0, g2 = g0;
  Mat4 M;
  if (hit) {
    M = load_mat4(xform + (int64_t)n * 16);
    const float4 q0 = mat4_apply(M, ldg4(verts + (int64_t)i0 * 4));
    const float4 q1 = mat4_apply(M, ldg4(verts + (int64_t)i1 * 4));
    const float4 q2 = mat4_apply(M, ldg4(verts + (int64_t)i2 * 4));
    raster_vjp_px<false>(pw, ph, H, W, u, v, du, dv, 0.0f, make_float4(0.f, 0.f, 0.f, 0.f), q0, q1, q2, g0, g1,
                         g2);
  }
  {
    float gv[12] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w, g2.x, g2.y, g2.z, g2.w};
    warp_seg_sum_n<12>(gv, lane, seg_end, span);
    g0 = make_float4(gv[0], gv[1], gv[2], gv[3]);
    g1 = make_float4(gv[4], gv[5], gv[6], gv[7]);
    g2 = make_float4(gv[8], gv[9], gv[10], gv[11]);
  }
  if (!(hit && head)) return;
  atomicAdd(reinterpret_cast<float4*>(d_verts + (int64_t)i0 * 4), mat4_apply_t(M, g0));
  atomicAdd(reinterpret_cast<float4*>(d_verts + (int64_t)i1 * 4), mat4_apply_t(M, g1));
  atomicAdd(reinterpret_cast<float4*>(d_verts + (int64_t)i2 * 4), mat4_apply_t(M, g2));
}

}  // namespace

using namespace dr;

namespace {

dr_status raster_bwd_launch(dr_ctx* ctx, const float* pos, const float* xform, int V, const int32_t* tri, int T,
                            bool shared_pos, int N, int H, int W, const float* rast, const float* d_rast,
                            const float* d_rast_db, float* d_pos) {
  DR_REQUIRE(ctx, rast && d_rast, "rasterize_bwd: rast and d_rast are required");
  DR_REQUIRE(ctx, aligned16(rast) && aligned16(d_rast) && (!d_rast_db || aligned16(d_rast_db)),
             "rasterize_bwd: rast/d_rast/d_rast_db must be 16-byte aligned");
  const int64_t P = (int64_t)N * H * W;
  const bool vec = aligned16(d_pos);
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* g4 = reinterpret_cast<const float4*>(d_rast);
  const float4* gd4 = reinterpret_cast<const float4*>(d_rast_db);
  const unsigned grid = grid_for(P, 256);
  DR_TB(ctx);
#define DR_RB(DBV, VECV, XFV) \
  k_raster_bwd<DBV, VECV, XFV><<<grid, 256, 0, ctx->stream>>>(pos, xform, V, tri, T, shared_pos, N, H, W, r4, g4, \
                                                              gd4, d_pos, ctx->d_err)
  const bool db = d_rast_db != nullptr, xf = xform != nullptr;
  if (xf) {
    if (db) { if (vec) DR_RB(true, true, true); else DR_RB(true, false, true); }
    else { if (vec) DR_RB(false, true, true); else DR_RB(false, false, true); }
  } else {
    if (db) { if (vec) DR_RB(true, true, false); else DR_RB(true, false, false); }
    else { if (vec) DR_RB(false, true, false); else DR_RB(false, false, false); }
  }
#undef DR_RB
  DR_LAUNCHED(ctx, "raster_bwd");
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_rasterize_bwd(dr_ctx* ctx, const float* pos, int V, const int32_t* tri, int T,
                                      const int32_t* ranges, int N, int H, int W, const float* rast,
                                      const float* d_rast, const float* d_rast_db, float* d_pos) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, pos && (tri || T == 0) && rast && d_rast && d_pos, "rasterize_bwd: null pointer");
  DR_REQUIRE(ctx, N > 0 && V > 0 && T >= 0 && H > 0 && W > 0, "rasterize_bwd: bad sizes");
  DR_REQUIRE(ctx, aligned16(pos), "rasterize_bwd: pos must be 16-byte aligned");
  const bool shared_pos = ranges != nullptr;
  const size_t npos = (size_t)(shared_pos ? 1 : N) * V * 4;
  DR_CUDA(ctx, cudaMemsetAsync(d_pos, 0, sizeof(float) * npos, ctx->stream), "rasterize_bwd memset");
  return raster_bwd_launch(ctx, pos, nullptr, V, tri, T, shared_pos, N, H, W, rast, d_rast, d_rast_db, d_pos);
}

namespace {

dr_status layers_bwd(dr_ctx* ctx, const float* pos, const float* xform, int V, const int32_t* tri, int T,
                     const int32_t* ranges, int N, int H, int W, int num_layers, const float* const* rast,
                     const float* const* d_rast, const float* const* d_rast_db, float* d_pos) {
  DR_REQUIRE(ctx, pos && (tri || T == 0) && rast && d_rast && d_pos && num_layers >= 1,
             "rasterize_layers_bwd: null pointer");
  DR_REQUIRE(ctx, N > 0 && V > 0 && T >= 0 && H > 0 && W > 0, "rasterize_layers_bwd: bad sizes");
  DR_REQUIRE(ctx, aligned16(pos), "rasterize_layers_bwd: pos must be 16-byte aligned");
  const bool shared_pos = ranges != nullptr;
  const size_t npos = (size_t)((shared_pos || xform) ? 1 : N) * V * 4;
  DR_CUDA(ctx, cudaMemsetAsync(d_pos, 0, sizeof(float) * npos, ctx->stream), "rasterize_layers_bwd memset");
  for (int l = 0; l < num_layers; ++l) {
    if (!d_rast[l]) continue;  // a layer whose outputs did not reach the loss
    dr_status st = raster_bwd_launch(ctx, pos, xform, V, tri, T, shared_pos, N, H, W, rast[l], d_rast[l],
                                     d_rast_db ? d_rast_db[l] : nullptr, d_pos);
    if (st != DR_OK) return st;
  }
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_rasterize_layers_bwd(dr_ctx* ctx, const float* pos, int V, const int32_t* tri, int T,
                                             const int32_t* ranges, int N, int H, int W, int num_layers,
                                             const float* const* rast, const float* const* d_rast,
                                             const float* const* d_rast_db, float* d_pos) {
  DR_ENTER(ctx);
  return layers_bwd(ctx, pos, nullptr, V, tri, T, ranges, N, H, W, num_layers, rast, d_rast, d_rast_db, d_pos);
}

extern "C" dr_status dr_rasterize_xf_bwd(dr_ctx* ctx, const float* verts, int V, const float* xform,
                                         const int32_t* tri, int T, int N, int H, int W, int num_layers,
                                         const float* const* rast, const float* const* d_rast,
                                         const float* const* d_rast_db, float* d_verts) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform != nullptr && ((uintptr_t)xform & 15) == 0,
             "rasterize_xf_bwd: xform [N,4,4] must be given and 16-byte aligned");
  return layers_bwd(ctx, verts, xform, V, tri, T, nullptr, N, H, W, num_layers, rast, d_rast, d_rast_db, d_verts);
}

extern "C" dr_status dr_rasterize_xf_interp_bwd(dr_ctx* ctx, const float* verts, int V, const float* xform,
                                                const int32_t* tri, int T, int N, int H, int W, const float* attr,
                                                int attr_batch, int A, const float* const* rast,
                                                const float* const* d_out, const float* const* out,
                                                const float* const* target, float scale,
                                                const float* const* d_loss, float* d_attr, float* d_verts) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, verts && xform && (tri || T == 0) && rast && d_attr && d_verts,
             "rasterize_interp_bwd: verts, xform, tri, rast, d_attr and d_verts are required");
  DR_REQUIRE(ctx, N > 0 && H > 0 && W > 0 && V > 0 && T >= 0,
             "rasterize_interp_bwd: bad sizes N=%d H=%d W=%d V=%d T=%d", N, H, W, V, T);
  DR_REQUIRE(ctx, aligned16(verts) && aligned16(xform) && aligned16(d_verts),
             "rasterize_interp_bwd: verts, xform and d_verts must be 16-byte aligned");
  DR_REQUIRE(ctx, attr && aligned16(attr) && aligned16(d_attr) && A > 0 && A % 4 == 0,
             "rasterize_interp_bwd: attr and d_attr must be 16-byte aligned with A a multiple of 4 (A=%d)", A);
  DR_REQUIRE(ctx, attr_batch == 1 || attr_batch == N,
             "rasterize_interp_bwd: attr batch dim %d incompatible with %d views", attr_batch, N);
  InterpRasterLayers lay{};
  int nl = 0;
  for (int l = 0; l < 2; ++l) {
    const float* d = d_out ? d_out[l] : nullptr;
    const float* o = out ? out[l] : nullptr;
    const float* tg = target ? target[l] : nullptr;
    const float* dl = d_loss ? d_loss[l] : nullptr;
    DR_REQUIRE(ctx, (o == nullptr) == (tg == nullptr) && (o == nullptr) == (dl == nullptr),
               "rasterize_interp_bwd: layer %d: out, target and d_loss go together", l);
    DR_REQUIRE(ctx, !(d && o), "rasterize_interp_bwd: layer %d: d_out or a fused loss, not both", l);
    if (!d && !o) continue;  // out of this layer takes no cotangent
    DR_REQUIRE(ctx, rast[l] && aligned16(rast[l]) && aligned16(d) && aligned16(o) && aligned16(tg),
               "rasterize_interp_bwd: layer %d: rast and the cotangent's rows must be given, 16-byte aligned", l);
    lay.rast[nl] = reinterpret_cast<const float4*>(rast[l]);
    lay.cot[nl] = Cot{d, o, tg, 2.0f * scale, dl};
    ++nl;
  }
  DR_CUDA(ctx, cudaMemsetAsync(d_attr, 0, sizeof(float) * (size_t)attr_batch * V * A, ctx->stream),
          "rasterize_interp_bwd memset");
  DR_CUDA(ctx, cudaMemsetAsync(d_verts, 0, sizeof(float) * (size_t)V * 4, ctx->stream),
          "rasterize_interp_bwd memset");
  if (nl == 0) return DR_OK;
  unsigned grid;
  const PixOrder po = pix_order(ctx, N, H, W, grid);
  DR_TB(ctx);
  k_interp_raster_bwd<<<dim3(grid, nl), 256, 0, ctx->stream>>>(verts, xform, V, tri, T, H, W, (int64_t)N * H * W,
                                                               attr, attr_batch == 1, A, lay, d_attr, d_verts, po,
                                                               ctx->d_err);
  DR_LAUNCHED(ctx, "interp_raster_bwd");
  return DR_OK;
}
