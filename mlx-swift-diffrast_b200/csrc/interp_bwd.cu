// interp_bwd.cu — the fused interpolate VJP (d_attr, d_rast, d_rast_db), the
// reference's four kernels _grad_attr, _grad_attr_da, _grad_rast,
// _grad_rast_db (Interpolate.swift:231-417) in one pass.
//
// Built without FMA contraction, as the forward: its per-pixel d_rast and
// d_rast_db (sums over channels with cancellation) are compared with the CPU
// oracle elementwise within 1e-5 relative / 1e-6 absolute, which contraction's
// different rounding can exceed.
#include "interp_common.cuh"

namespace {

template <bool VEC4, bool DA, bool IDX>
__global__ void k_interp_bwd(const float* __restrict__ attr, bool attr_shared, int V, int A,
                             const float4* __restrict__ rast, int64_t P, int64_t HW,
                             const int32_t* __restrict__ tri, int T,
                             const float4* __restrict__ rast_db, const DiffIdx idx, int K,
                             const Cot d_out, const float* __restrict__ d_out_da,
                             float* __restrict__ d_attr, float4* __restrict__ d_rast,
                             float4* __restrict__ d_rast_db, const PixOrder po, unsigned* err) {
  bool in;
  const int64_t pix = pix_of(po, P, in);
  const int lane = threadIdx.x & 31;
  float4 r = make_float4(0.f, 0.f, 0.f, -1.f);
  if (in) r = __ldcs(rast + pix);
  int t = (int)r.w - 1;
  int i0 = 0, i1 = 0, i2 = 0;
  bool hit = in && t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  if (hit && !tri_verts(tri, t, V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  const int n = (in && !attr_shared) ? view_of(pix, HW) : 0;
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
  const int64_t g = pix * A;  // the pixel's cotangent row in d_out
  const float gl = cot_g(d_out);
  const float* gd = DA ? d_out_da + pix * 2 * K : nullptr;
  float4 db = make_float4(0.f, 0.f, 0.f, 0.f);
  if (DA && hit) db = __ldcs(rast_db + pix);
  float du = 0.0f, dv = 0.0f;
  float d_udx = 0.0f, d_udy = 0.0f, d_vdx = 0.0f, d_vdy = 0.0f;
  for (int a = 0; a < A; a += 4) {
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
    if (hit) {
      float ga[4], x0[4], x1[4], x2[4];
      if (VEC4) {
        const float4 q = cot_at4<true>(d_out, gl, g + a), p0 = ldg4(a0p + a), p1 = ldg4(a1p + a), p2 = ldg4(a2p + a);
        ga[0] = q.x; ga[1] = q.y; ga[2] = q.z; ga[3] = q.w;
        x0[0] = p0.x; x0[1] = p0.y; x0[2] = p0.z; x0[3] = p0.w;
        x1[0] = p1.x; x1[1] = p1.y; x1[2] = p1.z; x1[3] = p1.w;
        x2[0] = p2.x; x2[1] = p2.y; x2[2] = p2.z; x2[3] = p2.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool ok = a + j < A;
          ga[j] = ok ? cot_at<true>(d_out, gl, g + a + j) : 0.f;
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
          const float gx = __ldcs(gd + 2 * (a + j)), gy = __ldcs(gd + 2 * (a + j) + 1);
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
    {
      float cv[12] = {c0[0], c0[1], c0[2], c0[3], c1[0], c1[1], c1[2], c1[3], c2[0], c2[1], c2[2], c2[3]};
      warp_seg_sum_n<12>(cv, lane, seg_end, span);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c0[j] = cv[j];
        c1[j] = cv[4 + j];
        c2[j] = cv[8 + j];
      }
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
    __stcs(d_rast + pix, make_float4(0.f, 0.f, 0.f, 0.f));
    if (DA) __stcs(d_rast_db + pix, make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }
  __stcs(d_rast + pix, make_float4(du, dv, 0.0f, 0.0f));
  if (DA) {
    if (IDX) {
      // .indices: arbitrary (possibly repeated) attribute indices.
      for (int k = 0; k < K; ++k) {
        const int a = idx.k[k];
        const float gx = __ldcs(gd + 2 * k), gy = __ldcs(gd + 2 * k + 1);
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
    __stcs(d_rast_db + pix, make_float4(d_udx, d_udy, d_vdx, d_vdy));
  }
}

}  // namespace

using namespace dr;

namespace {

dr_status interp_bwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A, const float* rast, int N, int H,
                     int W, const int32_t* tri, int T, const float* rast_db, const int32_t* diff_idx, int K,
                     const Cot& d_out, const float* d_out_da, float* d_attr, float* d_rast, float* d_rast_db) {
  DiffIdx idx;
  dr_status st = check_common(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, idx);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, (d_out.d || (d_out.pred && d_out.target && d_out.d_loss)) && d_attr && d_rast &&
                      (K == 0 || (d_out_da && d_rast_db)),
             "interpolate_bwd: d_out (or out, target and d_loss), d_attr, d_rast (and d_out_da, d_rast_db with "
             "diffAttrs) required");
  DR_REQUIRE(ctx, aligned16(d_rast) && (K == 0 || aligned16(d_rast_db)),
             "interpolate_bwd: d_rast / d_rast_db must be 16-byte aligned");
  DR_CUDA(ctx, cudaMemsetAsync(d_attr, 0, sizeof(float) * (size_t)attr_batch * V * A, ctx->stream),
          "interpolate_bwd memset");
  const int64_t P = (int64_t)N * H * W;
  const bool vec = (A % 4 == 0) && aligned16(attr) && aligned16(d_out.d) && aligned16(d_out.pred) &&
                   aligned16(d_out.target) && aligned16(d_attr);
  const bool use_idx = diff_idx != nullptr;
  unsigned grid;
  const PixOrder po = pix_order(ctx, N, H, W, grid);
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* db4 = reinterpret_cast<const float4*>(rast_db);
  float4* dr4 = reinterpret_cast<float4*>(d_rast);
  float4* ddb4 = reinterpret_cast<float4*>(d_rast_db);
  DR_TB(ctx);
  DR_INTERP_DISPATCH(k_interp_bwd, attr, attr_batch == 1, V, A, r4, P, (int64_t)H * W, tri, T, db4, idx, K, d_out,
                     d_out_da, d_attr, dr4, ddb4, po, ctx->d_err);
  DR_LAUNCHED(ctx, "interp_bwd");
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_interpolate_bwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                        const float* rast, int N, int H, int W, const int32_t* tri,
                                        int T, const float* rast_db, const int32_t* diff_idx, int K,
                                        const float* d_out, const float* d_out_da, float* d_attr,
                                        float* d_rast, float* d_rast_db) {
  DR_ENTER(ctx);
  return interp_bwd(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K,
                    Cot{d_out, nullptr, nullptr, 0.0f, nullptr}, d_out_da, d_attr, d_rast, d_rast_db);
}

// VJP of dr_interpolate_fwd_mse: out's cotangent is the fused loss's gradient
// 2 * scale * (out - target) * (*d_loss), formed where it is read; d_out_da
// (NULL when out_da does not reach a loss) is the cotangent of out_da.
extern "C" dr_status dr_interpolate_bwd_mse(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                            const float* rast, int N, int H, int W, const int32_t* tri, int T,
                                            const float* rast_db, const int32_t* diff_idx, int K, const float* out,
                                            const float* target, float scale, const float* d_loss,
                                            const float* d_out_da, float* d_attr, float* d_rast, float* d_rast_db) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, out && target && d_loss, "interpolate_bwd_mse: out, target and d_loss required");
  return interp_bwd(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K,
                    Cot{nullptr, out, target, 2.0f * scale, d_loss}, d_out_da, d_attr, d_rast, d_rast_db);
}
