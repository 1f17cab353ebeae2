// interp.cu — interpolate forward (with the pixel-derivative "DA" path); the
// fused backward is in interp_bwd.cu.
//
// Reference: Sources/MLXDiffRast/Interpolate.swift.  Forward = kernels
// diffrast_interp_fwd / _fwd_da (Interpolate.swift:137-228) in one kernel; the
// four VJP kernels _grad_attr, _grad_attr_da, _grad_rast, _grad_rast_db
// (Interpolate.swift:231-417) are one fused pass here, so rast / attr are read
// once.  attr_batch == 1 (the reference's broadcast of [V,A] / [1,V,A]) reads and
// accumulates one shared attribute table: the reference materialises N copies
// and lets MLX sum their gradients (Interpolate.swift:67-73).
#include "interp_common.cuh"

namespace {

// One pixel.  VEC4: A % 4 == 0 and 16-byte aligned attr/out (and target), so
// the vertex gathers and the output row are float4.  With a target (the fused
// loss) it adds sum((out - target)^2) over the row to lsum.
template <bool VEC4, bool DA, bool IDX>
__device__ __forceinline__ void interp_fwd_pixel(const float* __restrict__ attr, bool attr_shared, int V, int A,
                                                 const float4* __restrict__ rast, int64_t pix, int64_t HW,
                                                 const int32_t* __restrict__ tri, int T,
                                                 const float4* __restrict__ rast_db, const DiffIdx& idx, int K,
                                                 float* __restrict__ out, float* __restrict__ out_da,
                                                 const float* __restrict__ tgt, float& lsum, unsigned* err) {
  const float4 r = __ldcs(rast + pix);
  // rast_db is independent of the triangle gathers: issue it with rast.
  float4 db = make_float4(0.f, 0.f, 0.f, 0.f);
  if (DA) db = __ldcs(rast_db + pix);
  int t = (int)r.w - 1;
  float* o = out + pix * A;
  float* od = DA ? out_da + pix * 2 * K : nullptr;
  const float* tp = tgt ? tgt + pix * A : nullptr;
  int i0, i1, i2;
  bool hit = t >= 0;
  if (hit && t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); hit = false; }
  if (hit && !tri_verts(tri, t, V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  if (!hit) {
    if (VEC4) {
      for (int a = 0; a < A; a += 4) {
        stcs4(o + a, make_float4(0.f, 0.f, 0.f, 0.f));
        if (tp) lsum += sq_diff4(make_float4(0.f, 0.f, 0.f, 0.f), ldcs4(tp + a));
      }
    } else {
      for (int a = 0; a < A; ++a) {
        __stcs(o + a, 0.0f);
        if (tp) { const float d = 0.0f - __ldcs(tp + a); lsum += d * d; }
      }
    }
    if (DA) {
      if (VEC4 && !IDX) {
        for (int k = 0; k < 2 * K; k += 4) stcs4(od + k, make_float4(0.f, 0.f, 0.f, 0.f));
      } else {
        for (int k = 0; k < 2 * K; ++k) __stcs(od + k, 0.0f);
      }
    }
    return;
  }
  const float u = r.x, v = r.y;
  const float bw = 1.0f - u - v;
  const int n = attr_shared ? 0 : view_of(pix, HW);
  const float* an = attr + (attr_shared ? 0 : (int64_t)n * V * A);
  const float* a0p = an + (int64_t)i0 * A;
  const float* a1p = an + (int64_t)i1 * A;
  const float* a2p = an + (int64_t)i2 * A;
  if (VEC4 && DA && !IDX) {
    // .all with A % 4 == 0: out and out_da from the same float4 gathers.
    interp_row4_da(a0p, a1p, a2p, A, bw, u, v, db, o, od, tp, lsum);
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
      stcs4(o + a, y);
      if (tp) lsum += sq_diff4(y, ldcs4(tp + a));
    }
  } else {
    for (int a = 0; a < A; ++a) {
      const float y = bw * __ldg(a0p + a) + u * __ldg(a1p + a) + v * __ldg(a2p + a);
      __stcs(o + a, y);
      if (tp) { const float d = y - __ldcs(tp + a); lsum += d * d; }
    }
  }
  if (DA) {
    for (int k = 0; k < K; ++k) {
      const int a = IDX ? idx.k[k] : k;
      const float x0 = __ldg(a0p + a), x1 = __ldg(a1p + a), x2 = __ldg(a2p + a);
      const float d01 = x1 - x0, d02 = x2 - x0;
      __stcs(od + 2 * k + 0, d01 * db.x + d02 * db.z);
      __stcs(od + 2 * k + 1, d01 * db.y + d02 * db.w);
    }
  }
}

// One thread per pixel; with a fused loss (LOSS) every block adds lscale * its
// sum of squared differences to a partial sum.  The loss is a separate
// instance so the plain forward keeps its register count; both are held to
// four resident blocks per SM (the dependent gathers need the occupancy).
template <bool VEC4, bool DA, bool IDX, bool LOSS>
__global__ void __launch_bounds__(256, 4) k_interp_fwd(const float* __restrict__ attr, bool attr_shared, int V, int A,
                             const float4* __restrict__ rast, int64_t P, int64_t HW,
                             const int32_t* __restrict__ tri, int T,
                             const float4* __restrict__ rast_db, const DiffIdx idx, int K,
                             float* __restrict__ out, float* __restrict__ out_da, const float* __restrict__ tgt,
                             float lscale, float* __restrict__ part, const PixOrder po, unsigned* err) {
  bool in;
  const int64_t pix = pix_of(po, P, in);
  float lsum = 0.0f;
  if (in)
    interp_fwd_pixel<VEC4, DA, IDX>(attr, attr_shared, V, A, rast, pix, HW, tri, T, rast_db, idx, K, out, out_da,
                                    LOSS ? tgt : nullptr, lsum, err);
  if (LOSS) block_loss_add(lsum, lscale, part);
}

template <bool LOSS>
struct InterpFwd {
  template <bool VEC4, bool DA, bool IDX>
  static __host__ void launch(unsigned grid, cudaStream_t s, const float* attr, bool attr_shared, int V, int A,
                              const float4* rast, int64_t P, int64_t HW, const int32_t* tri, int T,
                              const float4* rast_db, const DiffIdx& idx, int K, float* out, float* out_da,
                              const float* tgt, float lscale, float* part, const PixOrder& po, unsigned* err) {
    k_interp_fwd<VEC4, DA, IDX, LOSS><<<grid, 256, 0, s>>>(attr, attr_shared, V, A, rast, P, HW, tri, T, rast_db, idx,
                                                           K, out, out_da, tgt, lscale, part, po, err);
  }
};

// Fused VJP: d_attr, d_rast, d_rast_db in one pass.  Pixels of a warp that hit
// the same triangle (runs along the row) first sum their d_attr contributions
// with warp shuffles, so each run issues one set of atomics instead of one per
// pixel.  Channels go in groups of four (float4 atomics when VEC4).
}  // namespace

using namespace dr;

namespace {

dr_status interp_fwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A, const float* rast, int N, int H,
                     int W, const int32_t* tri, int T, const float* rast_db, const int32_t* diff_idx, int K,
                     float* out, float* out_da, const float* target, float lscale, float* loss) {
  DiffIdx idx;
  dr_status st = check_common(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, idx);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, out && (K == 0 || out_da), "interpolate: out / out_da required");
  const int64_t P = (int64_t)N * H * W;
  const bool vec = (A % 4 == 0) && aligned16(attr) && aligned16(out) && aligned16(target);
  const bool use_idx = diff_idx != nullptr;
  unsigned grid;
  const PixOrder po = pix_order(ctx, N, H, W, grid);
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* db4 = reinterpret_cast<const float4*>(rast_db);
  float* part = nullptr;
  if (target) {
    DR_REQUIRE(ctx, loss, "interpolate_mse: loss required");
    if ((st = loss_begin(ctx, &part)) != DR_OK) return st;
  }
  DR_TB(ctx);
#define DR_IF(VEC4V, DAV, IDXV)                                                                                 \
  do {                                                                                                          \
    if (part)                                                                                                   \
      InterpFwd<true>::launch<VEC4V, DAV, IDXV>(grid, ctx->stream, attr, attr_batch == 1, V, A, r4, P,          \
                                                (int64_t)H * W, tri, T, db4, idx, K, out, out_da, target,       \
                                                lscale, part, po, ctx->d_err);                                  \
    else                                                                                                        \
      InterpFwd<false>::launch<VEC4V, DAV, IDXV>(grid, ctx->stream, attr, attr_batch == 1, V, A, r4, P,         \
                                                 (int64_t)H * W, tri, T, db4, idx, K, out, out_da, nullptr,     \
                                                 0.0f, nullptr, po, ctx->d_err);                                \
  } while (0)
  if (vec) {
    if (K == 0) DR_IF(true, false, false);
    else if (use_idx) DR_IF(true, true, true);
    else DR_IF(true, true, false);
  } else {
    if (K == 0) DR_IF(false, false, false);
    else if (use_idx) DR_IF(false, true, true);
    else DR_IF(false, true, false);
  }
#undef DR_IF
  DR_LAUNCHED(ctx, "interp_fwd");
  if (part) return loss_end(ctx, part, loss);
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_interpolate_fwd(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                        const float* rast, int N, int H, int W, const int32_t* tri,
                                        int T, const float* rast_db, const int32_t* diff_idx, int K,
                                        float* out, float* out_da) {
  DR_ENTER(ctx);
  return interp_fwd(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, out, out_da, nullptr,
                    0.0f, nullptr);
}

// Interpolate with a fused mean-squared-error loss of out against `target`
// ([N, H, W, A]): also writes scale * sum((out - target)^2) to the device
// scalar *loss.  Its VJP is dr_interpolate_bwd_mse.
extern "C" dr_status dr_interpolate_fwd_mse(dr_ctx* ctx, const float* attr, int attr_batch, int V, int A,
                                            const float* rast, int N, int H, int W, const int32_t* tri, int T,
                                            const float* rast_db, const int32_t* diff_idx, int K, float* out,
                                            float* out_da, const float* target, float scale, float* loss) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, target && loss, "interpolate_mse: target and loss required");
  return interp_fwd(ctx, attr, attr_batch, V, A, rast, N, H, W, tri, T, rast_db, diff_idx, K, out, out_da, target,
                    scale, loss);
}

