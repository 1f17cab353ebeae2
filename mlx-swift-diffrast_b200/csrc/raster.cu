// raster.cu — rasterize forward (setup, binning, per-tile fine raster, rast_db,
// depth peeling).  The backward (d_pos) is in raster_bwd.cu.
//
// Reference: Sources/MLXDiffRast/Rasterize.swift.  The reference rasterizes one
// thread per pixel over a capped (128) tile bin list; this implementation is
// triangle-centric inside each 16x16 tile:
//   1. k_raster_setup    one thread per (view, triangle): range / w<=0 reject,
//                        perspective divide, signed area (Rasterize.swift:280-328),
//                        the EXACT pixel rectangle of the NDC AABB test the
//                        reference applies per pixel (Rasterize.swift:426-433),
//                        and a count per touched tile.
//   2. scan               exclusive scan of the per-tile counts (no cap, no drop).
//   3. k_raster_scatter   per-tile candidate lists (order irrelevant, see 4).
//   4. k_raster_tiles     one CTA per (view, tile): every candidate visits the
//                        pixels of its rectangle inside the tile, runs the
//                        reference's edge / inside / z / peel tests with the same
//                        IEEE operations, and folds (z, tri) into a per-pixel
//                        64-bit shared-memory atomicMin.  The minimum of the
//                        packed key is the lexicographic minimum of (z, tri) — the
//                        winner the reference's ascending strict-< loop picks — so
//                        the result does not depend on list order.  The winner's
//                        (u, v, z) and rast_db are then recomputed bit-identically.
// All coverage-critical arithmetic uses explicit round-to-nearest intrinsics
// (never contracted into FMA), so tri_id, u, v and z match the CPU oracle bit for
// bit.
#include <algorithm>

#include "common.cuh"
#include "interp_common.cuh"

namespace {

constexpr int TILE = 16;
constexpr int TILE_PIX = TILE * TILE;

#define FM(a, b) __fmul_rn((a), (b))
#define FA(a, b) __fadd_rn((a), (b))
#define FS(a, b) __fsub_rn((a), (b))
#define FD(a, b) __fdiv_rn((a), (b))

// a / d for the image sizes d of the NDC conversions.  For a power of two
// d = 2^k the quotient is a * 2^-k exactly (a >= 1 here, so no underflow),
// which saves the IEEE division; otherwise the division itself.
__device__ __forceinline__ float div_by_size(float a, int d) {
  if ((d & (d - 1)) == 0) return FM(a, __int_as_float((127 - (__ffs(d) - 1)) << 23));
  return FD(a, (float)d);
}

// Pixel-centre NDC exactly as Rasterize.swift:381-382 computes it.
__device__ __forceinline__ float ndc_x_of(int pw, int W) {
  return FS(div_by_size(FM(2.0f, FA((float)pw, 0.5f)), W), 1.0f);
}
__device__ __forceinline__ float ndc_y_of(int ph, int H) {
  return FS(1.0f, div_by_size(FM(2.0f, FA((float)ph, 0.5f)), H));
}

// Setup record: 48 bytes.
//   r0 = (sx0, sy0, sz0, sx1)   r1 = (sy1, sz1, sx2, sy2)
//   r2 = (sz2, area, bits(x0 | x1 << 16), bits(y0 | y1 << 16))
// area == 0 marks a triangle that can cover no pixel.
struct Rec {
  float sx0, sy0, sz0, sx1, sy1, sz1, sx2, sy2, sz2, area;
  int x0, x1, y0, y1;
};

__device__ __forceinline__ Rec load_rec(const float4* __restrict__ rec, int64_t i) {
  float4 a = __ldg(rec + 3 * i + 0), b = __ldg(rec + 3 * i + 1), c = __ldg(rec + 3 * i + 2);
  Rec r;
  r.sx0 = a.x; r.sy0 = a.y; r.sz0 = a.z; r.sx1 = a.w;
  r.sy1 = b.x; r.sz1 = b.y; r.sx2 = b.z; r.sy2 = b.w;
  r.sz2 = c.x; r.area = c.y;
  unsigned xs = __float_as_uint(c.z), ys = __float_as_uint(c.w);
  r.x0 = (int)(xs & 0xffffu); r.x1 = (int)(xs >> 16);
  r.y0 = (int)(ys & 0xffffu); r.y1 = (int)(ys >> 16);
  return r;
}

__device__ __forceinline__ float clampf_safe(float x, float lo, float hi) {
  return fminf(fmaxf(x, lo), hi);  // NaN never reaches here (records are finite)
}

// Smallest / largest pixel column whose centre NDC lies in [minx, maxx].  The
// float estimate is refined against the exact ndc_x_of, which is monotone in pw.
__device__ void exact_cols(float minx, float maxx, int W, int& lo, int& hi) {
  float fl = clampf_safe((minx + 1.0f) * 0.5f * (float)W - 0.5f, -2.0f, (float)W + 1.0f);
  float fh = clampf_safe((maxx + 1.0f) * 0.5f * (float)W - 0.5f, -2.0f, (float)W + 1.0f);
  lo = min(max((int)floorf(fl), 0), W);
  while (lo > 0 && ndc_x_of(lo - 1, W) >= minx) --lo;
  while (lo < W && ndc_x_of(lo, W) < minx) ++lo;
  hi = min(max((int)ceilf(fh), -1), W - 1);
  while (hi < W - 1 && ndc_x_of(hi + 1, W) <= maxx) ++hi;
  while (hi >= 0 && ndc_x_of(hi, W) > maxx) --hi;
}

// Rows whose centre NDC y lies in [miny, maxy] (ndc_y_of decreases with ph).
__device__ void exact_rows(float miny, float maxy, int H, int& lo, int& hi) {
  float gl = clampf_safe((1.0f - maxy) * 0.5f * (float)H - 0.5f, -2.0f, (float)H + 1.0f);
  float gh = clampf_safe((1.0f - miny) * 0.5f * (float)H - 0.5f, -2.0f, (float)H + 1.0f);
  lo = min(max((int)floorf(gl), 0), H);
  while (lo > 0 && ndc_y_of(lo - 1, H) <= maxy) --lo;
  while (lo < H && ndc_y_of(lo, H) > maxy) ++lo;
  hi = min(max((int)ceilf(gh), -1), H - 1);
  while (hi < H - 1 && ndc_y_of(hi + 1, H) >= miny) ++hi;
  while (hi >= 0 && ndc_y_of(hi, H) < miny) --hi;
}

__device__ __forceinline__ bool finite3(float a, float b, float c) {
  return isfinite(a) && isfinite(b) && isfinite(c);
}

// Setup of triangle t in view n: writes its record and returns its exact pixel
// rectangle, or false (record zeroed) when it can cover no pixel.
__device__ __forceinline__ bool setup_one(const float* __restrict__ pos, const float* __restrict__ xform, int V,
                                          const int32_t* __restrict__ tri, int T,
                                          const int32_t* __restrict__ ranges, int H, int W, int n, int t,
                                          float4* __restrict__ out, int& x0, int& x1, int& y0, int& y1,
                                          unsigned* err) {
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok = true;
  int64_t pos_n_base = 0;
  if (ranges) {
    int rs = __ldg(ranges + 2 * n), rc = __ldg(ranges + 2 * n + 1);
    ok = !(t < rs || t >= rs + rc);
  } else if (!xform) {
    pos_n_base = (int64_t)n * V * 4;
  }
  int i0 = 0, i1 = 0, i2 = 0;
  if (ok) {
    i0 = __ldg(tri + 3 * t); i1 = __ldg(tri + 3 * t + 1); i2 = __ldg(tri + 3 * t + 2);
    if (i0 < 0 || i0 >= V || i1 < 0 || i1 >= V || i2 < 0 || i2 >= V) {
      dr_flag(err, DR_DEVERR_VERTEX);
      ok = false;
    }
  }
  float4 p0, p1, p2;
  if (ok) {
    p0 = ldg4(pos + pos_n_base + (int64_t)i0 * 4);
    p1 = ldg4(pos + pos_n_base + (int64_t)i1 * 4);
    p2 = ldg4(pos + pos_n_base + (int64_t)i2 * 4);
    if (xform) {
      const Mat4 M = load_mat4(xform + (int64_t)n * 16);
      p0 = mat4_apply(M, p0);
      p1 = mat4_apply(M, p1);
      p2 = mat4_apply(M, p2);
    }
    ok = !(p0.w <= 0.0f || p1.w <= 0.0f || p2.w <= 0.0f);
  }
  if (!ok) {
    out[0] = zero; out[1] = zero; out[2] = zero;
    return false;
  }
  float sx0 = FD(p0.x, p0.w), sy0 = FD(p0.y, p0.w), sz0 = FD(p0.z, p0.w);
  float sx1 = FD(p1.x, p1.w), sy1 = FD(p1.y, p1.w), sz1 = FD(p1.z, p1.w);
  float sx2 = FD(p2.x, p2.w), sy2 = FD(p2.y, p2.w), sz2 = FD(p2.z, p2.w);
  float area = FS(FM(FS(sx1, sx0), FS(sy2, sy0)), FM(FS(sx2, sx0), FS(sy1, sy0)));
  // |area| < 2^-128 (finite, non-zero) has 1/area = inf: every pixel test of
  // the record yields an infinite or NaN depth, which is never a fragment, so
  // the record is invalid (the oracle's setup applies the same rule).
  ok = finite3(sx0, sy0, sz0) && finite3(sx1, sy1, sz1) && finite3(sx2, sy2, sz2) &&
       isfinite(area) && area != 0.0f && isfinite(__frcp_rn(area));
  x0 = 0; x1 = -1; y0 = 0; y1 = -1;
  if (ok) {
    float minx = fminf(sx0, fminf(sx1, sx2)), maxx = fmaxf(sx0, fmaxf(sx1, sx2));
    float miny = fminf(sy0, fminf(sy1, sy2)), maxy = fmaxf(sy0, fmaxf(sy1, sy2));
    exact_cols(minx, maxx, W, x0, x1);
    exact_rows(miny, maxy, H, y0, y1);
    ok = (x0 <= x1) && (y0 <= y1);
  }
  if (!ok) {
    out[0] = zero; out[1] = zero; out[2] = zero;
    return false;
  }
  out[0] = make_float4(sx0, sy0, sz0, sx1);
  out[1] = make_float4(sy1, sz1, sx2, sy2);
  out[2] = make_float4(sz2, area, __uint_as_float((unsigned)x0 | ((unsigned)x1 << 16)),
                       __uint_as_float((unsigned)y0 | ((unsigned)y1 << 16)));
  return true;
}

// Binned setup: CTA (c, n) owns triangles [c*chunk, (c+1)*chunk) of view n and
// counts their tiles in a shared-memory histogram of the view's tiles, then
// writes the histogram to cnt[(n*ntiles + tile)*cpv + c].  The exclusive scan
// of cnt (tile-major, chunk-minor) gives every (tile, chunk) its list segment,
// so neither this kernel nor the scatter issues a global atomic.  Each
// triangle's pixel rectangle also goes to box[n*T + t] (the record's last two
// words, kInvalidBox for a record that covers nothing): the scatter reads
// those 8 bytes instead of a 32-byte sector of the record.
constexpr unsigned kInvalidBox = 0xFFFFFFFFu;

__global__ void __launch_bounds__(256)
k_raster_setup_binned(const float* __restrict__ pos, const float* __restrict__ xform, int V,
                      const int32_t* __restrict__ tri, int T, const int32_t* __restrict__ ranges, int H, int W,
                      int ntx, int nty, int chunk, int cpv, float4* __restrict__ rec, uint2* __restrict__ box,
                      uint32_t* __restrict__ cnt, unsigned* err) {
  extern __shared__ uint32_t s_hist[];
  const int c = blockIdx.x, n = blockIdx.y;
  const int ntiles = ntx * nty;
  for (int i = threadIdx.x; i < ntiles; i += blockDim.x) s_hist[i] = 0u;
  __syncthreads();
  const int t0 = c * chunk, t1 = min(T, t0 + chunk);
  for (int t = t0 + (int)threadIdx.x; t < t1; t += blockDim.x) {
    int x0, x1, y0, y1;
    if (!setup_one(pos, xform, V, tri, T, ranges, H, W, n, t, rec + 3 * ((int64_t)n * T + t), x0, x1, y0, y1,
                   err)) {
      box[(int64_t)n * T + t] = make_uint2(kInvalidBox, kInvalidBox);
      continue;
    }
    box[(int64_t)n * T + t] = make_uint2((unsigned)x0 | ((unsigned)x1 << 16), (unsigned)y0 | ((unsigned)y1 << 16));
    for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty)
      for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) atomicAdd(&s_hist[ty * ntx + tx], 1u);
  }
  __syncthreads();
  uint32_t* col = cnt + (int64_t)n * ntiles * cpv + c;
  for (int i = threadIdx.x; i < ntiles; i += blockDim.x) col[(int64_t)i * cpv] = s_hist[i];
}

// Binned scatter: CTA k walks the (view, chunk) pairs [k*per, (k+1)*per) of
// the setup's map (view-major) one after the other; each pair's (tile, chunk)
// segment starts come from the scan, and slots within them from shared
// atomics.  One wave of large CTAs keeps few pairs in flight: every pair
// appends to all of its view's tiles at once, and the partly written list
// sectors of all pairs in flight must stay in L2 until they fill (with one
// pair per 256-thread CTA they did not: about 1 GB of write-backs re-read).
constexpr int kScatterBlock = 1024;

__global__ void __launch_bounds__(kScatterBlock)
k_raster_scatter_binned(const uint2* __restrict__ box, int N, int T, int ntx, int nty, int chunk, int cpv, int per,
                        const uint32_t* __restrict__ off, int32_t* __restrict__ list, uint32_t cap) {
  extern __shared__ uint32_t s_base[];
  const int ntiles = ntx * nty;
  const int64_t pairs = (int64_t)N * cpv;
  for (int64_t q = (int64_t)blockIdx.x * per, qe = min(pairs, q + per); q < qe; ++q) {
    const int n = (int)(q / cpv), c = (int)(q - (int64_t)n * cpv);
    const uint32_t* col = off + (int64_t)n * ntiles * cpv + c;
    __syncthreads();  // the previous pair's appends are done with s_base
    for (int i = threadIdx.x; i < ntiles; i += blockDim.x) s_base[i] = __ldg(col + (int64_t)i * cpv);
    __syncthreads();
    const int t0 = c * chunk, t1 = min(T, t0 + chunk);
    // Four rectangles per thread per round, loaded before any is used, so
    // four independent loads are in flight.
    constexpr int R = 4;
    const uint2* bv = box + (int64_t)n * T;
    for (int tb = t0 + (int)threadIdx.x; tb < t1; tb += R * blockDim.x) {
      uint2 r2[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const int t = tb + k * (int)blockDim.x;
        r2[k] = t < t1 ? __ldcs(bv + t) : make_uint2(kInvalidBox, kInvalidBox);
      }
#pragma unroll
      for (int k = 0; k < R; ++k) {
        if (r2[k].x == kInvalidBox) continue;  // covers no pixel (or past the chunk)
        const int t = tb + k * (int)blockDim.x;
        const unsigned xs = r2[k].x, ys = r2[k].y;
        const int x0 = (int)(xs & 0xffffu), x1 = (int)(xs >> 16), y0 = (int)(ys & 0xffffu), y1 = (int)(ys >> 16);
        for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty)
          for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) {
            const uint32_t slot = atomicAdd(&s_base[ty * ntx + tx], 1u);
            if (slot < cap) list[slot] = t;  // past a fixed capacity: the tile scans instead
          }
      }
    }
  }
}

// Unbinned setup (views with more tiles than a shared histogram holds): one
// thread per (view, triangle), global atomics on the per-tile counts.
__global__ void k_raster_setup(const float* __restrict__ pos, const float* __restrict__ xform, int V,
                               const int32_t* __restrict__ tri,
                               int T, const int32_t* __restrict__ ranges, int N, int H, int W,
                               int ntx, int nty, float4* __restrict__ rec,
                               uint32_t* __restrict__ tile_count, unsigned* err) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)N * T) return;
  int t = (int)(idx % T);
  int n = (int)(idx / T);
  int x0, x1, y0, y1;
  if (!setup_one(pos, xform, V, tri, T, ranges, H, W, n, t, rec + 3 * idx, x0, x1, y0, y1, err)) return;
  uint32_t* tc = tile_count + (int64_t)n * ntx * nty;
  for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty)
    for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) atomicAdd(tc + ty * ntx + tx, 1u);
}

// Scatter every valid (view, triangle) into the lists of the tiles it touches.
// tile_cur starts as the exclusive offsets; atomicAdd hands out list slots.
__global__ void k_raster_scatter(const float4* __restrict__ rec, int N, int T, int ntx, int nty,
                                 uint32_t* __restrict__ tile_cur, int32_t* __restrict__ list, uint32_t cap) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)N * T) return;
  float4 c = __ldg(rec + 3 * idx + 2);
  if (c.y == 0.0f) return;  // area == 0: invalid
  int t = (int)(idx % T);
  int n = (int)(idx / T);
  unsigned xs = __float_as_uint(c.z), ys = __float_as_uint(c.w);
  int x0 = (int)(xs & 0xffffu), x1 = (int)(xs >> 16), y0 = (int)(ys & 0xffffu), y1 = (int)(ys >> 16);
  uint32_t* tc = tile_cur + (int64_t)n * ntx * nty;
  for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty)
    for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) {
      uint32_t slot = atomicAdd(tc + ty * ntx + tx, 1u);
      if (slot < cap) list[slot] = t;
    }
}

// Total order on (z, tri): z mapped to an order-preserving uint32 in the high
// word (-0 canonicalised to +0, which compares equal to it), tri in the low word.
__device__ __forceinline__ unsigned long long pack_key(float z, int t) {
  unsigned u = __float_as_uint(FA(z, 0.0f));
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)t;
}

// Two depth layers in one candidate pass.  Per pixel, k0 = the minimum key of
// all fragments and k1 = the minimum key among those whose z is strictly
// greater than z(k0) — exactly what a second pass peeling at layer 0's depth
// selects (Rasterize.swift:465-470: z <= peel_z is rejected).  Both are
// maintained with 64-bit atomicMin only: a fragment f exchanges with k0
// (old = atomicMin(k0, f)); of f and old, the larger key lost, and it is
// offered to k1 when its z is strictly greater than the winner's.
//   Every offered key is eligible (its z exceeds a k0 that can only fall).
//   The smallest eligible key m is offered: if m lost its own exchange, the
//   winner has a smaller key, hence (m being the smallest eligible) a smaller
//   z, so m was offered; if m won, a later fragment with z <= z(k0 final) <
//   z(m) displaced it and offered it.  A loser whose z ties the winner's is
//   dropped safely: the winner has the same z and a smaller key.
// Since k1 > k0 always, a fragment with key >= k1 changes neither: one 64-bit
// read of k1 filters almost every fragment.
__device__ __forceinline__ void fold_two(unsigned long long* k0, unsigned long long* k1,
                                         unsigned long long key) {
  const unsigned long long old = atomicMin(k0, key);
  const unsigned long long win = key < old ? key : old, lose = key < old ? old : key;
  if (lose != ~0ull && (lose >> 32) > (win >> 32)) atomicMin(k1, lose);
}

// What write_pixel wrote: the winner (hit, triangle), its (u, v) and rast_db.
struct PixOut {
  bool hit;
  int t;
  float u, v;
  float4 db;
};

// Recompute the winner's (u, v, z) and rast_db bit-identically from its record
// and write one output pixel (zeros where the key is empty).
// k_x = 2 / W and k_y = -2 / H (IEEE divisions, computed once per thread).
template <bool DB>
__device__ __forceinline__ PixOut write_pixel(const float4* __restrict__ rec, int64_t rec_view,
                                              unsigned long long key, float x, float y, float k_x, float k_y,
                                              float4* __restrict__ rast, float4* __restrict__ rast_db,
                                              int64_t pix) {
  PixOut po;
  po.hit = false;
  po.t = -1;
  po.u = po.v = 0.0f;
  po.db = make_float4(0.f, 0.f, 0.f, 0.f);
  if (key == ~0ull) {
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    rast[pix] = z4;
    if (DB) rast_db[pix] = z4;
    return po;
  }
  const int t = (int)(unsigned)(key & 0xffffffffull);
  const Rec r = load_rec(rec, rec_view + t);
  const float inv_area = __frcp_rn(r.area);  // correctly rounded: the same value as 1.0f / area
  const float dx0 = FS(r.sx0, x), dx1 = FS(r.sx1, x), dx2 = FS(r.sx2, x);
  const float dy0 = FS(r.sy0, y), dy1 = FS(r.sy1, y), dy2 = FS(r.sy2, y);
  const float e0 = FS(FM(dx1, dy2), FM(dx2, dy1));
  const float e1 = FS(FM(dx2, dy0), FM(dx0, dy2));
  const float e2 = FS(FM(dx0, dy1), FM(dx1, dy0));
  const float bw = FM(e0, inv_area), u = FM(e1, inv_area), v = FM(e2, inv_area);
  const float z = FA(FA(FM(bw, r.sz0), FM(u, r.sz1)), FM(v, r.sz2));
  rast[pix] = make_float4(u, v, z, (float)(t + 1));
  po.hit = true;
  po.t = t;
  po.u = u;
  po.v = v;
  if (DB) {
    // Rasterize.swift:586-598
    po.db = make_float4(FM(FM(FS(r.sy2, r.sy0), inv_area), k_x), FM(FM(FS(r.sx0, r.sx2), inv_area), k_y),
                        FM(FM(FS(r.sy0, r.sy1), inv_area), k_x), FM(FM(FS(r.sx1, r.sx0), inv_area), k_y));
    rast_db[pix] = po.db;
  }
  return po;
}

// Interpolation fused into the two-layer pass (dr_rasterize_xf_interp_fwd):
// per layer, interpolate's out / out_da (.all, A % 4 == 0) and, with a
// target, its mean-squared-error loss, computed from the winner the pass
// has just written instead of by a second kernel that reads rast back.
struct InterpEpi {
  const float* attr;  // [attr_batch, V, A]
  int attr_shared;    // attr_batch == 1
  int V, A;
  const int32_t* tri;
  float* out[2];
  float* out_da[2];
  const float* tgt[2];  // or nullptr
  float lscale[2];
  float* part[2];  // loss partial sums, or nullptr
};

__device__ __forceinline__ void epi_pixel(const InterpEpi& e, int l, const PixOut& p, int64_t pix, int n,
                                          float& lsum, unsigned* err) {
  float* o = e.out[l] + pix * e.A;
  float* od = e.out_da[l] + pix * 2 * e.A;
  const float* tp = e.tgt[l] ? e.tgt[l] + pix * e.A : nullptr;
  int i0, i1, i2;
  bool hit = p.hit;
  if (hit && !tri_verts(e.tri, p.t, e.V, i0, i1, i2)) { dr_flag(err, DR_DEVERR_VERTEX); hit = false; }
  if (!hit) {
    interp_row4_da_miss(e.A, o, od, tp, lsum);
    return;
  }
  // The interpolate forward's arithmetic on the rast it would read back.
  const float bw = 1.0f - p.u - p.v;
  const float* an = e.attr + (e.attr_shared ? 0 : (int64_t)n * e.V * e.A);
  interp_row4_da<1>(an + (int64_t)i0 * e.A, an + (int64_t)i1 * e.A, an + (int64_t)i2 * e.A, e.A, bw, p.u, p.v,
                    p.db, o, od, tp, lsum);
}

// Conservative column spans of one candidate, per tile row.
//
// The exact pixel test (inclusive edges, Rasterize.swift:442-447) stays the
// only authority on coverage; a span only drops pixels it provably rejects,
// so results are bit-identical, and about half of the pixels of a small
// triangle's rectangle are never tested (cfg4: 36.5 M -> 16.7 M tests per
// view for 16.65 M covered pixels).
//
// Edge i runs from a = vertex i+1 to b = vertex i+2; its exact edge function
// at a pixel centre p, e(p) = (a_x - p_x)(b_y - p_y) - (b_x - p_x)(a_y - p_y),
// is affine in p_x with slope g = a_y - b_y, and zero at the root
// x*(y) = a_x + (b_x - a_x)(y - a_y) / (b_y - a_y).  For pixels inside the
// candidate's bounding box (|p - vertex| <= Wb, Hb per axis), the float
// evaluation ê of the test differs from e by at most
//   D = 8u Wb Hb + 2^-149 (1 + 1/|area|)      (u = 2^-24)
// (three roundings of the products, one of the difference, subnormal
// products, and an e * area product that underflows to -0 and passes).  A
// pixel that passes has sign(area) * ê >= 0, so sign(area) * g (p_x - x*) >=
// -D: p_x >= x* - D/|g| when sign(area) g > 0 (a lower bound), else p_x <=
// x* + D/|g| (an upper bound).  The root is evaluated as fma(B, y, A) with
// B = (b_x - a_x) / (b_y - a_y) and A = a_x - B a_y; its error, that of
// folding the margin into A, of the pixel centres' own NDC rounding and of
// the conversion to a column index stay below
//   u (10|a_x| + 2|B||a_y| + 9|B| Hb + 42) + 4u Wb Hb / |g|.
// The margin used is twice the sum of both bounds; an edge with g = 0, a
// non-finite B or A, or a margin of 8 or more constrains nothing.  (Checked on
// the CPU against the exact test on full cfg4 views and on adversarial
// slivers, axis-aligned and near-degenerate edges, sub-pixel and huge
// triangles at several resolutions: no accepted pixel outside its span.)
//
// Every triangle has at most two lower-bound and two upper-bound edges (the
// exact slopes g of its three edges sum to zero and a correctly rounded
// difference keeps its sign), so each row's span is
//   [max of the two lower roots, min of the two upper roots],
// unused slots holding (B, A) = (0, -inf) or (0, +inf).
// Writes one byte per tile row of [ly0, ly1] with a non-empty span (first
// column | last column << 4, tile-local), returns the number of pixels and
// sets n_rows to the number of non-empty rows.
__device__ __forceinline__ int stage_spans(const float4& f0, const float4& f1, float area, float inv_area,
                                           int lx0, int lx1, int ly0, int ly1, int tx0, int W,
                                           const float* __restrict__ s_ndcy, unsigned char* __restrict__ span,
                                           int& n_rows) {
  constexpr float kU = 5.9604645e-08f;     // 2^-24
  constexpr float kTiny = 1.4012985e-45f;  // 2^-149
  const float sx[3] = {f0.x, f0.w, f1.z}, sy[3] = {f0.y, f1.x, f1.w};
  const float Wb = FS(fmaxf(sx[0], fmaxf(sx[1], sx[2])), fminf(sx[0], fminf(sx[1], sx[2])));
  const float Hb = FS(fmaxf(sy[0], fmaxf(sy[1], sy[2])), fminf(sy[0], fminf(sy[1], sy[2])));
  const float dnum = FA(FM(12.1f * kU, FM(Wb, Hb)), FM(kTiny, FA(1.0f, fabsf(inv_area))));
  float lb0 = 0.0f, la0 = -INFINITY, lb1 = 0.0f, la1 = -INFINITY;
  float hb0 = 0.0f, ha0 = INFINITY, hb1 = 0.0f, ha1 = INFINITY;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int ia = (i + 1) % 3, ib = (i + 2) % 3;
    const float ax = sx[ia], ay = sy[ia], bx = sx[ib], by = sy[ib];
    const float g = FS(ay, by);
    const float inv = __frcp_rn(FS(by, ay));
    const float B = FM(FS(bx, ax), inv);
    const float A = FS(ax, FM(B, ay));
    const float aB = fabsf(B);
    const float m = FM(2.0f, FA(FM(dnum, fabsf(inv)),
                                FM(kU, FA(FA(FA(FM(10.0f, fabsf(ax)), FM(FM(2.0f, aB), fabsf(ay))),
                                             FM(FM(9.0f, aB), Hb)), 42.0f))));
    if (g != 0.0f && isfinite(B) && isfinite(A) && m < 8.0f) {
      if ((area > 0.0f) == (g > 0.0f)) {  // a lower bound on the column
        const float a = FS(A, m);
        if (la0 == -INFINITY) { lb0 = B; la0 = a; } else { lb1 = B; la1 = a; }
      } else {
        const float a = FA(A, m);
        if (ha0 == INFINITY) { hb0 = B; ha0 = a; } else { hb1 = B; ha1 = a; }
      }
    }
  }
  const float half = (float)W * 0.5f;  // exact: W <= 32768
  const float off = half - 0.5f;
  const float clo_min = (float)(lx0 + tx0), chi_max = (float)(lx1 + tx0);
  int n = 0, rows = 0;
  for (int ly = ly0; ly <= ly1; ++ly) {
    const float y = s_ndcy[ly];
    const float lo = fmaxf(__fmaf_rn(lb0, y, la0), __fmaf_rn(lb1, y, la1));
    const float hi = fminf(__fmaf_rn(hb0, y, ha0), __fmaf_rn(hb1, y, ha1));
    const float cl = fmaxf(ceilf(__fmaf_rn(lo, half, off)), clo_min);
    const float ch = fminf(floorf(__fmaf_rn(hi, half, off)), chi_max);
    // Branch-free: an empty row keeps the empty code 0x0F (first column 15,
    // last 0).  cl and ch lie in [clo_min, chi_max] whenever cl <= ch.
    const bool on = cl <= ch;
    const int c0 = (int)cl - tx0, c1 = (int)ch - tx0;
    span[ly] = on ? (unsigned char)(c0 | (c1 << 4)) : (unsigned char)0x0F;
    n += on ? c1 - c0 + 1 : 0;
    rows += on ? 1 : 0;
  }
  n_rows = rows;
  return n;
}

// Per-tile fine raster.  The CTA stages up to 256 candidates at a time (one per
// thread): each thread loads its candidate's record, computes its per-row
// column spans inside the tile (stage_spans) and counts its pixels and
// non-empty rows.  One block scan of both counts gives every non-empty
// (candidate, row) span its slot in a shared list of spans and the index of
// its first pixel in the batch's item space, so the list is ordered by item
// and its start indices increase strictly.  Each warp then takes a contiguous
// range of items, 32 consecutive items per step, one per lane: a lane finds
// the span holding its item by counting the span starts among the next 32
// that do not exceed it (one shared load, an OR-reduction of one bit per
// start, a population count), so the walk has no per-lane loop.  Work is
// balanced to within one step per warp whatever the triangle sizes.
// MODE: 0 = one layer, 1 = one layer peeled at `peel`, 2 = layers 0 and 1 at once.
constexpr int WARPS = TILE_PIX / 32;
// A batch stages at most 255 candidates, so its items (at most 255 * 256)
// and span starts fit 16 bits with 0xFFFF left free as the end sentinel.
constexpr int BATCH = TILE_PIX - 1;
constexpr int MAX_SPANS = BATCH * TILE;  // every staged candidate non-empty on every row
constexpr unsigned short kNoStart = 0xFFFF;

// CAPPED: the list buffer holds `cap` entries (fixed capacity, no readback);
// a tile whose list runs past it stages every triangle of its view instead,
// giving those without pixels in the tile no work items.
// Five resident CTAs per SM: 48 registers (the hot instances do not spill)
// and about 44 KB of shared memory each; four with the interpolation
// epilogue, whose gathers need the registers.
// EPI (two layers with rast_db only): the interpolation epilogue (InterpEpi).
template <int MODE, bool DB, bool CAPPED, bool EPI = false>
__global__ void __launch_bounds__(TILE_PIX, EPI ? 4 : 5)
k_raster_tiles(const float4* __restrict__ rec, int T, int H, int W, int ntx, int nty,
               const uint32_t* __restrict__ tile_off, int off_stride,
               const int32_t* __restrict__ list, const float* __restrict__ peel,
               float4* __restrict__ rast, float4* __restrict__ rast_db,
               float4* __restrict__ rast1, float4* __restrict__ rast_db1, unsigned* err,
               uint32_t cap, unsigned* overflow, const InterpEpi epi) {
  static_assert(!EPI || (MODE == 2 && DB), "the interpolation epilogue runs on the two-layer pass with rast_db");
  constexpr bool PEEL = MODE == 1, TWO = MODE == 2;
  __shared__ unsigned long long s_k0[TILE_PIX], s_k1[TWO ? TILE_PIX : 1];
  __shared__ float s_peel[PEEL ? TILE_PIX : 1];
  __shared__ float s_ndcx[TILE], s_ndcy[TILE];
  __shared__ float4 s_rec[TILE_PIX * 3];        // staged records, by staging thread
  __shared__ uint4 s_rowspan[TILE_PIX];         // per staging thread: one span byte per tile row
  __shared__ unsigned short s_start[MAX_SPANS + 33];  // first item of each span (+ 33 entries past the last)
  // Staging thread | row << 8 | (first column - first item) << 12 (signed):
  // an item's column is its index plus the high bits, with no second load.
  __shared__ int s_info[MAX_SPANS];
  __shared__ int s_wsum[WARPS];

  const int ntiles = ntx * nty;
  const int n = blockIdx.x / ntiles;
  const int tile = blockIdx.x - n * ntiles;
  const int tx0 = (tile % ntx) * TILE, ty0 = (tile / ntx) * TILE;
  const int tid = threadIdx.x;
  const int px = tx0 + (tid & (TILE - 1)), py = ty0 + (tid >> 4);
  const bool inside_img = (px < W) && (py < H);
  const int64_t pix = ((int64_t)n * H + py) * W + px;

  s_k0[tid] = ~0ull;
  if (TWO) s_k1[tid] = ~0ull;
  if (PEEL) {
    float pz = -1e30f;
    if (inside_img) {
      float4 pl = ldg4(peel + 4 * pix);
      if (pl.w > 0.0f) pz = pl.z;
    }
    s_peel[tid] = pz;
  }
  if (tid < TILE) s_ndcx[tid] = ndc_x_of(tx0 + tid, W);
  else if (tid < 2 * TILE) s_ndcy[tid - TILE] = ndc_y_of(ty0 + tid - TILE, H);

  const uint32_t gt = (uint32_t)blockIdx.x;
  const uint32_t begin = __ldg(tile_off + (int64_t)gt * off_stride);
  const uint32_t end = __ldg(tile_off + (int64_t)(gt + 1) * off_stride);
  bool scan_all = false;  // CAPPED only: the tile's list did not fit
  if (CAPPED && end > cap) {
    scan_all = true;
    if (tid == 0) atomicAdd(overflow, 1u);
  }
  const uint32_t cnt = scan_all ? (uint32_t)T : end - begin;
  const int64_t rec_view = (int64_t)n * T;
  const int warp = tid >> 5, lane = tid & 31;

  // One pixel test (Rasterize.swift:426-470) of the staged candidate: true
  // when the fragment may lower the pixel's key(s), with its key and pixel.
  // f0 = (sx0, sy0, sz0, sx1), f1 = (sy1, sz1, sx2, sy2), f2 = (sz2, area, 1/area, t)
  auto test = [&](const float4& f0, const float4& f1, const float4& f2, int lx, int ly,
                  unsigned long long& key, int& p) -> bool {
    const float x = s_ndcx[lx], y = s_ndcy[ly];
    const float dx0 = FS(f0.x, x), dx1 = FS(f0.w, x), dx2 = FS(f1.z, x);
    const float dy0 = FS(f0.y, y), dy1 = FS(f1.x, y), dy2 = FS(f1.w, y);
    const float e0 = FS(FM(dx1, dy2), FM(dx2, dy1));
    const float e1 = FS(FM(dx2, dy0), FM(dx0, dy2));
    const float e2 = FS(FM(dx0, dy1), FM(dx1, dy0));
    const float area = f2.y;
    // Straight-line code: nearly every tested item covers its pixel (the
    // spans leave few misses), so the barycentrics and depth are computed
    // for all and the conditions combined into one predicate.
    const float bw = FM(e0, f2.z), u = FM(e1, f2.z), v = FM(e2, f2.z);
    const float z = FA(FA(FM(bw, f0.z), FM(u, f1.y)), FM(v, f2.x));
    // A NaN depth is never a fragment.  The reference stores one (every
    // comparison it makes is false) and lets the next candidate in its bin
    // order replace it; rejecting it keeps the winner independent of order,
    // and the oracle applies the same rule.
    p = ly * TILE + lx;
    bool ok = !(FM(e0, area) < 0.0f) & !(FM(e1, area) < 0.0f) & !(FM(e2, area) < 0.0f) & (z >= -1.0f) &
              (z <= 1.0f);
    if (PEEL) ok &= !(z <= s_peel[p]);
    key = pack_key(z, __float_as_int(f2.w));
    return ok & (TWO ? key < s_k1[p] : key < s_k0[p]);
  };
  // The test's read of the key is the filter; the atomics are correct for
  // any key, so a key lowered by another thread in between costs nothing.
  auto fold = [&](unsigned long long key, int p) {
    if (TWO) fold_two(&s_k0[p], &s_k1[p], key);
    else atomicMin(&s_k0[p], key);
  };
  for (uint32_t base = 0; base < cnt; base += BATCH) {
    __syncthreads();  // the previous batch's readers are done with the stage
    const uint32_t i = base + tid;
    int n_items = 0, n_rows = 0, ly0 = 0, ly1 = -1;
    unsigned char* span = reinterpret_cast<unsigned char*>(&s_rowspan[tid]);
    if (tid < BATCH && i < cnt) {
      const int t = scan_all ? (int)i : __ldg(list + begin + i);
      const float4 a = __ldg(rec + 3 * (rec_view + t) + 0);
      const float4 bb = __ldg(rec + 3 * (rec_view + t) + 1);
      const float4 c = __ldg(rec + 3 * (rec_view + t) + 2);
      const unsigned xs = __float_as_uint(c.z), ys = __float_as_uint(c.w);
      const int cx0 = max((int)(xs & 0xffffu), tx0), cx1 = min((int)(xs >> 16), tx0 + TILE - 1);
      const int cy0 = max((int)(ys & 0xffffu), ty0), cy1 = min((int)(ys >> 16), ty0 + TILE - 1);
      // The correctly rounded reciprocal: identical to the reference's 1.0f / area.
      const float inv_area = __frcp_rn(c.y);
      s_rowspan[tid] = make_uint4(0x0F0F0F0Fu, 0x0F0F0F0Fu, 0x0F0F0F0Fu, 0x0F0F0F0Fu);  // every row empty
      // A listed candidate's rectangle always meets its tile (it was binned by
      // it); a scanned one may not, and an invalid record (area 0) has none.
      if (c.y != 0.0f && cx0 <= cx1 && cy0 <= cy1) {
        ly0 = cy0 - ty0;
        ly1 = cy1 - ty0;
        n_items = stage_spans(a, bb, c.y, inv_area, cx0 - tx0, cx1 - tx0, ly0, ly1, tx0, W, s_ndcy, span, n_rows);
      }
      s_rec[3 * tid + 0] = a;
      s_rec[3 * tid + 1] = bb;
      s_rec[3 * tid + 2] = make_float4(c.x, c.y, inv_area, __int_as_float(t));
    }
    // Block exclusive scan of (pixels, non-empty rows), packed: a batch holds
    // at most 255 * 256 pixels (17 bits) and 255 * 16 rows (13 bits).
    const int mine = n_items | (n_rows << 17);
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const int ws = s_wsum[w];
      if (w < warp) before += ws;
      all += ws;
    }
    const int n_total = all & 0x1FFFF, n_spans = all >> 17;
    if (n_rows > 0) {
      // This candidate's non-empty rows, in item order, into the span list
      // (stage_spans wrote only the rows in [ly0, ly1] with a span).
      const int excl = before + incl - mine;
      int item = excl & 0x1FFFF, slot = excl >> 17;
      for (int ly = ly0; ly <= ly1; ++ly) {
        const unsigned sp = span[ly];
        const int c0 = (int)(sp & 15u), c1 = (int)(sp >> 4);
        if (c1 >= c0) {
          s_start[slot] = (unsigned short)item;
          s_info[slot] = tid | (ly << 8) | (int)((unsigned)(c0 - item) << 12);
          ++slot;
          item += c1 - c0 + 1;
        }
      }
    }
    if (tid < 33) s_start[n_spans + tid] = kNoStart;  // no start past the last span
    __syncthreads();
    // Warp w tests items [wlo, whi), 32 consecutive items per step.
    const int wlo = (int)(((long long)warp * n_total) / WARPS);
    const int whi = (int)(((long long)(warp + 1) * n_total) / WARPS);
    if (wlo < whi) {
      // The span holding item wlo: the last s with s_start[s] <= wlo (starts
      // increase strictly, every span owning at least one item).
      int s0 = 0, sh = n_spans - 1;
      while (s0 < sh) {
        const int mid = (s0 + sh + 1) >> 1;
        if (s_start[mid] <= wlo) s0 = mid; else sh = mid - 1;
      }
      for (int b0 = wlo; b0 < whi; b0 += 32) {
        // s0 holds item b0, so the starts after it are >= b0 and at most 32
        // of them (one per later item of the step) can fall inside the step:
        // the span of item b0 + lane is s0 plus the number of starts among
        // s_start[s0 + 1 .. s0 + 32] that are <= b0 + lane.
        const int d = (int)s_start[s0 + 1 + lane] - b0;
        const unsigned M = __reduce_or_sync(0xffffffffu, d < 32 ? (1u << d) : 0u);
        // Lanes past the warp's range (last step only) get a valid span and
        // an in-tile column, test without effect and fold nothing: no branch.
        const int s = min(s0 + __popc(M & (0xffffffffu >> (31 - lane))), n_spans - 1);
        s0 = __shfl_sync(0xffffffffu, s, 31);
        const int item = b0 + lane;
        const int info = s_info[s];
        const int j = info & 255, ly = (info >> 8) & 15;
        const int lx = (item + (info >> 12)) & (TILE - 1);
        unsigned long long key = 0;
        int p = 0;
        if (test(s_rec[3 * j], s_rec[3 * j + 1], s_rec[3 * j + 2], lx, ly, key, p) & (item < whi)) fold(key, p);
      }
    }
  }
  __syncthreads();
  const float k_x = DB ? FD(2.0f, (float)W) : 0.0f, k_y = DB ? FD(-2.0f, (float)H) : 0.0f;
  if (!EPI) {
    if (!inside_img) return;
    const float x = s_ndcx[px - tx0], y = s_ndcy[py - ty0];
    write_pixel<DB>(rec, rec_view, s_k0[tid], x, y, k_x, k_y, rast, rast_db, pix);
    if (TWO) write_pixel<DB>(rec, rec_view, s_k1[tid], x, y, k_x, k_y, rast1, rast_db1, pix);
    return;
  }
  // Every thread stays for the block sums of the fused losses.
  float l0 = 0.0f, l1 = 0.0f;
  if (inside_img) {
    const float x = s_ndcx[px - tx0], y = s_ndcy[py - ty0];
    const PixOut p0 = write_pixel<DB>(rec, rec_view, s_k0[tid], x, y, k_x, k_y, rast, rast_db, pix);
    epi_pixel(epi, 0, p0, pix, n, l0, err);
    const PixOut p1 = write_pixel<DB>(rec, rec_view, s_k1[tid], x, y, k_x, k_y, rast1, rast_db1, pix);
    epi_pixel(epi, 1, p1, pix, n, l1, err);
  }
  if (epi.part[0]) block_loss_add(l0, epi.lscale[0], epi.part[0]);
  if (epi.part[0] && epi.part[1]) __syncthreads();  // block_loss_add's shared slots are reused
  if (epi.part[1]) block_loss_add(l1, epi.lscale[1], epi.part[1]);
}

}  // namespace

using namespace dr;

namespace {

struct Prepared {
  const float4* rec;
  const uint32_t* tile_off;  // tile gt's list is [tile_off[gt*off_stride], tile_off[(gt+1)*off_stride])
  int off_stride;
  const int32_t* list;
  int ntx, nty;
  int64_t ntiles_all;
  uint32_t cap;  // list entries held; UINT32_MAX when sized exactly
  bool capped;   // fixed capacity: tiles past it scan every triangle
};

// Largest per-view tile count whose histogram (4 B per tile) the binned
// setup / scatter keep in shared memory.
constexpr int kMaxHistTiles = 40960;

// Setup, tile counts, scan, one readback of the list length, scatter.
dr_status raster_prepare(dr_ctx* ctx, const float* pos, const float* xform, int V, const int32_t* tri, int T,
                         const int32_t* ranges, int N, int H, int W, Prepared& pr) {
  DR_REQUIRE(ctx, pos && (tri || T == 0), "rasterize: pos and tri are required");
  DR_REQUIRE(ctx, N > 0 && V > 0 && T >= 0 && H > 0 && W > 0,
             "rasterize: bad sizes N=%d V=%d T=%d H=%d W=%d", N, V, T, H, W);
  DR_REQUIRE(ctx, H <= 32768 && W <= 32768, "rasterize: resolution above 32768 is not supported");
  DR_REQUIRE(ctx, T < (1 << 24), "rasterize: T must be < 2^24 (tri_id+1 is stored as float)");
  DR_REQUIRE(ctx, aligned16(pos), "rasterize: pos must be 16-byte aligned");
  const int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE;
  const int ntiles = ntx * nty;
  const int64_t ntiles_all = (int64_t)N * ntiles;
  const int64_t NT = (int64_t)N * T;
  DR_REQUIRE(ctx, ntiles_all < (1ll << 31), "rasterize: too many tiles");

  // Binned mode: cpv CTAs per view, each with a chunk of at least max(1024,
  // ntiles) triangles (so its histogram flush is amortised), about 8 CTAs per
  // SM in total.
  const bool binned = ntiles <= kMaxHistTiles && T > 0 && N <= 65535;  // views on grid.y
  int cpv = 1, chunk = T;
  if (binned) {
    const int64_t by_size = ((int64_t)T + std::max(1024, ntiles) - 1) / std::max(1024, ntiles);
    const int64_t by_grid = ((int64_t)8 * ctx->num_sms + N - 1) / N;
    cpv = (int)std::max<int64_t>(1, std::min<int64_t>(std::min(by_size, by_grid), 65535));
    chunk = (int)(((int64_t)T + cpv - 1) / cpv);
  }
  const int64_t ncnt = ntiles_all * cpv;
  DR_REQUIRE(ctx, ncnt < (1ll << 31), "rasterize: too many tile segments");

  // Records (48 B) then, binned, the pixel rectangles (8 B) of every (view, triangle).
  float4* rec = (float4*)ws_get(ctx, WS_RASTER_REC, (sizeof(float4) * 3 + sizeof(uint2)) * (size_t)(NT > 0 ? NT : 1));
  uint2* box = rec ? reinterpret_cast<uint2*>(rec + 3 * (NT > 0 ? NT : 1)) : nullptr;
  // cnt[ncnt] | off[ncnt + 1] | cur[ntiles_all] (unbinned only) | total
  uint32_t* tc = (uint32_t*)ws_get(ctx, WS_TILE_COUNT, sizeof(uint32_t) * (size_t)(2 * ncnt + ntiles_all + 4));
  if (!rec || !tc) return DR_ENOMEM;
  uint32_t* cnt = tc;
  uint32_t* off = tc + ncnt;
  uint32_t* cur = off + ncnt + 1;
  uint32_t* total = cur + ntiles_all;
  const size_t hist_bytes = sizeof(uint32_t) * (size_t)ntiles;

  if (binned) {
    if (hist_bytes > 48 * 1024) {
      DR_CUDA(ctx, cudaFuncSetAttribute(k_raster_setup_binned, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)hist_bytes), "rasterize smem");
      DR_CUDA(ctx, cudaFuncSetAttribute(k_raster_scatter_binned, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)hist_bytes), "rasterize smem");
    }
    DR_TB(ctx);
    k_raster_setup_binned<<<dim3(cpv, N), 256, hist_bytes, ctx->stream>>>(pos, xform, V, tri, T, ranges, H, W, ntx,
                                                                         nty, chunk, cpv, rec, box, cnt,
                                                                         ctx->d_err);
    DR_LAUNCHED(ctx, "raster_setup");
  } else {
    DR_CUDA(ctx, cudaMemsetAsync(cnt, 0, sizeof(uint32_t) * (size_t)ncnt, ctx->stream), "rasterize memset");
    if (NT > 0) {
      DR_TB(ctx);
      k_raster_setup<<<grid_for(NT, 256), 256, 0, ctx->stream>>>(pos, xform, V, tri, T, ranges, N, H, W, ntx,
                                                                 nty, rec, cnt, ctx->d_err);
      DR_LAUNCHED(ctx, "raster_setup");
    }
  }
  dr_status st = scan_u32(ctx, cnt, off, ncnt, total);
  if (st != DR_OK) return st;
  // off[ncnt] = total closes the last tile's range.
  DR_CUDA(ctx, cudaMemcpyAsync(off + ncnt, total, sizeof(uint32_t), cudaMemcpyDeviceToDevice, ctx->stream),
          "rasterize copy");
  if (!binned)
    DR_CUDA(ctx, cudaMemcpyAsync(cur, off, sizeof(uint32_t) * (size_t)ntiles_all, cudaMemcpyDeviceToDevice,
                                 ctx->stream), "rasterize copy");
  int32_t* list;
  uint32_t cap;
  bool launch_scatter = NT > 0;
  if (ctx->list_cap > 0) {
    // Fixed capacity (dr_ctx_set_raster_list_capacity): nothing is read back.
    cap = (uint32_t)ctx->list_cap;
    list = (int32_t*)ws_get(ctx, WS_TILE_LIST, sizeof(int32_t) * (size_t)(cap + 1));
  } else {
    // The list length is data dependent: read it back (one small sync) and
    // size the list buffer exactly, so no candidate is ever dropped.
    DR_CUDA(ctx, cudaMemcpyAsync(ctx->h_pinned, total, sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream),
            "rasterize readback");
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return fail(ctx, DR_ECUDA, "rasterize: %s", cudaGetErrorString(e));
    const uint32_t n_pairs = (uint32_t)ctx->h_pinned[0];
    list = (int32_t*)ws_get(ctx, WS_TILE_LIST, sizeof(int32_t) * (size_t)(n_pairs + 1));
    cap = UINT32_MAX;
    launch_scatter = launch_scatter && n_pairs > 0;
  }
  if (!list) return DR_ENOMEM;
  if (launch_scatter) {
    DR_TB(ctx);
    if (binned) {
      // One wave: as many pairs per CTA as fill the resident CTAs once.
      const int per_sm = (int)std::max<size_t>(1, std::min<size_t>(2048 / kScatterBlock,
                                                                   (227 * 1024) / (hist_bytes + 1024)));
      const int64_t pairs = (int64_t)N * cpv;
      const int64_t slots = (int64_t)per_sm * ctx->num_sms;
      const int per = (int)((pairs + slots - 1) / slots);
      const unsigned grid = (unsigned)((pairs + per - 1) / per);
      k_raster_scatter_binned<<<grid, kScatterBlock, hist_bytes, ctx->stream>>>(box, N, T, ntx, nty, chunk, cpv,
                                                                                per, off, list, cap);
    } else
      k_raster_scatter<<<grid_for(NT, 256), 256, 0, ctx->stream>>>(rec, N, T, ntx, nty, cur, list, cap);
    DR_LAUNCHED(ctx, "raster_scatter");
  }
  pr.rec = rec;
  pr.tile_off = off;
  pr.off_stride = cpv;
  pr.list = list;
  pr.ntx = ntx;
  pr.nty = nty;
  pr.ntiles_all = ntiles_all;
  pr.cap = cap;
  pr.capped = ctx->list_cap > 0;
  return DR_OK;
}

// One depth layer over prepared tile lists (peel: previous layer or NULL), or
// layers 0 and 1 together when rast1 is given (then peel must be NULL).
dr_status raster_layer(dr_ctx* ctx, const Prepared& pr, int T, int H, int W, const float* peel_layer,
                       float* rast, float* rast_db, float* rast1 = nullptr, float* rast_db1 = nullptr,
                       const InterpEpi* epi = nullptr) {
  DR_REQUIRE(ctx, rast != nullptr, "rasterize: rast output is required");
  DR_REQUIRE(ctx, aligned16(rast) && (!rast_db || aligned16(rast_db)) && (!peel_layer || aligned16(peel_layer)) &&
                      (!rast1 || aligned16(rast1)) && (!rast_db1 || aligned16(rast_db1)),
             "rasterize: rast/rast_db/peel_layer must be 16-byte aligned");
  const unsigned grid = (unsigned)pr.ntiles_all;
  float4* r4 = reinterpret_cast<float4*>(rast);
  float4* d4 = reinterpret_cast<float4*>(rast_db);
  float4* r41 = reinterpret_cast<float4*>(rast1);
  float4* d41 = reinterpret_cast<float4*>(rast_db1);
  const int ntx = pr.ntx, nty = pr.nty;
  DR_TB(ctx);
  if (epi) {  // two layers with rast_db and the interpolation epilogue
    if (pr.capped)
      k_raster_tiles<2, true, true, true><<<grid, TILE_PIX, 0, ctx->stream>>>(
          pr.rec, T, H, W, ntx, nty, pr.tile_off, pr.off_stride, pr.list, nullptr, r4, d4, r41, d41, ctx->d_err,
          pr.cap, ctx->d_overflow, *epi);
    else
      k_raster_tiles<2, true, false, true><<<grid, TILE_PIX, 0, ctx->stream>>>(
          pr.rec, T, H, W, ntx, nty, pr.tile_off, pr.off_stride, pr.list, nullptr, r4, d4, r41, d41, ctx->d_err,
          pr.cap, ctx->d_overflow, *epi);
    DR_LAUNCHED(ctx, "raster_tiles_interp");
    return DR_OK;
  }
#define DR_RT(MODEV, DBV, PEELP)                                                                               \
  do {                                                                                                         \
    if (pr.capped)                                                                                             \
      k_raster_tiles<MODEV, DBV, true><<<grid, TILE_PIX, 0, ctx->stream>>>(                                    \
          pr.rec, T, H, W, ntx, nty, pr.tile_off, pr.off_stride, pr.list, PEELP, r4, d4, r41, d41, ctx->d_err, \
          pr.cap, ctx->d_overflow, InterpEpi{});                                                               \
    else                                                                                                       \
      k_raster_tiles<MODEV, DBV, false><<<grid, TILE_PIX, 0, ctx->stream>>>(                                   \
          pr.rec, T, H, W, ntx, nty, pr.tile_off, pr.off_stride, pr.list, PEELP, r4, d4, r41, d41, ctx->d_err, \
          pr.cap, ctx->d_overflow, InterpEpi{});                                                               \
  } while (0)
  if (rast1) {
    if (rast_db) DR_RT(2, true, nullptr); else DR_RT(2, false, nullptr);
  } else if (peel_layer) {
    if (rast_db) DR_RT(1, true, peel_layer); else DR_RT(1, false, peel_layer);
  } else {
    if (rast_db) DR_RT(0, true, nullptr); else DR_RT(0, false, nullptr);
  }
#undef DR_RT
  DR_LAUNCHED(ctx, "raster_tiles");
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_rasterize_fwd(dr_ctx* ctx, const float* pos, int V, const int32_t* tri,
                                      int T, const int32_t* ranges, int N, int H, int W,
                                      const float* peel_layer, float* rast, float* rast_db) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, pos && (tri || T == 0) && rast, "rasterize: pos, tri and rast are required");
  Prepared pr;
  dr_status st = raster_prepare(ctx, pos, nullptr, V, tri, T, ranges, N, H, W, pr);
  if (st != DR_OK) return st;
  return raster_layer(ctx, pr, T, H, W, peel_layer, rast, rast_db);
}

namespace {

dr_status layers_fwd(dr_ctx* ctx, const float* pos, const float* xform, int V, const int32_t* tri, int T,
                     const int32_t* ranges, int N, int H, int W, int num_layers, float* const* rast,
                     float* const* rast_db) {
  DR_REQUIRE(ctx, num_layers >= 1 && rast, "rasterize_layers: num_layers >= 1 and rast[] required");
  for (int l = 0; l < num_layers; ++l) DR_REQUIRE(ctx, rast[l] != nullptr, "rasterize_layers: rast[%d] is NULL", l);
  Prepared pr;
  dr_status st = raster_prepare(ctx, pos, xform, V, tri, T, ranges, N, H, W, pr);
  if (st != DR_OK) return st;
  auto db_of = [&](int l) { return rast_db ? rast_db[l] : nullptr; };
  int l = 0;
  // Layers 0 and 1 come out of one candidate pass when both or neither carry rast_db.
  if (num_layers >= 2 && ((db_of(0) == nullptr) == (db_of(1) == nullptr))) {
    st = raster_layer(ctx, pr, T, H, W, nullptr, rast[0], db_of(0), rast[1], db_of(1));
    if (st != DR_OK) return st;
    l = 2;
  }
  for (; l < num_layers; ++l) {
    st = raster_layer(ctx, pr, T, H, W, l ? rast[l - 1] : nullptr, rast[l], db_of(l));
    if (st != DR_OK) return st;
  }
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_rasterize_layers_fwd(dr_ctx* ctx, const float* pos, int V, const int32_t* tri, int T,
                                             const int32_t* ranges, int N, int H, int W, int num_layers,
                                             float* const* rast, float* const* rast_db) {
  DR_ENTER(ctx);
  return layers_fwd(ctx, pos, nullptr, V, tri, T, ranges, N, H, W, num_layers, rast, rast_db);
}

extern "C" dr_status dr_rasterize_xf_fwd(dr_ctx* ctx, const float* verts, int V, const float* xform,
                                         const int32_t* tri, int T, int N, int H, int W, int num_layers,
                                         float* const* rast, float* const* rast_db) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform != nullptr && ((uintptr_t)xform & 15) == 0,
             "rasterize_xf: xform [N,4,4] must be given and 16-byte aligned");
  return layers_fwd(ctx, verts, xform, V, tri, T, nullptr, N, H, W, num_layers, rast, rast_db);
}

extern "C" dr_status dr_rasterize_xf_interp_fwd(dr_ctx* ctx, const float* verts, int V, const float* xform,
                                                const int32_t* tri, int T, int N, int H, int W, const float* attr,
                                                int attr_batch, int A, float* const* rast, float* const* rast_db,
                                                float* const* out, float* const* out_da,
                                                const float* const* target, float scale, float* const* loss) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform != nullptr && ((uintptr_t)xform & 15) == 0,
             "rasterize_interp: xform [N,4,4] must be given and 16-byte aligned");
  DR_REQUIRE(ctx, rast && rast_db && out && out_da, "rasterize_interp: rast, rast_db, out and out_da are required");
  DR_REQUIRE(ctx, attr && aligned16(attr) && A > 0 && A % 4 == 0,
             "rasterize_interp: attr must be 16-byte aligned with A a multiple of 4 (A=%d)", A);
  DR_REQUIRE(ctx, attr_batch == 1 || attr_batch == N,
             "rasterize_interp: attr batch dim %d incompatible with %d views", attr_batch, N);
  InterpEpi e{};
  e.attr = attr;
  e.attr_shared = attr_batch == 1;
  e.V = V;
  e.A = A;
  e.tri = tri;
  bool any_loss = false;
  for (int l = 0; l < 2; ++l) {
    DR_REQUIRE(ctx, rast[l] && rast_db[l] && out[l] && out_da[l], "rasterize_interp: layer %d output missing", l);
    DR_REQUIRE(ctx, aligned16(out[l]) && aligned16(out_da[l]), "rasterize_interp: out / out_da must be 16-byte aligned");
    const float* t = target ? target[l] : nullptr;
    float* lo = loss ? loss[l] : nullptr;
    DR_REQUIRE(ctx, (t == nullptr) == (lo == nullptr), "rasterize_interp: layer %d: target and loss go together", l);
    DR_REQUIRE(ctx, !t || aligned16(t), "rasterize_interp: target must be 16-byte aligned");
    e.out[l] = out[l];
    e.out_da[l] = out_da[l];
    e.tgt[l] = t;
    e.lscale[l] = scale;
    any_loss = any_loss || t;
  }
  Prepared pr;
  dr_status st = raster_prepare(ctx, verts, xform, V, tri, T, nullptr, N, H, W, pr);
  if (st != DR_OK) return st;
  if (any_loss) {
    // Both layers' partial sums, side by side in the fused-loss slot.
    float* part = (float*)ws_get(ctx, WS_LOSS, sizeof(float) * 2 * kLossSlots);
    if (!part) return DR_ENOMEM;
    DR_CUDA(ctx, cudaMemsetAsync(part, 0, sizeof(float) * 2 * kLossSlots, ctx->stream), "loss memset");
    for (int l = 0; l < 2; ++l) e.part[l] = e.tgt[l] ? part + l * kLossSlots : nullptr;
  }
  st = raster_layer(ctx, pr, T, H, W, nullptr, rast[0], rast_db[0], rast[1], rast_db[1], &e);
  if (st != DR_OK) return st;
  for (int l = 0; l < 2; ++l)
    if (e.part[l] && (st = loss_end(ctx, e.part[l], loss[l])) != DR_OK) return st;
  return DR_OK;
}
