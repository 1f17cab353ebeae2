// diffrast_oracle.cpp — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
//
// CPU restatement of the per-thread arithmetic of mlx-swift-diffrast's Metal
// kernels (Sources/MLXDiffRast/*.swift).  It is the parity checker for the
// CUDA library: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg are its only callers.  Build with -O2 -ffp-contract=off (no fast-math)
// so every float operation rounds exactly as written, in the written order.
//
// Conventions and deliberate definitions: see diffrast_oracle.h.

#include "diffrast_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// threading helpers

int clamp_threads(int nthreads) {
  if (nthreads <= 0) {
    unsigned hc = std::thread::hardware_concurrency();
    nthreads = hc ? (int)hc : 1;
  }
  return nthreads;
}

// Static partition of [0, n) into `nthreads` contiguous chunks; f(begin, end, tid).
template <class F>
void parallel_for(int64_t n, int nthreads, F f) {
  nthreads = clamp_threads(nthreads);
  if (n <= 0) return;
  if (nthreads == 1 || n < 64) {
    f((int64_t)0, n, 0);
    return;
  }
  std::vector<std::thread> th;
  int64_t chunk = (n + nthreads - 1) / nthreads;
  for (int i = 0; i < nthreads; ++i) {
    int64_t b = i * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    th.emplace_back([=, &f]() { f(b, e, i); });
  }
  for (auto& t : th) t.join();
}

// Per-thread float64 accumulators standing in for the reference's relaxed
// float atomics; reduced in thread order so the result is deterministic.  The
// buffers come from a process-wide pool (kept between calls, so large meshes do
// not page-fault fresh memory on every call); each thread zeroes its own buffer
// on first use and the reduction is split across threads by index range.
struct AccumPool {
  std::mutex m;
  std::vector<std::vector<double>> bufs;
};
AccumPool& accum_pool() {
  static AccumPool p;
  return p;
}

struct Accum {
  std::vector<double*> buf;
  std::vector<char> touched;
  size_t n;
  int nthreads;
  Accum(int nthreads_, size_t n_) : n(n_), nthreads(clamp_threads(nthreads_)) {
    AccumPool& p = accum_pool();
    std::lock_guard<std::mutex> g(p.m);
    if ((int)p.bufs.size() < nthreads) p.bufs.resize(nthreads);
    buf.resize(nthreads);
    touched.assign(nthreads, 0);
    for (int t = 0; t < nthreads; ++t) {
      if (p.bufs[t].size() < n) p.bufs[t].resize(n);
      buf[t] = p.bufs[t].data();
    }
  }
  double* get(int tid) {
    if (!touched[tid]) {
      std::memset(buf[tid], 0, sizeof(double) * n);
      touched[tid] = 1;
    }
    return buf[tid];
  }
  void reduce_to(float* out) {
    parallel_for((int64_t)n, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t i = b; i < e; ++i) {
        double s = 0.0;
        for (int t = 0; t < nthreads; ++t)
          if (touched[t]) s += buf[t][i];
        out[i] = (float)s;
      }
    });
  }
};

inline bool finitef(float x) { return std::isfinite(x); }

// Pixel-centre NDC (Rasterize.swift:381-382).
inline float ndc_x_of(int pw, int W) { return 2.0f * ((float)pw + 0.5f) / (float)W - 1.0f; }
inline float ndc_y_of(int ph, int H) { return 1.0f - 2.0f * ((float)ph + 0.5f) / (float)H; }

// ---------------------------------------------------------------------------
// rasterize

// K1 diffrast_rasterize_precompute (Rasterize.swift:280-328): one record of
// (sx0,sy0,sz0, sx1,sy1,sz1, sx2,sy2,sz2, area); area = 0 marks invalid.
void raster_setup(const float* pos, int64_t pos_n_base, const int32_t* tri,
                  int t, int V, bool in_range, float* rec) {
  for (int k = 0; k < 10; ++k) rec[k] = 0.0f;
  if (!in_range) return;
  int i0 = tri[t * 3 + 0], i1 = tri[t * 3 + 1], i2 = tri[t * 3 + 2];
  if (i0 < 0 || i0 >= V || i1 < 0 || i1 >= V || i2 < 0 || i2 >= V) return;
  const float* p0 = pos + pos_n_base + (int64_t)i0 * 4;
  const float* p1 = pos + pos_n_base + (int64_t)i1 * 4;
  const float* p2 = pos + pos_n_base + (int64_t)i2 * 4;
  float w0 = p0[3], w1 = p1[3], w2 = p2[3];
  if (w0 <= 0.0f || w1 <= 0.0f || w2 <= 0.0f) return;
  float sx0 = p0[0] / w0, sy0 = p0[1] / w0, sz0 = p0[2] / w0;
  float sx1 = p1[0] / w1, sy1 = p1[1] / w1, sz1 = p1[2] / w1;
  float sx2 = p2[0] / w2, sy2 = p2[1] / w2, sz2 = p2[2] / w2;
  float area = (sx1 - sx0) * (sy2 - sy0) - (sx2 - sx0) * (sy1 - sy0);
  float v[10] = {sx0, sy0, sz0, sx1, sy1, sz1, sx2, sy2, sz2, area};
  for (int k = 0; k < 10; ++k)
    if (!finitef(v[k])) return;
  // A finite, non-zero but tiny area (|area| < 2^-128) has 1/area = inf: every
  // pixel of such a record gets bw/u/v of +-inf or NaN (0 * inf), hence a depth
  // that is infinite or NaN and never a fragment (see the z test in the pixel
  // loop).  Marking it invalid here changes no output and skips the work.
  if (!finitef(1.0f / area)) return;
  for (int k = 0; k < 10; ++k) rec[k] = v[k];
}

// Conservative (superset) pixel range of a record's NDC AABB, widened by one
// pixel on each side; the per-pixel NDC test stays authoritative, so the
// candidate set contains every triangle the reference's unbinned loop would
// accept (Rasterize.swift:199-223 for the reference's own binning formula).
bool raster_pixel_range(const float* r, int H, int W, int* x0, int* x1, int* y0, int* y1) {
  double minx = std::min(r[0], std::min(r[3], r[6]));
  double maxx = std::max(r[0], std::max(r[3], r[6]));
  double miny = std::min(r[1], std::min(r[4], r[7]));
  double maxy = std::max(r[1], std::max(r[4], r[7]));
  double pxmin = std::floor((minx + 1.0) * W * 0.5 - 0.5) - 1.0;
  double pxmax = std::floor((maxx + 1.0) * W * 0.5 - 0.5) + 1.0;
  double pymin = std::floor((1.0 - maxy) * H * 0.5 - 0.5) - 1.0;
  double pymax = std::floor((1.0 - miny) * H * 0.5 - 0.5) + 1.0;
  pxmin = std::max(pxmin, 0.0);
  pymin = std::max(pymin, 0.0);
  pxmax = std::min(pxmax, (double)(W - 1));
  pymax = std::min(pymax, (double)(H - 1));
  if (pxmin > pxmax || pymin > pymax) return false;
  *x0 = (int)pxmin; *x1 = (int)pxmax; *y0 = (int)pymin; *y1 = (int)pymax;
  return true;
}

constexpr int TILE = 16;

}  // namespace

// K3/K4 diffrast_rasterize_fwd/_fwd_db (Rasterize.swift:371-599), with the
// candidate list of each 16x16 tile = every valid triangle whose AABB may touch
// it, in ascending index (the reference's pre-binning semantics, todo.md M2.4).
extern "C" int orc_rasterize_fwd(const float* pos, int V, const int32_t* tri, int T,
                                 const int32_t* ranges, int N, int H, int W,
                                 const float* peel, float* rast, float* rast_db,
                                 int nthreads) {
  if (N <= 0 || H <= 0 || W <= 0 || T < 0 || V <= 0) return 1;
  const int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE;
  std::vector<float> recs((size_t)T * 10);
  std::vector<std::vector<int>> bins((size_t)ntx * nty);
  for (int pn = 0; pn < N; ++pn) {
    int64_t pos_n_base = ranges ? 0 : (int64_t)pn * V * 4;
    int rs = ranges ? ranges[pn * 2 + 0] : 0;
    int rc = ranges ? ranges[pn * 2 + 1] : T;
    parallel_for(T, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t t = b; t < e; ++t) {
        bool in_range = !((int)t < rs || (int)t >= rs + rc);
        raster_setup(pos, pos_n_base, tri, (int)t, V, in_range, &recs[(size_t)t * 10]);
      }
    });
    for (auto& bl : bins) bl.clear();
    for (int t = 0; t < T; ++t) {
      const float* r = &recs[(size_t)t * 10];
      if (r[9] == 0.0f) continue;
      int x0, x1, y0, y1;
      if (!raster_pixel_range(r, H, W, &x0, &x1, &y0, &y1)) continue;
      for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty)
        for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) bins[(size_t)ty * ntx + tx].push_back(t);
    }
    parallel_for((int64_t)ntx * nty, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t tile = b; tile < e; ++tile) {
        int tx = (int)(tile % ntx), ty = (int)(tile / ntx);
        const auto& cand = bins[(size_t)tile];
        for (int ph = ty * TILE; ph < std::min(H, ty * TILE + TILE); ++ph)
          for (int pw = tx * TILE; pw < std::min(W, tx * TILE + TILE); ++pw) {
            float ndc_x = ndc_x_of(pw, W);
            float ndc_y = ndc_y_of(ph, H);
            int64_t base = (((int64_t)pn * H + ph) * W + pw) * 4;
            float peel_z = -1e30f;
            if (peel) {
              float prev_tri = peel[base + 3];
              if (prev_tri > 0.0f) peel_z = peel[base + 2];
            }
            float best_z = 1e30f, best_u = 0.0f, best_v = 0.0f;
            int best_t = -1;
            for (int t : cand) {
              const float* r = &recs[(size_t)t * 10];
              float area = r[9];
              if (area == 0.0f) continue;
              float sx0 = r[0], sy0 = r[1], sz0 = r[2];
              float sx1 = r[3], sy1 = r[4], sz1 = r[5];
              float sx2 = r[6], sy2 = r[7], sz2 = r[8];
              float minx = std::fmin(sx0, std::fmin(sx1, sx2));
              if (ndc_x < minx) continue;
              float maxx = std::fmax(sx0, std::fmax(sx1, sx2));
              if (ndc_x > maxx) continue;
              float miny = std::fmin(sy0, std::fmin(sy1, sy2));
              if (ndc_y < miny) continue;
              float maxy = std::fmax(sy0, std::fmax(sy1, sy2));
              if (ndc_y > maxy) continue;
              float inv_area = 1.0f / area;
              float e0 = (sx1 - ndc_x) * (sy2 - ndc_y) - (sx2 - ndc_x) * (sy1 - ndc_y);
              float e1 = (sx2 - ndc_x) * (sy0 - ndc_y) - (sx0 - ndc_x) * (sy2 - ndc_y);
              float e2 = (sx0 - ndc_x) * (sy1 - ndc_y) - (sx1 - ndc_x) * (sy0 - ndc_y);
              if ((e0 * area) < 0.0f || (e1 * area) < 0.0f || (e2 * area) < 0.0f) continue;
              float bw = e0 * inv_area;
              float u = e1 * inv_area;
              float v = e2 * inv_area;
              float z_pix = bw * sz0 + u * sz1 + v * sz2;
              if (z_pix < -1.0f || z_pix > 1.0f) continue;
              // Deviation from Rasterize.swift:455-458: there a NaN depth
              // (e.g. e = inf - inf for vertices near w = 0, or 0 * inf) passes
              // every comparison, is stored as best_z, and is then replaced by
              // whichever candidate comes next, so the result depends on the
              // bin's atomic append order.  Here a NaN depth is never a
              // fragment, which keeps the winner order independent.
              if (std::isnan(z_pix)) continue;
              if (z_pix <= peel_z) continue;
              if (z_pix >= best_z) continue;
              best_z = z_pix; best_t = t; best_u = u; best_v = v;
            }
            if (best_t < 0) {
              for (int c = 0; c < 4; ++c) rast[base + c] = 0.0f;
              if (rast_db)
                for (int c = 0; c < 4; ++c) rast_db[base + c] = 0.0f;
              continue;
            }
            rast[base + 0] = best_u;
            rast[base + 1] = best_v;
            rast[base + 2] = best_z;
            rast[base + 3] = (float)(best_t + 1);
            if (rast_db) {
              const float* r = &recs[(size_t)best_t * 10];
              float sx0 = r[0], sy0 = r[1], sx1 = r[3], sy1 = r[4], sx2 = r[6], sy2 = r[7];
              float inv_area = 1.0f / r[9];
              float k_x = 2.0f / (float)W;
              float k_y = -2.0f / (float)H;
              rast_db[base + 0] = (sy2 - sy0) * inv_area * k_x;
              rast_db[base + 1] = (sx0 - sx2) * inv_area * k_y;
              rast_db[base + 2] = (sy0 - sy1) * inv_area * k_x;
              rast_db[base + 3] = (sx1 - sx0) * inv_area * k_y;
            }
          }
      }
    });
  }
  return 0;
}

// K5 diffrast_rasterize_bwd (Rasterize.swift:637-812).  Range mode sums the
// per-view gradients onto the shared [V,4] buffer (MLX broadcast-backward,
// Rasterize.swift:72-76).
extern "C" int orc_rasterize_bwd(const float* pos, int V, const int32_t* tri, int T,
                                 const int32_t* ranges, int N, int H, int W,
                                 const float* rast, const float* d_rast,
                                 const float* d_rast_db, float* d_pos, int nthreads) {
  if (N <= 0 || H <= 0 || W <= 0 || V <= 0) return 1;
  size_t out_n = (size_t)(ranges ? 1 : N) * V * 4;
  Accum acc(nthreads, out_n);
  int64_t P = (int64_t)N * H * W;
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
    double* dp = nullptr;
    for (int64_t pix = b; pix < e; ++pix) {
      int pw = (int)(pix % W);
      int ph = (int)((pix / W) % H);
      int pn = (int)(pix / ((int64_t)H * W));
      int64_t rb = pix * 4;
      int t = (int)rast[rb + 3] - 1;
      if (t < 0 || t >= T) continue;
      float u_val = rast[rb + 0], v_val = rast[rb + 1];
      float bw_val = 1.0f - u_val - v_val;
      float d_u = d_rast[rb + 0], d_v = d_rast[rb + 1], d_z = d_rast[rb + 2];
      float d_db0 = 0, d_db1 = 0, d_db2 = 0, d_db3 = 0;
      if (d_rast_db) {
        d_db0 = d_rast_db[rb + 0]; d_db1 = d_rast_db[rb + 1];
        d_db2 = d_rast_db[rb + 2]; d_db3 = d_rast_db[rb + 3];
      }
      float Px = 2.0f * ((float)pw + 0.5f) / (float)W - 1.0f;
      float Py = 1.0f - 2.0f * ((float)ph + 0.5f) / (float)H;
      int64_t pos_n_base = ranges ? 0 : (int64_t)pn * V * 4;
      int i0 = tri[t * 3 + 0], i1 = tri[t * 3 + 1], i2 = tri[t * 3 + 2];
      if (i0 < 0 || i0 >= V || i1 < 0 || i1 >= V || i2 < 0 || i2 >= V) continue;
      const float* q0 = pos + pos_n_base + (int64_t)i0 * 4;
      const float* q1 = pos + pos_n_base + (int64_t)i1 * 4;
      const float* q2 = pos + pos_n_base + (int64_t)i2 * 4;
      float x0 = q0[0], y0 = q0[1], z0 = q0[2], w0 = q0[3];
      float x1 = q1[0], y1 = q1[1], z1 = q1[2], w1 = q1[3];
      float x2 = q2[0], y2 = q2[1], z2 = q2[2], w2 = q2[3];
      float sx0 = x0 / w0, sy0 = y0 / w0, sz0 = z0 / w0;
      float sx1 = x1 / w1, sy1 = y1 / w1, sz1 = z1 / w1;
      float sx2 = x2 / w2, sy2 = y2 / w2, sz2 = z2 / w2;
      float area = (sx1 - sx0) * (sy2 - sy0) - (sx2 - sx0) * (sy1 - sy0);
      float inv_area = 1.0f / area;
      float dadsx0 = sy1 - sy2, dadsx1 = sy2 - sy0, dadsx2 = sy0 - sy1;
      float dadsy0 = sx2 - sx1, dadsy1 = sx0 - sx2, dadsy2 = sx1 - sx0;
      float de1dsx0 = Py - sy2, de1dsx2 = sy0 - Py, de1dsy0 = sx2 - Px, de1dsy2 = Px - sx0;
      float de2dsx0 = sy1 - Py, de2dsx1 = Py - sy0, de2dsy0 = Px - sx1, de2dsy1 = sx0 - Px;
      float dudsx0 = (de1dsx0 - u_val * dadsx0) * inv_area;
      float dudsx1 = (0.0f - u_val * dadsx1) * inv_area;
      float dudsx2 = (de1dsx2 - u_val * dadsx2) * inv_area;
      float dudsy0 = (de1dsy0 - u_val * dadsy0) * inv_area;
      float dudsy1 = (0.0f - u_val * dadsy1) * inv_area;
      float dudsy2 = (de1dsy2 - u_val * dadsy2) * inv_area;
      float dvdsx0 = (de2dsx0 - v_val * dadsx0) * inv_area;
      float dvdsx1 = (de2dsx1 - v_val * dadsx1) * inv_area;
      float dvdsx2 = (0.0f - v_val * dadsx2) * inv_area;
      float dvdsy0 = (de2dsy0 - v_val * dadsy0) * inv_area;
      float dvdsy1 = (de2dsy1 - v_val * dadsy1) * inv_area;
      float dvdsy2 = (0.0f - v_val * dadsy2) * inv_area;
      float dsz10 = sz1 - sz0, dsz20 = sz2 - sz0;
      float dsx0 = d_u * dudsx0 + d_v * dvdsx0 + d_z * (dudsx0 * dsz10 + dvdsx0 * dsz20);
      float dsx1 = d_u * dudsx1 + d_v * dvdsx1 + d_z * (dudsx1 * dsz10 + dvdsx1 * dsz20);
      float dsx2 = d_u * dudsx2 + d_v * dvdsx2 + d_z * (dudsx2 * dsz10 + dvdsx2 * dsz20);
      float dsy0 = d_u * dudsy0 + d_v * dvdsy0 + d_z * (dudsy0 * dsz10 + dvdsy0 * dsz20);
      float dsy1 = d_u * dudsy1 + d_v * dvdsy1 + d_z * (dudsy1 * dsz10 + dvdsy1 * dsz20);
      float dsy2 = d_u * dudsy2 + d_v * dvdsy2 + d_z * (dudsy2 * dsz10 + dvdsy2 * dsz20);
      float dsz0_s = d_z * bw_val, dsz1_s = d_z * u_val, dsz2_s = d_z * v_val;
      float Kx = 2.0f / (float)W, Ky = -2.0f / (float)H;
      float rdb0 = (sy2 - sy0) * Kx * inv_area;
      float rdb1 = (sx0 - sx2) * Ky * inv_area;
      float rdb2 = (sy0 - sy1) * Kx * inv_area;
      float rdb3 = (sx1 - sx0) * Ky * inv_area;
      float s = d_db0 * rdb0 + d_db1 * rdb1 + d_db2 * rdb2 + d_db3 * rdb3;
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
      float inv_w0 = 1.0f / w0, inv_w1 = 1.0f / w1, inv_w2 = 1.0f / w2;
      float g[12] = {
          dsx0 * inv_w0, dsy0 * inv_w0, dsz0_s * inv_w0, -(sx0 * dsx0 + sy0 * dsy0 + sz0 * dsz0_s) * inv_w0,
          dsx1 * inv_w1, dsy1 * inv_w1, dsz1_s * inv_w1, -(sx1 * dsx1 + sy1 * dsy1 + sz1 * dsz1_s) * inv_w1,
          dsx2 * inv_w2, dsy2 * inv_w2, dsz2_s * inv_w2, -(sx2 * dsx2 + sy2 * dsy2 + sz2 * dsz2_s) * inv_w2};
      if (!dp) dp = acc.get(tid);
      int idx[3] = {i0, i1, i2};
      for (int k = 0; k < 3; ++k)
        for (int c = 0; c < 4; ++c) dp[pos_n_base + (int64_t)idx[k] * 4 + c] += (double)g[k * 4 + c];
    }
  });
  acc.reduce_to(d_pos);
  return 0;
}

// ---------------------------------------------------------------------------
// interpolate

namespace {
// Resolve the triangle of a rast pixel: -1 for empty / out-of-range.
inline int pixel_tri(const float* rast, int64_t rb, int T, const int32_t* tri, int V,
                     int* i0, int* i1, int* i2) {
  int t = (int)rast[rb + 3] - 1;
  if (t < 0 || t >= T) return -1;
  *i0 = tri[t * 3 + 0]; *i1 = tri[t * 3 + 1]; *i2 = tri[t * 3 + 2];
  if (*i0 < 0 || *i0 >= V || *i1 < 0 || *i1 >= V || *i2 < 0 || *i2 >= V) return -1;
  return t;
}
}  // namespace

// K6/K7 diffrast_interp_fwd/_fwd_da (Interpolate.swift:137-228).
extern "C" int orc_interpolate_fwd(const float* attr, int attr_batch, int V, int A,
                                   const float* rast, int N, int H, int W,
                                   const int32_t* tri, int T, const float* rast_db,
                                   const int32_t* diff_idx, int K, float* out,
                                   float* out_da, int nthreads) {
  int64_t P = (int64_t)N * H * W;
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
    for (int64_t pix = b; pix < e; ++pix) {
      int n = (int)(pix / ((int64_t)H * W));
      int64_t rb = pix * 4;
      float u = rast[rb + 0], v = rast[rb + 1];
      int i0, i1, i2;
      int t = pixel_tri(rast, rb, T, tri, V, &i0, &i1, &i2);
      float* o = out + pix * A;
      float* od = K > 0 ? out_da + pix * 2 * K : nullptr;
      if (t < 0) {
        for (int a = 0; a < A; ++a) o[a] = 0.0f;
        for (int k = 0; k < 2 * K; ++k) od[k] = 0.0f;
        continue;
      }
      float bw = 1.0f - u - v;
      const float* an = attr + (int64_t)(attr_batch == 1 ? 0 : n) * V * A;
      for (int a = 0; a < A; ++a) {
        float a0 = an[(int64_t)i0 * A + a], a1 = an[(int64_t)i1 * A + a], a2 = an[(int64_t)i2 * A + a];
        o[a] = bw * a0 + u * a1 + v * a2;
      }
      if (K > 0) {
        float udx = rast_db[rb + 0], udy = rast_db[rb + 1], vdx = rast_db[rb + 2], vdy = rast_db[rb + 3];
        for (int k = 0; k < K; ++k) {
          int a = diff_idx ? diff_idx[k] : k;
          float a0 = an[(int64_t)i0 * A + a], a1 = an[(int64_t)i1 * A + a], a2 = an[(int64_t)i2 * A + a];
          float d01 = a1 - a0, d02 = a2 - a0;
          od[2 * k + 0] = d01 * udx + d02 * vdx;
          od[2 * k + 1] = d01 * udy + d02 * vdy;
        }
      }
    }
  });
  return 0;
}

// K8-K11 diffrast_interp_grad_attr/_grad_attr_da/_grad_rast/_grad_rast_db
// (Interpolate.swift:231-417); attr_batch == 1 sums over views (67-73).
extern "C" int orc_interpolate_bwd(const float* attr, int attr_batch, int V, int A,
                                   const float* rast, int N, int H, int W,
                                   const int32_t* tri, int T, const float* rast_db,
                                   const int32_t* diff_idx, int K, const float* d_out,
                                   const float* d_out_da, float* d_attr, float* d_rast,
                                   float* d_rast_db, int nthreads) {
  int64_t P = (int64_t)N * H * W;
  Accum acc(nthreads, (size_t)attr_batch * V * A);
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
    double* da = nullptr;
    for (int64_t pix = b; pix < e; ++pix) {
      int n = (int)(pix / ((int64_t)H * W));
      int64_t rb = pix * 4;
      float u = rast[rb + 0], v = rast[rb + 1];
      int i0, i1, i2;
      int t = pixel_tri(rast, rb, T, tri, V, &i0, &i1, &i2);
      d_rast[rb + 2] = 0.0f;
      d_rast[rb + 3] = 0.0f;
      if (t < 0) {
        d_rast[rb + 0] = 0.0f;
        d_rast[rb + 1] = 0.0f;
        if (K > 0)
          for (int c = 0; c < 4; ++c) d_rast_db[rb + c] = 0.0f;
        continue;
      }
      float bw = 1.0f - u - v;
      int64_t nb = (int64_t)(attr_batch == 1 ? 0 : n) * V * A;
      const float* an = attr + nb;
      const float* g = d_out + pix * A;
      if (!da) da = acc.get(tid);
      double* dan = da + nb;
      float du = 0.0f, dv = 0.0f;
      for (int a = 0; a < A; ++a) {
        float ga = g[a];
        dan[(int64_t)i0 * A + a] += (double)(bw * ga);
        dan[(int64_t)i1 * A + a] += (double)(u * ga);
        dan[(int64_t)i2 * A + a] += (double)(v * ga);
        float a0 = an[(int64_t)i0 * A + a], a1 = an[(int64_t)i1 * A + a], a2 = an[(int64_t)i2 * A + a];
        du += (a1 - a0) * ga;
        dv += (a2 - a0) * ga;
      }
      d_rast[rb + 0] = du;
      d_rast[rb + 1] = dv;
      if (K > 0) {
        float udx = rast_db[rb + 0], udy = rast_db[rb + 1], vdx = rast_db[rb + 2], vdy = rast_db[rb + 3];
        const float* gd = d_out_da + pix * 2 * K;
        float d_udx = 0.0f, d_udy = 0.0f, d_vdx = 0.0f, d_vdy = 0.0f;
        for (int k = 0; k < K; ++k) {
          int a = diff_idx ? diff_idx[k] : k;
          float gx = gd[2 * k + 0], gy = gd[2 * k + 1];
          float u_term = gx * udx + gy * udy;
          float v_term = gx * vdx + gy * vdy;
          dan[(int64_t)i0 * A + a] += (double)(-u_term - v_term);
          dan[(int64_t)i1 * A + a] += (double)u_term;
          dan[(int64_t)i2 * A + a] += (double)v_term;
          float a0 = an[(int64_t)i0 * A + a], a1 = an[(int64_t)i1 * A + a], a2 = an[(int64_t)i2 * A + a];
          float d01 = a1 - a0, d02 = a2 - a0;
          d_udx += d01 * gx;
          d_udy += d01 * gy;
          d_vdx += d02 * gx;
          d_vdy += d02 * gy;
        }
        d_rast_db[rb + 0] = d_udx;
        d_rast_db[rb + 1] = d_udy;
        d_rast_db[rb + 2] = d_vdx;
        d_rast_db[rb + 3] = d_vdy;
      }
    }
  });
  acc.reduce_to(d_attr);
  return 0;
}

// ---------------------------------------------------------------------------
// texture

namespace {

// apply_boundary (Texture.swift:336-354): mode 0 wrap, 1 clamp, 2 zero.
inline int apply_boundary(int t, int size, int mode, float& oob) {
  if (mode == 2) {
    if (t < 0 || t >= size) { oob = 1.0f; return 0; }
    oob = 0.0f;
    return t;
  }
  if (mode == 1) {
    oob = 0.0f;
    return t < 0 ? 0 : (t >= size ? size - 1 : t);
  }
  oob = 0.0f;
  int r = t % size;
  if (r < 0) r += size;
  return r;
}

// float -> int of floor(x), defined for every float (saturating; NaN -> 0),
// matching the GPU's conversion so out-of-range coordinates agree.
inline int floor_to_int(float x) {
  float f = std::floor(x);
  if (!(f == f)) return 0;
  if (f >= 2147483520.0f) return 2147483647;
  if (f <= -2147483648.0f) return (-2147483647 - 1);
  return (int)f;
}

struct Level { const float* data; int H, W; };

struct Bilin {
  int ix0, ix1, iy0, iy1;
  float fx, fy;
  float ox0, ox1, oy0, oy1;
  float w00, w10, w01, w11;
};

// Bilinear taps with texel-centre convention tx = u*W - 0.5 (Texture.swift:372-391).
inline Bilin bilin(float u, float v, int Wk, int Hk, int mode) {
  Bilin b;
  float tx = u * (float)Wk - 0.5f;
  float ty = v * (float)Hk - 0.5f;
  int tx0 = floor_to_int(tx), ty0 = floor_to_int(ty);
  int tx1 = (int)((unsigned)tx0 + 1u), ty1 = (int)((unsigned)ty0 + 1u);
  b.fx = tx - (float)tx0;
  b.fy = ty - (float)ty0;
  b.ix0 = apply_boundary(tx0, Wk, mode, b.ox0);
  b.ix1 = apply_boundary(tx1, Wk, mode, b.ox1);
  b.iy0 = apply_boundary(ty0, Hk, mode, b.oy0);
  b.iy1 = apply_boundary(ty1, Hk, mode, b.oy1);
  float fx = b.fx, fy = b.fy;
  b.w00 = (1.0f - fx) * (1.0f - fy) * (1.0f - b.ox0) * (1.0f - b.oy0);
  b.w10 = (fx) * (1.0f - fy) * (1.0f - b.ox1) * (1.0f - b.oy0);
  b.w01 = (1.0f - fx) * (fy) * (1.0f - b.ox0) * (1.0f - b.oy1);
  b.w11 = (fx) * (fy) * (1.0f - b.ox1) * (1.0f - b.oy1);
  return b;
}

struct MipLayout {
  int L;
  int64_t off[64];
  int h[64], w[64];
  int64_t total;
};

// Level rule of textureConstructMip (Texture.swift:149-159).
MipLayout mip_layout(int Nt, int Ht, int Wt, int C, int max_level) {
  MipLayout m;
  m.L = 1;
  m.off[0] = -1; m.h[0] = Ht; m.w[0] = Wt;
  m.total = 0;
  int H = Ht, W = Wt;
  while (H >= 2 && W >= 2 && H % 2 == 0 && W % 2 == 0) {
    if (max_level >= 0 && m.L > max_level) break;
    if (m.L >= 32) break;
    H /= 2; W /= 2;
    m.off[m.L] = m.total; m.h[m.L] = H; m.w[m.L] = W;
    m.total += (int64_t)Nt * H * W * C;
    m.L++;
  }
  return m;
}

// 2^x and log2(x) in double, rounded once to float (the CUDA path does the
// same): the reference's float pow / log2 are not observable here, and the float
// library versions differ by an ulp between libraries.
inline float exp2_rn(float x) { return (float)std::exp2((double)x); }
inline float log2_rn(float x) { return (float)std::log2((double)x); }

// Per-pixel LOD block (Texture.swift:764-790).
struct Lod { int k0, k1; float frac; };
inline Lod lod_of(const float* da, int Ht, int Wt, int L, bool mip_linear) {
  float du_dx = da[0], du_dy = da[1], dv_dx = da[2], dv_dy = da[3];
  float sx = du_dx * (float)Wt, sy = du_dy * (float)Wt;
  float tx = dv_dx * (float)Ht, ty = dv_dy * (float)Ht;
  float rho_sq = std::fmax(sx * sx + tx * tx, sy * sy + ty * ty);
  float lod = 0.5f * log2_rn(std::fmax(rho_sq, 1e-20f));
  lod = std::fmax(0.0f, std::fmin((float)(L - 1), lod));
  Lod r;
  if (mip_linear) {
    r.k0 = floor_to_int(lod);
    r.k1 = r.k0 + 1;
    if (r.k1 >= L) r.k1 = L - 1;
    r.frac = lod - (float)r.k0;
  } else {
    r.k0 = floor_to_int(lod + 0.5f);
    if (r.k0 >= L) r.k0 = L - 1;
    r.k1 = r.k0;
    r.frac = 0.0f;
  }
  return r;
}

// Effective uvDA with the mipLevelBias / mipLevelBiasMap fold
// (Texture.swift:104-126): uvDA * 2^map * 2^bias.
inline void effective_da(const float* da4, int64_t pix, float bias, const float* bias_map,
                         float* eff, float* scale_out) {
  float s = 1.0f;
  bool scaled = false;
  if (bias_map) {
    s = exp2_rn(bias_map[pix]);
    if (bias != 0.0f) s = s * exp2_rn(bias);
    scaled = true;
  } else if (bias != 0.0f) {
    s = exp2_rn(bias);
    scaled = true;
  }
  for (int c = 0; c < 4; ++c) eff[c] = scaled ? da4[c] * s : da4[c];
  *scale_out = s;
}

// Cube projection (Texture.swift:616-636).
inline void cube_project(float x, float y, float z, int& face, float& u, float& v) {
  float ax = std::fabs(x), ay = std::fabs(y), az = std::fabs(z);
  float sc, tc, ma;
  if (ax >= ay && ax >= az) {
    ma = ax;
    if (x > 0.0f) { face = 0; sc = -z; tc = -y; } else { face = 1; sc = z; tc = -y; }
  } else if (ay >= az) {
    ma = ay;
    if (y > 0.0f) { face = 2; sc = x; tc = z; } else { face = 3; sc = x; tc = -z; }
  } else {
    ma = az;
    if (z > 0.0f) { face = 4; sc = x; tc = -y; } else { face = 5; sc = -x; tc = -y; }
  }
  float inv_ma = 1.0f / ma;
  u = (sc * inv_ma + 1.0f) * 0.5f;
  v = (tc * inv_ma + 1.0f) * 0.5f;
}

// Cube frame of a direction: the face and its (s, t, major) axes with their
// signs, as cube_project selects them, so that sc = s_sign * d[s_axis] etc.
struct CubeFrame {
  int face, sa, ta, ma;
  float ss, ts, ms, sc, tc, inv_ma;
  float u, v;  // face coordinates, exactly as cube_project returns them
};
inline CubeFrame cube_frame(const float* d) {
  static const int kAxes[6][3] = {{2, 1, 0}, {2, 1, 0}, {0, 2, 1}, {0, 2, 1}, {0, 1, 2}, {0, 1, 2}};
  static const float kSigns[6][3] = {{-1.f, -1.f, 1.f}, {1.f, -1.f, -1.f}, {1.f, 1.f, 1.f},
                                     {1.f, -1.f, -1.f}, {1.f, -1.f, 1.f}, {-1.f, -1.f, -1.f}};
  CubeFrame f;
  cube_project(d[0], d[1], d[2], f.face, f.u, f.v);
  f.sa = kAxes[f.face][0]; f.ta = kAxes[f.face][1]; f.ma = kAxes[f.face][2];
  f.ss = kSigns[f.face][0]; f.ts = kSigns[f.face][1]; f.ms = kSigns[f.face][2];
  f.sc = f.ss * d[f.sa];
  f.tc = f.ts * d[f.ta];
  f.inv_ma = 1.0f / (f.ms * d[f.ma]);
  return f;
}

// Screen-space derivatives of the face coordinates (u, v) from the
// direction's derivatives dd = [dx/dX, dx/dY, dy/dX, dy/dY, dz/dX, dz/dY]
// (interpolate's interleaved attribute-derivative layout):
//   u = (sc / ma + 1) / 2  =>  du = (dsc - (sc / ma) dma) / (2 ma).
// Output order matches uvDA: (du/dX, du/dY, dv/dX, dv/dY).  Extension (the
// reference's cube path samples level 0 only).
inline void cube_uv_da(const CubeFrame& f, const float* dd, float* e) {
  const float h = 0.5f * f.inv_ma;
  const float ks = (f.sc * f.inv_ma) * f.ms, kt = (f.tc * f.inv_ma) * f.ms;
  e[0] = h * (f.ss * dd[2 * f.sa] - ks * dd[2 * f.ma]);
  e[1] = h * (f.ss * dd[2 * f.sa + 1] - ks * dd[2 * f.ma + 1]);
  e[2] = h * (f.ts * dd[2 * f.ta] - kt * dd[2 * f.ma]);
  e[3] = h * (f.ts * dd[2 * f.ta + 1] - kt * dd[2 * f.ma + 1]);
}

// Transpose of cube_uv_da: g = d(loss)/d(du/dX, du/dY, dv/dX, dv/dY) ->
// d(loss)/d(dd).
inline void cube_uv_da_vjp(const CubeFrame& f, const float* g, float* dd) {
  const float h = 0.5f * f.inv_ma;
  const float ks = (f.sc * f.inv_ma) * f.ms, kt = (f.tc * f.inv_ma) * f.ms;
  dd[2 * f.sa] = g[0] * (h * f.ss);
  dd[2 * f.sa + 1] = g[1] * (h * f.ss);
  dd[2 * f.ta] = g[2] * (h * f.ts);
  dd[2 * f.ta + 1] = g[3] * (h * f.ts);
  dd[2 * f.ma] = -(g[0] * (h * ks) + g[2] * (h * kt));
  dd[2 * f.ma + 1] = -(g[1] * (h * ks) + g[3] * (h * kt));
}

// d(loss)/d(dir) through the face coordinates (extension; the reference's
// cube VJP returns zero, Texture.swift:196-197): u = (sc/ma + 1)/2, v alike,
// sc = ss d[sa], tc = ts d[ta], ma = ms d[ma].  d_u, d_v: d(loss)/d(u, v).
inline void cube_dir_vjp(const CubeFrame& f, float d_u, float d_v, float* dd) {
  const float h = 0.5f * f.inv_ma;
  dd[f.sa] = d_u * (h * f.ss);
  dd[f.ta] = d_v * (h * f.ts);
  dd[f.ma] = -((d_u * f.sc + d_v * f.tc) * (h * f.inv_ma)) * f.ms;
}

// The LOD's dependence on the direction: eff = s * cube_uv_da(dir, dirDA), so
// with G = d(loss)/d(eff) * s, add d(loss)/d(dir) of the four derivatives
// (Jacobian of cube_uv_da with respect to sc, tc and ma).
inline void cube_dir_lod_vjp(const CubeFrame& f, const float* dda, const float* G, float* dd) {
  const float a = f.inv_ma, a2 = a * a;
  const float Dsx = dda[2 * f.sa], Dsy = dda[2 * f.sa + 1];
  const float Dtx = dda[2 * f.ta], Dty = dda[2 * f.ta + 1];
  const float Dmx = dda[2 * f.ma], Dmy = dda[2 * f.ma + 1];
  const float gsm = G[0] * Dmx + G[1] * Dmy, gtm = G[2] * Dmx + G[3] * Dmy;
  const float gss = G[0] * Dsx + G[1] * Dsy, gtt = G[2] * Dtx + G[3] * Dty;
  const float hm = (0.5f * a2) * f.ms;
  dd[f.sa] += -(hm * f.ss) * gsm;
  dd[f.ta] += -(hm * f.ts) * gtm;
  dd[f.ma] += -(hm * (f.ss * gss + f.ts * gtt)) + (a2 * a) * (f.sc * gsm + f.tc * gtm);
}

void build_pyramid(const float* tex, int Nt, int C, const MipLayout& m, float* pyr, int nthreads) {
  for (int k = 1; k < m.L; ++k) {
    const float* src = (k == 1) ? tex : pyr + m.off[k - 1];
    int Hs = m.h[k - 1], Ws = m.w[k - 1];
    int Hd = m.h[k], Wd = m.w[k];
    float* dst = pyr + m.off[k];
    int64_t n_out = (int64_t)Nt * Hd * Wd * C;
    parallel_for(n_out, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t i = b; i < e; ++i) {
        int c = (int)(i % C);
        int x = (int)((i / C) % Wd);
        int y = (int)((i / ((int64_t)C * Wd)) % Hd);
        int n = (int)(i / ((int64_t)C * Wd * Hd));
        const float* s = src + (int64_t)n * Hs * Ws * C;
        float a = s[((int64_t)(2 * y) * Ws + 2 * x) * C + c];
        float bb = s[((int64_t)(2 * y) * Ws + 2 * x + 1) * C + c];
        float cc = s[((int64_t)(2 * y + 1) * Ws + 2 * x) * C + c];
        float d = s[((int64_t)(2 * y + 1) * Ws + 2 * x + 1) * C + c];
        dst[i] = ((a + bb) + (cc + d)) * 0.25f;
      }
    });
  }
}


// K22 (Texture.swift:1011-1102): d(loss)/d(eff) for the effective uvDA `eff`
// through the LOD, independent of MIP_LINEAR.  `img` selects the image (the
// texture batch entry, or batch * 6 + face for a cube) in every level.
void lod_vjp(const float* eff, const MipLayout& m, const float* tex, const float* pyr, int64_t img, int C,
             float u, float v, int boundary, const float* g, float* g4) {
  const int Ht = m.h[0], Wt = m.w[0];
  float du_dx = eff[0], du_dy = eff[1], dv_dx = eff[2], dv_dy = eff[3];
  float sx = du_dx * (float)Wt, sy = du_dy * (float)Wt;
  float tx_ = dv_dx * (float)Ht, ty_ = dv_dy * (float)Ht;
  float Asq = sx * sx + tx_ * tx_, Bsq = sy * sy + ty_ * ty_;
  float rho_sq = std::fmax(Asq, Bsq);
  float lod_raw = 0.5f * log2_rn(std::fmax(rho_sq, 1e-20f));
  for (int c = 0; c < 4; ++c) g4[c] = 0.0f;
  if (lod_raw <= 0.0f || lod_raw >= (float)(m.L - 1)) return;
  int k0 = floor_to_int(lod_raw);
  int k1 = k0 + 1;
  if (k1 >= m.L) k1 = m.L - 1;
  float d_lod = 0.0f;
  for (int li = 0; li < 2; ++li) {
    int k = li == 0 ? k0 : k1;
    float sign = li == 0 ? -1.0f : 1.0f;
    int Hk = m.h[k], Wk = m.w[k];
    const float* lb = (k == 0 ? tex : pyr + m.off[k]) + img * Hk * Wk * C;
    Bilin bl = bilin(u, v, Wk, Hk, boundary);
    for (int c = 0; c < C; ++c) {
      float t00 = lb[((int64_t)bl.iy0 * Wk + bl.ix0) * C + c];
      float t10 = lb[((int64_t)bl.iy0 * Wk + bl.ix1) * C + c];
      float t01 = lb[((int64_t)bl.iy1 * Wk + bl.ix0) * C + c];
      float t11 = lb[((int64_t)bl.iy1 * Wk + bl.ix1) * C + c];
      float sample = bl.w00 * t00 + bl.w10 * t10 + bl.w01 * t01 + bl.w11 * t11;
      d_lod += sign * sample * g[c];
    }
  }
  float ln2 = 0.6931471805599453f;
  float dlod_drho_sq = 1.0f / (2.0f * rho_sq * ln2);
  float A_is_max = (Asq >= Bsq) ? 1.0f : 0.0f;
  float B_is_max = 1.0f - A_is_max;
  g4[0] = d_lod * dlod_drho_sq * A_is_max * 2.0f * sx * (float)Wt;
  g4[1] = d_lod * dlod_drho_sq * B_is_max * 2.0f * sy * (float)Wt;
  g4[2] = d_lod * dlod_drho_sq * A_is_max * 2.0f * tx_ * (float)Ht;
  g4[3] = d_lod * dlod_drho_sq * B_is_max * 2.0f * ty_ * (float)Ht;
}

// Adjoint of the pyramid build: fold level gradients into level 0,
// d_{k-1} += upsample(d_k) / 4, coarsest first.  dall = [level 0 | levels >= 1].
void fold_pyramid(float* dall, int64_t l0, const MipLayout& m, int Nimg, int C) {
  for (int k = m.L - 1; k >= 1; --k) {
    float* dk = dall + l0 + m.off[k];
    float* dp = (k == 1) ? dall : dall + l0 + m.off[k - 1];
    int Hd = m.h[k], Wd = m.w[k], Ws = m.w[k - 1];
    for (int n = 0; n < Nimg; ++n)
      for (int y = 0; y < Hd; ++y)
        for (int x = 0; x < Wd; ++x)
          for (int c = 0; c < C; ++c) {
            float g = dk[(((int64_t)n * Hd + y) * Wd + x) * C + c] * 0.25f;
            int64_t pb = (int64_t)n * m.h[k - 1] * Ws;
            dp[(pb + (int64_t)(2 * y) * Ws + 2 * x) * C + c] += g;
            dp[(pb + (int64_t)(2 * y) * Ws + 2 * x + 1) * C + c] += g;
            dp[(pb + (int64_t)(2 * y + 1) * Ws + 2 * x) * C + c] += g;
            dp[(pb + (int64_t)(2 * y + 1) * Ws + 2 * x + 1) * C + c] += g;
          }
  }
}

}  // namespace

extern "C" int orc_texture_mip_layout(int Nt, int Ht, int Wt, int C, int max_level,
                                      int* num_levels, int64_t* level_offset,
                                      int* level_h, int* level_w, int64_t* total) {
  MipLayout m = mip_layout(Nt, Ht, Wt, C, max_level);
  *num_levels = m.L;
  for (int k = 0; k < m.L; ++k) {
    level_offset[k] = m.off[k];
    level_h[k] = m.h[k];
    level_w[k] = m.w[k];
  }
  *total = m.total;
  return 0;
}

// textureConstructMip (Texture.swift:144-161): mean of each 2x2 block.  MLX's
// reduction order is not observable here; the restatement sums
// ((t00 + t01) + (t10 + t11)) / 4.
extern "C" int orc_texture_construct_mip(const float* tex, int Nt, int Ht, int Wt, int C,
                                         int max_level, float* pyramid, int nthreads) {
  MipLayout m = mip_layout(Nt, Ht, Wt, C, max_level);
  build_pyramid(tex, Nt, C, m, pyramid, nthreads);
  return 0;
}

// K12 _fwd, K15 _nearest_fwd, K17 _cube_fwd, K19 _trilinear_fwd
// (Texture.swift:359-403, 545-572, 638-684, 795-863).
extern "C" int orc_texture_fwd(int filter, int boundary, const float* tex, int Nt, int Ht,
                               int Wt, int C, int max_level, const float* uv,
                               const float* uv_da, float bias, const float* bias_map, int N,
                               int Hi, int Wi, float* out, int nthreads) {
  int64_t P = (int64_t)N * Hi * Wi;
  if (boundary == 3 && (filter == 2 || filter == 3)) {
    // Mipmapped cube (extension): the pyramid of the Nt * 6 faces, LOD from
    // the face-coordinate derivatives, per-level per-face clamp bilinear.
    if (!uv_da) return 1;
    MipLayout m = mip_layout(Nt * 6, Ht, Wt, C, max_level);
    std::vector<float> pyr((size_t)std::max<int64_t>(m.total, 1));
    build_pyramid(tex, Nt * 6, C, m, pyr.data(), nthreads);
    bool mip_linear = (filter == 3);
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        CubeFrame f = cube_frame(uv + pix * 3);
        int64_t img = (int64_t)(Nt == 1 ? 0 : pn) * 6 + f.face;
        float da4[4], eff[4], s;
        cube_uv_da(f, uv_da + pix * 6, da4);
        effective_da(da4, pix, bias, bias_map, eff, &s);
        Lod ld = lod_of(eff, Ht, Wt, m.L, mip_linear);
        for (int li = 0; li < 2; ++li) {
          int k = li == 0 ? ld.k0 : ld.k1;
          int Hk = m.h[k], Wk = m.w[k];
          const float* lb = (k == 0 ? tex : pyr.data() + m.off[k]) + img * Hk * Wk * C;
          Bilin bl = bilin(f.u, f.v, Wk, Hk, 1);
          for (int c = 0; c < C; ++c) {
            float t00 = lb[((int64_t)bl.iy0 * Wk + bl.ix0) * C + c];
            float t10 = lb[((int64_t)bl.iy0 * Wk + bl.ix1) * C + c];
            float t01 = lb[((int64_t)bl.iy1 * Wk + bl.ix0) * C + c];
            float t11 = lb[((int64_t)bl.iy1 * Wk + bl.ix1) * C + c];
            float sample = bl.w00 * t00 + bl.w10 * t10 + bl.w01 * t01 + bl.w11 * t11;
            if (li == 0) out[pix * C + c] = (1.0f - ld.frac) * sample;
            else out[pix * C + c] += ld.frac * sample;
          }
        }
      }
    });
    return 0;
  }
  if (boundary == 3) {
    if (filter != 1) return 1;
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        const float* d = uv + pix * 3;
        int face; float u, v;
        cube_project(d[0], d[1], d[2], face, u, v);
        Bilin bl = bilin(u, v, Wt, Ht, 1);
        float w00 = (1.0f - bl.fx) * (1.0f - bl.fy), w10 = bl.fx * (1.0f - bl.fy);
        float w01 = (1.0f - bl.fx) * bl.fy, w11 = bl.fx * bl.fy;
        const float* fb = tex + ((int64_t)(Nt == 1 ? 0 : pn) * 6 + face) * Ht * Wt * C;
        for (int c = 0; c < C; ++c) {
          float t00 = fb[((int64_t)bl.iy0 * Wt + bl.ix0) * C + c];
          float t10 = fb[((int64_t)bl.iy0 * Wt + bl.ix1) * C + c];
          float t01 = fb[((int64_t)bl.iy1 * Wt + bl.ix0) * C + c];
          float t11 = fb[((int64_t)bl.iy1 * Wt + bl.ix1) * C + c];
          out[pix * C + c] = w00 * t00 + w10 * t10 + w01 * t01 + w11 * t11;
        }
      }
    });
    return 0;
  }
  if (filter == 0) {
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        float u = uv[pix * 2], v = uv[pix * 2 + 1];
        int tx = floor_to_int(u * (float)Wt), ty = floor_to_int(v * (float)Ht);
        float ox, oy;
        int ix = apply_boundary(tx, Wt, boundary, ox), iy = apply_boundary(ty, Ht, boundary, oy);
        float mask = (1.0f - ox) * (1.0f - oy);
        const float* tb = tex + (int64_t)(Nt == 1 ? 0 : pn) * Ht * Wt * C;
        for (int c = 0; c < C; ++c) out[pix * C + c] = tb[((int64_t)iy * Wt + ix) * C + c] * mask;
      }
    });
    return 0;
  }
  if (filter == 1) {
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        Bilin bl = bilin(uv[pix * 2], uv[pix * 2 + 1], Wt, Ht, boundary);
        const float* tb = tex + (int64_t)(Nt == 1 ? 0 : pn) * Ht * Wt * C;
        for (int c = 0; c < C; ++c) {
          float t00 = tb[((int64_t)bl.iy0 * Wt + bl.ix0) * C + c];
          float t10 = tb[((int64_t)bl.iy0 * Wt + bl.ix1) * C + c];
          float t01 = tb[((int64_t)bl.iy1 * Wt + bl.ix0) * C + c];
          float t11 = tb[((int64_t)bl.iy1 * Wt + bl.ix1) * C + c];
          out[pix * C + c] = bl.w00 * t00 + bl.w10 * t10 + bl.w01 * t01 + bl.w11 * t11;
        }
      }
    });
    return 0;
  }
  // mipmap filters
  if (!uv_da) return 1;
  MipLayout m = mip_layout(Nt, Ht, Wt, C, max_level);
  std::vector<float> pyr((size_t)std::max<int64_t>(m.total, 1));
  build_pyramid(tex, Nt, C, m, pyr.data(), nthreads);
  bool mip_linear = (filter == 3);
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
    for (int64_t pix = b; pix < e; ++pix) {
      int pn = (int)(pix / ((int64_t)Hi * Wi));
      int nt = (Nt == 1 ? 0 : pn);
      float eff[4], s;
      effective_da(uv_da + pix * 4, pix, bias, bias_map, eff, &s);
      Lod ld = lod_of(eff, Ht, Wt, m.L, mip_linear);
      float u = uv[pix * 2], v = uv[pix * 2 + 1];
      for (int li = 0; li < 2; ++li) {
        int k = li == 0 ? ld.k0 : ld.k1;
        int Hk = m.h[k], Wk = m.w[k];
        const float* lb = (k == 0 ? tex : pyr.data() + m.off[k]) + (int64_t)nt * Hk * Wk * C;
        Bilin bl = bilin(u, v, Wk, Hk, boundary);
        for (int c = 0; c < C; ++c) {
          float t00 = lb[((int64_t)bl.iy0 * Wk + bl.ix0) * C + c];
          float t10 = lb[((int64_t)bl.iy0 * Wk + bl.ix1) * C + c];
          float t01 = lb[((int64_t)bl.iy1 * Wk + bl.ix0) * C + c];
          float t11 = lb[((int64_t)bl.iy1 * Wk + bl.ix1) * C + c];
          float sample = bl.w00 * t00 + bl.w10 * t10 + bl.w01 * t01 + bl.w11 * t11;
          if (li == 0) out[pix * C + c] = (1.0f - ld.frac) * sample;
          else out[pix * C + c] += ld.frac * sample;
        }
      }
    }
  });
  return 0;
}

// VJPs: K13/K14 (Texture.swift:407-521), K16 (576-605), K18 (686-738),
// K20-K22 (870-1102), plus the autograd of the pyramid build, folded to level 0.
extern "C" int orc_texture_bwd(int filter, int boundary, const float* tex, int Nt, int Ht,
                               int Wt, int C, int max_level, const float* uv,
                               const float* uv_da, float bias, const float* bias_map, int N,
                               int Hi, int Wi, const float* d_out, float* d_tex, float* d_uv,
                               float* d_uv_da, float* d_bias_map, int nthreads) {
  int64_t P = (int64_t)N * Hi * Wi;
  // Flag bits above the boundary mode: 0x100 = the d_dir chain rule for cube
  // textures (extension; the reference returns d_dir = 0).
  const int flags = boundary & ~0xff;
  boundary &= 0xff;
  const bool dir_grad = (flags & 0x100) != 0;
  if ((flags & ~0x100) != 0 || (dir_grad && boundary != 3)) return 1;
  if (boundary == 3 && (filter == 2 || filter == 3)) {
    // Mipmapped cube VJP (extension): d_tex through the pyramid of the
    // Nt * 6 faces, d_dir = 0 as the reference's cube VJP, d_dirDA through
    // the LOD (K22's d(eff) mapped back through cube_uv_da).
    if (!uv_da) return 1;
    const int Nf = Nt * 6;
    MipLayout m = mip_layout(Nf, Ht, Wt, C, max_level);
    std::vector<float> pyr((size_t)std::max<int64_t>(m.total, 1));
    build_pyramid(tex, Nf, C, m, pyr.data(), nthreads);
    bool mip_linear = (filter == 3);
    int64_t l0 = (int64_t)Nf * Ht * Wt * C;
    Accum acc(nthreads, (size_t)(l0 + m.total));
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
      double* dt = acc.get(tid);
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        CubeFrame f = cube_frame(uv + pix * 3);
        int64_t img = (int64_t)(Nt == 1 ? 0 : pn) * 6 + f.face;
        float da4[4], eff[4], s;
        cube_uv_da(f, uv_da + pix * 6, da4);
        effective_da(da4, pix, bias, bias_map, eff, &s);
        Lod ld = lod_of(eff, Ht, Wt, m.L, mip_linear);
        float d_u = 0.0f, d_v = 0.0f;
        for (int li = 0; li < 2; ++li) {
          int k = li == 0 ? ld.k0 : ld.k1;
          float scale = li == 0 ? (1.0f - ld.frac) : ld.frac;
          int Hk = m.h[k], Wk = m.w[k];
          int64_t lvl_off = (k == 0 ? 0 : l0 + m.off[k]) + img * Hk * Wk * C;
          const float* lb = (k == 0 ? tex : pyr.data() + m.off[k]) + img * Hk * Wk * C;
          Bilin bl = bilin(f.u, f.v, Wk, Hk, 1);
          float dfx = 0.0f, dfy = 0.0f;
          for (int c = 0; c < C; ++c) {
            float g = d_out[pix * C + c] * scale;
            int64_t a00 = ((int64_t)bl.iy0 * Wk + bl.ix0) * C + c, a10 = ((int64_t)bl.iy0 * Wk + bl.ix1) * C + c;
            int64_t a01 = ((int64_t)bl.iy1 * Wk + bl.ix0) * C + c, a11 = ((int64_t)bl.iy1 * Wk + bl.ix1) * C + c;
            dt[lvl_off + a00] += (double)(bl.w00 * g);
            dt[lvl_off + a10] += (double)(bl.w10 * g);
            dt[lvl_off + a01] += (double)(bl.w01 * g);
            dt[lvl_off + a11] += (double)(bl.w11 * g);
            if (dir_grad) {
              dfx += g * ((1.0f - bl.fy) * (lb[a10] - lb[a00]) + bl.fy * (lb[a11] - lb[a01]));
              dfy += g * ((1.0f - bl.fx) * (lb[a01] - lb[a00]) + bl.fx * (lb[a11] - lb[a10]));
            }
          }
          d_u += dfx * (float)Wk;
          d_v += dfy * (float)Hk;
        }
        float* dd = d_uv + pix * 3;
        if (dir_grad) cube_dir_vjp(f, d_u, d_v, dd);
        else for (int c = 0; c < 3; ++c) dd[c] = 0.0f;
        float g4[4];
        lod_vjp(eff, m, tex, pyr.data(), img, C, f.u, f.v, 1, d_out + pix * C, g4);
        float gs[4] = {g4[0] * s, g4[1] * s, g4[2] * s, g4[3] * s};
        if (dir_grad) cube_dir_lod_vjp(f, uv_da + pix * 6, gs, dd);
        if (d_uv_da) cube_uv_da_vjp(f, gs, d_uv_da + pix * 6);
        if (d_bias_map) {
          float acc_m = 0.0f;
          for (int c = 0; c < 4; ++c) acc_m += g4[c] * eff[c];
          d_bias_map[pix] = bias_map ? acc_m * 0.6931471805599453f : 0.0f;
        }
      }
    });
    size_t tot = (size_t)(l0 + m.total);
    std::vector<float> dall(tot);
    acc.reduce_to(dall.data());
    fold_pyramid(dall.data(), l0, m, Nf, C);
    std::memcpy(d_tex, dall.data(), sizeof(float) * (size_t)l0);
    return 0;
  }
  if (boundary == 3) {
    if (filter != 1) return 1;
    Accum acc(nthreads, (size_t)Nt * 6 * Ht * Wt * C);
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
      double* dt = acc.get(tid);
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        const float* d = uv + pix * 3;
        CubeFrame f = cube_frame(d);
        Bilin bl = bilin(f.u, f.v, Wt, Ht, 1);
        float w00 = (1.0f - bl.fx) * (1.0f - bl.fy), w10 = bl.fx * (1.0f - bl.fy);
        float w01 = (1.0f - bl.fx) * bl.fy, w11 = bl.fx * bl.fy;
        const int64_t fo = ((int64_t)(Nt == 1 ? 0 : pn) * 6 + f.face) * Ht * Wt * C;
        double* fb = dt + fo;
        const float* tb = tex + fo;
        float dfx = 0.0f, dfy = 0.0f;
        for (int c = 0; c < C; ++c) {
          float g = d_out[pix * C + c];
          int64_t a00 = ((int64_t)bl.iy0 * Wt + bl.ix0) * C + c, a10 = ((int64_t)bl.iy0 * Wt + bl.ix1) * C + c;
          int64_t a01 = ((int64_t)bl.iy1 * Wt + bl.ix0) * C + c, a11 = ((int64_t)bl.iy1 * Wt + bl.ix1) * C + c;
          fb[a00] += (double)(w00 * g);
          fb[a10] += (double)(w10 * g);
          fb[a01] += (double)(w01 * g);
          fb[a11] += (double)(w11 * g);
          if (dir_grad) {
            dfx += g * ((1.0f - bl.fy) * (tb[a10] - tb[a00]) + bl.fy * (tb[a11] - tb[a01]));
            dfy += g * ((1.0f - bl.fx) * (tb[a01] - tb[a00]) + bl.fx * (tb[a11] - tb[a10]));
          }
        }
        if (dir_grad) cube_dir_vjp(f, dfx * (float)Wt, dfy * (float)Ht, d_uv + pix * 3);
        else for (int c = 0; c < 3; ++c) d_uv[pix * 3 + c] = 0.0f;
      }
    });
    acc.reduce_to(d_tex);
    return 0;
  }
  if (filter == 0) {
    Accum acc(nthreads, (size_t)Nt * Ht * Wt * C);
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
      double* dt = acc.get(tid);
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        float u = uv[pix * 2], v = uv[pix * 2 + 1];
        int tx = floor_to_int(u * (float)Wt), ty = floor_to_int(v * (float)Ht);
        float ox, oy;
        int ix = apply_boundary(tx, Wt, boundary, ox), iy = apply_boundary(ty, Ht, boundary, oy);
        float mask = (1.0f - ox) * (1.0f - oy);
        double* tb = dt + (int64_t)(Nt == 1 ? 0 : pn) * Ht * Wt * C;
        for (int c = 0; c < C; ++c) tb[((int64_t)iy * Wt + ix) * C + c] += (double)(d_out[pix * C + c] * mask);
        d_uv[pix * 2] = 0.0f;
        d_uv[pix * 2 + 1] = 0.0f;
      }
    });
    acc.reduce_to(d_tex);
    return 0;
  }
  if (filter == 1) {
    Accum acc(nthreads, (size_t)Nt * Ht * Wt * C);
    parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
      double* dt = acc.get(tid);
      for (int64_t pix = b; pix < e; ++pix) {
        int pn = (int)(pix / ((int64_t)Hi * Wi));
        Bilin bl = bilin(uv[pix * 2], uv[pix * 2 + 1], Wt, Ht, boundary);
        const float* tb = tex + (int64_t)(Nt == 1 ? 0 : pn) * Ht * Wt * C;
        double* db = dt + (int64_t)(Nt == 1 ? 0 : pn) * Ht * Wt * C;
        float m00 = (1.0f - bl.ox0) * (1.0f - bl.oy0), m10 = (1.0f - bl.ox1) * (1.0f - bl.oy0);
        float m01 = (1.0f - bl.ox0) * (1.0f - bl.oy1), m11 = (1.0f - bl.ox1) * (1.0f - bl.oy1);
        float dfx_sum = 0.0f, dfy_sum = 0.0f;
        float fx = bl.fx, fy = bl.fy;
        for (int c = 0; c < C; ++c) {
          float g = d_out[pix * C + c];
          int64_t a00 = ((int64_t)bl.iy0 * Wt + bl.ix0) * C + c, a10 = ((int64_t)bl.iy0 * Wt + bl.ix1) * C + c;
          int64_t a01 = ((int64_t)bl.iy1 * Wt + bl.ix0) * C + c, a11 = ((int64_t)bl.iy1 * Wt + bl.ix1) * C + c;
          db[a00] += (double)(bl.w00 * g);
          db[a10] += (double)(bl.w10 * g);
          db[a01] += (double)(bl.w01 * g);
          db[a11] += (double)(bl.w11 * g);
          float t00 = tb[a00] * m00, t10 = tb[a10] * m10, t01 = tb[a01] * m01, t11 = tb[a11] * m11;
          dfx_sum += g * ((1.0f - fy) * (t10 - t00) + fy * (t11 - t01));
          dfy_sum += g * ((1.0f - fx) * (t01 - t00) + fx * (t11 - t10));
        }
        d_uv[pix * 2 + 0] = dfx_sum * (float)Wt;
        d_uv[pix * 2 + 1] = dfy_sum * (float)Ht;
      }
    });
    acc.reduce_to(d_tex);
    return 0;
  }
  // mipmap filters
  if (!uv_da) return 1;
  MipLayout m = mip_layout(Nt, Ht, Wt, C, max_level);
  std::vector<float> pyr((size_t)std::max<int64_t>(m.total, 1));
  build_pyramid(tex, Nt, C, m, pyr.data(), nthreads);
  bool mip_linear = (filter == 3);
  int64_t l0 = (int64_t)Nt * Ht * Wt * C;
  Accum acc(nthreads, (size_t)(l0 + m.total));  // [level0 | pyramid levels]
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
    double* dt = acc.get(tid);
    for (int64_t pix = b; pix < e; ++pix) {
      int pn = (int)(pix / ((int64_t)Hi * Wi));
      int nt = (Nt == 1 ? 0 : pn);
      float eff[4], s;
      effective_da(uv_da + pix * 4, pix, bias, bias_map, eff, &s);
      Lod ld = lod_of(eff, Ht, Wt, m.L, mip_linear);
      float u = uv[pix * 2], v = uv[pix * 2 + 1];
      float dfx_sum_total = 0.0f, dfy_sum_total = 0.0f;
      for (int li = 0; li < 2; ++li) {
        int k = li == 0 ? ld.k0 : ld.k1;
        float scale = li == 0 ? (1.0f - ld.frac) : ld.frac;
        int Hk = m.h[k], Wk = m.w[k];
        int64_t lvl_off = (k == 0 ? 0 : l0 + m.off[k]) + (int64_t)nt * Hk * Wk * C;
        const float* lb = (k == 0 ? tex : pyr.data() + m.off[k]) + (int64_t)nt * Hk * Wk * C;
        Bilin bl = bilin(u, v, Wk, Hk, boundary);
        float m00 = (1.0f - bl.ox0) * (1.0f - bl.oy0), m10 = (1.0f - bl.ox1) * (1.0f - bl.oy0);
        float m01 = (1.0f - bl.ox0) * (1.0f - bl.oy1), m11 = (1.0f - bl.ox1) * (1.0f - bl.oy1);
        float dfx_level = 0.0f, dfy_level = 0.0f;
        float fx = bl.fx, fy = bl.fy;
        for (int c = 0; c < C; ++c) {
          float g = d_out[pix * C + c] * scale;
          int64_t a00 = ((int64_t)bl.iy0 * Wk + bl.ix0) * C + c, a10 = ((int64_t)bl.iy0 * Wk + bl.ix1) * C + c;
          int64_t a01 = ((int64_t)bl.iy1 * Wk + bl.ix0) * C + c, a11 = ((int64_t)bl.iy1 * Wk + bl.ix1) * C + c;
          dt[lvl_off + a00] += (double)(bl.w00 * g);
          dt[lvl_off + a10] += (double)(bl.w10 * g);
          dt[lvl_off + a01] += (double)(bl.w01 * g);
          dt[lvl_off + a11] += (double)(bl.w11 * g);
          float t00 = lb[a00] * m00, t10 = lb[a10] * m10, t01 = lb[a01] * m01, t11 = lb[a11] * m11;
          dfx_level += g * ((1.0f - fy) * (t10 - t00) + fy * (t11 - t01));
          dfy_level += g * ((1.0f - fx) * (t01 - t00) + fx * (t11 - t10));
        }
        dfx_sum_total += dfx_level * (float)Wk;
        dfy_sum_total += dfy_level * (float)Hk;
      }
      d_uv[pix * 2 + 0] = dfx_sum_total;
      d_uv[pix * 2 + 1] = dfy_sum_total;

      // K22 d_uvDA (Texture.swift:1011-1102): independent of MIP_LINEAR.
      float g4[4];
      lod_vjp(eff, m, tex, pyr.data(), nt, C, u, v, boundary, d_out + pix * C, g4);
      // Backward of eff = uvDA * s: d_uvDA = g * s; d_map = ln2 * sum(g * eff).
      if (d_uv_da)
        for (int c = 0; c < 4; ++c) d_uv_da[pix * 4 + c] = g4[c] * s;
      if (d_bias_map) {
        float acc_m = 0.0f;
        for (int c = 0; c < 4; ++c) acc_m += g4[c] * eff[c];
        d_bias_map[pix] = bias_map ? acc_m * 0.6931471805599453f : 0.0f;
      }
    }
  });
  size_t tot = (size_t)(l0 + m.total);
  std::vector<float> dall(tot);
  acc.reduce_to(dall.data());
  fold_pyramid(dall.data(), l0, m, Nt, C);
  std::memcpy(d_tex, dall.data(), sizeof(float) * (size_t)l0);
  return 0;
}

// ---------------------------------------------------------------------------
// antialias

// antialiasConstructTopologyHash (Antialias.swift:19-66).
extern "C" int orc_topology_hash(const int32_t* tri, int T, int32_t* topo) {
  struct E { int32_t a, b; int t, k; };
  std::vector<E> edges;
  edges.reserve((size_t)T * 3);
  for (int t = 0; t < T; ++t) {
    int32_t v0 = tri[t * 3], v1 = tri[t * 3 + 1], v2 = tri[t * 3 + 2];
    int32_t pr[3][2] = {{v1, v2}, {v2, v0}, {v0, v1}};
    for (int k = 0; k < 3; ++k)
      edges.push_back({std::min(pr[k][0], pr[k][1]), std::max(pr[k][0], pr[k][1]), t, k});
  }
  std::stable_sort(edges.begin(), edges.end(), [](const E& l, const E& r) {
    return l.a != r.a ? l.a < r.a : l.b < r.b;
  });
  for (int i = 0; i < T * 3; ++i) topo[i] = -1;
  size_t i = 0;
  while (i < edges.size()) {
    size_t j = i + 1;
    while (j < edges.size() && edges[j].a == edges[i].a && edges[j].b == edges[i].b) ++j;
    size_t run = j - i;
    if (run == 2) {
      topo[edges[i].t * 3 + edges[i].k] = edges[i + 1].t;
      topo[edges[i + 1].t * 3 + edges[i + 1].k] = edges[i].t;
    } else if (run > 2) {
      for (size_t q = i; q < j; ++q) topo[edges[q].t * 3 + edges[q].k] = -2;
    }
    i = j;
  }
  return 0;
}

namespace {

struct Sil {
  float alpha[4];
  bool active[4];
  int64_t nbase[4];  // neighbour pixel index
  int ie0[4], ie1[4];
  float e0x[4], e0y[4], e1x[4], e1y[4], t[4], denom[4], dadxy[4];
  bool horiz[4];
  float alpha_sum;
};

inline int rast_tri(const float* rast, int64_t pix, int T) {
  int t = (int)rast[pix * 4 + 3] - 1;
  return (t >= T) ? -1 : t;
}

// silhouetteBlock (Antialias.swift:168-326).
void silhouette(const float* rast, const float* pos, const int32_t* tri, const int32_t* topo,
                int H, int W, int V, int T, int pn, int ph, int pw, Sil& s) {
  int64_t pix = ((int64_t)pn * H + ph) * W + pw;
  int tri_p = rast_tri(rast, pix, T);
  int64_t pos_n_base = (int64_t)pn * V * 4;
  s.alpha_sum = 0.0f;
  for (int d = 0; d < 4; ++d) { s.alpha[d] = 0.0f; s.active[d] = false; }
  for (int dir = 0; dir < 4; ++dir) {
    int dh = 0, dw = 0;
    if (dir == 0) dw = 1;
    else if (dir == 1) dh = 1;
    else if (dir == 2) dw = -1;
    else dh = -1;
    int nh = ph + dh, nw = pw + dw;
    if (nh < 0 || nh >= H || nw < 0 || nw >= W) continue;
    int64_t npix = ((int64_t)pn * H + nh) * W + nw;
    int tri_n = rast_tri(rast, npix, T);
    if (tri_p == tri_n) continue;
    if (tri_p < 0 && tri_n < 0) continue;
    int fg_tri, target;
    if (tri_p >= 0 && tri_n >= 0) {
      int k_at_p = -1;
      if (topo[tri_p * 3 + 0] == tri_n) k_at_p = 0;
      else if (topo[tri_p * 3 + 1] == tri_n) k_at_p = 1;
      else if (topo[tri_p * 3 + 2] == tri_n) k_at_p = 2;
      if (k_at_p < 0) continue;
      fg_tri = tri_p; target = tri_n;
    } else if (tri_p >= 0) {
      fg_tri = tri_p; target = -1;
    } else {
      fg_tri = tri_n; target = -1;
    }
    int i_e0 = -1, i_e1 = -1;
    float e0x = 0, e0y = 0, e1x = 0, e1y = 0;
    {
      float pcx = (float)pw + 0.5f, pcy = (float)ph + 0.5f;
      float ncx = (float)nw + 0.5f, ncy = (float)nh + 0.5f;
      int k_sel = -1;
      for (int kk = 0; kk < 3; ++kk) {
        if (topo[fg_tri * 3 + kk] != target) continue;
        int a = tri[fg_tri * 3 + ((kk + 1) % 3)];
        int b = tri[fg_tri * 3 + ((kk + 2) % 3)];
        if (a < 0 || a >= V || b < 0 || b >= V) continue;
        const float* pa = pos + pos_n_base + (int64_t)a * 4;
        const float* pb = pos + pos_n_base + (int64_t)b * 4;
        float wc0 = pa[3], wc1 = pb[3];
        float E0x = (pa[0] / wc0 + 1.0f) * (float)W * 0.5f;
        float E0y = (1.0f - pa[1] / wc0) * (float)H * 0.5f;
        float E1x = (pb[0] / wc1 + 1.0f) * (float)W * 0.5f;
        float E1y = (1.0f - pb[1] / wc1) * (float)H * 0.5f;
        float ex = E1x - E0x, ey = E1y - E0y;
        float side_p = ex * (pcy - E0y) - ey * (pcx - E0x);
        float side_n = ex * (ncy - E0y) - ey * (ncx - E0x);
        if (side_p * side_n < 0.0f) {
          k_sel = kk; i_e0 = a; i_e1 = b;
          e0x = E0x; e0y = E0y; e1x = E1x; e1y = E1y;
          break;
        }
      }
      if (k_sel < 0) continue;
    }
    float beta = 0.0f, t_val = 0.0f, denom = 0.0f, dbeta = 0.0f;
    bool is_horiz = (dh == 0);
    float p_center_x = (float)pw + 0.5f, p_center_y = (float)ph + 0.5f;
    if (is_horiz) {
      float dyv = e1y - e0y;
      denom = dyv;
      if (std::fabs(dyv) >= 1e-7f) {
        float tval = (p_center_y - e0y) / dyv;
        t_val = tval;
        if (tval >= 0.0f && tval <= 1.0f) {
          float xe = e0x + tval * (e1x - e0x);
          if (xe > (float)pw && xe < (float)(pw + 1)) {
            float d = xe - p_center_x;
            beta = 0.5f - std::fabs(d);
            dbeta = (d > 0.0f) ? -1.0f : 1.0f;
          }
        }
      }
    } else {
      float dxv = e1x - e0x;
      denom = dxv;
      if (std::fabs(dxv) >= 1e-7f) {
        float tval = (p_center_x - e0x) / dxv;
        t_val = tval;
        if (tval >= 0.0f && tval <= 1.0f) {
          float ye = e0y + tval * (e1y - e0y);
          if (ye > (float)ph && ye < (float)(ph + 1)) {
            float d = ye - p_center_y;
            beta = 0.5f - std::fabs(d);
            dbeta = (d > 0.0f) ? -1.0f : 1.0f;
          }
        }
      }
    }
    if (beta <= 0.0f) continue;
    s.alpha[dir] = beta;
    s.nbase[dir] = npix;
    s.active[dir] = true;
    s.alpha_sum += beta;
    s.ie0[dir] = i_e0; s.ie1[dir] = i_e1;
    s.e0x[dir] = e0x; s.e0y[dir] = e0y; s.e1x[dir] = e1x; s.e1y[dir] = e1y;
    s.t[dir] = t_val; s.denom[dir] = denom; s.dadxy[dir] = dbeta; s.horiz[dir] = is_horiz;
  }
}

}  // namespace

// K23 diffrast_antialias_fwd (Antialias.swift:333-358).
extern "C" int orc_antialias_fwd(const float* color, int N, int H, int W, int C,
                                 const float* rast, const float* pos, int V,
                                 const int32_t* tri, int T, const int32_t* topo, float* out,
                                 int nthreads) {
  int64_t P = (int64_t)N * H * W;
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
    for (int64_t pix = b; pix < e; ++pix) {
      int pw = (int)(pix % W), ph = (int)((pix / W) % H), pn = (int)(pix / ((int64_t)H * W));
      Sil s;
      silhouette(rast, pos, tri, topo, H, W, V, T, pn, ph, pw, s);
      for (int c = 0; c < C; ++c) {
        float cp = color[pix * C + c];
        float acc = cp;
        for (int d = 0; d < 4; ++d) {
          if (!s.active[d]) continue;
          float cn = color[s.nbase[d] * C + c];
          acc += s.alpha[d] * (cn - cp);
        }
        out[pix * C + c] = acc;
      }
    }
  });
  return 0;
}

// K24/K25 diffrast_antialias_bwd_color/_bwd_pos (Antialias.swift:388-524).
// d_color is evaluated in gather form (each pixel sums its own (1 - sum beta)
// term and the beta terms its neighbours scatter toward it): the same sum
// as the reference's scatter, deterministic.
extern "C" int orc_antialias_bwd(const float* color, int N, int H, int W, int C,
                                 const float* rast, const float* pos, int V,
                                 const int32_t* tri, int T, const int32_t* topo,
                                 const float* d_out, float* d_color, float* d_pos,
                                 int nthreads) {
  int64_t P = (int64_t)N * H * W;
  std::vector<float> alpha((size_t)P * 4);
  std::vector<float> asum((size_t)P);
  Accum acc(nthreads, (size_t)N * V * 4);
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int tid) {
    double* dp = nullptr;
    float halfW = (float)W * 0.5f, halfH = (float)H * 0.5f;
    for (int64_t pix = b; pix < e; ++pix) {
      int pw = (int)(pix % W), ph = (int)((pix / W) % H), pn = (int)(pix / ((int64_t)H * W));
      Sil s;
      silhouette(rast, pos, tri, topo, H, W, V, T, pn, ph, pw, s);
      for (int d = 0; d < 4; ++d) alpha[pix * 4 + d] = s.active[d] ? s.alpha[d] : 0.0f;
      asum[pix] = s.alpha_sum;
      int64_t pos_n_base = (int64_t)pn * V * 4;
      for (int dir = 0; dir < 4; ++dir) {
        if (!s.active[dir]) continue;
        float a = s.alpha[dir];
        if (a <= 0.0f || a >= 1.0f) continue;
        float d_alpha = 0.0f;
        for (int c = 0; c < C; ++c) {
          float cp = color[pix * C + c], cn = color[s.nbase[dir] * C + c];
          float g = d_out[pix * C + c];
          d_alpha += g * (cn - cp);
        }
        if (d_alpha == 0.0f) continue;
        float e0x = s.e0x[dir], e0y = s.e0y[dir], e1x = s.e1x[dir], e1y = s.e1y[dir];
        float t = s.t[dir], denom = s.denom[dir], dad = s.dadxy[dir];
        float dade0x, dade0y, dade1x, dade1y;
        if (s.horiz[dir]) {
          float row_y = (float)ph + 0.5f;
          float ex_diff = e1x - e0x;
          float inv_denom_sq = 1.0f / (denom * denom);
          dade0x = dad * (1.0f - t);
          dade1x = dad * t;
          dade0y = dad * ex_diff * (row_y - e1y) * inv_denom_sq;
          dade1y = dad * (-ex_diff) * (row_y - e0y) * inv_denom_sq;
        } else {
          float col_x = (float)pw + 0.5f;
          float ey_diff = e1y - e0y;
          float inv_denom_sq = 1.0f / (denom * denom);
          dade0y = dad * (1.0f - t);
          dade1y = dad * t;
          dade0x = dad * ey_diff * (col_x - e1x) * inv_denom_sq;
          dade1x = dad * (-ey_diff) * (col_x - e0x) * inv_denom_sq;
        }
        if (!dp) dp = acc.get(tid);
        int ivs[2] = {s.ie0[dir], s.ie1[dir]};
        float dx[2] = {dade0x, dade1x}, dy[2] = {dade0y, dade1y};
        for (int q = 0; q < 2; ++q) {
          const float* pv = pos + pos_n_base + (int64_t)ivs[q] * 4;
          float wv = pv[3];
          float inv_w = 1.0f / wv;
          float nd_x = pv[0] * inv_w, nd_y = pv[1] * inv_w;
          float d_px = d_alpha * dx[q] * halfW * inv_w;
          float d_py = d_alpha * dy[q] * (-halfH) * inv_w;
          float d_pw = d_alpha * (dx[q] * (-halfW * nd_x) + dy[q] * (halfH * nd_y)) * inv_w;
          double* o = dp + pos_n_base + (int64_t)ivs[q] * 4;
          o[0] += (double)d_px;
          o[1] += (double)d_py;
          o[3] += (double)d_pw;
        }
      }
    }
  });
  acc.reduce_to(d_pos);
  // Gather d_color: self term plus every neighbour's beta toward this pixel.
  // Neighbour in direction d of p is q; q sees p in the opposite direction.
  parallel_for(P, nthreads, [&](int64_t b, int64_t e, int) {
    for (int64_t q = b; q < e; ++q) {
      int pw = (int)(q % W), ph = (int)((q / W) % H), pn = (int)(q / ((int64_t)H * W));
      for (int c = 0; c < C; ++c) {
        double v = (double)(d_out[q * C + c] * (1.0f - asum[q]));
        // p = q - (dw,dh) of direction d  (dir 0: +x, 1: +y, 2: -x, 3: -y)
        const int ddw[4] = {1, 0, -1, 0}, ddh[4] = {0, 1, 0, -1};
        for (int d = 0; d < 4; ++d) {
          int sw = pw - ddw[d], sh = ph - ddh[d];
          if (sw < 0 || sw >= W || sh < 0 || sh >= H) continue;
          int64_t p = ((int64_t)pn * H + sh) * W + sw;
          float a = alpha[p * 4 + d];
          if (a != 0.0f) v += (double)(d_out[p * C + c] * a);
        }
        d_color[q * C + c] = (float)v;
      }
    }
  });
  return 0;
}

extern "C" double orc_mse_fwd_bwd(const float* pred, const float* target, int64_t n, float scale,
                                  float* d_pred, int nthreads) {
  int nt = clamp_threads(nthreads);
  std::vector<double> part(nt, 0.0);
  parallel_for(n, nthreads, [&](int64_t b, int64_t e, int tid) {
    double s = 0.0;
    for (int64_t i = b; i < e; ++i) {
      float d = pred[i] - target[i];
      s += (double)d * (double)d;
      if (d_pred) d_pred[i] = 2.0f * scale * d;
    }
    part[tid] = s;
  });
  double tot = 0.0;
  for (double p : part) tot += p;
  return tot * (double)scale;
}
