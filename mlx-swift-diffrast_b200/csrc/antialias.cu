// antialias.cu — topology hash on the GPU, silhouette antialiasing forward and
// backward.
//
// Reference: Sources/MLXDiffRast/Antialias.swift.
//   antialiasConstructTopologyHash (19-66) runs on the CPU in the reference
//   (device->host copy, sort of 3T edges, run classification).  Here it is an
//   open-addressing hash table on the GPU: every edge (min, max) is inserted
//   with a 64-bit CAS; the slot counts its users and keeps the first two
//   (triangle, edge) references.  A second pass classifies each reference:
//   count 1 -> -1 (boundary), 2 -> the other triangle, >= 3 -> -2
//   (non-manifold).  The classification is order independent, so the table is
//   bit-identical to the reference's sort-based result.
//
//   silhouetteBlock (168-326) is evaluated per (pixel, direction) by sil_dir().
//   Forward = diffrast_antialias_fwd (333-358).  Backward fuses _bwd_color
//   (498-524) and _bwd_pos (388-496): d_color is computed in gather form — each
//   pixel adds its own g*(1 - sum beta) and the beta*g its four neighbours
//   would have scattered toward it — so it needs no atomics and is
//   deterministic; only d_pos uses (float) atomics.
#include <climits>
#include <mutex>

#include "common.cuh"

namespace {

constexpr unsigned long long EMPTY_KEY = 0xFFFFFFFF00000000ull;  // lo > hi: never a real edge

__device__ __forceinline__ unsigned long long edge_key(int a, int b) {
  const int lo = min(a, b), hi = max(a, b);
  return ((unsigned long long)((unsigned)lo ^ 0x80000000u) << 32) | (unsigned)((unsigned)hi ^ 0x80000000u);
}

__device__ __forceinline__ uint32_t hash64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return (uint32_t)k;
}

__global__ void k_topo_init(unsigned long long* __restrict__ keys, uint32_t* __restrict__ cnt, uint32_t cap) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= cap) return;
  keys[i] = EMPTY_KEY;
  cnt[i] = 0u;
}

// Edge k of triangle t joins vertices (k+1)%3 and (k+2)%3 (Antialias.swift:33).
__global__ void k_topo_insert(const int32_t* __restrict__ tri, int T, unsigned long long* __restrict__ keys,
                              uint32_t* __restrict__ cnt, int32_t* __restrict__ ref_a,
                              int32_t* __restrict__ ref_b, uint32_t* __restrict__ ref_slot, uint32_t mask,
                              unsigned* err) {
  const int64_t ref = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ref >= (int64_t)T * 3) return;
  const int t = (int)(ref / 3), k = (int)(ref % 3);
  const int va = __ldg(tri + 3 * t + (k + 1) % 3), vb = __ldg(tri + 3 * t + (k + 2) % 3);
  const unsigned long long key = edge_key(va, vb);
  uint32_t slot = hash64(key) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const unsigned long long prev = atomicCAS(keys + slot, EMPTY_KEY, key);
    if (prev == EMPTY_KEY || prev == key) {
      const uint32_t c = atomicAdd(cnt + slot, 1u);
      if (c == 0) ref_a[slot] = (int32_t)ref;
      else if (c == 1) ref_b[slot] = (int32_t)ref;
      ref_slot[ref] = slot;
      return;
    }
    slot = (slot + 1) & mask;
  }
  dr_flag(err, DR_DEVERR_CAPACITY);  // unreachable at load factor <= 1/2
  ref_slot[ref] = 0xFFFFFFFFu;
}

__global__ void k_topo_classify(int T, const uint32_t* __restrict__ cnt, const int32_t* __restrict__ ref_a,
                                const int32_t* __restrict__ ref_b, const uint32_t* __restrict__ ref_slot,
                                int32_t* __restrict__ topo) {
  const int64_t ref = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ref >= (int64_t)T * 3) return;
  const uint32_t slot = ref_slot[ref];
  if (slot == 0xFFFFFFFFu) { topo[ref] = -1; return; }
  const uint32_t c = cnt[slot];
  int32_t v = -1;
  if (c == 2) {
    const int32_t a = ref_a[slot], b = ref_b[slot];
    v = (a == (int32_t)ref ? b : a) / 3;
  } else if (c > 2) {
    v = -2;
  }
  topo[ref] = v;
}

// ------------------------------------------------------------ silhouettes

struct SilDir {
  bool active;
  float beta;
  int kk, ie0, ie1;
  float e0x, e0y, e1x, e1y, t, denom, dbeta;
  bool horiz;
};

__device__ __forceinline__ int rast_tri(const float4* __restrict__ rast, int64_t pix, int T, unsigned* err) {
  const int t = (int)__ldg(&rast[pix].w) - 1;
  if (t >= T) { dr_flag(err, DR_DEVERR_TRI_ID); return -1; }
  return t;
}

// Clip position of vertex a in view pn: pos[pn, a] (instanced) or M_pn verts[a].
template <bool XF>
__device__ __forceinline__ float4 vpos(const float* __restrict__ pos, const Mat4& M, int V, int pn, int a) {
  if (XF) return mat4_apply(M, ldg4(pos + (int64_t)a * 4));
  return ldg4(pos + ((int64_t)pn * V + a) * 4);
}

// Pixel-space projection E = ((x/w + 1) W/2, (1 - y/w) H/2) (Antialias.swift:240-247).
__device__ __forceinline__ void screen_of(const float4& p, int H, int W, float& ex, float& ey) {
  ex = (p.x / p.w + 1.0f) * (float)W * 0.5f;
  ey = (1.0f - p.y / p.w) * (float)H * 0.5f;
}

// Where the edge (e0, e1) crosses the segment between the centres of pixel
// (ph, pw) and its neighbour (Antialias.swift:264-325): beta > 0 iff the
// crossing lies inside this pixel's cell.  Shared by the forward's search and
// the backward's replay, so both produce the same bits.
__device__ __forceinline__ void crossing(bool horiz, int ph, int pw, float e0x, float e0y, float e1x, float e1y,
                                         float& beta, float& t_val, float& denom, float& dbeta) {
  const float pcx = (float)pw + 0.5f, pcy = (float)ph + 0.5f;
  beta = 0.0f; t_val = 0.0f; dbeta = 0.0f;
  if (horiz) {
    const float dyv = e1y - e0y;
    denom = dyv;
    if (fabsf(dyv) >= 1e-7f) {
      const float tval = (pcy - e0y) / dyv;
      t_val = tval;
      if (tval >= 0.0f && tval <= 1.0f) {
        const float xe = e0x + tval * (e1x - e0x);
        if (xe > (float)pw && xe < (float)(pw + 1)) {
          const float d = xe - pcx;
          beta = 0.5f - fabsf(d);
          dbeta = (d > 0.0f) ? -1.0f : 1.0f;
        }
      }
    }
  } else {
    const float dxv = e1x - e0x;
    denom = dxv;
    if (fabsf(dxv) >= 1e-7f) {
      const float tval = (pcx - e0x) / dxv;
      t_val = tval;
      if (tval >= 0.0f && tval <= 1.0f) {
        const float ye = e0y + tval * (e1y - e0y);
        if (ye > (float)ph && ye < (float)(ph + 1)) {
          const float d = ye - pcy;
          beta = 0.5f - fabsf(d);
          dbeta = (d > 0.0f) ? -1.0f : 1.0f;
        }
      }
    }
  }
}

// One direction of silhouetteBlock (Antialias.swift:189-325) for pixel
// (pn, ph, pw) whose triangle is tri_p.  dir: 0 +x, 1 +y, 2 -x, 3 -y.
template <bool XF>
__device__ SilDir sil_dir(const float4* __restrict__ rast, const float* __restrict__ pos, const Mat4& M,
                          const int32_t* __restrict__ tri, const int32_t* __restrict__ topo, int H, int W,
                          int V, int T, int pn, int ph, int pw, int tri_p, int dir, unsigned* err) {
  SilDir s;
  s.active = false;
  s.beta = 0.0f;
  const int dw = dir == 0 ? 1 : (dir == 2 ? -1 : 0);
  const int dh = dir == 1 ? 1 : (dir == 3 ? -1 : 0);
  const int nh = ph + dh, nw = pw + dw;
  if (nh < 0 || nh >= H || nw < 0 || nw >= W) return s;
  const int tri_n = rast_tri(rast, ((int64_t)pn * H + nh) * W + nw, T, err);
  if (tri_p == tri_n) return s;
  if (tri_p < 0 && tri_n < 0) return s;
  int fg, target;
  if (tri_p >= 0 && tri_n >= 0) {
    const int n0 = __ldg(topo + 3 * tri_p), n1 = __ldg(topo + 3 * tri_p + 1), n2 = __ldg(topo + 3 * tri_p + 2);
    if (!(n0 == tri_n || n1 == tri_n || n2 == tri_n)) return s;
    fg = tri_p; target = tri_n;
  } else if (tri_p >= 0) {
    fg = tri_p; target = -1;
  } else {
    fg = tri_n; target = -1;
  }
  const float pcx = (float)pw + 0.5f, pcy = (float)ph + 0.5f;
  const float ncx = (float)nw + 0.5f, ncy = (float)nh + 0.5f;
  int k_sel = -1, ie0 = -1, ie1 = -1;
  float e0x = 0.f, e0y = 0.f, e1x = 0.f, e1y = 0.f;
  for (int kk = 0; kk < 3; ++kk) {
    if (__ldg(topo + 3 * fg + kk) != target) continue;
    const int a = __ldg(tri + 3 * fg + (kk + 1) % 3), b = __ldg(tri + 3 * fg + (kk + 2) % 3);
    if (a < 0 || a >= V || b < 0 || b >= V) { dr_flag(err, DR_DEVERR_VERTEX); continue; }
    float E0x, E0y, E1x, E1y;
    screen_of(vpos<XF>(pos, M, V, pn, a), H, W, E0x, E0y);
    screen_of(vpos<XF>(pos, M, V, pn, b), H, W, E1x, E1y);
    const float ex = E1x - E0x, ey = E1y - E0y;
    const float side_p = ex * (pcy - E0y) - ey * (pcx - E0x);
    const float side_n = ex * (ncy - E0y) - ey * (ncx - E0x);
    if (side_p * side_n < 0.0f) {
      k_sel = kk; ie0 = a; ie1 = b;
      e0x = E0x; e0y = E0y; e1x = E1x; e1y = E1y;
      break;
    }
  }
  if (k_sel < 0) return s;
  const bool horiz = (dh == 0);
  float beta, t_val, denom, dbeta;
  crossing(horiz, ph, pw, e0x, e0y, e1x, e1y, beta, t_val, denom, dbeta);
  if (beta <= 0.0f) return s;
  s.active = true;
  s.beta = beta;
  s.kk = k_sel;
  s.ie0 = ie0; s.ie1 = ie1;
  s.e0x = e0x; s.e0y = e0y; s.e1x = e1x; s.e1y = e1y;
  s.t = t_val; s.denom = denom; s.dbeta = dbeta; s.horiz = horiz;
  return s;
}

// Directions of pixel (pn, ph, pw) that can hold a silhouette: exactly the
// pairs sil_dir does not reject before its edge search (neighbour inside the
// image, different ids, not both empty, and — both covered — the neighbour
// listed in tri_p's topology row).  All neighbour ids and the topology row
// are loaded up front, independently, so the common case (no candidate) costs
// one round of loads instead of four dependent chains.
__device__ __forceinline__ unsigned sil_candidates(const float4* __restrict__ rast,
                                                   const int32_t* __restrict__ topo, int H, int W, int T,
                                                   int pn, int ph, int pw, int tri_p, unsigned* err) {
  int tn[4];
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int nh = ph + (d == 1 ? 1 : (d == 3 ? -1 : 0)), nw = pw + (d == 0 ? 1 : (d == 2 ? -1 : 0));
    tn[d] = (nh < 0 || nh >= H || nw < 0 || nw >= W) ? INT_MIN
                                                     : rast_tri(rast, ((int64_t)pn * H + nh) * W + nw, T, err);
  }
  int n0 = INT_MIN, n1 = INT_MIN, n2 = INT_MIN;
  if (tri_p >= 0) {
    n0 = __ldg(topo + 3 * tri_p); n1 = __ldg(topo + 3 * tri_p + 1); n2 = __ldg(topo + 3 * tri_p + 2);
  }
  unsigned m = 0;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int t = tn[d];
    if (t == INT_MIN || t == tri_p || (tri_p < 0 && t < 0)) continue;
    if (tri_p >= 0 && t >= 0 && !(n0 == t || n1 == t || n2 == t)) continue;
    m |= 1u << d;
  }
  return m;
}

// The forward's per-pixel record for the VJP (the optional `aa_work` buffer):
// beta[P] float4 (one beta per direction, 0 where inactive), then code[P]
// bytes, 2 bits per direction: 0 inactive, else the selected edge kk + 1.
__host__ __device__ __forceinline__ size_t aa_work_bytes(int64_t P) {
  return (size_t)P * 16 + (((size_t)P + 15) & ~(size_t)15);
}

// Rebuild an active direction's edge from the recorded kk: the same vertex
// loads, projection and crossing arithmetic the search ran, minus the search.
template <bool XF>
__device__ SilDir sil_replay(const float4* __restrict__ rast, const float* __restrict__ pos, const Mat4& M,
                             const int32_t* __restrict__ tri, int H, int W, int V, int T, int pn, int ph,
                             int pw, int tri_p, int dir, int kk, unsigned* err) {
  SilDir s;
  s.active = false;
  const int dw = dir == 0 ? 1 : (dir == 2 ? -1 : 0);
  const int dh = dir == 1 ? 1 : (dir == 3 ? -1 : 0);
  const int nh = ph + dh, nw = pw + dw;
  if (nh < 0 || nh >= H || nw < 0 || nw >= W) return s;  // a record from another rast
  const int fg = tri_p >= 0 ? tri_p : rast_tri(rast, ((int64_t)pn * H + nh) * W + nw, T, err);
  if (fg < 0) return s;
  const int a = __ldg(tri + 3 * fg + (kk + 1) % 3), b = __ldg(tri + 3 * fg + (kk + 2) % 3);
  if (a < 0 || a >= V || b < 0 || b >= V) { dr_flag(err, DR_DEVERR_VERTEX); return s; }
  screen_of(vpos<XF>(pos, M, V, pn, a), H, W, s.e0x, s.e0y);
  screen_of(vpos<XF>(pos, M, V, pn, b), H, W, s.e1x, s.e1y);
  s.horiz = (dh == 0);
  crossing(s.horiz, ph, pw, s.e0x, s.e0y, s.e1x, s.e1y, s.beta, s.t, s.denom, s.dbeta);
  s.active = s.beta > 0.0f;
  s.kk = kk; s.ie0 = a; s.ie1 = b;
  return s;
}

__device__ __forceinline__ int64_t nbr_pix(int pn, int ph, int pw, int dir, int H, int W) {
  const int dw = dir == 0 ? 1 : (dir == 2 ? -1 : 0);
  const int dh = dir == 1 ? 1 : (dir == 3 ? -1 : 0);
  return ((int64_t)pn * H + (ph + dh)) * W + (pw + dw);
}

// A device list of pixels for the two-pass kernels below.  Appends are
// warp-aggregated, and the list is split into kListShards shards by block
// index so the append counters are not all one contended address: block b
// appends to shard b % kListShards, whose region holds every pixel of its
// blocks (cap entries).  count[s] is shard s's length.
constexpr int kListShards = 64;

struct PixList {
  unsigned long long* count;
  unsigned long long* list;
  int64_t cap;
};

__device__ __forceinline__ void list_append(const PixList& L, bool want, unsigned long long entry) {
  const unsigned m = __ballot_sync(0xffffffffu, want);
  if (!m) return;
  const int lane = threadIdx.x & 31, leader = __ffs(m) - 1;
  const int sh = (int)(blockIdx.x % kListShards);
  unsigned long long base = 0;
  if (lane == leader) base = atomicAdd(L.count + sh, (unsigned long long)__popc(m));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (want) L.list[sh * L.cap + (int64_t)base + __popc(m & ((1u << lane) - 1u))] = entry;
}

// Forward in two passes, so the rare silhouette search runs at full occupancy
// instead of holding up whole warps and blocks:
//   k_aa_fwd_scan   every pixel finds its candidate directions with one round
//                   of independent loads (sil_candidates); pixels with none
//                   are finished there (colour copied, empty record), the rest
//                   are appended to a list as (pixel << 4 | candidate bits);
//   k_aa_fwd_edges  a grid-stride pass over the list: sil_dir for each
//                   candidate direction, then the record and the blend.
template <bool WORK>
__global__ void __launch_bounds__(256) k_aa_fwd_scan(const float* __restrict__ color, int N, int H, int W, int C,
                                                     const float4* __restrict__ rast, int T,
                                                     const int32_t* __restrict__ topo, float* __restrict__ out,
                                                     float4* __restrict__ work_beta, uint8_t* __restrict__ work_code,
                                                     const PixList L, const float* __restrict__ tgt, float lscale,
                                                     float* __restrict__ part, unsigned* err) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = pix < (int64_t)N * H * W;
  const float* cp = color + pix * C;
  float* o = out + pix * C;
  // The common case (no candidate, C == 8, colour, out and target 16-byte
  // aligned) copies the colour row: load it first so it overlaps the
  // topology gather.
  const bool vec8 = C == 8 && ((((uintptr_t)color) | ((uintptr_t)out) | ((uintptr_t)tgt)) & 15) == 0;
  float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = c0;
  if (valid && vec8) { c0 = ldg4(cp); c1 = ldg4(cp + 4); }
  unsigned cand = 0;
  if (valid) {
    int pn, ph, pw;
    dr::pix_nyx(pix, (int64_t)N * H * W, H, W, pn, ph, pw);
    cand = sil_candidates(rast, topo, H, W, T, pn, ph, pw, rast_tri(rast, pix, T, err), err);
  }
  list_append(L, cand != 0u, ((unsigned long long)pix << 4) | cand);
  // Pixels without a candidate keep their colour (and add their share of a
  // fused loss: out == colour).
  float l = 0.0f;
  if (valid && !cand) {
    if (WORK) {
      work_beta[pix] = make_float4(0.f, 0.f, 0.f, 0.f);
      work_code[pix] = 0;
    }
    const float* tp = tgt ? tgt + pix * C : nullptr;
    if (vec8) {
      *reinterpret_cast<float4*>(o) = c0;
      *reinterpret_cast<float4*>(o + 4) = c1;
      if (tp) l = sq_diff4(c0, ldg4(tp)) + sq_diff4(c1, ldg4(tp + 4));
    } else if ((C & 3) == 0 && ((((uintptr_t)color) | ((uintptr_t)out) | ((uintptr_t)tgt)) & 15) == 0) {
      for (int c = 0; c < C; c += 4) {
        const float4 x = ldg4(cp + c);
        *reinterpret_cast<float4*>(o + c) = x;
        if (tp) l += sq_diff4(x, ldg4(tp + c));
      }
    } else {
      for (int c = 0; c < C; ++c) {
        const float x = __ldg(cp + c);
        o[c] = x;
        if (tp) { const float r = x - __ldg(tp + c); l += r * r; }
      }
    }
  }
  if (part) block_loss_add(l, lscale, part);
}

template <bool XF, bool WORK>
__global__ void __launch_bounds__(256, 4) k_aa_fwd_edges(const float* __restrict__ color, int N, int H, int W, int C,
                                                      const float4* __restrict__ rast, const float* __restrict__ pos,
                                                      const float* __restrict__ xform, int V,
                                                      const int32_t* __restrict__ tri, int T,
                                                      const int32_t* __restrict__ topo, float* __restrict__ out,
                                                      float4* __restrict__ work_beta, uint8_t* __restrict__ work_code,
                                                      const PixList L, const float* __restrict__ tgt, float lscale,
                                                      float* __restrict__ part, unsigned* err) {
  // Grid (x, shard): the blocks of row y walk shard y, a warp 32 listed
  // pixels at a time.  The warp's (pixel, candidate direction) pairs are
  // searched one per lane (a pixel has one to four, so a lane per pixel
  // left most lanes idle), into per-warp shared slots; then every lane
  // blends its own pixel.
  constexpr int kWarps = 256 / 32;
  __shared__ unsigned char s_item[kWarps][128];  // source lane | direction << 5
  __shared__ float s_beta[kWarps][128];          // [source lane * 4 + direction]
  __shared__ unsigned char s_kk[kWarps][128];    // selected edge + 1, 0 inactive
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned long long n = L.count[blockIdx.y];
  float l = 0.0f;
  const unsigned long long* sl = L.list + (int64_t)blockIdx.y * L.cap;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long wb = (unsigned long long)blockIdx.x * blockDim.x + (unsigned)(warp * 32); wb < n;
       wb += stride) {
    const bool has = wb + lane < n;
    const unsigned long long e = has ? sl[wb + lane] : 0ull;
    const int64_t pix = (int64_t)(e >> 4);
    const unsigned cand = (unsigned)(e & 15u);
    const int tri_p = has ? rast_tri(rast, pix, T, err) : -1;
    // The warp's items, in lane order, and this lane's result slots cleared.
    const int cnt = __popc(cand);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    int k = incl - cnt;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      if ((cand >> d) & 1u) s_item[warp][k++] = (unsigned char)(lane | (d << 5));
      s_beta[warp][lane * 4 + d] = 0.0f;
      s_kk[warp][lane * 4 + d] = 0;
    }
    __syncwarp();
    for (int r = 0; r < total; r += 32) {
      const bool act = r + lane < total;
      const unsigned it = act ? s_item[warp][r + lane] : 0u;
      const int src = (int)(it & 31u), d = (int)(it >> 5);
      const int64_t spix = __shfl_sync(0xffffffffu, pix, src);
      const int stri = __shfl_sync(0xffffffffu, tri_p, src);
      if (act) {
        int pn, ph, pw;
        dr::pix_nyx(spix, (int64_t)N * H * W, H, W, pn, ph, pw);
        Mat4 M;
        if (XF) M = load_mat4(xform + (int64_t)pn * 16);
        const SilDir sd = sil_dir<XF>(rast, pos, M, tri, topo, H, W, V, T, pn, ph, pw, stri, d, err);
        if (sd.active) {
          s_beta[warp][src * 4 + d] = sd.beta;
          s_kk[warp][src * 4 + d] = (unsigned char)(sd.kk + 1);
        }
      }
    }
    __syncwarp();
    if (!has) continue;
    int pn, ph, pw;
    dr::pix_nyx(pix, (int64_t)N * H * W, H, W, pn, ph, pw);
    float beta[4];
    unsigned code = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      beta[d] = s_beta[warp][lane * 4 + d];
      code |= (unsigned)s_kk[warp][lane * 4 + d] << (2 * d);
    }
    if (WORK) {
      work_beta[pix] = make_float4(beta[0], beta[1], beta[2], beta[3]);
      work_code[pix] = (uint8_t)code;
    }
    const float* cp = color + pix * C;
    float* o = out + pix * C;
    const float* tp = tgt ? tgt + pix * C : nullptr;
    if (code == 0u) {
      for (int c = 0; c < C; ++c) {
        const float x = __ldg(cp + c);
        o[c] = x;
        if (tp) { const float r = x - __ldg(tp + c); l += r * r; }
      }
      continue;
    }
    int64_t nb[4];
#pragma unroll
    for (int d = 0; d < 4; ++d) nb[d] = beta[d] > 0.0f ? nbr_pix(pn, ph, pw, d, H, W) : -1;
    for (int c = 0; c < C; ++c) {
      const float p = __ldg(cp + c);
      float acc = p;
#pragma unroll
      for (int d = 0; d < 4; ++d)
        if (nb[d] >= 0) acc += beta[d] * (__ldg(color + nb[d] * C + c) - p);
      o[c] = acc;
      if (tp) { const float r = acc - __ldg(tp + c); l += r * r; }
    }
  }
  if (part) block_loss_add(l, lscale, part);
}

template <bool VEC, bool XF>
__device__ __forceinline__ void add_pos(float* p, const Mat4& M, float x, float y, float w) {
  if (XF) {
    atomicAdd(reinterpret_cast<float4*>(p), mat4_apply_t(M, make_float4(x, y, 0.0f, w)));
  } else if (VEC) {
    atomicAdd(reinterpret_cast<float4*>(p), make_float4(x, y, 0.0f, w));
  } else {
    atomicAdd(p + 0, x);
    atomicAdd(p + 1, y);
    atomicAdd(p + 3, w);
  }
}

// d_pos contribution of one active silhouette direction of pixel (pn, ph, pw)
// (Antialias.swift:405-495): d_alpha = sum_c g (c_n - c_p); skipped outside
// beta in (0, 1) or for d_alpha == 0.
template <bool VEC, bool XF>
__device__ __forceinline__ void aa_dir_dpos(const SilDir& s, const float* __restrict__ color, int C,
                                            const Cot& cot, float gl, int64_t pix, int64_t nb,
                                            const float* __restrict__ pos, const Mat4& M, int V, int pn, int ph,
                                            int pw, int H, int W, float* __restrict__ d_pos) {
  if (s.beta <= 0.0f || s.beta >= 1.0f) return;
  const float halfW = (float)W * 0.5f, halfH = (float)H * 0.5f;
  float d_alpha = 0.0f;
  for (int c = 0; c < C; ++c) {
    const float cp = __ldg(color + pix * C + c), cn = __ldg(color + nb * C + c);
    d_alpha += cot_at(cot, gl, pix * C + c) * (cn - cp);
  }
  if (d_alpha == 0.0f) return;
  float dade0x, dade0y, dade1x, dade1y;
  const float inv_denom_sq = __fdividef(1.0f, s.denom * s.denom);  // gradient only: fast reciprocal
  if (s.horiz) {
    const float row_y = (float)ph + 0.5f;
    const float ex_diff = s.e1x - s.e0x;
    dade0x = s.dbeta * (1.0f - s.t);
    dade1x = s.dbeta * s.t;
    dade0y = s.dbeta * ex_diff * (row_y - s.e1y) * inv_denom_sq;
    dade1y = s.dbeta * (-ex_diff) * (row_y - s.e0y) * inv_denom_sq;
  } else {
    const float col_x = (float)pw + 0.5f;
    const float ey_diff = s.e1y - s.e0y;
    dade0y = s.dbeta * (1.0f - s.t);
    dade1y = s.dbeta * s.t;
    dade0x = s.dbeta * ey_diff * (col_x - s.e1x) * inv_denom_sq;
    dade1x = s.dbeta * (-ey_diff) * (col_x - s.e0x) * inv_denom_sq;
  }
  const int64_t pb = XF ? 0 : (int64_t)pn * V * 4;
  {
    const float4 pv = vpos<XF>(pos, M, V, pn, s.ie0);
    const float inv_w = __fdividef(1.0f, pv.w);
    const float nd_x = pv.x * inv_w, nd_y = pv.y * inv_w;
    add_pos<VEC, XF>(d_pos + pb + (int64_t)s.ie0 * 4, M, d_alpha * dade0x * halfW * inv_w,
                     d_alpha * dade0y * (-halfH) * inv_w,
                     d_alpha * (dade0x * (-halfW * nd_x) + dade0y * (halfH * nd_y)) * inv_w);
  }
  {
    const float4 pv = vpos<XF>(pos, M, V, pn, s.ie1);
    const float inv_w = __fdividef(1.0f, pv.w);
    const float nd_x = pv.x * inv_w, nd_y = pv.y * inv_w;
    add_pos<VEC, XF>(d_pos + pb + (int64_t)s.ie1 * 4, M, d_alpha * dade1x * halfW * inv_w,
                     d_alpha * dade1y * (-halfH) * inv_w,
                     d_alpha * (dade1x * (-halfW * nd_x) + dade1y * (halfH * nd_y)) * inv_w);
  }
}

// d_color in gather form: g (1 - sum of own betas) plus beta * g of every
// neighbour whose silhouette points at this pixel.
__device__ __forceinline__ void aa_dcolor(const Cot& cot, float gl, float* __restrict__ d_color, int C,
                                          int64_t pix, float keep, const float nbeta[4], const int64_t nsrc[4]) {
  if ((C & 3) == 0 &&
      ((((uintptr_t)cot.d) | ((uintptr_t)cot.pred) | ((uintptr_t)cot.target) | ((uintptr_t)d_color)) & 15) == 0) {
    for (int c = 0; c < C; c += 4) {
      const float4 gs = cot_at4(cot, gl, pix * C + c);
      float4 v = make_float4(gs.x * keep, gs.y * keep, gs.z * keep, gs.w * keep);
#pragma unroll
      for (int d = 0; d < 4; ++d)
        if (nsrc[d] >= 0) {
          const float4 gn = cot_at4(cot, gl, nsrc[d] * C + c);
          const float b = nbeta[d];
          v.x += gn.x * b; v.y += gn.y * b; v.z += gn.z * b; v.w += gn.w * b;
        }
      *reinterpret_cast<float4*>(d_color + pix * C + c) = v;
    }
    return;
  }
  for (int c = 0; c < C; ++c) {
    float v = cot_at(cot, gl, pix * C + c) * keep;
#pragma unroll
    for (int d = 0; d < 4; ++d)
      if (nsrc[d] >= 0) v += cot_at(cot, gl, nsrc[d] * C + c) * nbeta[d];
    d_color[pix * C + c] = v;
  }
}

// VJP from the forward's record, in two passes: k_aa_bwd_gather forms every
// pixel's d_color from its own and its neighbours' recorded betas and appends
// pixels with active directions to a list as (pixel << 8 | record code);
// k_aa_bwd_edges replays those edges (a grid-stride pass, full occupancy)
// for the d_pos atomics.  The gather is a stream of independent loads held to
// five resident blocks per SM (48 registers) for more loads in flight.
__global__ void __launch_bounds__(256, 5) k_aa_bwd_gather(int N, int H, int W, int C,
                                                       const Cot cot, float* __restrict__ d_color,
                                                       const float4* __restrict__ work_beta,
                                                       const uint8_t* __restrict__ work_code, const PixList L) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = pix < (int64_t)N * H * W;
  // C == 8 with 16-byte aligned streams: the pixel's own cotangent is loaded
  // together with its record, ahead of the neighbours' betas, so all of the
  // pixel's loads are in flight at once (the same arithmetic as aa_dcolor).
  const bool vec8 = C == 8 && ((((uintptr_t)cot.d) | ((uintptr_t)cot.pred) | ((uintptr_t)cot.target) |
                                ((uintptr_t)d_color)) & 15) == 0;
  unsigned code = 0;
  if (valid) {
    int pn, ph, pw;
    dr::pix_nyx(pix, (int64_t)N * H * W, H, W, pn, ph, pw);
    const float gl = cot_g(cot);
    float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
    if (vec8) {
      g0 = cot_at4<true>(cot, gl, pix * 8);
      g1 = cot_at4<true>(cot, gl, pix * 8 + 4);
    }
    code = __ldg(work_code + pix);
    const float4 b4 = __ldg(work_beta + pix);
    // The same sum the search path forms: 0 + the active betas in direction order.
    const float keep = 1.0f - ((((0.0f + b4.x) + b4.y) + b4.z) + b4.w);
    float nbeta[4];
    int64_t nsrc[4];
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      nbeta[d] = 0.0f;
      nsrc[d] = -1;
      const int sw = pw - (d == 0 ? 1 : (d == 2 ? -1 : 0));
      const int sh = ph - (d == 1 ? 1 : (d == 3 ? -1 : 0));
      if (sw < 0 || sw >= W || sh < 0 || sh >= H) continue;
      const int64_t p = ((int64_t)pn * H + sh) * W + sw;
      const float b = __ldg(reinterpret_cast<const float*>(work_beta + p) + d);
      if (b > 0.0f) { nbeta[d] = b; nsrc[d] = p; }
    }
    if (vec8) {
      float4 v0 = make_float4(g0.x * keep, g0.y * keep, g0.z * keep, g0.w * keep);
      float4 v1 = make_float4(g1.x * keep, g1.y * keep, g1.z * keep, g1.w * keep);
#pragma unroll
      for (int d = 0; d < 4; ++d)
        if (nsrc[d] >= 0) {
          const float4 n0 = cot_at4(cot, gl, nsrc[d] * 8), n1 = cot_at4(cot, gl, nsrc[d] * 8 + 4);
          const float b = nbeta[d];
          v0.x += n0.x * b; v0.y += n0.y * b; v0.z += n0.z * b; v0.w += n0.w * b;
          v1.x += n1.x * b; v1.y += n1.y * b; v1.z += n1.z * b; v1.w += n1.w * b;
        }
      stcs4(d_color + pix * 8, v0);
      stcs4(d_color + pix * 8 + 4, v1);
    } else {
      aa_dcolor(cot, gl, d_color, C, pix, keep, nbeta, nsrc);
    }
  }
  list_append(L, code != 0u, ((unsigned long long)pix << 8) | code);
}

template <bool VEC, bool XF>
__global__ void __launch_bounds__(256, DR_MINB_AA_BWD) k_aa_bwd_edges(
    const float* __restrict__ color, int N, int H, int W, int C, const float4* __restrict__ rast,
    const float* __restrict__ pos, const float* __restrict__ xform, int V, const int32_t* __restrict__ tri, int T,
    const Cot cot, float* __restrict__ d_pos, const PixList L, unsigned* err) {
  // Grid (x, shard): the blocks of row y walk shard y, a warp 32 listed
  // pixels at a time; their recorded (pixel, direction) edges are replayed
  // one per lane (a pixel has one to four).
  constexpr int kWarps = 256 / 32;
  __shared__ unsigned char s_item[kWarps][128];  // source lane | direction << 5
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float gl = cot_g(cot);
  const unsigned long long n = L.count[blockIdx.y];
  const unsigned long long* sl = L.list + (int64_t)blockIdx.y * L.cap;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long wb = (unsigned long long)blockIdx.x * blockDim.x + (unsigned)(warp * 32); wb < n;
       wb += stride) {
    const bool has = wb + lane < n;
    const unsigned long long e = has ? sl[wb + lane] : 0ull;
    const int64_t pix = (int64_t)(e >> 8);
    const unsigned code = (unsigned)(e & 255u);
    const int tri_p = has ? rast_tri(rast, pix, T, err) : -1;
    unsigned dirs = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) dirs |= (((code >> (2 * d)) & 3u) != 0u ? 1u : 0u) << d;
    const int cnt = __popc(dirs);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    int k = incl - cnt;
#pragma unroll
    for (int d = 0; d < 4; ++d)
      if ((dirs >> d) & 1u) s_item[warp][k++] = (unsigned char)(lane | (d << 5));
    __syncwarp();
    for (int r = 0; r < total; r += 32) {
      const bool act = r + lane < total;
      const unsigned it = act ? s_item[warp][r + lane] : 0u;
      const int src = (int)(it & 31u), d = (int)(it >> 5);
      const int64_t spix = __shfl_sync(0xffffffffu, pix, src);
      const int stri = __shfl_sync(0xffffffffu, tri_p, src);
      const unsigned scode = __shfl_sync(0xffffffffu, code, src);
      if (!act) continue;
      int pn, ph, pw;
      dr::pix_nyx(spix, (int64_t)N * H * W, H, W, pn, ph, pw);
      const int kk = (int)((scode >> (2 * d)) & 3u) - 1;
      Mat4 M;
      if (XF) M = load_mat4(xform + (int64_t)pn * 16);
      const SilDir sd = sil_replay<XF>(rast, pos, M, tri, H, W, V, T, pn, ph, pw, stri, d, kk, err);
      if (!sd.active) continue;
      aa_dir_dpos<VEC, XF>(sd, color, C, cot, gl, spix, nbr_pix(pn, ph, pw, d, H, W), pos, M, V, pn, ph, pw, H, W,
                           d_pos);
    }
    __syncwarp();
  }
}

// VJP that searches the silhouettes again (no forward record), as the
// reference does: own directions for (1 - sum beta) and d_pos, and each
// neighbour's direction toward this pixel for the gathered d_color.
template <bool VEC, bool XF>
__global__ void __launch_bounds__(256, DR_MINB_AA_BWD) k_aa_bwd(const float* __restrict__ color, int N, int H, int W, int C,
                         const float4* __restrict__ rast, const float* __restrict__ pos,
                         const float* __restrict__ xform, int V,
                         const int32_t* __restrict__ tri, int T, const int32_t* __restrict__ topo,
                         const Cot cot, float* __restrict__ d_color, float* __restrict__ d_pos,
                         unsigned* err) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= (int64_t)N * H * W) return;
  const float gl = cot_g(cot);
  int pn, ph, pw;
  dr::pix_nyx(pix, (int64_t)N * H * W, H, W, pn, ph, pw);
  const int tri_p = rast_tri(rast, pix, T, err);
  Mat4 M;
  if (XF) M = load_mat4(xform + (int64_t)pn * 16);
  float alpha_sum = 0.0f;
#pragma unroll 1
  for (int dir = 0; dir < 4; ++dir) {
    const SilDir s = sil_dir<XF>(rast, pos, M, tri, topo, H, W, V, T, pn, ph, pw, tri_p, dir, err);
    if (!s.active) continue;
    alpha_sum += s.beta;
    aa_dir_dpos<VEC, XF>(s, color, C, cot, gl, pix, nbr_pix(pn, ph, pw, dir, H, W), pos, M, V, pn, ph, pw, H, W,
                         d_pos);
  }
  float nbeta[4];
  int64_t nsrc[4];
#pragma unroll 1
  for (int d = 0; d < 4; ++d) {
    nbeta[d] = 0.0f;
    nsrc[d] = -1;
    const int sw = pw - (d == 0 ? 1 : (d == 2 ? -1 : 0));
    const int sh = ph - (d == 1 ? 1 : (d == 3 ? -1 : 0));
    if (sw < 0 || sw >= W || sh < 0 || sh >= H) continue;
    const int64_t p = ((int64_t)pn * H + sh) * W + sw;
    const int tri_s = rast_tri(rast, p, T, err);
    if (tri_s == tri_p) continue;  // no silhouette between equal ids
    const SilDir s = sil_dir<XF>(rast, pos, M, tri, topo, H, W, V, T, pn, sh, sw, tri_s, d, err);
    if (s.active) { nbeta[d] = s.beta; nsrc[d] = p; }
  }
  aa_dcolor(cot, gl, d_color, C, pix, 1.0f - alpha_sum, nbeta, nsrc);
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

dr_status check_aa(dr_ctx* ctx, const float* color, int N, int H, int W, int C, const float* rast,
                   const float* pos, int V, const int32_t* tri, int T, const int32_t* topo) {
  DR_REQUIRE(ctx, color && rast && pos && ((tri && topo) || T == 0), "antialias: null input");
  DR_REQUIRE(ctx, N > 0 && H > 0 && W > 0 && C > 0 && V > 0 && T >= 0, "antialias: bad sizes");
  DR_REQUIRE(ctx, aligned16(rast) && aligned16(pos), "antialias: rast / pos must be 16-byte aligned");
  return DR_OK;
}

}  // namespace

using namespace dr;

extern "C" dr_status dr_antialias_construct_topology_hash(dr_ctx* ctx, const int32_t* tri, int T, int32_t* topo) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, T >= 0 && (T == 0 || (tri && topo)), "antialiasConstructTopologyHash: bad arguments");
  DR_REQUIRE(ctx, T < (1 << 29), "antialiasConstructTopologyHash: T too large");
  if (T == 0) return DR_OK;
  const int64_t E = (int64_t)T * 3;
  uint64_t cap = 1024;
  while (cap < (uint64_t)(2 * E)) cap <<= 1;
  const size_t bytes = cap * (8 + 4 + 4 + 4) + (size_t)E * 4 + 256;
  char* w = (char*)ws_get(ctx, WS_HASH, bytes);
  if (!w) return DR_ENOMEM;
  unsigned long long* keys = (unsigned long long*)w;
  uint32_t* cnt = (uint32_t*)(keys + cap);
  int32_t* ra = (int32_t*)(cnt + cap);
  int32_t* rb = ra + cap;
  uint32_t* rs = (uint32_t*)(rb + cap);
  DR_TB(ctx);
  k_topo_init<<<grid_for((int64_t)cap, 256), 256, 0, ctx->stream>>>(keys, cnt, (uint32_t)cap);
  DR_LAUNCHED(ctx, "topo_init");
  DR_TB(ctx);
  k_topo_insert<<<grid_for(E, 256), 256, 0, ctx->stream>>>(tri, T, keys, cnt, ra, rb, rs, (uint32_t)(cap - 1),
                                                            ctx->d_err);
  DR_LAUNCHED(ctx, "topo_insert");
  DR_TB(ctx);
  k_topo_classify<<<grid_for(E, 256), 256, 0, ctx->stream>>>(T, cnt, ra, rb, rs, topo);
  DR_LAUNCHED(ctx, "topo_classify");
  return DR_OK;
}

namespace {

// Pixel list in the WS_AA slot: kListShards 64-bit counts, then the shards,
// each with room for every pixel of its blocks (see PixList).
dr_status aa_list(dr_ctx* ctx, int64_t P, PixList* L) {
  const int64_t nblocks = (P + 255) / 256;
  const int64_t cap = (nblocks + kListShards - 1) / kListShards * 256;
  const size_t head = sizeof(unsigned long long) * kListShards;
  char* w = (char*)ws_get(ctx, WS_AA, head + sizeof(unsigned long long) * (size_t)(cap * kListShards));
  if (!w) return DR_ENOMEM;
  L->count = reinterpret_cast<unsigned long long*>(w);
  L->list = reinterpret_cast<unsigned long long*>(w + head);
  L->cap = cap;
  DR_CUDA(ctx, cudaMemsetAsync(w, 0, head, ctx->stream), "antialias list");
  return DR_OK;
}

// Grid of a grid-stride pass over a sharded list: one row of blocks per shard,
// about 8 blocks per SM in total.
inline dim3 list_grid(dr_ctx* ctx, int64_t P) {
  const int64_t total = std::max<int64_t>(1, std::min<int64_t>((P + 255) / 256, (int64_t)ctx->num_sms * 8));
  return dim3((unsigned)std::max<int64_t>(1, (total + kListShards - 1) / kListShards), kListShards);
}

// With a target, also writes lscale * sum((out - target)^2) to the device
// scalar *loss (the fused MSE of the *_mse entry points).
dr_status aa_fwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C, const float* rast,
                 const float* pos, const float* xform, int V, const int32_t* tri, int T, const int32_t* topo,
                 float* out, void* work, const float* target = nullptr, float lscale = 0.0f,
                 float* loss = nullptr) {
  dr_status st = check_aa(ctx, color, N, H, W, C, rast, pos, V, tri, T, topo);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, out, "antialias: out required");
  DR_REQUIRE(ctx, !work || aligned16(work), "antialias: aa_work must be 16-byte aligned");
  const int64_t P = (int64_t)N * H * W;
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  float4* wb = reinterpret_cast<float4*>(work);
  uint8_t* wc = work ? reinterpret_cast<uint8_t*>(work) + (size_t)P * 16 : nullptr;
  PixList L;
  if ((st = aa_list(ctx, P, &L)) != DR_OK) return st;
  float* part = nullptr;
  if (target) {
    DR_REQUIRE(ctx, loss, "antialias_mse: loss required");
    if ((st = loss_begin(ctx, &part)) != DR_OK) return st;
  }
  DR_TB(ctx);
  if (work)
    k_aa_fwd_scan<true><<<grid_for(P, 256), 256, 0, ctx->stream>>>(color, N, H, W, C, r4, T, topo, out, wb, wc, L,
                                                                    target, lscale, part, ctx->d_err);
  else
    k_aa_fwd_scan<false><<<grid_for(P, 256), 256, 0, ctx->stream>>>(color, N, H, W, C, r4, T, topo, out, wb, wc, L,
                                                                     target, lscale, part, ctx->d_err);
  DR_LAUNCHED(ctx, "aa_fwd");
  DR_TB(ctx);
#define DR_AF(XFV, WV, XP)                                                                                       \
  k_aa_fwd_edges<XFV, WV><<<list_grid(ctx, P), 256, 0, ctx->stream>>>(color, N, H, W, C, r4, pos, XP, V, tri, T,  \
                                                                      topo, out, wb, wc, L, target, lscale, part, \
                                                                      ctx->d_err)
  if (xform) {
    if (work) DR_AF(true, true, xform); else DR_AF(true, false, xform);
  } else {
    if (work) DR_AF(false, true, nullptr); else DR_AF(false, false, nullptr);
  }
#undef DR_AF
  DR_LAUNCHED(ctx, "aa_fwd_edges");
  if (part) return loss_end(ctx, part, loss);
  return DR_OK;
}

dr_status aa_bwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C, const float* rast,
                 const float* pos, const float* xform, int V, const int32_t* tri, int T, const int32_t* topo,
                 const Cot& d_out, float* d_color, float* d_pos, const void* work) {
  dr_status st = check_aa(ctx, color, N, H, W, C, rast, pos, V, tri, T, topo);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, (d_out.d || (d_out.pred && d_out.target && d_out.d_loss)) && d_color && d_pos,
             "antialias_bwd: d_out (or out, target and d_loss), d_color, d_pos required");
  DR_REQUIRE(ctx, !work || aligned16(work), "antialias_bwd: aa_work must be 16-byte aligned");
  const size_t npos = (size_t)(xform ? 1 : N) * V * 4;
  DR_CUDA(ctx, cudaMemsetAsync(d_pos, 0, sizeof(float) * npos, ctx->stream), "antialias_bwd memset");
  const int64_t P = (int64_t)N * H * W;
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* wb = reinterpret_cast<const float4*>(work);
  const uint8_t* wc = work ? reinterpret_cast<const uint8_t*>(work) + (size_t)P * 16 : nullptr;
  if (xform) DR_REQUIRE(ctx, aligned16(d_pos), "antialias_xf_bwd: d_verts must be 16-byte aligned");
  const bool vec = xform || aligned16(d_pos);
  if (work) {
    PixList L;
    if ((st = aa_list(ctx, P, &L)) != DR_OK) return st;
    DR_TB(ctx);
    k_aa_bwd_gather<<<grid_for(P, 256), 256, 0, ctx->stream>>>(N, H, W, C, d_out, d_color, wb, wc, L);
    DR_LAUNCHED(ctx, "aa_bwd");
    DR_TB(ctx);
#define DR_AE(VECV, XFV, XP)                                                                                     \
  k_aa_bwd_edges<VECV, XFV><<<list_grid(ctx, P), 256, 0, ctx->stream>>>(color, N, H, W, C, r4, pos, XP, V, tri, T, \
                                                                        d_out, d_pos, L, ctx->d_err)
    if (xform) DR_AE(true, true, xform);
    else if (vec) DR_AE(true, false, nullptr);
    else DR_AE(false, false, nullptr);
#undef DR_AE
    DR_LAUNCHED(ctx, "aa_bwd_edges");
    return DR_OK;
  }
  DR_TB(ctx);
#define DR_AB(VECV, XFV, XP)                                                                                     \
  k_aa_bwd<VECV, XFV><<<grid_for(P, 256), 256, 0, ctx->stream>>>(color, N, H, W, C, r4, pos, XP, V, tri, T, topo,  \
                                                                 d_out, d_color, d_pos, ctx->d_err)
  if (xform) DR_AB(true, true, xform);
  else if (vec) DR_AB(true, false, nullptr);
  else DR_AB(false, false, nullptr);
#undef DR_AB
  DR_LAUNCHED(ctx, "aa_bwd");
  return DR_OK;
}

}  // namespace

extern "C" size_t dr_antialias_work_bytes(int N, int H, int W) {
  if (N <= 0 || H <= 0 || W <= 0) return 0;
  return aa_work_bytes((int64_t)N * H * W);
}

extern "C" dr_status dr_antialias_fwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                      const float* rast, const float* pos, int V, const int32_t* tri, int T,
                                      const int32_t* topo, float* out, void* aa_work) {
  DR_ENTER(ctx);
  return aa_fwd(ctx, color, N, H, W, C, rast, pos, nullptr, V, tri, T, topo, out, aa_work);
}

extern "C" dr_status dr_antialias_bwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                      const float* rast, const float* pos, int V, const int32_t* tri, int T,
                                      const int32_t* topo, const float* d_out, float* d_color, float* d_pos,
                                      const void* aa_work) {
  DR_ENTER(ctx);
  return aa_bwd(ctx, color, N, H, W, C, rast, pos, nullptr, V, tri, T, topo, Cot{d_out, nullptr, nullptr, 0.0f, nullptr},
                d_color, d_pos, aa_work);
}

extern "C" dr_status dr_antialias_xf_fwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                         const float* rast, const float* verts, int V, const float* xform,
                                         const int32_t* tri, int T, const int32_t* topo, float* out,
                                         void* aa_work) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform && aligned16(xform), "antialias_xf: xform [N,4,4] must be given and 16-byte aligned");
  return aa_fwd(ctx, color, N, H, W, C, rast, verts, xform, V, tri, T, topo, out, aa_work);
}

extern "C" dr_status dr_antialias_xf_bwd(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                         const float* rast, const float* verts, int V, const float* xform,
                                         const int32_t* tri, int T, const int32_t* topo, const float* d_out,
                                         float* d_color, float* d_verts, const void* aa_work) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform && aligned16(xform), "antialias_xf_bwd: xform [N,4,4] must be given and 16-byte aligned");
  return aa_bwd(ctx, color, N, H, W, C, rast, verts, xform, V, tri, T, topo,
                Cot{d_out, nullptr, nullptr, 0.0f, nullptr}, d_color, d_verts, aa_work);
}

// Antialias with a fused mean-squared-error loss against `target` (same shape
// as out): the forward also writes scale * sum((out - target)^2) to the device
// scalar *loss, and the VJP forms its cotangent 2 * scale * (out - target) *
// (*d_loss) where it reads it, so no separate loss pass or d_out tensor runs.
extern "C" dr_status dr_antialias_fwd_mse(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                          const float* rast, const float* pos, int V, const int32_t* tri, int T,
                                          const int32_t* topo, float* out, void* aa_work, const float* target,
                                          float scale, float* loss) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, target && loss, "antialias_mse: target and loss required");
  return aa_fwd(ctx, color, N, H, W, C, rast, pos, nullptr, V, tri, T, topo, out, aa_work, target, scale, loss);
}

extern "C" dr_status dr_antialias_bwd_mse(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                          const float* rast, const float* pos, int V, const int32_t* tri, int T,
                                          const int32_t* topo, const float* out, const float* target, float scale,
                                          const float* d_loss, float* d_color, float* d_pos, const void* aa_work) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, out && target && d_loss, "antialias_bwd_mse: out, target and d_loss required");
  return aa_bwd(ctx, color, N, H, W, C, rast, pos, nullptr, V, tri, T, topo,
                Cot{nullptr, out, target, 2.0f * scale, d_loss}, d_color, d_pos, aa_work);
}

extern "C" dr_status dr_antialias_xf_fwd_mse(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                             const float* rast, const float* verts, int V, const float* xform,
                                             const int32_t* tri, int T, const int32_t* topo, float* out,
                                             void* aa_work, const float* target, float scale, float* loss) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform && aligned16(xform), "antialias_xf: xform [N,4,4] must be given and 16-byte aligned");
  DR_REQUIRE(ctx, target && loss, "antialias_mse: target and loss required");
  return aa_fwd(ctx, color, N, H, W, C, rast, verts, xform, V, tri, T, topo, out, aa_work, target, scale, loss);
}

extern "C" dr_status dr_antialias_xf_bwd_mse(dr_ctx* ctx, const float* color, int N, int H, int W, int C,
                                             const float* rast, const float* verts, int V, const float* xform,
                                             const int32_t* tri, int T, const int32_t* topo, const float* out,
                                             const float* target, float scale, const float* d_loss,
                                             float* d_color, float* d_verts, const void* aa_work) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, xform && aligned16(xform), "antialias_xf_bwd: xform [N,4,4] must be given and 16-byte aligned");
  DR_REQUIRE(ctx, out && target && d_loss, "antialias_bwd_mse: out, target and d_loss required");
  return aa_bwd(ctx, color, N, H, W, C, rast, verts, xform, V, tri, T, topo,
                Cot{nullptr, out, target, 2.0f * scale, d_loss}, d_color, d_verts, aa_work);
}

// ---------------------------------------------------------------------------
// Allocation-free topology hash.
//
// Some callers cannot allocate device memory: a host that owns every byte of
// the GPU through its own pool (a game engine or inference server), or code that
// must not trigger the device-wide synchronisation cudaMalloc implies.  For
// them dr_antialias_construct_topology_hash_static takes no context and
// allocates nothing: its hash table lives in the fixed array below, which every
// GPU that loads this library holds until the process exits.
//
// The table is sized for DR_STATIC_TOPO_MAX_TRIS triangles (3 edges each, load
// factor <= 1/2): 2^19 slots of (key 8 B, count 4 B, two references 4 B each)
// plus one slot index per edge, about 10.8 MB.  Every call clears the part it
// uses before inserting.  All calls share the one array, so calls whose work
// overlaps on the GPU (different streams, or threads sharing a device) race and
// must be serialised by the caller.

namespace {

constexpr uint32_t kStaticCap = 1u << 19;
constexpr size_t kStaticEdges = 3 * (size_t)DR_STATIC_TOPO_MAX_TRIS;
constexpr size_t kStaticBytes = (size_t)kStaticCap * (8 + 4 + 4 + 4) + kStaticEdges * 4;
static_assert(2 * kStaticEdges <= kStaticCap, "static topology table below load factor 1/2");

static __device__ __align__(256) unsigned char g_topo_scratch[kStaticBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
unsigned char* g_static_base[kMaxDevices] = {};

// Device address of g_topo_scratch on the current device.  Host code only sees
// the array's host-side shadow; the device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
dr_status static_scratch(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return DR_ECUDA;
  }
  std::lock_guard<std::mutex> g(g_static_mu);
  if (!g_static_base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_topo_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return DR_ECUDA;
    }
    g_static_base[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_static_base[dev];
  return DR_OK;
}

}  // namespace

extern "C" dr_status dr_antialias_construct_topology_hash_static(const int32_t* tri, int T, int32_t* topo,
                                                                 void* stream) {
  if (T < 0 || T > DR_STATIC_TOPO_MAX_TRIS) return DR_EINVAL;
  if (T == 0) return DR_OK;
  if (!tri || !topo) return DR_EINVAL;
  unsigned char* base = nullptr;
  dr_status st = static_scratch(&base);
  if (st != DR_OK) return st;
  const int64_t E = (int64_t)T * 3;
  uint32_t cap = 1024;
  while (cap < (uint32_t)(2 * E)) cap <<= 1;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(base);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(keys + kStaticCap);
  int32_t* ra = reinterpret_cast<int32_t*>(cnt + kStaticCap);
  int32_t* rb = ra + kStaticCap;
  uint32_t* rs = reinterpret_cast<uint32_t*>(rb + kStaticCap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // An error already pending on this thread belongs to the caller's earlier
  // work: report it without launching, and leave it in place for the caller.
  if (cudaPeekAtLastError() != cudaSuccess) return DR_ECUDA;
  k_topo_init<<<dr::grid_for((int64_t)cap, 256), 256, 0, s>>>(keys, cnt, cap);
  if (cudaGetLastError() != cudaSuccess) return DR_ECUDA;
  k_topo_insert<<<dr::grid_for(E, 256), 256, 0, s>>>(tri, T, keys, cnt, ra, rb, rs, cap - 1, nullptr);
  if (cudaGetLastError() != cudaSuccess) return DR_ECUDA;
  k_topo_classify<<<dr::grid_for(E, 256), 256, 0, s>>>(T, cnt, ra, rb, rs, topo);
  if (cudaGetLastError() != cudaSuccess) return DR_ECUDA;
  return DR_OK;
}
