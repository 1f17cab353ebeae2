// texture_impl.cuh — the texture kernels and their host-side checks, shared
// by texture.cu (forward entry points, pyramid construction) and
// texture_bwd.cu (the VJP entry point, built with FMA contraction: its
// outputs are gradients, compared within tolerances).  Everything here has
// internal linkage; each translation unit instantiates the kernels it
// launches.
//
// The kernels: texture sampling forward / backward for every filter and
// boundary mode, mip pyramid construction and the pyramid-gradient fold.
//
// Reference: Sources/MLXDiffRast/Texture.swift.
//   bilinear       diffrast_texture_fwd / _grad_tex / _grad_uv  (359-521)
//   nearest        _nearest_fwd / _nearest_grad_tex             (545-605)
//   cube           _cube_fwd / _cube_grad_tex                   (616-738)
//   mipmap         _trilinear_fwd / _grad_pyramid / _grad_uv / _grad_uvda
//                  (764-1102), pyramid = textureConstructMip (144-161)
//   mip-mapped cube and the cube d_dir chain rule: extensions (the reference
//                  takes .linear only for cube maps and returns d_dir = 0)
// Each backward here is ONE kernel (d_tex scatter + d_uv + d_uvDA together)
// instead of the reference's two or three passes; its d_tex scatter sums the
// pixels of a warp that hit the same texel first and issues float2 / float4
// atomics.  A texture with batch 1 is
// sampled directly (the reference broadcasts it to N copies and builds N
// pyramids, Texture.swift:282-285); gradients accumulate into the one copy.
// Pyramid gradients of levels >= 1 are folded into d_tex level 0 by one kernel,
// which is what MLX's autograd of reshape/mean/concatenate computes.
#pragma once
#include "common.cuh"

using dr::grid_for;

namespace {

struct MipDesc {
  int L;                       // number of levels, level 0 = tex
  int h[DR_MAX_MIP_LEVELS];
  int w[DR_MAX_MIP_LEVELS];
  int64_t off[DR_MAX_MIP_LEVELS];  // float offset of level k (k >= 1) in the pyramid
};

MipDesc mip_desc(int Nt, int Ht, int Wt, int C, int max_level, int64_t* total) {
  MipDesc m{};
  m.L = 1;
  m.h[0] = Ht; m.w[0] = Wt; m.off[0] = -1;
  int64_t tot = 0;
  int H = Ht, W = Wt;
  // Texture.swift:153-159: halve while both dims are even and >= 2.
  while (H >= 2 && W >= 2 && (H % 2) == 0 && (W % 2) == 0) {
    if (max_level >= 0 && m.L > max_level) break;
    if (m.L >= DR_MAX_MIP_LEVELS) break;
    H /= 2; W /= 2;
    m.h[m.L] = H; m.w[m.L] = W; m.off[m.L] = tot;
    tot += (int64_t)Nt * H * W * C;
    m.L++;
  }
  *total = tot;
  return m;
}

// apply_boundary (Texture.swift:336-354).  MODE 0 wrap, 1 clamp, 2 zero.
template <int MODE>
__device__ __forceinline__ int apply_boundary(int t, int size, float& oob) {
  if (MODE == 2) {
    if (t < 0 || t >= size) { oob = 1.0f; return 0; }
    oob = 0.0f;
    return t;
  }
  oob = 0.0f;
  if (MODE == 1) return t < 0 ? 0 : (t >= size ? size - 1 : t);
  int r = t % size;
  if (r < 0) r += size;
  return r;
}

struct Taps {
  int64_t a00, a10, a01, a11;  // texel index (times C added by caller)
  float fx, fy;
  float w00, w10, w01, w11;
  float m00, m10, m01, m11;
};

// Bilinear taps with texel centres at tx = u*W - 0.5 (Texture.swift:372-391).
template <int MODE>
__device__ __forceinline__ Taps bilin_taps(float u, float v, int Wk, int Hk) {
  Taps q;
  const float tx = u * (float)Wk - 0.5f;
  const float ty = v * (float)Hk - 0.5f;
  const int tx0 = dr_floor_i(tx), ty0 = dr_floor_i(ty);
  const int tx1 = (int)((unsigned)tx0 + 1u), ty1 = (int)((unsigned)ty0 + 1u);
  q.fx = tx - (float)tx0;
  q.fy = ty - (float)ty0;
  float ox0, ox1, oy0, oy1;
  const int ix0 = apply_boundary<MODE>(tx0, Wk, ox0), ix1 = apply_boundary<MODE>(tx1, Wk, ox1);
  const int iy0 = apply_boundary<MODE>(ty0, Hk, oy0), iy1 = apply_boundary<MODE>(ty1, Hk, oy1);
  const float fx = q.fx, fy = q.fy;
  q.w00 = (1.0f - fx) * (1.0f - fy) * (1.0f - ox0) * (1.0f - oy0);
  q.w10 = (fx) * (1.0f - fy) * (1.0f - ox1) * (1.0f - oy0);
  q.w01 = (1.0f - fx) * (fy) * (1.0f - ox0) * (1.0f - oy1);
  q.w11 = (fx) * (fy) * (1.0f - ox1) * (1.0f - oy1);
  q.m00 = (1.0f - ox0) * (1.0f - oy0);
  q.m10 = (1.0f - ox1) * (1.0f - oy0);
  q.m01 = (1.0f - ox0) * (1.0f - oy1);
  q.m11 = (1.0f - ox1) * (1.0f - oy1);
  q.a00 = (int64_t)iy0 * Wk + ix0;
  q.a10 = (int64_t)iy0 * Wk + ix1;
  q.a01 = (int64_t)iy1 * Wk + ix0;
  q.a11 = (int64_t)iy1 * Wk + ix1;
  return q;
}

__device__ __forceinline__ float sample4(const float* __restrict__ b, const Taps& q, int C, int c) {
  const float t00 = __ldg(b + q.a00 * C + c), t10 = __ldg(b + q.a10 * C + c);
  const float t01 = __ldg(b + q.a01 * C + c), t11 = __ldg(b + q.a11 * C + c);
  return q.w00 * t00 + q.w10 * t10 + q.w01 * t01 + q.w11 * t11;
}

// Per-CTA cache of "hot" texels for the d_tex scatter: a warp whose 32 lanes
// all hit one texel (typically background pixels that share one sample
// point) adds its sum here instead of to global memory, so the many warps of
// a CTA that hit the same texel issue one global atomic per channel between
// them.  8 direct-mapped slots keyed by the destination address, C <= 4.
constexpr int kHotSlots = 8, kHotC = 4;
struct HotCache {
  unsigned long long key[kHotSlots];
  float val[kHotSlots][kHotC];
};

__device__ __forceinline__ void hot_init(HotCache* hc) {
  if (threadIdx.x < kHotSlots) {
    hc->key[threadIdx.x] = 0ull;
#pragma unroll
    for (int c = 0; c < kHotC; ++c) hc->val[threadIdx.x][c] = 0.0f;
  }
}

// After every warp's last scatter_tap (a CTA barrier first): one atomic per
// cached texel and channel.
__device__ __forceinline__ void hot_flush(HotCache* hc, int C) {
  __syncthreads();
  if (threadIdx.x < kHotSlots && hc->key[threadIdx.x] != 0ull) {
    float* p = reinterpret_cast<float*>(hc->key[threadIdx.x]);
    for (int c = 0; c < C && c < kHotC; ++c) {
      const float v = hc->val[threadIdx.x][c];
      if (v != 0.0f) atomicAdd(p + c, v);
    }
  }
}

// Global float atomics of one texel's C <= 4 channel sums, as wide as the
// address allows: one float4 (16-byte aligned C == 4), else float2 pairs on
// 8-byte boundaries and scalars around them.  All-zero groups issue nothing
// (d_tex starts at +0 and adding +-0 leaves every value unchanged).
__device__ __forceinline__ void red_add(float* p, float a) {
  if (a != 0.0f) atomicAdd(p, a);
}
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  if (a != 0.0f || b != 0.0f) atomicAdd(reinterpret_cast<float2*>(p), make_float2(a, b));
}
__device__ __forceinline__ void red_add_texel(float* p, int C, float v0, float v1, float v2, float v3) {
  const uintptr_t ad = (uintptr_t)p;
  const bool a8 = (ad & 7) == 0;
  switch (C) {
    case 1:
      red_add(p, v0);
      return;
    case 2:
      if (a8) {
        red_add2(p, v0, v1);
      } else {
        red_add(p, v0);
        red_add(p + 1, v1);
      }
      return;
    case 3: {
      // Texels of 12 bytes alternate between 8-byte aligned and not: every
      // lane issues one float2 (channels 0-1 or 1-2) and one scalar (2 or 0)
      // with per-lane addresses, so the warp runs two atomics, not two paths.
      red_add2(a8 ? p : p + 1, a8 ? v0 : v1, a8 ? v1 : v2);
      red_add(a8 ? p + 2 : p, a8 ? v2 : v0);
      return;
    }
    default:  // 4
      if ((ad & 15) == 0) {
        if (v0 != 0.0f || v1 != 0.0f || v2 != 0.0f || v3 != 0.0f)
          atomicAdd(reinterpret_cast<float4*>(p), make_float4(v0, v1, v2, v3));
      } else if (a8) {
        red_add2(p, v0, v1);
        red_add2(p + 2, v2, v3);
      } else {
        red_add(p, v0);
        red_add2(p + 1, v1, v2);
        red_add(p + 3, v3);
      }
      return;
  }
}

// d_tex scatter of one tap for C <= 4: adds v.{x,y,z,w}[c] (c < C) to p[c] for
// every lane.  Lanes of a warp that hit the same texel (runs of neighbouring
// pixels: a magnified texture, or background pixels that all sample one
// texel) are summed first with a segmented warp reduction, so each run issues
// one (vector) atomic instead of one per pixel; a run covering the whole warp
// goes to the CTA's hot cache when one is given.  All 32 lanes of the warp
// must call it; lanes with on == false add nothing.
// so >= 0: the tap's texel is held at s_small[so .. so + C) (the CTA's shared
// copy of the small levels, see SmallLevels below) instead of at p.
__device__ __forceinline__ void scatter_tap4(float* p, float4 v, int C, bool on, int lane, HotCache* hc,
                                             float* s_small = nullptr, int so = -1) {
  const bool smem = so >= 0;
  float* sp = s_small + so;
  const long long key = on ? (long long)(uintptr_t)p : -1ll - (long long)lane;
  bool head;
  const int seg_end = warp_runs(key, lane, head);
  const int span = warp_max_run(lane, seg_end, head);
  if (!on) v = make_float4(0.f, 0.f, 0.f, 0.f);
  // A run spanning the warp has one key, so all 32 lanes are on and share p
  // (or all share sp: the small levels are already reduced per CTA).
  if (hc && span == 32 && !smem) {
    // One run spans the warp: all 32 lanes are on and share p.
    float sum[kHotC] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < kHotC; ++c) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum[c] += __shfl_xor_sync(0xffffffffu, sum[c], o);
    }
    if (lane == 0) {
      const unsigned long long k = (unsigned long long)(uintptr_t)p;
      const int slot = (int)((k >> 4) % kHotSlots);
      const unsigned long long prev = atomicCAS(&hc->key[slot], 0ull, k);
      if (prev == 0ull || prev == k) {
#pragma unroll
        for (int c = 0; c < kHotC; ++c)
          if (c < C && sum[c] != 0.0f) atomicAdd(&hc->val[slot][c], sum[c]);
      } else {
        red_add_texel(p, C, sum[0], sum[1], sum[2], sum[3]);
      }
    }
    return;
  }
  if (span > 1) {
    // All four lanes of the float4 in one step loop (channels past C are
    // zero and never stored).
    float vv[4] = {v.x, v.y, v.z, v.w};
    warp_seg_sum_n<4>(vv, lane, seg_end, span);
    v = make_float4(vv[0], vv[1], vv[2], vv[3]);
  }
  if (on && head) {
    if (smem) {
      // The CTA's shared copy of the small levels: scalar shared atomics.
      if (v.x != 0.0f) atomicAdd(sp, v.x);
      if (C > 1 && v.y != 0.0f) atomicAdd(sp + 1, v.y);
      if (C > 2 && v.z != 0.0f) atomicAdd(sp + 2, v.z);
      if (C > 3 && v.w != 0.0f) atomicAdd(sp + 3, v.w);
    } else {
      red_add_texel(p, C, v.x, v.y, v.z, v.w);
    }
  }
}

// Contribution w * (g[c] * gscale) of one tap, C <= 4 (unused channels 0).
__device__ __forceinline__ float4 tap_contrib(float w, const float4 g, float gscale) {
  return make_float4(w * (g.x * gscale), w * (g.y * gscale), w * (g.z * gscale), w * (g.w * gscale));
}

__device__ __forceinline__ float4 load_cot(const float* __restrict__ g, int C, bool vec4) {
  if (vec4) return ldg4(g);
  return make_float4(__ldg(g), C > 1 ? __ldg(g + 1) : 0.f, C > 2 ? __ldg(g + 2) : 0.f, C > 3 ? __ldg(g + 3) : 0.f);
}

// d_tex scatter of one tap: adds w * (g[c] * gscale) to p[c] (c < C).  As
// scatter_tap4 for C <= 4; wider texels sum each channel over the runs and
// issue scalar atomics from the run heads.  A zero contribution issues no
// atomic (d_tex starts at +0, and adding +-0 to +0 leaves +0).
__device__ __forceinline__ void scatter_tap(float* p, float w, const float* __restrict__ g, float gscale, int C,
                                            bool on, int lane, HotCache* hc = nullptr, float* s_small = nullptr,
                                            int so = -1) {
  if (C <= 4) {
    const float4 gv = on ? load_cot(g, C, false) : make_float4(0.f, 0.f, 0.f, 0.f);
    scatter_tap4(p, tap_contrib(w, gv, gscale), C, on, lane, hc, s_small, so);
    return;
  }
  const bool smem = so >= 0;
  const long long key = on ? (long long)(uintptr_t)p : -1ll - (long long)lane;
  bool head;
  const int seg_end = warp_runs(key, lane, head);
  const int span = warp_max_run(lane, seg_end, head);
  for (int c = 0; c < C; ++c) {
    float v = on ? w * (__ldg(g + c) * gscale) : 0.0f;
    if (span > 1) v = warp_seg_sum(v, lane, seg_end, span);
    if (on && head && v != 0.0f) {
      if (smem) atomicAdd(s_small + so + c, v);
      else atomicAdd(p + c, v);
    }
  }
}

// The four taps of one bilinear sample (weights q.w**, clamp / wrap / zero
// masks included): the pixel's cotangent g (C channels; gv = its first four)
// times `scale` and each tap's weight.
// slev >= 0: the level is held in the CTA's shared copy of the small levels,
// starting at s_small[slev]; its taps go there.
__device__ __forceinline__ void scatter_bilin(float* db, const Taps& q, const float* __restrict__ g, float4 gv,
                                              float scale, int C, bool on, int lane, HotCache* hc,
                                              float* s_small = nullptr, int slev = -1) {
  if (C <= 4) {
    // A rolled loop: one copy of the scatter code (the unrolled four copies
    // measured slower, instruction-fetch bound).
#pragma unroll 1
    for (int tp = 0; tp < 4; ++tp) {
      const int64_t a = tp == 0 ? q.a00 : (tp == 1 ? q.a10 : (tp == 2 ? q.a01 : q.a11));
      const float w = tp == 0 ? q.w00 : (tp == 1 ? q.w10 : (tp == 2 ? q.w01 : q.w11));
      scatter_tap4(db + a * C, tap_contrib(w, gv, scale), C, on, lane, hc, s_small,
                   slev >= 0 ? slev + (int)a * C : -1);
    }
  } else {
    scatter_tap(db + q.a00 * C, q.w00, g, scale, C, on, lane, hc, s_small, slev >= 0 ? slev + (int)q.a00 * C : -1);
    scatter_tap(db + q.a10 * C, q.w10, g, scale, C, on, lane, hc, s_small, slev >= 0 ? slev + (int)q.a10 * C : -1);
    scatter_tap(db + q.a01 * C, q.w01, g, scale, C, on, lane, hc, s_small, slev >= 0 ? slev + (int)q.a01 * C : -1);
    scatter_tap(db + q.a11 * C, q.w11, g, scale, C, on, lane, hc, s_small, slev >= 0 ? slev + (int)q.a11 * C : -1);
  }
}

// Shared-memory reduction of the pyramid's smallest levels.  Every pixel whose
// LOD reaches a level of a few texels scatters into the same handful of
// addresses; the mip VJPs keep the gradient of the levels [ks, L) of a shared
// texture (the tail of the pyramid gradient buffer, contiguous from
// base = off[ks]) in shared memory and add it to global memory once per CTA,
// one atomic per non-zero float.  ks == L (n == 0) holds nothing.
// 4 KB: the shared copy is carved out of the L1 the texel gathers use, so it
// holds only the top levels, where the contention is (a few texels per level).
constexpr int kSmallCap = 1024;  // floats
struct SmallLevels {
  int ks;
  int n;
  int64_t base;
};

__device__ __forceinline__ void small_init(float* s, const SmallLevels& sl) {
  for (int i = threadIdx.x; i < sl.n; i += blockDim.x) s[i] = 0.0f;
}

// After a CTA barrier: the CTA's sums into the pyramid gradient.
__device__ __forceinline__ void small_flush(const float* s, const SmallLevels& sl, float* __restrict__ d_pyr) {
  for (int i = threadIdx.x; i < sl.n; i += blockDim.x) {
    const float v = s[i];
    if (v != 0.0f) atomicAdd(d_pyr + sl.base + i, v);
  }
}

template <int MODE>
__global__ void k_tex_linear_fwd(const float* __restrict__ tex, bool tex_shared, int Ht, int Wt, int C,
                                 const float2* __restrict__ uv, int64_t P, int64_t HWi,
                                 float* __restrict__ out) {
  int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= P) return;
  const float2 t = __ldg(uv + pix);
  const Taps q = bilin_taps<MODE>(t.x, t.y, Wt, Ht);
  const float* b = tex + (tex_shared ? 0 : (pix / HWi) * Ht * Wt * C);
  float* o = out + pix * C;
  for (int c = 0; c < C; ++c) o[c] = sample4(b, q, C, c);
}

// d_tex scatter (Texture.swift:407-459) and d_uv (472-521) in one pass.
template <int MODE>
__global__ void __launch_bounds__(256, DR_MINB_TEX_BWD) k_tex_linear_bwd(const float* __restrict__ tex, bool tex_shared, int Ht, int Wt, int C,
                                 const float2* __restrict__ uv, int64_t P, int64_t HWi,
                                 const float* __restrict__ d_out, float* __restrict__ d_tex,
                                 float2* __restrict__ d_uv) {
  const int64_t pix0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool on = pix0 < P;
  const int64_t pix = on ? pix0 : P - 1;  // out-of-range lanes follow a valid pixel, adding nothing
  const int lane = threadIdx.x & 31;
  const float2 t = __ldg(uv + pix);
  const Taps q = bilin_taps<MODE>(t.x, t.y, Wt, Ht);
  const int64_t base = tex_shared ? 0 : (pix / HWi) * Ht * Wt * C;
  const float* b = tex + base;
  float* db = d_tex + base;
  const float* g = d_out + pix * C;
  const float4 gv = (on && C <= 4) ? load_cot(g, C, false) : make_float4(0.f, 0.f, 0.f, 0.f);
  __shared__ HotCache hc;
  hot_init(&hc);
  __syncthreads();
  scatter_bilin(db, q, g, gv, 1.0f, C, on, lane, &hc);
  hot_flush(&hc, C);
  if (!on) return;
  const float fx = q.fx, fy = q.fy;
  float dfx_sum = 0.0f, dfy_sum = 0.0f;
  for (int c = 0; c < C; ++c) {
    const float gc = __ldg(g + c);
    const float t00 = __ldg(b + q.a00 * C + c) * q.m00, t10 = __ldg(b + q.a10 * C + c) * q.m10;
    const float t01 = __ldg(b + q.a01 * C + c) * q.m01, t11 = __ldg(b + q.a11 * C + c) * q.m11;
    dfx_sum += gc * ((1.0f - fy) * (t10 - t00) + fy * (t11 - t01));
    dfy_sum += gc * ((1.0f - fx) * (t01 - t00) + fx * (t11 - t10));
  }
  d_uv[pix] = make_float2(dfx_sum * (float)Wt, dfy_sum * (float)Ht);
}

// ----------------------------------------------------------------- nearest

template <int MODE>
__global__ void k_tex_nearest(const float* __restrict__ tex, bool tex_shared, int Ht, int Wt, int C,
                              const float2* __restrict__ uv, int64_t P, int64_t HWi,
                              float* __restrict__ out, const float* __restrict__ d_out,
                              float* __restrict__ d_tex, float2* __restrict__ d_uv) {
  const int64_t pix0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (out && pix0 >= P) return;  // the forward has no warp collectives
  const bool on = pix0 < P;
  const int64_t pix = on ? pix0 : P - 1;
  const float2 t = __ldg(uv + pix);
  const int tx = dr_floor_i(t.x * (float)Wt), ty = dr_floor_i(t.y * (float)Ht);
  float ox, oy;
  const int ix = apply_boundary<MODE>(tx, Wt, ox), iy = apply_boundary<MODE>(ty, Ht, oy);
  const float mask = (1.0f - ox) * (1.0f - oy);
  const int64_t base = (tex_shared ? 0 : (pix / HWi) * Ht * Wt * C) + ((int64_t)iy * Wt + ix) * C;
  if (out) {
    for (int c = 0; c < C; ++c) out[pix * C + c] = __ldg(tex + base + c) * mask;
  } else {
    // d_tex += g * mask: the tap weight is the mask (Texture.swift:576-605).
    scatter_tap(d_tex + base, mask, d_out + pix * C, 1.0f, C, on, threadIdx.x & 31);
    if (on) d_uv[pix] = make_float2(0.0f, 0.0f);
  }
}

// -------------------------------------------------------------------- cube

// Cube projection (Texture.swift:616-636), face order +X,-X,+Y,-Y,+Z,-Z.
__device__ __forceinline__ void cube_project(float x, float y, float z, int& face, float& u, float& v) {
  const float ax = fabsf(x), ay = fabsf(y), az = fabsf(z);
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
  const float inv_ma = 1.0f / ma;
  u = (sc * inv_ma + 1.0f) * 0.5f;
  v = (tc * inv_ma + 1.0f) * 0.5f;
}

// Face of a direction with its (s, t, major) axes and signs, chosen as
// cube_project chooses them: sc = ss * d[sa], tc = ts * d[ta], ma = ms * d[ma].
struct CubeFrame {
  int face, sa, ta, ma;
  float ss, ts, ms, sc, tc, inv_ma, u, v;
};

__device__ __forceinline__ float pick3(int a, float x, float y, float z) { return a == 0 ? x : (a == 1 ? y : z); }

__device__ __forceinline__ CubeFrame cube_frame(float x, float y, float z) {
  CubeFrame f;
  cube_project(x, y, z, f.face, f.u, f.v);
  // Faces +X,-X,+Y,-Y,+Z,-Z: sc = (-z, z, x, x, x, -x), tc = (-y, -y, z, -z, -y, -y).
  switch (f.face) {
    case 0: f.sa = 2; f.ta = 1; f.ma = 0; f.ss = -1.f; f.ts = -1.f; f.ms = 1.f; break;
    case 1: f.sa = 2; f.ta = 1; f.ma = 0; f.ss = 1.f; f.ts = -1.f; f.ms = -1.f; break;
    case 2: f.sa = 0; f.ta = 2; f.ma = 1; f.ss = 1.f; f.ts = 1.f; f.ms = 1.f; break;
    case 3: f.sa = 0; f.ta = 2; f.ma = 1; f.ss = 1.f; f.ts = -1.f; f.ms = -1.f; break;
    case 4: f.sa = 0; f.ta = 1; f.ma = 2; f.ss = 1.f; f.ts = -1.f; f.ms = 1.f; break;
    default: f.sa = 0; f.ta = 1; f.ma = 2; f.ss = -1.f; f.ts = -1.f; f.ms = -1.f; break;
  }
  f.sc = f.ss * pick3(f.sa, x, y, z);
  f.tc = f.ts * pick3(f.ta, x, y, z);
  f.inv_ma = 1.0f / (f.ms * pick3(f.ma, x, y, z));
  return f;
}

// Per-pixel direction derivatives, interpolate's interleaved layout:
// [dx/dX, dx/dY, dy/dX, dy/dY, dz/dX, dz/dY].
struct DirDA {
  float2 a[3];  // a[axis] = (d/dX, d/dY)
};

__device__ __forceinline__ float2 pick_axis(const DirDA& d, int a) {
  return a == 0 ? d.a[0] : (a == 1 ? d.a[1] : d.a[2]);
}

// (du/dX, du/dY, dv/dX, dv/dY) of the face coordinates:
//   u = (sc / ma + 1) / 2  =>  du = (dsc - (sc / ma) dma) / (2 ma).
__device__ __forceinline__ float4 cube_uv_da(const CubeFrame& f, const DirDA& d) {
  const float h = 0.5f * f.inv_ma;
  const float ks = (f.sc * f.inv_ma) * f.ms, kt = (f.tc * f.inv_ma) * f.ms;
  const float2 ds = pick_axis(d, f.sa), dt = pick_axis(d, f.ta), dm = pick_axis(d, f.ma);
  return make_float4(h * (f.ss * ds.x - ks * dm.x), h * (f.ss * ds.y - ks * dm.y),
                     h * (f.ts * dt.x - kt * dm.x), h * (f.ts * dt.y - kt * dm.y));
}

// Transpose of cube_uv_da.
__device__ __forceinline__ DirDA cube_uv_da_vjp(const CubeFrame& f, const float4 g) {
  const float h = 0.5f * f.inv_ma;
  const float ks = (f.sc * f.inv_ma) * f.ms, kt = (f.tc * f.inv_ma) * f.ms;
  const float2 gs = make_float2(g.x * (h * f.ss), g.y * (h * f.ss));
  const float2 gt = make_float2(g.z * (h * f.ts), g.w * (h * f.ts));
  const float2 gm = make_float2(-(g.x * (h * ks) + g.z * (h * kt)), -(g.y * (h * ks) + g.w * (h * kt)));
  DirDA r;
#pragma unroll
  for (int a = 0; a < 3; ++a) r.a[a] = a == f.sa ? gs : (a == f.ta ? gt : gm);
  return r;
}

// d(loss)/d(dir) (extension; the reference returns zero, Texture.swift:196-197)
// from d(loss)/d(u, v) through u = (sc/ma + 1)/2, v alike, as per-axis values
// (s axis, t axis, major axis).
struct AxisGrad {
  float s, t, m;
};

__device__ __forceinline__ AxisGrad cube_dir_vjp(const CubeFrame& f, float d_u, float d_v) {
  const float h = 0.5f * f.inv_ma;
  AxisGrad r;
  r.s = d_u * (h * f.ss);
  r.t = d_v * (h * f.ts);
  r.m = -((d_u * f.sc + d_v * f.tc) * (h * f.inv_ma)) * f.ms;
  return r;
}

// The LOD's dependence on the direction: with G = d(loss)/d(eff) * s, add
// the Jacobian of cube_uv_da with respect to sc, tc and ma, transposed.
__device__ __forceinline__ void cube_dir_lod_vjp(const CubeFrame& f, const DirDA& d, const float4 G,
                                                 AxisGrad& r) {
  const float a = f.inv_ma, a2 = a * a;
  const float2 ds = pick_axis(d, f.sa), dt = pick_axis(d, f.ta), dm = pick_axis(d, f.ma);
  const float gsm = G.x * dm.x + G.y * dm.y, gtm = G.z * dm.x + G.w * dm.y;
  const float gss = G.x * ds.x + G.y * ds.y, gtt = G.z * dt.x + G.w * dt.y;
  const float hm = (0.5f * a2) * f.ms;
  r.s += -(hm * f.ss) * gsm;
  r.t += -(hm * f.ts) * gtm;
  r.m += -(hm * (f.ss * gss + f.ts * gtt)) + (a2 * a) * (f.sc * gsm + f.tc * gtm);
}

__device__ __forceinline__ void store_dir_grad(float* __restrict__ d_dir, int64_t pix, const CubeFrame& f,
                                               const AxisGrad& r) {
  float v[3];
#pragma unroll
  for (int a = 0; a < 3; ++a) v[a] = a == f.sa ? r.s : (a == f.ta ? r.t : r.m);
  d_dir[3 * pix] = v[0];
  d_dir[3 * pix + 1] = v[1];
  d_dir[3 * pix + 2] = v[2];
}

__device__ __forceinline__ DirDA load_dir_da(const float2* __restrict__ p, int64_t pix) {
  DirDA d;
  d.a[0] = __ldg(p + 3 * pix);
  d.a[1] = __ldg(p + 3 * pix + 1);
  d.a[2] = __ldg(p + 3 * pix + 2);
  return d;
}

__global__ void __launch_bounds__(256, DR_MINB_TEX_BWD) k_tex_cube(const float* __restrict__ tex, bool tex_shared, int Ht, int Wt, int C,
                           const float* __restrict__ dir, int64_t P, int64_t HWi, float* __restrict__ out,
                           const float* __restrict__ d_out, float* __restrict__ d_tex,
                           float* __restrict__ d_dir, bool dir_grad) {
  const int64_t pix0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (out && pix0 >= P) return;  // the forward has no warp collectives
  const bool on = pix0 < P;
  const int64_t pix = on ? pix0 : P - 1;
  const CubeFrame f = cube_frame(__ldg(dir + 3 * pix), __ldg(dir + 3 * pix + 1), __ldg(dir + 3 * pix + 2));
  const int face = f.face;
  // Per-face clamp bilinear (Texture.swift:656-672): weights carry no OOB mask.
  Taps q = bilin_taps<1>(f.u, f.v, Wt, Ht);
  const float fx = q.fx, fy = q.fy;
  const float w00 = (1.0f - fx) * (1.0f - fy), w10 = fx * (1.0f - fy);
  const float w01 = (1.0f - fx) * fy, w11 = fx * fy;
  const int64_t fb = ((tex_shared ? 0 : (pix / HWi)) * 6 + face) * (int64_t)Ht * Wt * C;
  if (out) {
    for (int c = 0; c < C; ++c) {
      const float t00 = __ldg(tex + fb + q.a00 * C + c), t10 = __ldg(tex + fb + q.a10 * C + c);
      const float t01 = __ldg(tex + fb + q.a01 * C + c), t11 = __ldg(tex + fb + q.a11 * C + c);
      out[pix * C + c] = w00 * t00 + w10 * t10 + w01 * t01 + w11 * t11;
    }
  } else {
    const int lane = threadIdx.x & 31;
    const float* g = d_out + pix * C;
    const float4 gv = (on && C <= 4) ? load_cot(g, C, false) : make_float4(0.f, 0.f, 0.f, 0.f);
    __shared__ HotCache hc;
    hot_init(&hc);
    __syncthreads();
    // q.w** equal w** here: clamp taps carry no OOB mask.
    scatter_bilin(d_tex + fb, q, g, gv, 1.0f, C, on, lane, &hc);
    hot_flush(&hc, C);
    if (!on) return;
    // d_dir is identically zero in the reference (Texture.swift:196-197); the
    // chain rule through the projection is an opt-in extension.
    AxisGrad ag = {0.0f, 0.0f, 0.0f};
    if (dir_grad) {
      float dfx = 0.0f, dfy = 0.0f;
      for (int c = 0; c < C; ++c) {
        const float gc = __ldg(g + c);
        const float t00 = __ldg(tex + fb + q.a00 * C + c), t10 = __ldg(tex + fb + q.a10 * C + c);
        const float t01 = __ldg(tex + fb + q.a01 * C + c), t11 = __ldg(tex + fb + q.a11 * C + c);
        dfx += gc * ((1.0f - fy) * (t10 - t00) + fy * (t11 - t01));
        dfy += gc * ((1.0f - fx) * (t01 - t00) + fx * (t11 - t10));
      }
      ag = cube_dir_vjp(f, dfx * (float)Wt, dfy * (float)Ht);
    }
    store_dir_grad(d_dir, pix, f, ag);
  }
}

// ------------------------------------------------------------------ mipmap

// 2x2 box filter of one level, 4 channels per thread (C == 4, 16-byte
// aligned): the same ((t00 + t01) + (t10 + t11)) / 4 per channel.  n_out
// counts output texels.
__global__ void k_mip_down4(const float4* __restrict__ src, int Hs, int Ws, float4* __restrict__ dst, int Hd,
                            int Wd, int64_t n_out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_out) return;
  const int x = (int)(i % Wd);
  const int64_t ny = i / Wd;  // n * Hd + y
  const int y = (int)(ny % Hd);
  const int64_t n = ny / Hd;
  const float4* s = src + n * Hs * Ws;
  const float4 a = __ldg(s + (int64_t)(2 * y) * Ws + 2 * x);
  const float4 b = __ldg(s + (int64_t)(2 * y) * Ws + 2 * x + 1);
  const float4 c = __ldg(s + (int64_t)(2 * y + 1) * Ws + 2 * x);
  const float4 d = __ldg(s + (int64_t)(2 * y + 1) * Ws + 2 * x + 1);
  dst[i] = make_float4(((a.x + b.x) + (c.x + d.x)) * 0.25f, ((a.y + b.y) + (c.y + d.y)) * 0.25f,
                       ((a.z + b.z) + (c.z + d.z)) * 0.25f, ((a.w + b.w) + (c.w + d.w)) * 0.25f);
}

// 2x2 box filter of one level: ((t00 + t01) + (t10 + t11)) / 4.
__global__ void k_mip_down(const float* __restrict__ src, int Hs, int Ws, float* __restrict__ dst, int Hd,
                           int Wd, int C, int64_t n_out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_out) return;
  const int c = (int)(i % C);
  const int x = (int)((i / C) % Wd);
  const int64_t ny = i / ((int64_t)C * Wd);  // n * Hd + y
  const int y = (int)(ny % Hd);
  const int64_t n = ny / Hd;
  const float* s = src + n * Hs * Ws * C;
  const float a = __ldg(s + ((int64_t)(2 * y) * Ws + 2 * x) * C + c);
  const float b = __ldg(s + ((int64_t)(2 * y) * Ws + 2 * x + 1) * C + c);
  const float cc = __ldg(s + ((int64_t)(2 * y + 1) * Ws + 2 * x) * C + c);
  const float d = __ldg(s + ((int64_t)(2 * y + 1) * Ws + 2 * x + 1) * C + c);
  dst[i] = ((a + b) + (cc + d)) * 0.25f;
}

// 2^x and log2(x) evaluated in double and rounded once to float, so the CPU
// oracle (which does the same with the C library) agrees to the bit in all but
// vanishingly rare rounding ties; the float versions differ by an ulp between
// CUDA and glibc, which moves the LOD.
__device__ __forceinline__ float exp2_rn(float x) { return (float)exp2((double)x); }
__device__ __forceinline__ float log2_rn(float x) { return (float)log2((double)x); }

// Effective uvDA = uvDA * 2^map * 2^bias (Texture.swift:104-126).
__device__ __forceinline__ float4 effective_da(const float4 da, int64_t pix, float bias,
                                               const float* __restrict__ bias_map, float& s) {
  s = 1.0f;
  bool scaled = false;
  if (bias_map) {
    s = exp2_rn(__ldg(bias_map + pix));
    if (bias != 0.0f) s = s * exp2_rn(bias);
    scaled = true;
  } else if (bias != 0.0f) {
    s = exp2_rn(bias);
    scaled = true;
  }
  if (!scaled) return da;
  return make_float4(da.x * s, da.y * s, da.z * s, da.w * s);
}

struct LodSel {
  int k0, k1;
  float frac;
  float raw;  // the unclamped LOD (K22 uses it)
};

// Texture.swift:764-790.
template <bool MIP_LINEAR>
__device__ __forceinline__ LodSel lod_select(const float4 e, int Ht, int Wt, int L) {
  const float sx = e.x * (float)Wt, sy = e.y * (float)Wt;
  const float tx = e.z * (float)Ht, ty = e.w * (float)Ht;
  const float rho_sq = fmaxf(sx * sx + tx * tx, sy * sy + ty * ty);
  float lod = 0.5f * log2_rn(fmaxf(rho_sq, 1e-20f));
  LodSel s;
  s.raw = lod;
  lod = fmaxf(0.0f, fminf((float)(L - 1), lod));
  if (MIP_LINEAR) {
    s.k0 = dr_floor_i(lod);
    s.k1 = s.k0 + 1;
    if (s.k1 >= L) s.k1 = L - 1;
    s.frac = lod - (float)s.k0;
  } else {
    s.k0 = dr_floor_i(lod + 0.5f);
    if (s.k0 >= L) s.k0 = L - 1;
    s.k1 = s.k0;
    s.frac = 0.0f;
  }
  return s;
}

__device__ __forceinline__ const float* level_ptr(const float* tex, const float* pyr, const MipDesc& m, int k,
                                                  int64_t nt, int C) {
  const float* b = (k == 0) ? tex : pyr + m.off[k];
  return b + nt * (int64_t)m.h[k] * m.w[k] * C;
}

// K22 (Texture.swift:1011-1102): d(loss)/d(eff) of the effective uvDA through
// the LOD, independent of MIP_LINEAR.  lod_interior: whether the unclamped
// LOD has a gradient; lod_grad: the gradient given
// d_lod = sum over the two levels floor(lod), floor(lod) + 1 of
// (-1, +1) * sample_c * g_c, accumulated level by level, channel by channel.
__device__ __forceinline__ bool lod_interior(float lod_raw, int L) {
  return !(lod_raw <= 0.0f || lod_raw >= (float)(L - 1));
}

__device__ __forceinline__ float4 lod_grad(const float4 e, int Ht, int Wt, float d_lod) {
  const float sx = e.x * (float)Wt, sy = e.y * (float)Wt;
  const float tx_ = e.z * (float)Ht, ty_ = e.w * (float)Ht;
  const float Asq = sx * sx + tx_ * tx_, Bsq = sy * sy + ty_ * ty_;
  const float rho_sq = fmaxf(Asq, Bsq);
  const float ln2 = 0.6931471805599453f;
  const float dlod_drho_sq = 1.0f / (2.0f * rho_sq * ln2);
  const float A_is_max = (Asq >= Bsq) ? 1.0f : 0.0f;
  const float B_is_max = 1.0f - A_is_max;
  return make_float4(d_lod * dlod_drho_sq * A_is_max * 2.0f * sx * (float)Wt,
                     d_lod * dlod_drho_sq * B_is_max * 2.0f * sy * (float)Wt,
                     d_lod * dlod_drho_sq * A_is_max * 2.0f * tx_ * (float)Ht,
                     d_lod * dlod_drho_sq * B_is_max * 2.0f * ty_ * (float)Ht);
}

// The same, sampling the two levels itself (mip-nearest, whose sampled level
// is not floor(lod), and callers that did not keep the samples).  `img`
// selects the image in each level (texture batch entry, or batch * 6 + face
// for a cube).
template <int MODE>
__device__ __forceinline__ float4 lod_vjp(const float4 e, const MipDesc& m, const float* __restrict__ tex,
                                          const float* __restrict__ pyr, int64_t img, int C, float u, float v,
                                          float lod_raw, const float* __restrict__ g) {
  const int L = m.L;
  if (!lod_interior(lod_raw, L)) return make_float4(0.f, 0.f, 0.f, 0.f);
  const int k0 = dr_floor_i(lod_raw);
  int k1 = k0 + 1;
  if (k1 >= L) k1 = L - 1;
  float d_lod = 0.0f;
  for (int li = 0; li < 2; ++li) {
    const int k = li == 0 ? k0 : k1;
    const float sign = li == 0 ? -1.0f : 1.0f;
    const Taps q = bilin_taps<MODE>(u, v, m.w[k], m.h[k]);
    const float* b = level_ptr(tex, pyr, m, k, img, C);
    for (int c = 0; c < C; ++c) d_lod += sign * sample4(b, q, C, c) * __ldg(g + c);
  }
  return lod_grad(e, m.h[0], m.w[0], d_lod);
}

// Bilinear sample of all four channels of a C == 4 level (16-byte texels),
// per channel the same arithmetic as sample4.
__device__ __forceinline__ float4 sample4v(const float* __restrict__ b, const Taps& q) {
  const float4 t00 = ldg4(b + q.a00 * 4), t10 = ldg4(b + q.a10 * 4);
  const float4 t01 = ldg4(b + q.a01 * 4), t11 = ldg4(b + q.a11 * 4);
  return make_float4(q.w00 * t00.x + q.w10 * t10.x + q.w01 * t01.x + q.w11 * t11.x,
                     q.w00 * t00.y + q.w10 * t10.y + q.w01 * t01.y + q.w11 * t11.y,
                     q.w00 * t00.z + q.w10 * t10.z + q.w01 * t01.z + q.w11 * t11.z,
                     q.w00 * t00.w + q.w10 * t10.w + q.w01 * t01.w + q.w11 * t11.w);
}

// VEC4: C == 4 with 16-byte aligned texture, pyramid and output.
template <int MODE, bool MIP_LINEAR, bool VEC4>
__global__ void __launch_bounds__(256, DR_MINB_TEX_FWD) k_tex_mip_fwd(const float* __restrict__ tex, const float* __restrict__ pyr, const MipDesc m,
                              bool tex_shared, int C, const float2* __restrict__ uv,
                              const float4* __restrict__ uv_da, float bias, const float* __restrict__ bias_map,
                              int64_t P, int64_t HWi, float* __restrict__ out) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= P) return;  // no warp collectives
  const int64_t nt = tex_shared ? 0 : pix / HWi;
  float s;
  const float4 e = effective_da(__ldg(uv_da + pix), pix, bias, bias_map, s);
  const LodSel ls = lod_select<MIP_LINEAR>(e, m.h[0], m.w[0], m.L);
  const float2 t = __ldg(uv + pix);
  const Taps q0 = bilin_taps<MODE>(t.x, t.y, m.w[ls.k0], m.h[ls.k0]);
  const Taps q1 = bilin_taps<MODE>(t.x, t.y, m.w[ls.k1], m.h[ls.k1]);
  const float* b0 = level_ptr(tex, pyr, m, ls.k0, nt, C);
  const float* b1 = level_ptr(tex, pyr, m, ls.k1, nt, C);
  float* o = out + pix * C;
  // out = (1-frac)*s0, then += frac*s1 (Texture.swift:853-859)
  const float a = 1.0f - ls.frac, f = ls.frac;
  if constexpr (VEC4) {
    const float4 s0 = sample4v(b0, q0), s1 = sample4v(b1, q1);
    *reinterpret_cast<float4*>(o) =
        make_float4(a * s0.x + f * s1.x, a * s0.y + f * s1.y, a * s0.z + f * s1.z, a * s0.w + f * s1.w);
  } else {
    for (int c = 0; c < C; ++c) {
      const float o0 = a * sample4(b0, q0, C, c);
      o[c] = o0 + f * sample4(b1, q1, C, c);
    }
  }
}

// One channel of the mipmap VJP's per-level texel pass: d(out)/d(u, v)
// (with the OOB masks) and, when `acc`, the K22 term sign * sample * g.
__device__ __forceinline__ void mip_texel_terms(const Taps& q, float r00, float r10, float r01, float r11, float gv,
                                               float scale, float sign, bool acc, float& dfx, float& dfy,
                                               float& d_lod) {
  const float gc = gv * scale;
  if (acc) d_lod += sign * (q.w00 * r00 + q.w10 * r10 + q.w01 * r01 + q.w11 * r11) * gv;
  const float t00 = r00 * q.m00, t10 = r10 * q.m10, t01 = r01 * q.m01, t11 = r11 * q.m11;
  dfx += gc * ((1.0f - q.fy) * (t10 - t00) + q.fy * (t11 - t01));
  dfy += gc * ((1.0f - q.fx) * (t01 - t00) + q.fx * (t11 - t10));
}

// Fused mipmap VJP: d_tex / d_pyramid scatter (K20), d_uv (K21), d_uvDA (K22)
// and the optional gradient of the bias map.  For MIP_LINEAR the K22 samples
// are those of the two levels already read for d_uv (the unclamped LOD's
// floor and floor + 1 are the sampled levels whenever K22 is non-zero).
// VEC4: C == 4 with 16-byte aligned texture, pyramid and cotangent.
template <int MODE, bool MIP_LINEAR, bool VEC4>
__device__ __forceinline__ void mip_bwd_pixel(const int64_t pix0, const float* __restrict__ tex,
                                              const float* __restrict__ pyr, const MipDesc& m, bool tex_shared,
                                              int C, const float2* __restrict__ uv,
                                              const float4* __restrict__ uv_da, float bias,
                                              const float* __restrict__ bias_map, int64_t P, int64_t HWi,
                                              const float* __restrict__ d_out, float* __restrict__ d_tex,
                                              float* __restrict__ d_pyr, float2* __restrict__ d_uv,
                                              float4* __restrict__ d_uv_da, float* __restrict__ d_bias_map,
                                              HotCache* hc, float* s_small, const SmallLevels& sl) {
  const bool on = pix0 < P;
  const int64_t pix = on ? pix0 : P - 1;  // out-of-range lanes follow a valid pixel, adding nothing
  const int lane = threadIdx.x & 31;
  const int64_t nt = tex_shared ? 0 : pix / HWi;
  float s;
  const float4 e = effective_da(__ldg(uv_da + pix), pix, bias, bias_map, s);
  const int Ht = m.h[0], Wt = m.w[0], L = m.L;
  const LodSel ls = lod_select<MIP_LINEAR>(e, Ht, Wt, L);
  const float2 t = __ldg(uv + pix);
  const float* g = d_out + pix * C;
  const bool want_lod = d_uv_da || d_bias_map;
  const bool acc = MIP_LINEAR && want_lod && lod_interior(ls.raw, L);
  const float4 gv = C <= 4 ? load_cot(g, C, VEC4) : make_float4(0.f, 0.f, 0.f, 0.f);
  float dfx_total = 0.0f, dfy_total = 0.0f, d_lod = 0.0f;
#pragma unroll
  for (int li = 0; li < 2; ++li) {
    const int k = li == 0 ? ls.k0 : ls.k1;
    const float scale = li == 0 ? (1.0f - ls.frac) : ls.frac;
    const float sign = li == 0 ? -1.0f : 1.0f;
    const Taps q = bilin_taps<MODE>(t.x, t.y, m.w[k], m.h[k]);
    const float* b = level_ptr(tex, pyr, m, k, nt, C);
    float* db = (k == 0 ? d_tex : d_pyr + m.off[k]) + nt * (int64_t)m.h[k] * m.w[k] * C;
    float dfx = 0.0f, dfy = 0.0f;
    scatter_bilin(db, q, g, gv, scale, C, on && scale != 0.0f, lane, hc, s_small,
                  k >= sl.ks ? (int)(m.off[k] - sl.base) : -1);  // a small level: shared texture, nt == 0
    if constexpr (VEC4) {
      const float4 T00 = ldg4(b + q.a00 * 4), T10 = ldg4(b + q.a10 * 4);
      const float4 T01 = ldg4(b + q.a01 * 4), T11 = ldg4(b + q.a11 * 4);
      mip_texel_terms(q, T00.x, T10.x, T01.x, T11.x, gv.x, scale, sign, acc, dfx, dfy, d_lod);
      mip_texel_terms(q, T00.y, T10.y, T01.y, T11.y, gv.y, scale, sign, acc, dfx, dfy, d_lod);
      mip_texel_terms(q, T00.z, T10.z, T01.z, T11.z, gv.z, scale, sign, acc, dfx, dfy, d_lod);
      mip_texel_terms(q, T00.w, T10.w, T01.w, T11.w, gv.w, scale, sign, acc, dfx, dfy, d_lod);
    } else {
      for (int c = 0; c < C; ++c)
        mip_texel_terms(q, __ldg(b + q.a00 * C + c), __ldg(b + q.a10 * C + c), __ldg(b + q.a01 * C + c),
                        __ldg(b + q.a11 * C + c), __ldg(g + c), scale, sign, acc, dfx, dfy, d_lod);
    }
    dfx_total += dfx * (float)m.w[k];
    dfy_total += dfy * (float)m.h[k];
  }
  if (!on) return;
  d_uv[pix] = make_float2(dfx_total, dfy_total);

  if (!want_lod) return;
  float4 g4;
  if (MIP_LINEAR) g4 = acc ? lod_grad(e, Ht, Wt, d_lod) : make_float4(0.f, 0.f, 0.f, 0.f);
  else g4 = lod_vjp<MODE>(e, m, tex, pyr, nt, C, t.x, t.y, ls.raw, g);
  // Backward of eff = uvDA * s: d_uvDA = g * s, d_map = ln2 * sum(g * eff).
  if (d_uv_da) d_uv_da[pix] = make_float4(g4.x * s, g4.y * s, g4.z * s, g4.w * s);
  if (d_bias_map) {
    const float acc_m = g4.x * e.x + g4.y * e.y + g4.z * e.z + g4.w * e.w;
    d_bias_map[pix] = bias_map ? acc_m * 0.6931471805599453f : 0.0f;
  }
}

// Mip-mapped VJP: d_tex / pyramid gradient, d_uv, d_uvDA (and the bias map's
// gradient), one pixel per thread.
template <int MODE, bool MIP_LINEAR, bool VEC4>
__global__ void __launch_bounds__(256, DR_MINB_TEX_BWD) k_tex_mip_bwd(const float* __restrict__ tex, const float* __restrict__ pyr, const MipDesc m,
                              bool tex_shared, int C, const float2* __restrict__ uv,
                              const float4* __restrict__ uv_da, float bias, const float* __restrict__ bias_map,
                              int64_t P, int64_t HWi, const float* __restrict__ d_out,
                              float* __restrict__ d_tex, float* __restrict__ d_pyr, float2* __restrict__ d_uv,
                              float4* __restrict__ d_uv_da, float* __restrict__ d_bias_map, const SmallLevels sl) {
  __shared__ HotCache hc;
  __shared__ float s_small[kSmallCap];
  hot_init(&hc);
  small_init(s_small, sl);
  __syncthreads();
  mip_bwd_pixel<MODE, MIP_LINEAR, VEC4>((int64_t)blockIdx.x * blockDim.x + threadIdx.x, tex, pyr, m, tex_shared, C,
                                        uv, uv_da, bias, bias_map, P, HWi, d_out, d_tex, d_pyr, d_uv, d_uv_da,
                                        d_bias_map, &hc, s_small, sl);
  hot_flush(&hc, C);  // a CTA barrier first
  small_flush(s_small, sl, d_pyr);
}

// ------------------------------------------------------- mip-mapped cube
// Extension (the reference's cube path samples level 0 with .linear only):
// the pyramid of the Nt * 6 faces, LOD from the screen-space derivatives of
// the face coordinates, per-level per-face clamp bilinear.  d_dir = 0 as the
// reference's cube VJP; dirDA gets the LOD gradient.

template <bool MIP_LINEAR>
__global__ void __launch_bounds__(256, DR_MINB_TEX_FWD) k_tex_cube_mip_fwd(const float* __restrict__ tex, const float* __restrict__ pyr, const MipDesc m,
                                   bool tex_shared, int C, const float* __restrict__ dir,
                                   const float2* __restrict__ dir_da, float bias,
                                   const float* __restrict__ bias_map, int64_t P, int64_t HWi,
                                   float* __restrict__ out) {
  const int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= P) return;  // no warp collectives
  const CubeFrame f = cube_frame(__ldg(dir + 3 * pix), __ldg(dir + 3 * pix + 1), __ldg(dir + 3 * pix + 2));
  const int64_t img = (tex_shared ? 0 : pix / HWi) * 6 + f.face;
  float s;
  const float4 e = effective_da(cube_uv_da(f, load_dir_da(dir_da, pix)), pix, bias, bias_map, s);
  const LodSel ls = lod_select<MIP_LINEAR>(e, m.h[0], m.w[0], m.L);
  const Taps q0 = bilin_taps<1>(f.u, f.v, m.w[ls.k0], m.h[ls.k0]);
  const Taps q1 = bilin_taps<1>(f.u, f.v, m.w[ls.k1], m.h[ls.k1]);
  const float* b0 = level_ptr(tex, pyr, m, ls.k0, img, C);
  const float* b1 = level_ptr(tex, pyr, m, ls.k1, img, C);
  float* o = out + pix * C;
  for (int c = 0; c < C; ++c) {
    const float o0 = (1.0f - ls.frac) * sample4(b0, q0, C, c);
    o[c] = o0 + ls.frac * sample4(b1, q1, C, c);
  }
}

template <bool MIP_LINEAR, bool DIR_GRAD>
__device__ __forceinline__ void cube_mip_bwd_pixel(const int64_t pix0, const float* __restrict__ tex,
                                                   const float* __restrict__ pyr, const MipDesc& m, bool tex_shared,
                                                   int C, const float* __restrict__ dir,
                                                   const float2* __restrict__ dir_da, float bias,
                                                   const float* __restrict__ bias_map, int64_t P, int64_t HWi,
                                                   const float* __restrict__ d_out, float* __restrict__ d_tex,
                                                   float* __restrict__ d_pyr, float* __restrict__ d_dir,
                                                   float2* __restrict__ d_dir_da, float* __restrict__ d_bias_map,
                                                   HotCache* hc, float* s_small, const SmallLevels& sl) {
  const bool on = pix0 < P;
  const int64_t pix = on ? pix0 : P - 1;  // out-of-range lanes follow a valid pixel, adding nothing
  const int lane = threadIdx.x & 31;
  const CubeFrame f = cube_frame(__ldg(dir + 3 * pix), __ldg(dir + 3 * pix + 1), __ldg(dir + 3 * pix + 2));
  const int64_t img = (tex_shared ? 0 : pix / HWi) * 6 + f.face;
  float s;
  const DirDA dda = load_dir_da(dir_da, pix);
  const float4 e = effective_da(cube_uv_da(f, dda), pix, bias, bias_map, s);
  const LodSel ls = lod_select<MIP_LINEAR>(e, m.h[0], m.w[0], m.L);
  const float* g = d_out + pix * C;
  const bool want_lod = d_dir_da || d_bias_map || DIR_GRAD;
  // MIP_LINEAR: the K22 samples are those of the two levels read here.
  const bool acc = MIP_LINEAR && want_lod && lod_interior(ls.raw, m.L);
  const float4 gv = C <= 4 ? load_cot(g, C, false) : make_float4(0.f, 0.f, 0.f, 0.f);
  float d_u = 0.0f, d_v = 0.0f, d_lod = 0.0f;
#pragma unroll
  for (int li = 0; li < 2; ++li) {
    const int k = li == 0 ? ls.k0 : ls.k1;
    const float scale = li == 0 ? (1.0f - ls.frac) : ls.frac;
    const float sign = li == 0 ? -1.0f : 1.0f;
    const Taps q = bilin_taps<1>(f.u, f.v, m.w[k], m.h[k]);
    float* db = (k == 0 ? d_tex : d_pyr + m.off[k]) + img * (int64_t)m.h[k] * m.w[k] * C;
    scatter_bilin(db, q, g, gv, scale, C, on && scale != 0.0f, lane, hc, s_small,
                  k >= sl.ks ? (int)(m.off[k] - sl.base + img * (int64_t)m.h[k] * m.w[k] * C) : -1);
    if (DIR_GRAD || acc) {
      const float* b = level_ptr(tex, pyr, m, k, img, C);
      float dfx = 0.0f, dfy = 0.0f;
      for (int c = 0; c < C; ++c)
        mip_texel_terms(q, __ldg(b + q.a00 * C + c), __ldg(b + q.a10 * C + c), __ldg(b + q.a01 * C + c),
                        __ldg(b + q.a11 * C + c), __ldg(g + c), scale, sign, acc, dfx, dfy, d_lod);
      d_u += dfx * (float)m.w[k];
      d_v += dfy * (float)m.h[k];
    }
  }
  if (!on) return;
  AxisGrad ag = {0.0f, 0.0f, 0.0f};
  if (DIR_GRAD) ag = cube_dir_vjp(f, d_u, d_v);
  if (!want_lod) {
    store_dir_grad(d_dir, pix, f, ag);
    return;
  }
  float4 g4;
  if (MIP_LINEAR) g4 = acc ? lod_grad(e, m.h[0], m.w[0], d_lod) : make_float4(0.f, 0.f, 0.f, 0.f);
  else g4 = lod_vjp<1>(e, m, tex, pyr, img, C, f.u, f.v, ls.raw, g);
  const float4 gs = make_float4(g4.x * s, g4.y * s, g4.z * s, g4.w * s);
  if (DIR_GRAD) cube_dir_lod_vjp(f, dda, gs, ag);
  store_dir_grad(d_dir, pix, f, ag);
  if (d_dir_da) {
    const DirDA r = cube_uv_da_vjp(f, gs);
    d_dir_da[3 * pix] = r.a[0];
    d_dir_da[3 * pix + 1] = r.a[1];
    d_dir_da[3 * pix + 2] = r.a[2];
  }
  if (d_bias_map) {
    const float acc_m = g4.x * e.x + g4.y * e.y + g4.z * e.z + g4.w * e.w;
    d_bias_map[pix] = bias_map ? acc_m * 0.6931471805599453f : 0.0f;
  }
}

template <bool MIP_LINEAR, bool DIR_GRAD>
__global__ void __launch_bounds__(256, DR_MINB_TEX_BWD) k_tex_cube_mip_bwd(const float* __restrict__ tex, const float* __restrict__ pyr, const MipDesc m,
                                   bool tex_shared, int C, const float* __restrict__ dir,
                                   const float2* __restrict__ dir_da, float bias,
                                   const float* __restrict__ bias_map, int64_t P, int64_t HWi,
                                   const float* __restrict__ d_out, float* __restrict__ d_tex,
                                   float* __restrict__ d_pyr, float* __restrict__ d_dir,
                                   float2* __restrict__ d_dir_da, float* __restrict__ d_bias_map,
                                   const SmallLevels sl) {
  __shared__ HotCache hc;
  __shared__ float s_small[kSmallCap];
  hot_init(&hc);
  small_init(s_small, sl);
  __syncthreads();
  cube_mip_bwd_pixel<MIP_LINEAR, DIR_GRAD>((int64_t)blockIdx.x * blockDim.x + threadIdx.x, tex, pyr, m, tex_shared,
                                           C, dir, dir_da, bias, bias_map, P, HWi, d_out, d_tex, d_pyr, d_dir,
                                           d_dir_da, d_bias_map, &hc, s_small, sl);
  hot_flush(&hc, C);  // a CTA barrier first
  small_flush(s_small, sl, d_pyr);
}

// d_tex[level 0] += sum_k d_pyr_k[y >> k, x >> k] / 4^k: the adjoint of the
// 2x2 mean pyramid, evaluated in one pass over level 0.
template <bool VEC4>
__global__ void k_mip_fold(float* __restrict__ d_tex, const float* __restrict__ d_pyr, const MipDesc m, int C) {
  // Grid (x blocks, y = level-0 row, z = texture): one thread per level-0
  // texel, all channels, 32-bit indexing within a level.  VEC4: C == 4 with
  // 16-byte aligned buffers, one float4 per texel and level (the same sums).
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= m.w[0]) return;
  const int y = blockIdx.y, n = blockIdx.z;
  float* dst = d_tex + (((int64_t)n * m.h[0] + y) * m.w[0] + x) * C;
  if constexpr (VEC4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float w = 1.0f;
    for (int k = 1; k < m.L; ++k) {
      w *= 0.25f;
      const float* lk = d_pyr + m.off[k] + (int64_t)n * m.h[k] * m.w[k] * 4;
      const float4 v = ldg4(lk + ((y >> k) * m.w[k] + (x >> k)) * 4);
      acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
    }
    float4 d = *reinterpret_cast<float4*>(dst);
    d.x += acc.x; d.y += acc.y; d.z += acc.z; d.w += acc.w;
    *reinterpret_cast<float4*>(dst) = d;
  } else {
    for (int c = 0; c < C; ++c) {
      float acc = 0.0f, w = 1.0f;
      for (int k = 1; k < m.L; ++k) {
        w *= 0.25f;
        const float* lk = d_pyr + m.off[k] + (int64_t)n * m.h[k] * m.w[k] * C;
        acc += w * __ldg(lk + ((y >> k) * m.w[k] + (x >> k)) * C + c);
      }
      dst[c] += acc;
    }
  }
}

inline bool aligned(const void* p, unsigned a) { return ((uintptr_t)p & (a - 1)) == 0; }

dr_status build_pyramid(dr_ctx* ctx, const float* tex, int Nt, int C, const MipDesc& m, float* pyr) {
  const bool vec4 = C == 4 && aligned(tex, 16) && aligned(pyr, 16);
  for (int k = 1; k < m.L; ++k) {
    const float* src = (k == 1) ? tex : pyr + m.off[k - 1];
    DR_TB(ctx);
    if (vec4) {
      const int64_t n_out = (int64_t)Nt * m.h[k] * m.w[k];
      k_mip_down4<<<grid_for(n_out, 256), 256, 0, ctx->stream>>>(
          reinterpret_cast<const float4*>(src), m.h[k - 1], m.w[k - 1], reinterpret_cast<float4*>(pyr + m.off[k]),
          m.h[k], m.w[k], n_out);
    } else {
      const int64_t n_out = (int64_t)Nt * m.h[k] * m.w[k] * C;
      k_mip_down<<<grid_for(n_out, 256), 256, 0, ctx->stream>>>(src, m.h[k - 1], m.w[k - 1], pyr + m.off[k],
                                                                 m.h[k], m.w[k], C, n_out);
    }
    DR_LAUNCHED(ctx, "mip_down");
  }
  return DR_OK;
}

struct TexArgs {
  bool cube, mip, mip_linear;
  bool dir_grad;  // d_dir through the cube projection (extension)
  int64_t P, HWi;
  int64_t nimg;  // images per level: Nt, or Nt * 6 faces for a cube
  MipDesc m;
  int64_t pyr_floats;
};

// `boundary` carries the boundary mode in its low byte and flag bits above it
// (DR_TEXTURE_CUBE_DIR_GRAD); check_tex strips the flags into `a`.
dr_status check_tex(dr_ctx* ctx, int filter, int& boundary, const float* tex, int Nt, int Ht, int Wt, int C,
                    int max_level, const float* uv, const float* uv_da, int N, int Hi, int Wi, TexArgs& a) {
  const int flags = boundary & ~0xff;
  boundary &= 0xff;
  DR_REQUIRE(ctx, (flags & ~DR_TEXTURE_CUBE_DIR_GRAD) == 0, "texture: unknown flag bits 0x%x", flags);
  a.dir_grad = (flags & DR_TEXTURE_CUBE_DIR_GRAD) != 0;
  DR_REQUIRE(ctx, !a.dir_grad || boundary == DR_BOUNDARY_CUBE,
             "texture: DR_TEXTURE_CUBE_DIR_GRAD applies to cube textures only");
  DR_REQUIRE(ctx, tex && uv, "texture: tex and uv are required");
  DR_REQUIRE(ctx, filter >= 0 && filter <= 3, "texture: bad filter mode %d", filter);
  DR_REQUIRE(ctx, boundary >= 0 && boundary <= 3, "texture: bad boundary mode %d", boundary);
  DR_REQUIRE(ctx, Nt > 0 && Ht > 0 && Wt > 0 && C > 0 && N > 0 && Hi > 0 && Wi > 0, "texture: bad sizes");
  DR_REQUIRE(ctx, Nt == 1 || Nt == N, "texture: tex batch dim %d incompatible with uv batch %d", Nt, N);
  a.cube = boundary == DR_BOUNDARY_CUBE;
  if (a.cube)
    DR_REQUIRE(ctx, filter != DR_FILTER_NEAREST, "texture: cube textures support the linear and mipmap filterModes");
  a.mip = filter == DR_FILTER_LINEAR_MIPMAP_NEAREST || filter == DR_FILTER_LINEAR_MIPMAP_LINEAR;
  a.mip_linear = filter == DR_FILTER_LINEAR_MIPMAP_LINEAR;
  if (a.mip) {
    DR_REQUIRE(ctx, uv_da != nullptr, "texture: mipmap filterModes require uvDA");
    // [.., 4] uvDA loads as float4; a cube's [.., 6] dirDA as three float2.
    DR_REQUIRE(ctx, aligned(uv_da, a.cube ? 8 : 16), "texture: uvDA must be %d-byte aligned", a.cube ? 8 : 16);
  }
  if (!a.cube) DR_REQUIRE(ctx, aligned(uv, 8), "texture: uv must be 8-byte aligned");
  a.P = (int64_t)N * Hi * Wi;
  a.HWi = (int64_t)Hi * Wi;
  a.nimg = a.cube ? 6 * (int64_t)Nt : Nt;
  DR_REQUIRE(ctx, a.nimg <= INT32_MAX, "texture: too many texture images");
  a.m = mip_desc((int)a.nimg, Ht, Wt, C, a.mip ? max_level : 0, &a.pyr_floats);
  return DR_OK;
}

}  // namespace

using namespace dr;

#define DR_MODE_SWITCH(MODE_VAR, ...)                 \
  switch (MODE_VAR) {                                 \
    case 0: { constexpr int MODE = 0; __VA_ARGS__; } break; \
    case 1: { constexpr int MODE = 1; __VA_ARGS__; } break; \
    default: { constexpr int MODE = 2; __VA_ARGS__; } break; \
  }

