// texture_bwd.cu — dr_texture_bwd, the VJP of every texture filter and
// boundary mode (kernels in texture_impl.cuh).  Built with FMA contraction
// (-fmad=true): gradients only, compared with the oracle within tolerances.
#include "texture_impl.cuh"

extern "C" dr_status dr_texture_bwd(dr_ctx* ctx, int filter, int boundary, const float* tex, int Nt, int Ht,
                                    int Wt, int C, const float* pyramid, int max_level, const float* uv,
                                    const float* uv_da, float mip_level_bias, const float* mip_level_bias_map,
                                    int N, int Hi, int Wi, const float* d_out, float* d_tex, float* d_uv,
                                    float* d_uv_da, float* d_bias_map) {
  DR_ENTER(ctx);
  TexArgs a;
  dr_status st = check_tex(ctx, filter, boundary, tex, Nt, Ht, Wt, C, max_level, uv, uv_da, N, Hi, Wi, a);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, d_out && d_tex && d_uv, "texture_bwd: d_out, d_tex and d_uv are required");
  if (d_uv_da)
    DR_REQUIRE(ctx, aligned(d_uv_da, a.cube ? 8 : 16), "texture_bwd: d_uv_da must be %d-byte aligned",
               a.cube ? 8 : 16);
  const unsigned grid = grid_for(a.P, 256);
  const bool shared = Nt == 1;
  const int64_t n_tex = (int64_t)Nt * (a.cube ? 6 : 1) * Ht * Wt * C;
  DR_CUDA(ctx, cudaMemsetAsync(d_tex, 0, sizeof(float) * (size_t)n_tex, ctx->stream), "texture_bwd memset");
  if (a.cube && !a.mip) {
    DR_TB(ctx);
    k_tex_cube<<<grid, 256, 0, ctx->stream>>>(tex, shared, Ht, Wt, C, uv, a.P, a.HWi, nullptr, d_out, d_tex,
                                              d_uv, a.dir_grad);
    DR_LAUNCHED(ctx, "tex_cube_bwd");
    return DR_OK;
  }
  const float2* uv2 = reinterpret_cast<const float2*>(uv);
  float2* duv2 = reinterpret_cast<float2*>(d_uv);
  if (!a.cube) DR_REQUIRE(ctx, aligned(d_uv, 8), "texture_bwd: d_uv must be 8-byte aligned");
  if (filter == DR_FILTER_NEAREST) {
    DR_TB(ctx);
    DR_MODE_SWITCH(boundary, (k_tex_nearest<MODE><<<grid, 256, 0, ctx->stream>>>(
                                 tex, shared, Ht, Wt, C, uv2, a.P, a.HWi, nullptr, d_out, d_tex, duv2)));
    DR_LAUNCHED(ctx, "tex_nearest_bwd");
    return DR_OK;
  }
  if (filter == DR_FILTER_LINEAR) {
    DR_TB(ctx);
    DR_MODE_SWITCH(boundary, (k_tex_linear_bwd<MODE><<<grid, 256, 0, ctx->stream>>>(
                                 tex, shared, Ht, Wt, C, uv2, a.P, a.HWi, d_out, d_tex, duv2)));
    DR_LAUNCHED(ctx, "tex_linear_bwd");
    return DR_OK;
  }
  const float* pyr = pyramid;
  if (!pyr && a.m.L > 1) {
    float* w = (float*)ws_get(ctx, WS_MIP, sizeof(float) * (size_t)a.pyr_floats);
    if (!w) return DR_ENOMEM;
    st = build_pyramid(ctx, tex, (int)a.nimg, C, a.m, w);
    if (st != DR_OK) return st;
    pyr = w;
  }
  float* dpyr = nullptr;
  if (a.m.L > 1) {
    dpyr = (float*)ws_get(ctx, WS_DMIP, sizeof(float) * (size_t)a.pyr_floats);
    if (!dpyr) return DR_ENOMEM;
    DR_CUDA(ctx, cudaMemsetAsync(dpyr, 0, sizeof(float) * (size_t)a.pyr_floats, ctx->stream),
            "texture_bwd memset");
  }
  // The smallest levels of a shared texture (all of them that fit together in
  // kSmallCap floats) are reduced in shared memory per CTA.
  SmallLevels sl{a.m.L, 0, 0};
  if (shared && a.m.L > 1) {
    for (int k = 1; k < a.m.L; ++k)
      if (a.pyr_floats - a.m.off[k] <= kSmallCap) {
        sl = SmallLevels{k, (int)(a.pyr_floats - a.m.off[k]), a.m.off[k]};
        break;
      }
  }
  const unsigned mgrid = grid;
  if (a.cube) {
    const float2* dda = reinterpret_cast<const float2*>(uv_da);
    float2* ddda = reinterpret_cast<float2*>(d_uv_da);
    DR_TB(ctx);
#define DR_CUBE_MIP_BWD(ML, DG)                                                                                     \
  k_tex_cube_mip_bwd<ML, DG><<<mgrid, 256, 0, ctx->stream>>>(tex, pyr, a.m, shared, C, uv, dda, mip_level_bias,      \
                                                             mip_level_bias_map, a.P, a.HWi, d_out, d_tex, dpyr,     \
                                                             d_uv, ddda, d_bias_map, sl)
    if (a.mip_linear) {
      if (a.dir_grad) DR_CUBE_MIP_BWD(true, true); else DR_CUBE_MIP_BWD(true, false);
    } else {
      if (a.dir_grad) DR_CUBE_MIP_BWD(false, true); else DR_CUBE_MIP_BWD(false, false);
    }
#undef DR_CUBE_MIP_BWD
    DR_LAUNCHED(ctx, "tex_cube_mip_bwd");
  } else {
  const float4* da4 = reinterpret_cast<const float4*>(uv_da);
  float4* dda4 = reinterpret_cast<float4*>(d_uv_da);
  const bool vec4 = C == 4 && aligned(tex, 16) && aligned(pyr, 16) && aligned(d_out, 16);
  DR_TB(ctx);
#define DR_MIP_BWD(ML, V4)                                                                                          \
  DR_MODE_SWITCH(boundary, (k_tex_mip_bwd<MODE, ML, V4><<<mgrid, 256, 0, ctx->stream>>>(                              \
                               tex, pyr, a.m, shared, C, uv2, da4, mip_level_bias, mip_level_bias_map, a.P, a.HWi, \
                               d_out, d_tex, dpyr, duv2, dda4, d_bias_map, sl)))
  if (a.mip_linear) {
    if (vec4) { DR_MIP_BWD(true, true); } else { DR_MIP_BWD(true, false); }
  } else {
    if (vec4) { DR_MIP_BWD(false, true); } else { DR_MIP_BWD(false, false); }
  }
#undef DR_MIP_BWD
  DR_LAUNCHED(ctx, "tex_mip_bwd");
  }
  if (a.m.L > 1) {
    DR_REQUIRE(ctx, Ht <= 65535 && a.nimg <= 65535, "texture_bwd: mip fold supports H, images <= 65535");
    DR_TB(ctx);
    const dim3 fg(grid_for(Wt, 256), Ht, (unsigned)a.nimg);
    if (C == 4 && aligned(d_tex, 16) && aligned(dpyr, 16))
      k_mip_fold<true><<<fg, 256, 0, ctx->stream>>>(d_tex, dpyr, a.m, C);
    else
      k_mip_fold<false><<<fg, 256, 0, ctx->stream>>>(d_tex, dpyr, a.m, C);
    DR_LAUNCHED(ctx, "mip_fold");
  }
  return DR_OK;
}
