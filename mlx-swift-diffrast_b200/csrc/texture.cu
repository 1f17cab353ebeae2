// texture.cu — the texture forward entry points and mip pyramid
// construction (dr_texture_mip_layout, dr_texture_construct_mip,
// dr_texture_fwd), built without FMA contraction like the other forward
// paths; the kernels and their reference mapping are in texture_impl.cuh.
#include "texture_impl.cuh"

extern "C" dr_status dr_texture_mip_layout(int Nt, int Ht, int Wt, int C, int max_level, int* num_levels,
                                           int64_t* level_offset, int* level_h, int* level_w,
                                           int64_t* pyramid_floats) {
  if (Nt <= 0 || Ht <= 0 || Wt <= 0 || C <= 0 || !num_levels) return DR_EINVAL;
  int64_t tot;
  MipDesc m = mip_desc(Nt, Ht, Wt, C, max_level, &tot);
  *num_levels = m.L;
  for (int k = 0; k < m.L; ++k) {
    if (level_offset) level_offset[k] = m.off[k];
    if (level_h) level_h[k] = m.h[k];
    if (level_w) level_w[k] = m.w[k];
  }
  if (pyramid_floats) *pyramid_floats = tot;
  return DR_OK;
}

extern "C" dr_status dr_texture_construct_mip(dr_ctx* ctx, const float* tex, int Nt, int Ht, int Wt, int C,
                                              int max_level, float* pyramid) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, tex && Nt > 0 && Ht > 0 && Wt > 0 && C > 0, "textureConstructMip: bad arguments");
  int64_t tot;
  MipDesc m = mip_desc(Nt, Ht, Wt, C, max_level, &tot);
  if (m.L > 1) DR_REQUIRE(ctx, pyramid != nullptr, "textureConstructMip: pyramid buffer required");
  return build_pyramid(ctx, tex, Nt, C, m, pyramid);
}

extern "C" dr_status dr_texture_fwd(dr_ctx* ctx, int filter, int boundary, const float* tex, int Nt, int Ht,
                                    int Wt, int C, const float* pyramid, int max_level, const float* uv,
                                    const float* uv_da, float mip_level_bias, const float* mip_level_bias_map,
                                    int N, int Hi, int Wi, float* out) {
  DR_ENTER(ctx);
  TexArgs a;
  dr_status st = check_tex(ctx, filter, boundary, tex, Nt, Ht, Wt, C, max_level, uv, uv_da, N, Hi, Wi, a);
  if (st != DR_OK) return st;
  DR_REQUIRE(ctx, out, "texture: out required");
  const unsigned grid = grid_for(a.P, 256);
  const bool shared = Nt == 1;
  if (a.cube && !a.mip) {
    DR_TB(ctx);
    k_tex_cube<<<grid, 256, 0, ctx->stream>>>(tex, shared, Ht, Wt, C, uv, a.P, a.HWi, out, nullptr, nullptr,
                                              nullptr, false);
    DR_LAUNCHED(ctx, "tex_cube_fwd");
    return DR_OK;
  }
  const float2* uv2 = reinterpret_cast<const float2*>(uv);
  if (filter == DR_FILTER_NEAREST) {
    DR_TB(ctx);
    DR_MODE_SWITCH(boundary, (k_tex_nearest<MODE><<<grid, 256, 0, ctx->stream>>>(
                                 tex, shared, Ht, Wt, C, uv2, a.P, a.HWi, out, nullptr, nullptr, nullptr)));
    DR_LAUNCHED(ctx, "tex_nearest_fwd");
    return DR_OK;
  }
  if (filter == DR_FILTER_LINEAR) {
    DR_TB(ctx);
    DR_MODE_SWITCH(boundary, (k_tex_linear_fwd<MODE><<<grid, 256, 0, ctx->stream>>>(tex, shared, Ht, Wt, C,
                                                                                    uv2, a.P, a.HWi, out)));
    DR_LAUNCHED(ctx, "tex_linear_fwd");
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
  if (a.cube) {
    const float2* dda = reinterpret_cast<const float2*>(uv_da);
    DR_TB(ctx);
    if (a.mip_linear)
      k_tex_cube_mip_fwd<true><<<grid, 256, 0, ctx->stream>>>(tex, pyr, a.m, shared, C, uv, dda, mip_level_bias,
                                                              mip_level_bias_map, a.P, a.HWi, out);
    else
      k_tex_cube_mip_fwd<false><<<grid, 256, 0, ctx->stream>>>(tex, pyr, a.m, shared, C, uv, dda, mip_level_bias,
                                                               mip_level_bias_map, a.P, a.HWi, out);
    DR_LAUNCHED(ctx, "tex_cube_mip_fwd");
    return DR_OK;
  }
  const float4* da4 = reinterpret_cast<const float4*>(uv_da);
  const bool vec4 = C == 4 && aligned(tex, 16) && aligned(pyr, 16) && aligned(out, 16);
  DR_TB(ctx);
#define DR_MIP_FWD(ML, V4)                                                                                          \
  DR_MODE_SWITCH(boundary, (k_tex_mip_fwd<MODE, ML, V4><<<grid, 256, 0, ctx->stream>>>(                               \
                               tex, pyr, a.m, shared, C, uv2, da4, mip_level_bias, mip_level_bias_map, a.P, a.HWi, \
                               out)))
  if (a.mip_linear) {
    if (vec4) { DR_MIP_FWD(true, true); } else { DR_MIP_FWD(true, false); }
  } else {
    if (vec4) { DR_MIP_FWD(false, true); } else { DR_MIP_FWD(false, false); }
  }
#undef DR_MIP_FWD
  DR_LAUNCHED(ctx, "tex_mip_fwd");
  return DR_OK;
}
