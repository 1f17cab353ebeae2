// dr_check — a C++ caller of libdiffrast that uses nothing but the public
// header (include/diffrast.h) and the CUDA runtime: the shape of any native
// host (Swift via its C module, a game engine, a C++ trainer).  It runs one
// small chain through the C ABI and checks known answers:
//   * rasterize: a triangle covering the image centre; coverage of the centre
//     and of a far corner, tri_id + 1, barycentric bounds;
//   * interpolate: out = (1 - u - v) a0 + u a1 + v a2 recomputed on the host;
//   * antialias: a constant colour is returned unchanged;
//   * the VJPs run and leave finite gradients; dr_ctx_sync reports no error;
//   * the fused two-layer pass's one-pass VJP equals the separate VJPs;
//   * misuse returns DR_EINVAL with a message instead of crashing.
// Exit status 0 when every check passes.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "diffrast.h"

static int g_fail = 0;
#define CHECK(cond, ...)                   \
  do {                                     \
    if (!(cond)) {                         \
      std::printf("FAIL %s:%d ", __FILE__, __LINE__); \
      std::printf(__VA_ARGS__);            \
      std::printf("\n");                   \
      ++g_fail;                            \
    }                                      \
  } while (0)
#define OK(call) CHECK((call) == DR_OK, "%s -> %s", #call, dr_last_error(ctx))

template <class T>
static T* dev(const std::vector<T>& h) {
  T* d = nullptr;
  if (cudaMalloc(&d, sizeof(T) * (h.empty() ? 1 : h.size())) != cudaSuccess) return nullptr;
  if (!h.empty()) cudaMemcpy(d, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice);
  return d;
}
template <class T>
static std::vector<T> host(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, sizeof(T) * n, cudaMemcpyDeviceToHost);
  return h;
}

int main() {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    std::printf("no CUDA device\n");
    return 2;
  }
  CHECK(dr_abi_version() == DR_ABI_VERSION, "ABI %d != header %d", dr_abi_version(), DR_ABI_VERSION);
  dr_ctx* ctx = nullptr;
  if (dr_ctx_create(0, &ctx) != DR_OK) {
    std::printf("dr_ctx_create failed\n");
    return 1;
  }
  const int N = 1, H = 16, W = 16, V = 3, T = 1, A = 3;
  const std::vector<float> pos = {-0.8f, -0.8f, 0.0f, 1.0f, 0.8f, -0.8f, 0.0f, 1.0f, 0.0f, 0.8f, 0.0f, 1.0f};
  const std::vector<int32_t> tri = {0, 1, 2};
  const std::vector<float> attr = {1, 0, 0, 0, 1, 0, 0, 0, 1};
  float* d_posv = dev(pos);
  int32_t* d_tri = dev(tri);
  float* d_attr = dev(attr);
  std::vector<float> zeros(N * H * W * 4, 0.0f);
  float* d_rast = dev(zeros);
  float* d_db = dev(zeros);

  // rasterize
  OK(dr_rasterize_fwd(ctx, d_posv, V, d_tri, T, nullptr, N, H, W, nullptr, d_rast, d_db));
  OK(dr_ctx_sync(ctx));
  const std::vector<float> rast = host(d_rast, zeros.size());
  const float* c = &rast[((H / 2) * W + W / 2) * 4];
  CHECK(c[3] == 1.0f, "centre pixel tri_id+1 = %g", c[3]);
  CHECK(c[0] >= 0.0f && c[1] >= 0.0f && c[0] + c[1] <= 1.0f, "centre barycentrics (%g, %g)", c[0], c[1]);
  CHECK(std::fabs(c[2]) < 1e-6f, "centre depth %g", c[2]);
  CHECK(rast[3] == 0.0f, "top-left corner must be empty (tri_id+1 = %g)", rast[3]);

  // interpolate, checked on the host from rast
  std::vector<float> out0(N * H * W * A, 0.0f);
  float* d_out = dev(out0);
  OK(dr_interpolate_fwd(ctx, d_attr, 1, V, A, d_rast, N, H, W, d_tri, T, nullptr, nullptr, 0, d_out, nullptr));
  const std::vector<float> out = host(d_out, out0.size());
  float maxerr = 0.0f;
  for (int p = 0; p < H * W; ++p) {
    const float u = rast[4 * p], v = rast[4 * p + 1];
    const bool hit = rast[4 * p + 3] > 0.0f;
    const float bw = 1.0f - u - v;
    for (int a = 0; a < A; ++a) {
      const float want = hit ? bw * attr[a] + u * attr[3 + a] + v * attr[6 + a] : 0.0f;
      maxerr = std::fmax(maxerr, std::fabs(out[3 * p + a] - want));
    }
  }
  CHECK(maxerr <= 1e-6f, "interpolate max error %g", maxerr);

  // antialias of a constant colour is the identity
  std::vector<int32_t> topo0(3 * T, 0);
  int32_t* d_topo = dev(topo0);
  OK(dr_antialias_construct_topology_hash(ctx, d_tri, T, d_topo));
  const std::vector<int32_t> topo = host(d_topo, 3);
  CHECK(topo[0] == -1 && topo[1] == -1 && topo[2] == -1, "single-triangle topology (%d %d %d)", topo[0], topo[1],
        topo[2]);
  std::vector<float> colh(N * H * W * A, 0.7f);
  float* d_col = dev(colh);
  float* d_aa = dev(out0);
  OK(dr_antialias_fwd(ctx, d_col, N, H, W, A, d_rast, d_posv, V, d_tri, T, d_topo, d_aa, nullptr));
  const std::vector<float> aa = host(d_aa, out0.size());
  float aerr = 0.0f;
  for (float x : aa) aerr = std::fmax(aerr, std::fabs(x - 0.7f));
  CHECK(aerr == 0.0f, "antialias of a constant colour changed it by %g", aerr);

  // VJPs: finite gradients, no device-side error
  std::vector<float> ones(N * H * W * A, 1.0f);
  float* d_g = dev(ones);
  float* d_dcol = dev(out0);
  std::vector<float> dpos0(N * V * 4, 0.0f);
  float* d_dpos = dev(dpos0);
  OK(dr_antialias_bwd(ctx, d_col, N, H, W, A, d_rast, d_posv, V, d_tri, T, d_topo, d_g, d_dcol, d_dpos, nullptr));
  float* d_dattr = dev(attr);
  float* d_drast = dev(zeros);
  OK(dr_interpolate_bwd(ctx, d_attr, 1, V, A, d_rast, N, H, W, d_tri, T, nullptr, nullptr, 0, d_g, nullptr, d_dattr,
                        d_drast, nullptr));
  float* d_dpos_r = dev(dpos0);  // each VJP zeroes its own output; a chain sums them
  OK(dr_rasterize_bwd(ctx, d_posv, V, d_tri, T, nullptr, N, H, W, d_rast, d_drast, nullptr, d_dpos_r));
  OK(dr_ctx_sync(ctx));
  std::vector<float> dpos = host(d_dpos, dpos0.size());
  const std::vector<float> dpos_r = host(d_dpos_r, dpos0.size());
  for (size_t k = 0; k < dpos.size(); ++k) dpos[k] += dpos_r[k];
  const std::vector<float> dat = host(d_dattr, attr.size());
  bool finite = true;
  for (float x : dpos) finite = finite && std::isfinite(x);
  for (float x : dat) finite = finite && std::isfinite(x);
  CHECK(finite, "non-finite gradient");
  // d_attr of a sum of all outputs: each vertex's total barycentric weight.
  float wsum = 0.0f;
  for (int a = 0; a < 3; ++a) wsum += dat[3 * a];
  int covered = 0;
  for (int p = 0; p < H * W; ++p) covered += rast[4 * p + 3] > 0.0f;
  CHECK(std::fabs(wsum - (float)covered) <= 1e-3f * covered, "sum of d_attr[:,0] %g != covered pixels %d", wsum,
        covered);

  // The fused two-layer pass (per-view transform mode, identity transform)
  // and its one-pass VJP against the separate VJP entry points: layer 0's
  // out takes a cotangent, layer 1 (empty for one triangle) none.
  {
    const int A4 = 4;
    const std::vector<float> attr4 = {1, 0, 0, 2, 0, 1, 0, 3, 0, 0, 1, 4};
    const std::vector<float> eye = {1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1};
    const std::vector<float> z4(N * H * W * 4, 0.0f), zA(N * H * W * A4, 0.0f), zA2(N * H * W * 2 * A4, 0.0f);
    float* d_attr4 = dev(attr4);
    float* d_xf = dev(eye);
    float* r[2] = {dev(z4), dev(z4)};
    float* db[2] = {dev(z4), dev(z4)};
    float* o[2] = {dev(zA), dev(zA)};
    float* od[2] = {dev(zA2), dev(zA2)};
    OK(dr_rasterize_xf_interp_fwd(ctx, d_posv, V, d_xf, d_tri, T, N, H, W, d_attr4, 1, A4, r, db, o, od, nullptr,
                                  0.0f, nullptr));
    std::vector<float> gh(N * H * W * A4);
    for (size_t k = 0; k < gh.size(); ++k) gh[k] = 0.25f + 0.01f * (float)(k % 7);
    float* dg = dev(gh);
    const float* rc[2] = {r[0], r[1]};
    const float* dout[2] = {dg, nullptr};
    float* fa = dev(attr4);
    float* fv = dev(dpos0);
    OK(dr_rasterize_xf_interp_bwd(ctx, d_posv, V, d_xf, d_tri, T, N, H, W, d_attr4, 1, A4, rc, dout, nullptr,
                                  nullptr, 0.0f, nullptr, fa, fv));
    float* sa = dev(attr4);
    float* sr = dev(z4);
    float* sv = dev(dpos0);
    OK(dr_interpolate_bwd(ctx, d_attr4, 1, V, A4, r[0], N, H, W, d_tri, T, nullptr, nullptr, 0, dg, nullptr, sa, sr,
                          nullptr));
    const float* drs[2] = {sr, nullptr};
    OK(dr_rasterize_xf_bwd(ctx, d_posv, V, d_xf, d_tri, T, N, H, W, 2, rc, drs, nullptr, sv));
    OK(dr_ctx_sync(ctx));
    const std::vector<float> ha = host(fa, attr4.size()), hsa = host(sa, attr4.size());
    const std::vector<float> hv = host(fv, dpos0.size()), hsv = host(sv, dpos0.size());
    float ea = 0.0f, ma = 0.0f, ev = 0.0f, mv = 0.0f;
    for (size_t k = 0; k < ha.size(); ++k) {
      ea = std::fmax(ea, std::fabs(ha[k] - hsa[k]));
      ma = std::fmax(ma, std::fabs(hsa[k]));
    }
    for (size_t k = 0; k < hv.size(); ++k) {
      ev = std::fmax(ev, std::fabs(hv[k] - hsv[k]));
      mv = std::fmax(mv, std::fabs(hsv[k]));
    }
    CHECK(ma > 0.0f && ea <= 1e-5f * ma, "fused VJP d_attr differs by %g (max %g)", ea, ma);
    CHECK(mv > 0.0f && ev <= 1e-4f * mv, "fused VJP d_verts differs by %g (max %g)", ev, mv);
    for (void* p : {(void*)d_attr4, (void*)d_xf, (void*)r[0], (void*)r[1], (void*)db[0], (void*)db[1], (void*)o[0],
                    (void*)o[1], (void*)od[0], (void*)od[1], (void*)dg, (void*)fa, (void*)fv, (void*)sa, (void*)sr,
                    (void*)sv})
      cudaFree(p);
  }

  // misuse is a status, not a crash
  const dr_status bad = dr_rasterize_fwd(ctx, nullptr, V, d_tri, T, nullptr, N, H, W, nullptr, d_rast, d_db);
  CHECK(bad == DR_EINVAL, "null pos gave %d", (int)bad);
  CHECK(std::strlen(dr_last_error(ctx)) > 0, "no error message");

  for (void* p : {(void*)d_posv, (void*)d_tri, (void*)d_attr, (void*)d_rast, (void*)d_db, (void*)d_out, (void*)d_topo,
                  (void*)d_col, (void*)d_aa, (void*)d_g, (void*)d_dcol, (void*)d_dpos, (void*)d_dpos_r, (void*)d_dattr,
                  (void*)d_drast})
    cudaFree(p);
  dr_ctx_destroy(ctx);
  if (g_fail) {
    std::printf("%d check(s) failed\n", g_fail);
    return 1;
  }
  std::printf("dr_check: all checks passed\n");
  return 0;
}
