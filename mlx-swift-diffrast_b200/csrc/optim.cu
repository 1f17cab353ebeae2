// optim.cu — the Adam step of the reference's examples, fused into one pass.
//
// Reference: Sources/MLXDiffRastExamples/Adam.swift:36-43.  Per element,
// with the gradient optionally masked first (the examples multiply it by a
// per-component mask, PoseFitExample/main.swift and MeshFitExample/main.swift):
//   m = b1 m + (1 - b1) g
//   v = b2 v + (1 - b2) (g g)
//   param = param - (lr mHat) / (sqrt(vHat) + eps),  mHat = m / c1, vHat = v / c2
// where c1 = 1 - b1^t and c2 = 1 - b2^t are formed by the caller (float
// arithmetic, as the reference's Float pow).  Every operation is a separate
// IEEE round-to-nearest step in the reference's order, so the update matches
// an unfused float32 evaluation bit for bit.
#include "common.cuh"

namespace {

__global__ void k_adam(float* __restrict__ param, const float* __restrict__ grad, const float* __restrict__ mask,
                       float* __restrict__ m, float* __restrict__ v, int64_t n, float lr, float b1, float b2,
                       float one_m_b1, float one_m_b2, float c1, float c2, float eps) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float g = grad[i];
    if (mask) g = __fmul_rn(g, mask[i]);
    const float mi = __fadd_rn(__fmul_rn(b1, m[i]), __fmul_rn(one_m_b1, g));
    const float vi = __fadd_rn(__fmul_rn(b2, v[i]), __fmul_rn(one_m_b2, __fmul_rn(g, g)));
    m[i] = mi;
    v[i] = vi;
    const float m_hat = __fdiv_rn(mi, c1), v_hat = __fdiv_rn(vi, c2);
    param[i] = __fsub_rn(param[i], __fdiv_rn(__fmul_rn(lr, m_hat), __fadd_rn(__fsqrt_rn(v_hat), eps)));
  }
}

}  // namespace

using namespace dr;

extern "C" dr_status dr_adam_step(dr_ctx* ctx, float* param, const float* grad, const float* mask, float* m,
                                  float* v, int64_t n, float lr, float beta1, float beta2, float eps,
                                  float bias_c1, float bias_c2) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, n >= 0 && (n == 0 || (param && grad && m && v)), "adam: null pointer or n < 0");
  DR_REQUIRE(ctx, bias_c1 != 0.0f && bias_c2 != 0.0f, "adam: bias corrections must be non-zero (step t >= 1)");
  if (n == 0) return DR_OK;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->num_sms * 8);
  DR_TB(ctx);
  k_adam<<<blocks, 256, 0, ctx->stream>>>(param, grad, mask, m, v, n, lr, beta1, beta2, 1.0f - beta1,
                                          1.0f - beta2, bias_c1, bias_c2, eps);
  DR_LAUNCHED(ctx, "adam");
  return DR_OK;
}
