// Activation functions and derivatives used in GEMM epilogues.
//
// The functions are the reference Triton helpers' (model/kernels.py:13-118):
//   squared_relu  f = relu(x)^2                 f' = 2 relu(x)
//   gelu (tanh)   f = 0.5 x (1 + tanh(u)),  u = k (x + c x^3),  k = sqrt(2/pi),  c = 0.044715
//                 f' = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3 c x^2),  t = tanh(u)
//   silu          f = x sigmoid(x)              f' = s (1 + x (1 - s)),  s = sigmoid(x)
//   mish          sp = x if x > 20 else log(1 + exp(x)); f = x tanh(sp)
//                 f' = tanh(sp) + x (1 - tanh(sp)^2) sigmoid(x)
//
// They are evaluated through exact algebraic rewrites that need one exponential and one reciprocal
// each, both the hardware approximations (ex2.approx, rcp.approx: relative errors near 2^-22, far
// below the bf16 rounding of the stored results):
//   sigmoid(x)         = 1 / (1 + 2^(-x log2 e))
//   0.5 (1 + tanh(u))  = sigmoid(2u), so GELU f = x s2 and f' = s2 + 2 x s2 (1 - s2) u',  s2 = sigmoid(2u)
//                        (0.5 (1 - t^2) = 2 s2 (1 - s2)); no 1 + tanh cancellation for negative u
//   tanh(log(1 + E))   = n / (n + 2)  and  1 - tanh^2 = 4 (n + 1) / (n + 2)^2,  E = e^x,  n = E (E + 2)
//                        (from tanh(y) = (e^2y - 1) / (e^2y + 1) with e^y = 1 + E); for x > 20 the
//                        reference's branch gives tanh(x) = 1 in fp32, kept here as t = 1, f' = 1
// tests/test_gpu_gemm.py checks every activation's forward and backward epilogue against torch's fp32
// evaluation of the reference formulas.
#pragma once

#include "common.cuh"

namespace rgpt {

enum ActKind : int { ACT_NONE = 0, ACT_SQRELU = 1, ACT_GELU = 2, ACT_SILU = 3, ACT_MISH = 4, ACT_SQRELU_POST = 5 };
// ACT_SQRELU_POST: squared ReLU whose forward stores only post = relu(x)^2 and whose backward takes its
// derivative from post: relu(x) = sqrt(post), so act'(x) = 2 sqrt(post). The pre-activation is never
// written, halving the forward GEMM's output bytes.

constexpr float ACT_LOG2E = 1.4426950408889634f;
constexpr float GELU_K = 0.7978845608028654f;  // sqrt(2 / pi)
constexpr float GELU_C = 0.044715f;

// sigmoid(x) = 1 / (1 + 2^(-x log2 e)); 2^(+large) = inf gives 0, 2^(-large) = 0 gives 1
__device__ __forceinline__ float sigmoid_fast(float x) { return rcp_approx(1.0f + ex2_approx(-x * ACT_LOG2E)); }

// Compile-time activation (one instantiation per kind keeps unrolled epilogues small).
template <int ACT>
__device__ __forceinline__ float act_fwd_t(float x) {
  if constexpr (ACT == ACT_SQRELU || ACT == ACT_SQRELU_POST) {
    const float r = fmaxf(x, 0.0f);
    return r * r;
  } else if constexpr (ACT == ACT_GELU) {
    const float u = GELU_K * fmaf(GELU_C * x, x * x, x);
    return x * sigmoid_fast(2.0f * u);
  } else if constexpr (ACT == ACT_SILU) {
    return x * sigmoid_fast(x);
  } else if constexpr (ACT == ACT_MISH) {
    if (x > 20.0f) return x;  // softplus(x) = x there, and tanh(x) = 1 in fp32
    const float e = ex2_approx(x * ACT_LOG2E);
    const float n = e * (e + 2.0f);
    return x * n * rcp_approx(n + 2.0f);
  } else {
    return x;
  }
}

template <int ACT>
__device__ __forceinline__ float act_grad_t(float x) {
  if constexpr (ACT == ACT_SQRELU) {
    return 2.0f * fmaxf(x, 0.0f);
  } else if constexpr (ACT == ACT_SQRELU_POST) {
    // x = post = relu(pre)^2 >= 0; one MUFU operation (an IEEE sqrtf here slowed the epilogue-bound
    // backward GEMM more than dropping the pre-activation saved in the forward)
    return 2.0f * sqrt_approx(fmaxf(x, 0.0f));
  } else if constexpr (ACT == ACT_GELU) {
    const float x2 = x * x;
    const float u = GELU_K * fmaf(GELU_C * x, x2, x);
    const float s = sigmoid_fast(2.0f * u);
    const float du = GELU_K * fmaf(3.0f * GELU_C, x2, 1.0f);
    return fmaf(2.0f * x * s * (1.0f - s), du, s);
  } else if constexpr (ACT == ACT_SILU) {
    const float s = sigmoid_fast(x);
    return s * fmaf(x, 1.0f - s, 1.0f);
  } else if constexpr (ACT == ACT_MISH) {
    if (x > 20.0f) return 1.0f;  // t = 1: t + x (1 - t^2) sigmoid(x) = 1
    const float e = ex2_approx(x * ACT_LOG2E);
    const float n = e * (e + 2.0f);
    const float r = rcp_approx(n + 2.0f);
    const float t = n * r;
    const float one_minus_t2 = 4.0f * (n + 1.0f) * r * r;
    const float sig = e * rcp_approx(1.0f + e);
    return fmaf(x * one_minus_t2, sig, t);
  } else {
    return 1.0f;
  }
}

}  // namespace rgpt
