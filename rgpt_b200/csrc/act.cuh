// Activation functions and derivatives used in GEMM epilogues.
//
// Formulas follow the reference Triton helpers (model/kernels.py:13-118):
//   squared_relu  f = relu(x)^2                 f' = 2 relu(x)
//   gelu (tanh)   f = 0.5 x (1 + tanh(k (x + 0.044715 x^3))),  k = sqrt(2/pi)
//                 f' = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3*0.044715 x^2)
//   silu          f = x sigmoid(x)              f' = s (1 + x (1 - s))
//   mish          sp = x if x > 20 else log(1 + exp(x)); f = x tanh(sp)
//                 f' = tanh(sp) + x (1 - tanh(sp)^2) sigmoid(x)
// All math is fp32 and calls CUDA's tanhf / expf / logf.
#pragma once

namespace rgpt {

enum ActKind : int { ACT_NONE = 0, ACT_SQRELU = 1, ACT_GELU = 2, ACT_SILU = 3, ACT_MISH = 4 };

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// Compile-time activation (one instantiation per kind keeps unrolled epilogues small).
template <int ACT>
__device__ __forceinline__ float act_fwd_t(float x) {
  if constexpr (ACT == ACT_SQRELU) {
    const float r = fmaxf(x, 0.0f);
    return r * r;
  } else if constexpr (ACT == ACT_GELU) {
    const float k = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
  } else if constexpr (ACT == ACT_SILU) {
    return x * sigmoidf_(x);
  } else if constexpr (ACT == ACT_MISH) {
    const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
    return x * tanhf(sp);
  } else {
    return x;
  }
}

template <int ACT>
__device__ __forceinline__ float act_grad_t(float x) {
  if constexpr (ACT == ACT_SQRELU) {
    return 2.0f * fmaxf(x, 0.0f);
  } else if constexpr (ACT == ACT_GELU) {
    const float k = 0.7978845608028654f;
    const float x2 = x * x;
    const float t = tanhf(k * (x + 0.044715f * x2 * x));
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * (k * (1.0f + 3.0f * 0.044715f * x2));
  } else if constexpr (ACT == ACT_SILU) {
    const float s = sigmoidf_(x);
    return s * (1.0f + x * (1.0f - s));
  } else if constexpr (ACT == ACT_MISH) {
    const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
    const float t = tanhf(sp);
    return t + x * (1.0f - t * t) * sigmoidf_(x);
  } else {
    return 1.0f;
  }
}

__device__ __forceinline__ float act_fwd(int act, float x) {
  switch (act) {
    case ACT_SQRELU: {
      float r = fmaxf(x, 0.0f);
      return r * r;
    }
    case ACT_GELU: {
      const float k = 0.7978845608028654f;
      float inner = k * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.0f + tanhf(inner));
    }
    case ACT_SILU:
      return x * sigmoidf_(x);
    case ACT_MISH: {
      float sp = x > 20.0f ? x : logf(1.0f + expf(x));
      return x * tanhf(sp);
    }
    default:
      return x;
  }
}

// Derivative f'(x) (the caller multiplies by the upstream gradient).
__device__ __forceinline__ float act_grad(int act, float x) {
  switch (act) {
    case ACT_SQRELU:
      return 2.0f * fmaxf(x, 0.0f);
    case ACT_GELU: {
      const float k = 0.7978845608028654f;
      float x2 = x * x;
      float t = tanhf(k * (x + 0.044715f * x2 * x));
      float dt = 1.0f - t * t;
      float dinner = k * (1.0f + 3.0f * 0.044715f * x2);
      return 0.5f * (1.0f + t) + 0.5f * x * dt * dinner;
    }
    case ACT_SILU: {
      float s = sigmoidf_(x);
      return s * (1.0f + x * (1.0f - s));
    }
    case ACT_MISH: {
      float sp = x > 20.0f ? x : logf(1.0f + expf(x));
      float t = tanhf(sp);
      return t + x * (1.0f - t * t) * sigmoidf_(x);
    }
    default:
      return 1.0f;
  }
}

}  // namespace rgpt
