// The norm family's row scale s(S) and its derivative ds/dS, S = sum of x^2 over a row of length d.
// Shared by the residual-stream norms (rowops.cu) and the standalone module norms (modules.cu).
//   RMS_AFFINE / RMS  s = rsqrt(S/d + eps)                               model/norm.py:21-38
//   L2_TEMP / L2      s = 1/(sqrt(S) + eps)                              model/norm.py:50-55
//   ELASTIC           h = sqrt(d) rsqrt(max(S, eps)); s = h if h < 1 else h^alpha   model/norm.py:83-95
//   ELASTICBALL       s = (sqrt(d) / sqrt(S + eps))^alpha                model/norm.py:118-132
//   HYPERBALL         s = rsqrt(1 + S/d)                                 model/norm.py:40-42
#pragma once
#include <math.h>

#include "rgpt.h"

namespace rgpt {

struct NS2 {
  float s, ds;
};

__device__ __forceinline__ NS2 norm_scale(int kind, float S, int d, float eps, float alpha) {
  NS2 r;
  switch (kind) {
    case RGPT_NORM_RMS_AFFINE:
    case RGPT_NORM_RMS: {
      const float v = S / d + eps;
      r.s = rsqrtf(v);
      r.ds = -0.5f * r.s / v / d;
      break;
    }
    case RGPT_NORM_L2_TEMP:
    case RGPT_NORM_L2: {
      const float n = sqrtf(S);
      r.s = 1.0f / (n + eps);
      r.ds = n > 0.f ? -r.s * r.s / (2.0f * n) : 0.f;
      break;
    }
    case RGPT_NORM_ELASTIC: {
      const float Sc = fmaxf(S, eps);
      const float hs = sqrtf((float)d) * rsqrtf(Sc);
      const float dh = (S >= eps) ? -hs / (2.0f * Sc) : 0.f;
      if (hs < 1.0f) {
        r.s = hs;
        r.ds = dh;
      } else {
        r.s = powf(hs, alpha);
        r.ds = alpha * powf(hs, alpha - 1.0f) * dh;
      }
      break;
    }
    case RGPT_NORM_ELASTICBALL: {
      const float v = S + eps;
      r.s = powf((float)d / v, 0.5f * alpha);
      r.ds = -0.5f * alpha * r.s / v;
      break;
    }
    case RGPT_NORM_HYPERBALL: {
      const float v = 1.0f + S / d;
      r.s = rsqrtf(v);
      r.ds = -0.5f * r.s / v / d;
      break;
    }
    default:
      r.s = 1.f;
      r.ds = 0.f;
  }
  return r;
}

}  // namespace rgpt
