// Bandwidth-bound row kernels of the training step.
//
//   rownorm_fwd      residual-stream norm (fp32 in, bf16 out) with an optional fused
//                    2-output q_head (rGPT halting logits)            model/norm.py, model/gpt.py:107-109
//   rownorm_bwd      norm backward fused with the residual-gradient add, the bf16 copy
//                    of the gradient scaled by the next branch's layer scale, the norm
//                    weight grad and the layer-scale grad              model/transformer_block.py:43-57
//   qkv_prep_fwd/bwd QK-norm + G1 gate (sigmoid(q_n Wg^T + b)) + RoPE per (token, head)
//                                                                      model/attention.py:38-54, model/rope.py
//   embedding_fwd/bwd                                                  model/gpt.py:95
//   cross_entropy    row-wise logsumexp, loss, argmax and in-place bf16 dlogits  trainer.py:148, model/gpt.py:119-120
//   halt_losses      the rGPT q-head BCE losses and their gradients   model/gpt.py:105-141, trainer.py:150-162
//
// Norm family (y = x * s(S) * a, S = sum x^2 over the row, a = affine):
//   RMS_AFFINE  Gemma RMSNorm, s = rsqrt(S/d + eps), a = 1 + w          model/norm.py:21-34
//   RMS         F.rms_norm with eps = FLT_EPSILON                       model/norm.py:37-38
//   L2_TEMP     s = 1/(sqrt(S) + eps), a = temp                         model/norm.py:50-51
//   L2          s = 1/(sqrt(S) + eps)                                   model/norm.py:54-55
//   ELASTIC     h = sqrt(d) rsqrt(max(S, eps)); s = h if h < 1 else h^alpha   model/norm.py:83-95
//   ELASTICBALL s = (sqrt(d) / sqrt(S + eps))^alpha                     model/norm.py:118-132
//   HYPERBALL   s = rsqrt(1 + S/d)                                      model/norm.py:40-42
// Backward: dx = s (a.dy) + 2 s'(S) (sum a.dy.x) x.
#include <math.h>

#include <cuda_fp16.h>

#include "common.cuh"
#include "norm.cuh"
#include "rgpt.h"

#include <atomic>
#include <type_traits>

namespace rgpt {

// ============================================================================ residual norm
// One warp per row; each lane owns NV float4 (d = 128 * NV).
template <int NV>
__global__ void rownorm_fwd_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, float* __restrict__ stat,
                                   const float* __restrict__ w, float temp, int kind, float eps, float alpha, int M,
                                   int d, const float* __restrict__ qw, const float* __restrict__ qb,
                                   float* __restrict__ qout) {
  griddep_wait();
  griddep_launch();
  const int warps = blockDim.x >> 5;
  const long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * d);
  float4 v[NV];
  float S = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[lane + 32 * i];
    S += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  S = warp_sum(S);
  const NS2 ns = norm_scale(kind, S, d, eps, alpha);
  if (stat) stat[row] = ns.s;
  float q0 = 0.f, q1 = 0.f;
  uint2* yr = reinterpret_cast<uint2*>(y + row * d);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 4 * (lane + 32 * i);
    float4 a = make_float4(1.f, 1.f, 1.f, 1.f);
    if (kind == RGPT_NORM_RMS_AFFINE) {
      float4 ww = reinterpret_cast<const float4*>(w)[lane + 32 * i];
      a = make_float4(1.f + ww.x, 1.f + ww.y, 1.f + ww.z, 1.f + ww.w);
    } else if (kind == RGPT_NORM_L2_TEMP) {
      const float t = w ? w[0] : temp;  // the learned temperature, read on the device when given
      a = make_float4(t, t, t, t);
    }
    float4 o = make_float4(v[i].x * ns.s * a.x, v[i].y * ns.s * a.y, v[i].z * ns.s * a.z, v[i].w * ns.s * a.w);
    yr[lane + 32 * i] = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
    if (qout) {
      // q_head sees the same rounded activations the lm_head GEMM sees
      const float ox = bf16_round(o.x), oy = bf16_round(o.y), oz = bf16_round(o.z), ow = bf16_round(o.w);
      float4 w0 = reinterpret_cast<const float4*>(qw)[c / 4];
      float4 w1 = reinterpret_cast<const float4*>(qw + d)[c / 4];
      q0 += ox * w0.x + oy * w0.y + oz * w0.z + ow * w0.w;
      q1 += ox * w1.x + oy * w1.y + oz * w1.z + ow * w1.w;
    }
  }
  if (qout) {
    q0 = warp_sum(q0);
    q1 = warp_sum(q1);
    if (lane == 0) {
      qout[row * 2 + 0] = q0 + qb[0];
      qout[row * 2 + 1] = q1 + qb[1];
    }
  }
}

// Backward. dy = grad of the norm output (fp32) or, in q_head mode (dq != null),
// dy = dq[row,0]*qw[0,:] + dq[row,1]*qw[1,:]. Then
//   g_out = g_in + dx          (fp32, may alias g_in; g_in may be null = 0)
//   g_bf16 = bf16(g_out * ls)  (optional; ls optional)
//   dls  += g_out * raw        (optional: layer-scale grad of the branch that produced raw)
//   dw   += dy * x * s         (RMS_AFFINE weight grad)     dtemp += sum(dy * x * s) (L2_TEMP)
//   dqw  += dq^T h, dqb += dq  (q_head mode, h = the forward norm output in bf16)
// NV float4s per lane; QM: q-head mode (dy = dq Wq); DW / DLS: accumulate the norm weight /
// layer-scale grads. For d <= 512 the residual-grad input row is fetched with x and dy so that
// its latency overlaps the row reductions.
template <int NV, bool QM, bool DW, bool DLS>
__global__ void __launch_bounds__(256, NV <= 4 ? 2 : 1) rownorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                   const float* __restrict__ w, float temp, int kind, float eps, float alpha, int M,
                                   int d, const float* __restrict__ g_in, float* __restrict__ g_out,
                                   __nv_bfloat16* __restrict__ g_bf16, const float* __restrict__ ls,
                                   const float* __restrict__ raw, float* __restrict__ dls, float* __restrict__ dw,
                                   float* __restrict__ dtemp, const float* __restrict__ dq,
                                   const float* __restrict__ qw, const __nv_bfloat16* __restrict__ h,
                                   float* __restrict__ dqw, float* __restrict__ dqb,
                                   const uint32_t* __restrict__ drop_mask, float drop_scale) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float red[];  // per-CTA column partials: [d] dw, [d] dls, [2d] dqw
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  constexpr bool need_dw = DW;
  constexpr bool need_dls = DLS;
  constexpr bool qmode = QM;
  constexpr bool PREF = NV <= 4;
  for (int i = threadIdx.x; i < 4 * d; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  float dtemp_acc = 0.f, dqb0 = 0.f, dqb1 = 0.f;
  // column partials owned by this lane, accumulated over the rows this warp visits
  float4 pdw[DW ? NV : 1], pdls[DLS ? NV : 1], pq0[QM ? NV : 1], pq1[QM ? NV : 1];
#pragma unroll
  for (int i = 0; i < (DW ? NV : 1); ++i) pdw[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < (DLS ? NV : 1); ++i) pdls[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < (QM ? NV : 1); ++i) pq0[i] = pq1[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto affine = [&](int i) -> float4 {
    if (kind == RGPT_NORM_RMS_AFFINE) {
      float4 ww = reinterpret_cast<const float4*>(w)[lane + 32 * i];
      return make_float4(1.f + ww.x, 1.f + ww.y, 1.f + ww.z, 1.f + ww.w);
    }
    if (kind == RGPT_NORM_L2_TEMP) {
      const float t = w ? w[0] : temp;
      return make_float4(t, t, t, t);
    }
    return make_float4(1.f, 1.f, 1.f, 1.f);
  };

  for (long long row = (long long)blockIdx.x * warps + wid; row < M; row += (long long)gridDim.x * warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * d);
    float4 xv[NV], dv[NV], gpre[PREF ? NV : 1];
    float S = 0.f;
    float q0 = 0.f, q1 = 0.f;
    if (qmode) {
      q0 = dq[row * 2 + 0];
      q1 = dq[row * 2 + 1];
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      xv[i] = xr[lane + 32 * i];
      S += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
      if (qmode) {
        float4 w0 = reinterpret_cast<const float4*>(qw)[lane + 32 * i];
        float4 w1 = reinterpret_cast<const float4*>(qw + d)[lane + 32 * i];
        dv[i] = make_float4(q0 * w0.x + q1 * w1.x, q0 * w0.y + q1 * w1.y, q0 * w0.z + q1 * w1.z,
                            q0 * w0.w + q1 * w1.w);
      } else {
        dv[i] = reinterpret_cast<const float4*>(dy + row * d)[lane + 32 * i];
      }
      if constexpr (PREF)
        gpre[i] = g_in ? reinterpret_cast<const float4*>(g_in + row * d)[lane + 32 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    S = warp_sum(S);
    const NS2 ns = norm_scale(kind, S, d, eps, alpha);
    float c = 0.f, xdy = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 av = affine(i);
      c += av.x * dv[i].x * xv[i].x + av.y * dv[i].y * xv[i].y + av.z * dv[i].z * xv[i].z + av.w * dv[i].w * xv[i].w;
      xdy += dv[i].x * xv[i].x + dv[i].y * xv[i].y + dv[i].z * xv[i].z + dv[i].w * xv[i].w;
    }
    c = warp_sum(c);
    const float k2 = 2.0f * ns.ds * c;
    if (kind == RGPT_NORM_L2_TEMP) dtemp_acc += warp_sum(xdy) * ns.s;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 av = affine(i);
      float4 g = make_float4(ns.s * av.x * dv[i].x + k2 * xv[i].x, ns.s * av.y * dv[i].y + k2 * xv[i].y,
                             ns.s * av.z * dv[i].z + k2 * xv[i].z, ns.s * av.w * dv[i].w + k2 * xv[i].w);
      if (PREF || g_in) {
        float4 gi;
        if constexpr (PREF) gi = gpre[i];
        else gi = reinterpret_cast<const float4*>(g_in + row * d)[lane + 32 * i];
        g.x += gi.x;
        g.y += gi.y;
        g.z += gi.z;
        g.w += gi.w;
      }
      reinterpret_cast<float4*>(g_out + row * d)[lane + 32 * i] = g;
      if (g_bf16) {
        float4 s4 = ls ? reinterpret_cast<const float4*>(ls)[lane + 32 * i] : make_float4(1.f, 1.f, 1.f, 1.f);
        if (drop_mask != nullptr) {  // the branch output was dropped: its gradient takes the same mask
          const int col = 4 * (lane + 32 * i);
          const uint32_t bits = (__ldg(drop_mask + row * (d >> 5) + (col >> 5)) >> (col & 31)) & 0xFu;
          s4.x = (bits & 1u) ? s4.x * drop_scale : 0.f;
          s4.y = (bits & 2u) ? s4.y * drop_scale : 0.f;
          s4.z = (bits & 4u) ? s4.z * drop_scale : 0.f;
          s4.w = (bits & 8u) ? s4.w * drop_scale : 0.f;
        }
        reinterpret_cast<uint2*>(g_bf16 + row * d)[lane + 32 * i] =
            make_uint2(pack_bf16x2(g.x * s4.x, g.y * s4.y), pack_bf16x2(g.z * s4.z, g.w * s4.w));
      }
      if constexpr (need_dls) {
        float4 rv = reinterpret_cast<const float4*>(raw + row * d)[lane + 32 * i];
        pdls[i].x += g.x * rv.x;
        pdls[i].y += g.y * rv.y;
        pdls[i].z += g.z * rv.z;
        pdls[i].w += g.w * rv.w;
      }
      if constexpr (need_dw) {
        pdw[i].x += dv[i].x * xv[i].x * ns.s;
        pdw[i].y += dv[i].y * xv[i].y * ns.s;
        pdw[i].z += dv[i].z * xv[i].z * ns.s;
        pdw[i].w += dv[i].w * xv[i].w * ns.s;
      }
      if constexpr (QM) if (dqw) {
        uint2 hv = reinterpret_cast<const uint2*>(h + row * d)[lane + 32 * i];
        float2 h01 = unpack_bf16x2(hv.x), h23 = unpack_bf16x2(hv.y);
        pq0[i].x += q0 * h01.x;
        pq0[i].y += q0 * h01.y;
        pq0[i].z += q0 * h23.x;
        pq0[i].w += q0 * h23.y;
        pq1[i].x += q1 * h01.x;
        pq1[i].y += q1 * h01.y;
        pq1[i].z += q1 * h23.x;
        pq1[i].w += q1 * h23.y;
      }
    }
    dqb0 += q0;
    dqb1 += q1;
  }
  // fold lane partials into the CTA's shared partials, then one atomic per column per CTA
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c0 = 4 * (lane + 32 * i);
    if constexpr (need_dw) {
      atomicAdd(&red[c0 + 0], pdw[i].x);
      atomicAdd(&red[c0 + 1], pdw[i].y);
      atomicAdd(&red[c0 + 2], pdw[i].z);
      atomicAdd(&red[c0 + 3], pdw[i].w);
    }
    if constexpr (need_dls) {
      atomicAdd(&red[d + c0 + 0], pdls[i].x);
      atomicAdd(&red[d + c0 + 1], pdls[i].y);
      atomicAdd(&red[d + c0 + 2], pdls[i].z);
      atomicAdd(&red[d + c0 + 3], pdls[i].w);
    }
    if constexpr (QM) if (dqw) {
      atomicAdd(&red[2 * d + c0 + 0], pq0[i].x);
      atomicAdd(&red[2 * d + c0 + 1], pq0[i].y);
      atomicAdd(&red[2 * d + c0 + 2], pq0[i].z);
      atomicAdd(&red[2 * d + c0 + 3], pq0[i].w);
      atomicAdd(&red[3 * d + c0 + 0], pq1[i].x);
      atomicAdd(&red[3 * d + c0 + 1], pq1[i].y);
      atomicAdd(&red[3 * d + c0 + 2], pq1[i].z);
      atomicAdd(&red[3 * d + c0 + 3], pq1[i].w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    if (need_dw) atomicAdd(&dw[i], red[i]);
    if (need_dls) atomicAdd(&dls[i], red[d + i]);
    if (qmode && dqw) {
      atomicAdd(&dqw[i], red[2 * d + i]);
      atomicAdd(&dqw[d + i], red[3 * d + i]);
    }
  }
  if (lane == 0) {
    if (kind == RGPT_NORM_L2_TEMP && dtemp) atomicAdd(dtemp, dtemp_acc);
    if (qmode && dqb) {
      atomicAdd(&dqb[0], dqb0);
      atomicAdd(&dqb[1], dqb1);
    }
  }
}

// ============================================================================ QKV prep
// A half-warp per (token, head): lane l handles elements 4*(l%16) .. +3 of head 2*hp + l/16,
// so a warp moves two contiguous 128-byte head rows and the norm sums are 4-step half-warp
// reductions. RoPE partners i and i + 32 live in lanes l and l ^ 8. Each warp walks a
// contiguous run of (token, head pair) units and recomputes the RoPE angles only when the
// token changes. Forward writes
//   qk [M, 2d]  roped, normalised q | k (the attention operands, bf16)
//   qn [M, d]   normalised q before RoPE (bf16), the input of the gate GEMM
// The G1 gate itself, sigmoid(q_n Wg^T + bg), is a tcgen05 GEMM with a bias+sigmoid
// epilogue, and its backward runs as GEMMs too (dqn += dgp Wg, dWg += dgp^T q_n).
struct QkNormArgs {
  int kind;
  float eps, alpha;
  const float* wq;  // RMS_AFFINE weights (64) for q / k, or null
  const float* wk;
  float tq, tk;     // L2_TEMP temps
  float sq, sk;     // constant post-scales (asymmetric hyperball: 1.0 / 1.1)
};

__device__ __forceinline__ float half_warp_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

__device__ __forceinline__ float4 ld_bf16x4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
__device__ __forceinline__ float4 mul4(float4 a, float4 b) {
  return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}

// per-element affine factor of the QK norm (RMS_AFFINE: 1 + w, L2_TEMP: temp) times the post-scale
__device__ __forceinline__ float4 qk_affine4(const QkNormArgs& a, bool is_q, int i0) {
  const float post = is_q ? a.sq : a.sk;
  if (a.kind == RGPT_NORM_RMS_AFFINE) {
    const float4 w = *reinterpret_cast<const float4*>((is_q ? a.wq : a.wk) + i0);
    return make_float4((1.0f + w.x) * post, (1.0f + w.y) * post, (1.0f + w.z) * post, (1.0f + w.w) * post);
  }
  float t = 1.0f;
  if (a.kind == RGPT_NORM_L2_TEMP) {
    const float* tp = is_q ? a.wq : a.wk;  // learned temperature on the device, else the by-value one
    t = tp ? *tp : (is_q ? a.tq : a.tk);
  }
  t *= post;
  return make_float4(t, t, t, t);
}

// rotate-half RoPE on a lane's 4 elements; the partners sit in lane ^ 8.
// forward: first half y = x c - partner s, second half y = x c + partner s (dir = +1);
// the backward (dir = -1) applies the transposed rotation.
__device__ __forceinline__ float4 rope4(float4 x, float4 c, float4 sn, bool second_half, float dir) {
  const float p0 = __shfl_xor_sync(0xffffffffu, x.x, 8), p1 = __shfl_xor_sync(0xffffffffu, x.y, 8);
  const float p2 = __shfl_xor_sync(0xffffffffu, x.z, 8), p3 = __shfl_xor_sync(0xffffffffu, x.w, 8);
  const float sg = (second_half ? 1.0f : -1.0f) * dir;
  return make_float4(x.x * c.x + sg * p0 * sn.x, x.y * c.y + sg * p1 * sn.y, x.z * c.z + sg * p2 * sn.z,
                     x.w * c.w + sg * p3 * sn.w);
}

struct PrepLane {
  int half, i0;  // head of the pair (0/1) and first element
  bool second;   // elements in [32, 64)
  float4 f;      // inverse frequencies of the 4 elements
};

__device__ __forceinline__ PrepLane prep_lane(const float* inv_freq) {
  PrepLane L;
  const int lane = threadIdx.x & 31;
  L.half = lane >> 4;
  L.i0 = 4 * (lane & 15);
  L.second = L.i0 >= 32;
  const int fi = L.i0 & 31;
  L.f = make_float4(inv_freq[fi], inv_freq[fi + 1], inv_freq[fi + 2], inv_freq[fi + 3]);
  return L;
}

// sin and cos of a RoPE angle x = t * inv_freq (|x| < 65536, enforced on the host through T).
// Cody-Waite reduction by pi/2 with a three-part split of pi/2 whose first part has 8
// significant bits (k * C1 is exact for |k| < 2^16), then the hardware sin/cos on |r| <= pi/4
// (absolute error below 4e-7 there) and the quadrant rotation.
__device__ __forceinline__ void rope_sincos(float x, float* sn, float* cs) {
  const float k = rintf(x * 0.636619772f);
  float r = fmaf(-k, 1.5703125f, x);
  r = fmaf(-k, 4.83826792e-4f, r);
  r = fmaf(-k, 2.56328292e-12f, r);
  const float sr = __sinf(r), cr = __cosf(r);
  const int q = static_cast<int>(k) & 3;
  const float s1 = (q & 1) ? cr : sr, c1 = (q & 1) ? sr : cr;
  *sn = (q & 2) ? -s1 : s1;
  *cs = ((q + 1) & 2) ? -c1 : c1;
}

__device__ __forceinline__ void rope_angles(const PrepLane& L, float t, float4& c, float4& sn) {
  rope_sincos(t * L.f.x, &sn.x, &c.x);
  rope_sincos(t * L.f.y, &sn.y, &c.y);
  rope_sincos(t * L.f.z, &sn.z, &c.z);
  rope_sincos(t * L.f.w, &sn.w, &c.w);
}

// contiguous run of units for this warp
__device__ __forceinline__ void prep_units(long long total, long long& u0, long long& u1) {
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long per = (total + nwarps - 1) / nwarps;
  u0 = w * per;
  u1 = u0 + per < total ? u0 + per : total;
}

template <int KIND>
__global__ void __launch_bounds__(256, 4) qkv_prep_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                           __nv_bfloat16* __restrict__ qk,
                                                           __nv_bfloat16* __restrict__ qn_out,
                                                           const float* __restrict__ inv_freq, QkNormArgs na,
                                                           int M, int T, int H) {
  griddep_wait();
  griddep_launch();
  const PrepLane L = prep_lane(inv_freq);
  const int d = H * 64;
  const int hp_n = (H + 1) >> 1;
  const float4 aq = qk_affine4(na, true, L.i0), ak = qk_affine4(na, false, L.i0);
  long long u0, u1;
  prep_units((long long)M * hp_n, u0, u1);
  float4 c = make_float4(1.f, 1.f, 1.f, 1.f), sn = make_float4(0.f, 0.f, 0.f, 0.f);
  // (token, head pair) of unit u, walked incrementally (no 64-bit division per unit)
  int tok = (int)(u0 / hp_n), hp = (int)(u0 % hp_n);
  if (u0 < u1) rope_angles(L, (float)(tok % T), c, sn);
  for (long long u = u0; u < u1; ++u, ++hp) {
    if (hp == hp_n) {
      hp = 0;
      ++tok;
      rope_angles(L, (float)(tok % T), c, sn);
    }
    const int h = hp * 2 + L.half;
    const bool live = h < H;
    const size_t col = (size_t)h * 64 + L.i0;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f), y = x;
    if (live) {
      x = ld_bf16x4(qkv + (size_t)tok * 3 * d + col);
      y = ld_bf16x4(qkv + (size_t)tok * 3 * d + d + col);
    }
    if (KIND != RGPT_NORM_IDENTITY) {
      const NS2 nq = norm_scale(KIND, half_warp_sum(dot4(x, x)), 64, na.eps, na.alpha);
      const NS2 nk = norm_scale(KIND, half_warp_sum(dot4(y, y)), 64, na.eps, na.alpha);
      x = mul4(x, make_float4(nq.s * aq.x, nq.s * aq.y, nq.s * aq.z, nq.s * aq.w));
      y = mul4(y, make_float4(nk.s * ak.x, nk.s * ak.y, nk.s * ak.z, nk.s * ak.w));
    } else {
      x = mul4(x, aq);
      y = mul4(y, ak);
    }
    if (qn_out && live) st_bf16x4(qn_out + (size_t)tok * d + col, x);
    x = rope4(x, c, sn, L.second, 1.0f);
    y = rope4(y, c, sn, L.second, 1.0f);
    if (live) {
      st_bf16x4(qk + (size_t)tok * 2 * d + col, x);
      st_bf16x4(qk + (size_t)tok * 2 * d + d + col, y);
    }
  }
}

// Backward of the norm + RoPE. dq, dk: fp32 [M, d] grads of the roped q / k;
// dqn_gate: fp32 [M, d] = dgp Wg (the gate GEMM's contribution to d q_n), may be null;
// dgp: bf16 [M, d] grad of the gate pre-activation, only summed here into dbg.
// Writes the q and k column blocks of dqkv (bf16); ACCUMULATES dbg, dwq/dwk, dtq/dtk.
template <int KIND>
__global__ void __launch_bounds__(256, 3) qkv_prep_bwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ dq, const float* __restrict__ dk,
    const float* __restrict__ dqn_gate, const __nv_bfloat16* __restrict__ dgp, __nv_bfloat16* __restrict__ dqkv,
    float* __restrict__ dbg, float* __restrict__ dwq, float* __restrict__ dwk, float* __restrict__ dtq,
    float* __restrict__ dtk, const float* __restrict__ inv_freq, QkNormArgs na, int M, int T, int H) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[3][64];  // per-CTA column partials: dbg, dwq, dwk
  const PrepLane L = prep_lane(inv_freq);
  const int d = H * 64;
  const int hp_n = (H + 1) >> 1;
  for (int i = threadIdx.x; i < 3 * 64; i += blockDim.x) (&red[0][0])[i] = 0.f;
  __syncthreads();
  const float4 aq = qk_affine4(na, true, L.i0), ak = qk_affine4(na, false, L.i0);
  constexpr bool affine = KIND == RGPT_NORM_RMS_AFFINE, temp = KIND == RGPT_NORM_L2_TEMP;
  float4 acc_b = make_float4(0.f, 0.f, 0.f, 0.f), acc_wq = acc_b, acc_wk = acc_b;
  float acc_tq = 0.f, acc_tk = 0.f;
  long long u0, u1;
  prep_units((long long)M * hp_n, u0, u1);
  float4 c = make_float4(1.f, 1.f, 1.f, 1.f), sn = make_float4(0.f, 0.f, 0.f, 0.f);
  // (token, head pair) of unit u, walked incrementally (no 64-bit division per unit)
  int tok = (int)(u0 / hp_n), hp = (int)(u0 % hp_n);
  if (u0 < u1) rope_angles(L, (float)(tok % T), c, sn);
  for (long long u = u0; u < u1; ++u, ++hp) {
    if (hp == hp_n) {
      hp = 0;
      ++tok;
      rope_angles(L, (float)(tok % T), c, sn);
    }
    const int h = hp * 2 + L.half;
    const bool live = h < H;
    const size_t col = (size_t)h * 64 + L.i0;
    const size_t rq = (size_t)tok * 3 * d + col;
    float4 gq = make_float4(0.f, 0.f, 0.f, 0.f), gk = gq, xq = gq, xk = gq, gg = gq, gp = gq;
    if (live) {
      gq = *reinterpret_cast<const float4*>(dq + (size_t)tok * d + col);
      gk = *reinterpret_cast<const float4*>(dk + (size_t)tok * d + col);
      xq = ld_bf16x4(qkv + rq);
      xk = ld_bf16x4(qkv + rq + d);
      if (dqn_gate) gg = *reinterpret_cast<const float4*>(dqn_gate + (size_t)tok * d + col);
      if (dgp) gp = ld_bf16x4(dgp + (size_t)tok * d + col);
    }
    acc_b.x += gp.x;
    acc_b.y += gp.y;
    acc_b.z += gp.z;
    acc_b.w += gp.w;
    gq = rope4(gq, c, sn, L.second, -1.0f);
    gk = rope4(gk, c, sn, L.second, -1.0f);
    gq = make_float4(gq.x + gg.x, gq.y + gg.y, gq.z + gg.z, gq.w + gg.w);
    NS2 nq{1.f, 0.f}, nk{1.f, 0.f};
    if (KIND != RGPT_NORM_IDENTITY) {
      nq = norm_scale(KIND, half_warp_sum(dot4(xq, xq)), 64, na.eps, na.alpha);
      nk = norm_scale(KIND, half_warp_sum(dot4(xk, xk)), 64, na.eps, na.alpha);
    }
    // y = x * s(S) * a  =>  dx = s a g + 2 s'(S) (sum a g x) x
    const float4 agq = mul4(aq, gq), agk = mul4(ak, gk);
    const float k2q = 2.0f * nq.ds * half_warp_sum(dot4(agq, xq));
    const float k2k = 2.0f * nk.ds * half_warp_sum(dot4(agk, xk));
    if (affine && live) {
      const float fq = nq.s * na.sq, fk = nk.s * na.sk;
      acc_wq = make_float4(acc_wq.x + gq.x * xq.x * fq, acc_wq.y + gq.y * xq.y * fq, acc_wq.z + gq.z * xq.z * fq,
                           acc_wq.w + gq.w * xq.w * fq);
      acc_wk = make_float4(acc_wk.x + gk.x * xk.x * fk, acc_wk.y + gk.y * xk.y * fk, acc_wk.z + gk.z * xk.z * fk,
                           acc_wk.w + gk.w * xk.w * fk);
    }
    if (temp && live) {
      acc_tq += dot4(gq, xq) * nq.s * na.sq;
      acc_tk += dot4(gk, xk) * nk.s * na.sk;
    }
    if (live) {
      st_bf16x4(dqkv + rq, make_float4(nq.s * agq.x + k2q * xq.x, nq.s * agq.y + k2q * xq.y,
                                       nq.s * agq.z + k2q * xq.z, nq.s * agq.w + k2q * xq.w));
      st_bf16x4(dqkv + rq + d, make_float4(nk.s * agk.x + k2k * xk.x, nk.s * agk.y + k2k * xk.y,
                                           nk.s * agk.z + k2k * xk.z, nk.s * agk.w + k2k * xk.w));
    }
  }
  // column partials: a lane owns columns i0..i0+3; fold the CTA's lanes in smem, then one atomic per column
  if (dbg) {
    atomicAdd(&red[0][L.i0 + 0], acc_b.x);
    atomicAdd(&red[0][L.i0 + 1], acc_b.y);
    atomicAdd(&red[0][L.i0 + 2], acc_b.z);
    atomicAdd(&red[0][L.i0 + 3], acc_b.w);
  }
  if (affine) {
    atomicAdd(&red[1][L.i0 + 0], acc_wq.x);
    atomicAdd(&red[1][L.i0 + 1], acc_wq.y);
    atomicAdd(&red[1][L.i0 + 2], acc_wq.z);
    atomicAdd(&red[1][L.i0 + 3], acc_wq.w);
    atomicAdd(&red[2][L.i0 + 0], acc_wk.x);
    atomicAdd(&red[2][L.i0 + 1], acc_wk.y);
    atomicAdd(&red[2][L.i0 + 2], acc_wk.z);
    atomicAdd(&red[2][L.i0 + 3], acc_wk.w);
  }
  __syncthreads();
  if (threadIdx.x < 64) {
    if (dbg) atomicAdd(&dbg[threadIdx.x], red[0][threadIdx.x]);
    if (affine) {
      if (dwq) atomicAdd(&dwq[threadIdx.x], red[1][threadIdx.x]);
      if (dwk) atomicAdd(&dwk[threadIdx.x], red[2][threadIdx.x]);
    }
  }
  if (temp) {
    const float tq = warp_sum(acc_tq), tk = warp_sum(acc_tk);
    if ((threadIdx.x & 31) == 0) {
      if (dtq) atomicAdd(dtq, tq);
      if (dtk) atomicAdd(dtk, tk);
    }
  }
}

// ============================================================================ embedding
// x = emb[ids] (model/gpt.py:95), then nn.Dropout (model/gpt.py:96) when drop_mask != null: keep bits
// of (row, column) from Philox block (column / 8, row, site, 0), written to drop_mask [M, d / 32].
__global__ void embedding_fwd_kernel(const long long* __restrict__ ids, const float* __restrict__ emb,
                                     float* __restrict__ x, int M, int d, int V, int* __restrict__ err,
                                     uint32_t* __restrict__ drop_mask, const unsigned long long* __restrict__ seed,
                                     uint32_t site, uint32_t thresh, float scale) {
  griddep_wait();
  griddep_launch();
  const int warps = blockDim.x >> 5;
  const long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= M) return;
  const long long id = ids[row];
  const int lane = threadIdx.x & 31;
  float4* dst = reinterpret_cast<float4*>(x + row * d);
  const bool bad = id < 0 || id >= V;
  if (bad && lane == 0) atomicCAS(err, 0, RGPT_DEVERR_BAD_ARGS);
  const float4* src = reinterpret_cast<const float4*>(emb + (bad ? 0 : id) * d);
  uint32_t k0 = 0, k1 = 0;
  if (drop_mask != nullptr) {
    const unsigned long long sd = *seed;
    k0 = (uint32_t)sd;
    k1 = (uint32_t)(sd >> 32);
  }
  for (int c0 = 0; c0 < d / 4; c0 += 32) {  // warp-uniform trip count (d % 128 == 0 with dropout)
    const int c = c0 + lane;
    float4 v = (c < d / 4 && !bad) ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (drop_mask != nullptr) {
      // this lane's 4 columns are half of Philox block c / 2; groups of 8 lanes share one mask word
      const uint32_t k8 = keep8(philox4x32_10(make_uint4((uint32_t)(c >> 1), (uint32_t)row, site, 0u), k0, k1),
                                thresh);
      const uint32_t b4 = (k8 >> (4 * (c & 1))) & 0xFu;
      v.x = (b4 & 1u) ? v.x * scale : 0.f;
      v.y = (b4 & 2u) ? v.y * scale : 0.f;
      v.z = (b4 & 4u) ? v.z * scale : 0.f;
      v.w = (b4 & 8u) ? v.w * scale : 0.f;
      uint32_t word = b4 << (4 * (lane & 7));
      word |= __shfl_xor_sync(0xffffffffu, word, 1);
      word |= __shfl_xor_sync(0xffffffffu, word, 2);
      word |= __shfl_xor_sync(0xffffffffu, word, 4);
      if ((lane & 7) == 0 && c < d / 4) drop_mask[row * (d >> 5) + (c >> 3)] = word;
    }
    if (c < d / 4) dst[c] = v;
  }
}

__global__ void embedding_bwd_kernel(const long long* __restrict__ ids, const float* __restrict__ dx,
                                     float* __restrict__ demb, int M, int d, int V,
                                     const uint32_t* __restrict__ drop_mask, float scale) {
  griddep_wait();
  griddep_launch();
  const int warps = blockDim.x >> 5;
  const long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= M) return;
  const long long id = ids[row];
  if (id < 0 || id >= V) return;
  const int lane = threadIdx.x & 31;
  const float4* src = reinterpret_cast<const float4*>(dx + row * d);
  float4* dst = reinterpret_cast<float4*>(demb + id * d);
  for (int c = lane; c < d / 4; c += 32) {
    float4 g = src[c];
    if (drop_mask != nullptr) {  // the forward's dropout mask of this row
      const uint32_t b4 = (__ldg(drop_mask + row * (d >> 5) + (c >> 3)) >> (4 * (c & 7))) & 0xFu;
      g.x = (b4 & 1u) ? g.x * scale : 0.f;
      g.y = (b4 & 2u) ? g.y * scale : 0.f;
      g.z = (b4 & 4u) ? g.z * scale : 0.f;
      g.w = (b4 & 8u) ? g.w * scale : 0.f;
    }
    atomicAdd(dst + c, g);
  }
}

// ============================================================================ cross entropy
// count valid labels; scale_out = grad_scale / count
__global__ void ce_count_kernel(const long long* __restrict__ labels, int M, int ignore_index, float grad_scale,
                                float* __restrict__ scale_out, float* __restrict__ count_out) {
  griddep_wait();
  griddep_launch();
  __shared__ int s[32];
  int c = 0;
  for (int i = threadIdx.x; i < M; i += blockDim.x) c += (labels[i] != ignore_index) ? 1 : 0;
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int tot = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += s[i];
    count_out[0] = (float)tot;
    scale_out[0] = tot > 0 ? grad_scale / (float)tot : 0.f;
  }
}

// One CTA per row of bf16 logits [M, V]. Online max / sum-exp with 16-byte loads,
// argmax (first index of the maximum), loss_row = lse - x[label] (0 if ignored).
// With write_grad, overwrites the row with bf16 (softmax - onehot) * (*scale).
__global__ void __launch_bounds__(512) cross_entropy_kernel(__nv_bfloat16* __restrict__ logits, long long ld, int V,
                                                            const long long* __restrict__ labels, int ignore_index,
                                                            float* __restrict__ loss_rows, int* __restrict__ argmax,
                                                            const float* __restrict__ scale, int write_grad) {
  griddep_wait();
  griddep_launch();
  const long long row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const int nvec = V / 8;
  float m = -INFINITY, s = 0.f, best = -INFINITY;
  int besti = 0x7fffffff;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(x)[v];
    uint32_t w4[4] = {u.x, u.y, u.z, u.w};
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 p = unpack_bf16x2(w4[e]);
      f[2 * e] = p.x;
      f[2 * e + 1] = p.y;
    }
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    if (lm > best) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (f[e] == lm) {
          best = lm;
          besti = v * 8 + e;
          break;
        }
    }
    const float nm = fmaxf(m, lm);
    float acc = s * expf(m - nm);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += expf(f[e] - nm);
    s = acc;
    m = nm;
  }
  for (int j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x) {  // tail (V % 8)
    const float f = __bfloat162float(x[j]);
    if (f > best) {
      best = f;
      besti = j;
    }
    const float nm = fmaxf(m, f);
    s = s * expf(m - nm) + expf(f - nm);
    m = nm;
  }
  // block reduction of (m, s) and (best, besti)
  __shared__ float sm[32], ss[32], sb[32];
  __shared__ int sbi[32];
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (nm == -INFINITY) ? 0.f : s * expf(m - nm) + os * expf(om - nm);
    m = nm;
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
    }
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sm[wid] = m;
    ss[wid] = s;
    sb[wid] = best;
    sbi[wid] = besti;
  }
  __syncthreads();
  if (wid == 0) {
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    best = lane < nw ? sb[lane] : -INFINITY;
    besti = lane < nw ? sbi[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (nm == -INFINITY) ? 0.f : s * expf(m - nm) + os * expf(om - nm);
      m = nm;
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ob > best || (ob == best && oi < besti)) {
        best = ob;
        besti = oi;
      }
    }
    if (lane == 0) {
      sm[0] = m;
      ss[0] = s;
      sbi[0] = besti;
    }
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
  const float lse = m + logf(s);
  const long long label = labels[row];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  if (threadIdx.x == 0) {
    if (loss_rows) loss_rows[row] = valid ? lse - __bfloat162float(x[label]) : 0.f;
    if (argmax) argmax[row] = sbi[0];
  }
  if (!write_grad) return;
  __syncthreads();  // the label logit was read above before any thread overwrites it
  const float sc = valid ? scale[0] : 0.f;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(x)[v];
    uint32_t w4[4] = {u.x, u.y, u.z, u.w};
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 p = unpack_bf16x2(w4[e]);
      const int j = v * 8 + 2 * e;
      float g0 = expf(p.x - lse) - (j == label ? 1.f : 0.f);
      float g1 = expf(p.y - lse) - (j + 1 == label ? 1.f : 0.f);
      o4[e] = pack_bf16x2(g0 * sc, g1 * sc);
    }
    reinterpret_cast<uint4*>(x)[v] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
  for (int j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x) {
    const float f = __bfloat162float(x[j]);
    x[j] = __float2bfloat16((expf(f - lse) - (j == label ? 1.f : 0.f)) * sc);
  }
}

// Row-in-shared-memory variant for V % 8 == 0 and V * 2 bytes <= CE_SMEM_MAX: one bulk copy
// brings the row into shared memory (two CTAs per SM, so one row's copy overlaps the other's
// math), then three passes over shared memory: max + argmax (packed bf16 compares), the sum of
// e = exp2((x - max) log2 e) with e written back in place as fp16, and the gradient e * scale / sum
// (minus scale at the label) written straight to HBM. Logits are read from HBM once, dlogits written
// once, and each logit costs one exp2 (the gradient's softmax carries e's fp16 rounding, <= 2^-11
// relative, before its bf16 rounding).
constexpr int CE_THREADS = 512;
constexpr uint32_t CE_SMEM_MAX = 112 * 1024;

__device__ __forceinline__ void ce_unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 p = unpack_bf16x2(w4[e]);
    f[2 * e] = p.x;
    f[2 * e + 1] = p.y;
  }
}

__global__ void __launch_bounds__(CE_THREADS, 2)
    cross_entropy_smem_kernel(__nv_bfloat16* __restrict__ logits, long long ld, int V,
                              const long long* __restrict__ labels, int ignore_index, float* __restrict__ loss_rows,
                              int* __restrict__ argmax, const float* __restrict__ scale, int write_grad) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(128) uint8_t ce_row[];
  __shared__ uint64_t bar;
  __shared__ float red_f[CE_THREADS / 32];
  __shared__ int red_i[CE_THREADS / 32];
  constexpr float LOG2E = 1.4426950408889634f;
  const long long row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const int nvec = V >> 3;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, (uint32_t)V * 2u);
    bulk_load_1d(ce_row, x, (uint32_t)V * 2u, &bar);
  }
  const long long label = labels[row];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  const float sc = (valid && write_grad) ? scale[0] : 0.f;
  if (!mbar_wait(&bar, 0, nullptr)) {
    mbar_wait(&bar, 0, nullptr);  // give the copy a second bound before the CTA retires
    return;
  }
  const uint4* s4 = reinterpret_cast<const uint4*>(ce_row);
  // the label's logit, read before pass 2 overwrites the row with exponentials
  const float xl = (threadIdx.x == 0 && valid) ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(ce_row)[label])
                                               : 0.f;

  // pass 1: max (packed bf16 compares; exact) and the first index of the max
  float m = -INFINITY;
  int besti = 0x7fffffff;
  for (int v = threadIdx.x; v < nvec; v += CE_THREADS) {
    const uint4 u = s4[v];
    const __nv_bfloat162 h01 = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&u.x),
                                       *reinterpret_cast<const __nv_bfloat162*>(&u.y));
    const __nv_bfloat162 h23 = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&u.z),
                                       *reinterpret_cast<const __nv_bfloat162*>(&u.w));
    const float2 hm = __bfloat1622float2(__hmax2(h01, h23));
    const float lm = fmaxf(hm.x, hm.y);
    if (lm > m) {  // strictly greater: the earliest vector holding the max keeps it
      float f[8];
      ce_unpack8(u, f);
      int e = 7;
#pragma unroll
      for (int k = 6; k >= 0; --k) e = (f[k] == lm) ? k : e;
      m = lm;
      besti = v * 8 + e;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (om > m || (om == m && oi < besti)) {
      m = om;
      besti = oi;
    }
  }
  if (lane == 0) {
    red_f[wid] = m;
    red_i[wid] = besti;
  }
  __syncthreads();
  m = red_f[0];
  besti = red_i[0];
#pragma unroll
  for (int w = 1; w < CE_THREADS / 32; ++w) {
    const float om = red_f[w];
    const int oi = red_i[w];
    if (om > m || (om == m && oi < besti)) {
      m = om;
      besti = oi;
    }
  }
  __syncthreads();  // red_f is reused below

  // pass 2: e = exp2((x - m) log2 e), summed, and kept in place as fp16 for pass 3 (e is in (0, 1])
  const float m2 = m * LOG2E;
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  uint4* s4w = reinterpret_cast<uint4*>(ce_row);
  const float2 l2e = make_float2(LOG2E, LOG2E), nm2 = make_float2(-m2, -m2);
  for (int v = threadIdx.x; v < nvec; v += CE_THREADS) {
    float f[8];
    ce_unpack8(s4[v], f);
    float e[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 t = ffma2(make_float2(f[2 * k], f[2 * k + 1]), l2e, nm2);
      e[2 * k] = ex2_approx(t.x);
      e[2 * k + 1] = ex2_approx(t.y);
    }
    acc0 = fadd2(acc0, make_float2(e[0], e[1]));
    acc1 = fadd2(acc1, make_float2(e[2], e[3]));
    acc0 = fadd2(acc0, make_float2(e[4], e[5]));
    acc1 = fadd2(acc1, make_float2(e[6], e[7]));
    if (write_grad) {
      __half2 h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(e[2 * k], e[2 * k + 1]);
      s4w[v] = *reinterpret_cast<const uint4*>(h);
    }
  }
  float sum = warp_sum((acc0.x + acc0.y) + (acc1.x + acc1.y));
  if (lane == 0) red_f[wid] = sum;
  __syncthreads();
  sum = 0.f;
#pragma unroll
  for (int w = 0; w < CE_THREADS / 32; ++w) sum += red_f[w];
  const float lse2 = m2 + log2f(sum);
  if (threadIdx.x == 0) {
    if (loss_rows) loss_rows[row] = valid ? lse2 * 0.69314718055994531f - xl : 0.f;
    if (argmax) argmax[row] = besti;
  }
  if (!write_grad) return;

  // pass 3: dlogits = (softmax - onehot) * scale = e * (scale / sum) - onehot * scale, overwriting the
  // row in HBM (each thread reads back only the vectors it wrote in pass 2)
  const int label_vec = valid ? (int)(label >> 3) : -1;
  const int label_e = (int)(label & 7);
  const float k = sc / sum;
  const float2 k2 = make_float2(k, k);
  uint4* xo = reinterpret_cast<uint4*>(x);
  for (int v = threadIdx.x; v < nvec; v += CE_THREADS) {
    const uint4 u = s4[v];
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
    float2 p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = fmul2(__half22float2(*reinterpret_cast<const __half2*>(&w4[q])), k2);
    if (v == label_vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (2 * q == label_e) p[q].x -= sc;
        if (2 * q + 1 == label_e) p[q].y -= sc;
      }
    }
    xo[v] = make_uint4(pack_bf16x2(p[0].x, p[0].y), pack_bf16x2(p[1].x, p[1].y), pack_bf16x2(p[2].x, p[2].y),
                       pack_bf16x2(p[3].x, p[3].y));
  }
}

// Launch the per-row cross entropy (shared-memory row when it fits, else the streaming kernel).
static int launch_cross_entropy_rows(__nv_bfloat16* logits, long long ld, int M, int V, const long long* labels,
                                     int ignore_index, float* loss_rows, int* argmax, const float* scale,
                                     int write_grad, cudaStream_t s) {
  if (V % 8 == 0 && (uint32_t)V * 2u <= CE_SMEM_MAX) {
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr[64] = {false};
    if (dev >= 0 && dev < 64 && !attr[dev]) {
      if (cudaFuncSetAttribute(cross_entropy_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)CE_SMEM_MAX) != cudaSuccess)
        return rgpt_check_launch("cross_entropy_smem set smem");
      attr[dev] = true;
    }
    launch_pdl(cross_entropy_smem_kernel, dim3(M), dim3(CE_THREADS), (size_t)V * 2, s, 1, logits, ld, V, labels, ignore_index, loss_rows,
                                                                    argmax, scale, write_grad);
  } else {
    launch_pdl(cross_entropy_kernel, dim3(M), dim3(512), 0, s, 1, logits, ld, V, labels, ignore_index, loss_rows, argmax, scale,
                                           write_grad);
  }
  return RGPT_OK;
}

// sum of loss rows / count -> out[0] (mean CE over valid labels), also adds into accum (optional)
__global__ void ce_finalize_kernel(const float* __restrict__ loss_rows, int M, const float* __restrict__ count,
                                   float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  __shared__ float s[32];
  float a = 0.f;
  for (int i = threadIdx.x; i < M; i += blockDim.x) a += loss_rows[i];
  a = warp_sum(a);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += s[i];
    out[0] = t / count[0];
  }
}

// ============================================================================ rGPT halting losses
// q [R, M, 2] (halt, continue logits per recurrence step), correct [R, M] (argmax == label)
// halt loss   = (1/R) sum_i mean_m BCE(q[i,m,0], correct[i,m])
// q_cont loss = (1/R) sum_i mean_m BCE(q[i,m,1], target[i,m]),
//   target[i] = sigmoid(max(q[i+1,m,0], q[i+1,m,1])) for i < R-1, sigmoid(q[R-1,m,0]) for the last step
// losses[0] += halt loss, losses[1] += q_cont loss; dq = d(total)/dq * grad_scale
__device__ __forceinline__ float bce_logits(float x, float y) {
  return fmaxf(x, 0.f) - x * y + log1pf(expf(-fabsf(x)));
}

__global__ void halt_losses_kernel(const float* __restrict__ q, const int* __restrict__ argmax,
                                   const long long* __restrict__ labels, int R, int M, float grad_scale,
                                   float* __restrict__ dq, float* __restrict__ losses) {
  griddep_wait();
  griddep_launch();
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  float lh = 0.f, lc = 0.f;
  if (m < M) {
    const long long lab = labels[m];
    const float inv = 1.0f / ((float)R * (float)M);
    for (int i = 0; i < R; ++i) {
      const float qh = q[((long long)i * M + m) * 2 + 0];
      const float qc = q[((long long)i * M + m) * 2 + 1];
      const float y = (argmax[(long long)i * M + m] == lab) ? 1.f : 0.f;
      float tgt;
      if (i < R - 1) {
        const float a = q[((long long)(i + 1) * M + m) * 2 + 0], b = q[((long long)(i + 1) * M + m) * 2 + 1];
        tgt = 1.0f / (1.0f + expf(-fmaxf(a, b)));
      } else {
        tgt = 1.0f / (1.0f + expf(-qh));
      }
      lh += bce_logits(qh, y);
      lc += bce_logits(qc, tgt);
      dq[((long long)i * M + m) * 2 + 0] = (1.0f / (1.0f + expf(-qh)) - y) * inv * grad_scale;
      dq[((long long)i * M + m) * 2 + 1] = (1.0f / (1.0f + expf(-qc)) - tgt) * inv * grad_scale;
    }
    lh /= (float)R * (float)M;
    lc /= (float)R * (float)M;
  }
  lh = warp_sum(lh);
  lc = warp_sum(lc);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&losses[0], lh);
    atomicAdd(&losses[1], lc);
  }
}

}  // namespace rgpt

using namespace rgpt;

static int norm_nv(int d) {
  if (d % 128 != 0) return 0;
  const int nv = d / 128;
  return (nv == 1 || nv == 2 || nv == 4 || nv == 8 || nv == 16) ? nv : 0;
}

extern "C" int rgpt_rownorm_fwd(const float* x, void* y, float* stat, const float* w, float temp, int kind, float eps,
                                float alpha, int M, int d, const float* qw, const float* qb, float* qout,
                                void* stream) {
  const int nv = norm_nv(d);
  if (nv == 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm needs d in {128,256,512,1024,2048} (got %d)", d);
  if (kind == RGPT_NORM_RMS_AFFINE && w == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rmsnorm needs w");
  if (qout && (qw == nullptr || qb == nullptr)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "q_head needs qw/qb");
  const int block = 256, rows_per = block / 32;
  const int grid = (M + rows_per - 1) / rows_per;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y);
#define RN_F(N) launch_pdl(rownorm_fwd_kernel<N>, dim3(grid), dim3(block), 0, s, 1, x, yb, stat, w, temp, kind, eps, alpha, M, d, qw, qb, qout)
  switch (nv) {
    case 1: RN_F(1); break;
    case 2: RN_F(2); break;
    case 4: RN_F(4); break;
    case 8: RN_F(8); break;
    default: RN_F(16); break;
  }
#undef RN_F
  return rgpt_check_launch("rownorm_fwd_kernel");
}

extern "C" int rgpt_rownorm_bwd(const float* x, const float* dy, const float* w, float temp, int kind, float eps,
                                float alpha, int M, int d, const float* g_in, float* g_out, void* g_bf16,
                                const float* ls, const float* raw, float* dls, float* dw, float* dtemp,
                                const float* dq, const float* qw, const void* h, float* dqw, float* dqb,
                                const unsigned* drop_mask, float drop_p, void* stream) {
  const int nv = norm_nv(d);
  if (drop_mask != nullptr && !(drop_p >= 0.0f && drop_p < 1.0f))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout p must be in [0, 1), got %g", drop_p);
  const float drop_scale = (float)(1.0 / (1.0 - (double)drop_p));
  if (nv == 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm needs d in {128,256,512,1024,2048} (got %d)", d);
  if (dy == nullptr && dq == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm_bwd needs dy or dq");
  if (dq && (qw == nullptr)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "q_head mode needs qw");
  if (dqw && h == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dqw needs h");
  int dev = 0;
  cudaGetDevice(&dev);
  const int block = 256, rows_per = block / 32;
  int grid = (M + rows_per - 1) / rows_per;
  const int cap = rgpt_num_sms(dev) * 4;
  if (grid > cap) grid = cap;
  const size_t smem = 4 * d * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  __nv_bfloat16* gb = reinterpret_cast<__nv_bfloat16*>(g_bf16);
  const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(h);
  const bool want_dw = dw != nullptr && kind == RGPT_NORM_RMS_AFFINE, want_dls = dls != nullptr && raw != nullptr;
  auto launch = [&](auto nv_tag, auto qm_tag, auto dw_tag, auto dls_tag) {
    constexpr int N = decltype(nv_tag)::value;
    const int cap2 = rgpt_num_sms(dev) * (N <= 4 ? 2 : 1);
    launch_pdl(rownorm_bwd_kernel<N, decltype(qm_tag)::value, decltype(dw_tag)::value, decltype(dls_tag)::value>, dim3(grid < cap2 ? grid : cap2), dim3(block), smem, s, 1, x, dy, w, temp, kind, eps, alpha, M, d, g_in, g_out, gb, ls,
                                                        raw, dls, dw, dtemp, dq, qw, hb, dqw, dqb,
                                                        reinterpret_cast<const uint32_t*>(drop_mask), drop_scale);
  };
  auto with_flags = [&](auto nv_tag) {
    using T_ = std::true_type;
    using F_ = std::false_type;
    if (dq) {
      if (want_dw) want_dls ? launch(nv_tag, T_{}, T_{}, T_{}) : launch(nv_tag, T_{}, T_{}, F_{});
      else want_dls ? launch(nv_tag, T_{}, F_{}, T_{}) : launch(nv_tag, T_{}, F_{}, F_{});
    } else {
      if (want_dw) want_dls ? launch(nv_tag, F_{}, T_{}, T_{}) : launch(nv_tag, F_{}, T_{}, F_{});
      else want_dls ? launch(nv_tag, F_{}, F_{}, T_{}) : launch(nv_tag, F_{}, F_{}, F_{});
    }
  };
  switch (nv) {
    case 1: with_flags(std::integral_constant<int, 1>{}); break;
    case 2: with_flags(std::integral_constant<int, 2>{}); break;
    case 4: with_flags(std::integral_constant<int, 4>{}); break;
    case 8: with_flags(std::integral_constant<int, 8>{}); break;
    default: with_flags(std::integral_constant<int, 16>{}); break;
  }
  return rgpt_check_launch("rownorm_bwd_kernel");
}

static QkNormArgs qk_args(int kind, float eps, float alpha, const float* wq, const float* wk, float tq, float tk,
                          float sq, float sk) {
  QkNormArgs a;
  a.kind = kind;
  a.eps = eps;
  a.alpha = alpha;
  a.wq = wq;
  a.wk = wk;
  a.tq = tq;
  a.tk = tk;
  a.sq = sq;
  a.sk = sk;
  return a;
}

// Calls f(std::integral_constant<int, kind>{}) for a runtime norm kind.
template <typename F>
static void dispatch_norm_kind(int kind, F&& f) {
  switch (kind) {
    case RGPT_NORM_IDENTITY: f(std::integral_constant<int, RGPT_NORM_IDENTITY>{}); break;
    case RGPT_NORM_RMS_AFFINE: f(std::integral_constant<int, RGPT_NORM_RMS_AFFINE>{}); break;
    case RGPT_NORM_RMS: f(std::integral_constant<int, RGPT_NORM_RMS>{}); break;
    case RGPT_NORM_L2_TEMP: f(std::integral_constant<int, RGPT_NORM_L2_TEMP>{}); break;
    case RGPT_NORM_L2: f(std::integral_constant<int, RGPT_NORM_L2>{}); break;
    case RGPT_NORM_ELASTIC: f(std::integral_constant<int, RGPT_NORM_ELASTIC>{}); break;
    case RGPT_NORM_ELASTICBALL: f(std::integral_constant<int, RGPT_NORM_ELASTICBALL>{}); break;
    default: f(std::integral_constant<int, RGPT_NORM_HYPERBALL>{}); break;
  }
}

static int prep_grid(long long tokens, int H, int ctas_per_sm) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long long units = tokens * ((H + 1) / 2);  // (token, head pair) units, one warp each at a time
  const long long want = (units + 7) / 8;           // 8 warps per 256-thread CTA
  const long long cap = (long long)rgpt_num_sms(dev) * ctas_per_sm;
  return (int)(want < cap ? want : cap);
}

extern "C" int rgpt_qkv_prep_fwd(const void* qkv, void* qk, void* qn, const float* inv_freq, int qk_kind, float eps,
                                 float alpha, const float* wq, const float* wk, float tq, float tk, float sq, float sk,
                                 int M, int T, int H, void* stream) {
  if (M % T != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rows (%d) must be a multiple of T (%d)", M, T);
  if (T > 65536) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "RoPE positions are limited to T <= 65536 (got %d)", T);
  if (qk_kind == RGPT_NORM_RMS_AFFINE && (wq == nullptr || wk == nullptr))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rmsnorm QK norm needs weights");
  if (qk_kind < RGPT_NORM_IDENTITY || qk_kind > RGPT_NORM_HYPERBALL)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown QK norm kind %d", qk_kind);
  const QkNormArgs na = qk_args(qk_kind, eps, alpha, wq, wk, tq, tk, sq, sk);
  auto launch = [&](auto kind_tag) {
    launch_pdl(qkv_prep_fwd_kernel<decltype(kind_tag)::value>, dim3(prep_grid(M, H, 4)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
            reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<__nv_bfloat16*>(qk),
            reinterpret_cast<__nv_bfloat16*>(qn), inv_freq, na, M, T, H);
  };
  dispatch_norm_kind(qk_kind, launch);
  return rgpt_check_launch("qkv_prep_fwd_kernel");
}

extern "C" int rgpt_qkv_prep_bwd(const void* qkv, const float* dq, const float* dk, const float* dqn_gate,
                                 const void* dgp, void* dqkv, float* dbg, float* dwq, float* dwk, float* dtq,
                                 float* dtk, const float* inv_freq, int qk_kind, float eps, float alpha,
                                 const float* wq, const float* wk, float tq, float tk, float sq, float sk, int M, int T,
                                 int H, void* stream) {
  if (M % T != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rows (%d) must be a multiple of T (%d)", M, T);
  if (T > 65536) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "RoPE positions are limited to T <= 65536 (got %d)", T);
  if (dbg && dgp == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dbg needs dgp");
  if (qk_kind < RGPT_NORM_IDENTITY || qk_kind > RGPT_NORM_HYPERBALL)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown QK norm kind %d", qk_kind);
  const QkNormArgs na = qk_args(qk_kind, eps, alpha, wq, wk, tq, tk, sq, sk);
  auto launch = [&](auto kind_tag) {
    launch_pdl(qkv_prep_bwd_kernel<decltype(kind_tag)::value>, dim3(prep_grid(M, H, 3)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
            reinterpret_cast<const __nv_bfloat16*>(qkv), dq, dk, dqn_gate,
            reinterpret_cast<const __nv_bfloat16*>(dgp), reinterpret_cast<__nv_bfloat16*>(dqkv), dbg, dwq, dwk, dtq,
            dtk, inv_freq, na, M, T, H);
  };
  dispatch_norm_kind(qk_kind, launch);
  return rgpt_check_launch("qkv_prep_bwd_kernel");
}

// Dropout arguments of the embedding kernels: a mask (null = no dropout), p in [0, 1), rows of
// d % 128 == 0 columns, and (forward only) the device seed.
// Row-layout dropout keep bits [M, N] (residual branches, model/transformer_block.py:45,52): the bit of
// (row, column) comes from Philox4x32-10 block (column / 8, row, site, 0) under key (seed low, high 32
// bits), the 16-bit uniform (column % 8) -> word (column % 8) / 2, half column % 2, kept iff >= thresh;
// one thread per 32-column word: mask[row * ldm + column / 32] bit column % 32.
__global__ void drop_mask_rows_kernel(uint32_t* __restrict__ mask, long long ldm, const unsigned long long* seed,
                                      uint32_t site, uint32_t thresh, int M, int words) {
  griddep_wait();
  griddep_launch();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)M * words) return;
  const int row = (int)(i / words), w = (int)(i - (long long)row * words);
  const unsigned long long sd = *seed;
  mask[row * ldm + w] = keep32((uint32_t)(w * 32), (uint32_t)row, site, 0u, (uint32_t)sd, (uint32_t)(sd >> 32), thresh);
}

static int check_drop(const void* mask, bool need_seed, const void* seed, float p, int d) {
  if (mask == nullptr) return 0;
  if (!(p >= 0.0f && p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout p must be in [0, 1), got %g", p);
  if (d % 128 != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout needs d %% 128 == 0 (got %d)", d);
  if (need_seed && seed == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout needs a device seed");
  return 0;
}

extern "C" int rgpt_embedding_fwd(const long long* ids, const float* emb, float* x, int M, int d, int V,
                                  unsigned* drop_mask, const unsigned long long* drop_seed, unsigned drop_site,
                                  float drop_p, void* stream) {
  if (d % 4 != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "embedding dim must be a multiple of 4");
  if (int st = check_drop(drop_mask, true, drop_seed, drop_p, d)) return st;
  const int block = 256, rows_per = block / 32;
  int* err = nullptr;
  cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_rgpt_device_error);
  const uint32_t thresh = (uint32_t)lrintf(drop_p * 65536.0f);
  const float scale = (float)(1.0 / (1.0 - (double)drop_p));
  launch_pdl(embedding_fwd_kernel, dim3((M + rows_per - 1) / rows_per), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      ids, emb, x, M, d, V, err, reinterpret_cast<uint32_t*>(drop_mask), drop_seed, (uint32_t)drop_site, thresh,
      scale);
  return rgpt_check_launch("embedding_fwd_kernel");
}

extern "C" int rgpt_embedding_bwd(const long long* ids, const float* dx, float* demb, int M, int d, int V,
                                  const unsigned* drop_mask, float drop_p, void* stream) {
  if (d % 4 != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "embedding dim must be a multiple of 4");
  if (int st = check_drop(drop_mask, false, nullptr, drop_p, d)) return st;
  const int block = 256, rows_per = block / 32;
  const float scale = (float)(1.0 / (1.0 - (double)drop_p));
  launch_pdl(embedding_bwd_kernel, dim3((M + rows_per - 1) / rows_per), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      ids, dx, demb, M, d, V, reinterpret_cast<const uint32_t*>(drop_mask), scale);
  return rgpt_check_launch("embedding_bwd_kernel");
}

extern "C" int rgpt_cross_entropy(void* logits, long long ld, int M, int V, const long long* labels, int ignore_index,
                                  float grad_scale, float* loss_rows, int* argmax, float* scale_buf, float* loss_out,
                                  int write_grad, void* stream) {
  if ((reinterpret_cast<uintptr_t>(logits) & 15) || (ld % 8))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "logits must be 16-byte aligned with ld %% 8 == 0");
  if ((write_grad || loss_out) && scale_buf == nullptr)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "scale_buf (2 floats) required for loss / grad");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (scale_buf) launch_pdl(ce_count_kernel, dim3(1), dim3(1024), 0, s, 1, labels, M, ignore_index, grad_scale, scale_buf, scale_buf + 1);
  int st = launch_cross_entropy_rows(reinterpret_cast<__nv_bfloat16*>(logits), ld, M, V, labels, ignore_index,
                                     loss_rows, argmax, scale_buf, write_grad, s);
  if (st) return st;
  if (loss_out && loss_rows) launch_pdl(ce_finalize_kernel, dim3(1), dim3(1024), 0, s, 1, loss_rows, M, scale_buf + 1, loss_out);
  return rgpt_check_launch("cross_entropy_kernel");
}

extern "C" int rgpt_halt_losses(const float* q, const int* argmax, const long long* labels, int R, int M,
                                float grad_scale, float* dq, float* losses, void* stream) {
  const int block = 256;
  launch_pdl(halt_losses_kernel, dim3((M + block - 1) / block), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      q, argmax, labels, R, M, grad_scale, dq, losses);
  return rgpt_check_launch("halt_losses_kernel");
}

// ============================================================================ allocation-free cross entropy
// For callers that cannot allocate device memory: plugin-style hosts whose enqueue
// contract hands over only the input/output buffers, and processes whose device memory
// is already fully reserved by another framework's pool, so a cudaMalloc would fail.
// The scratch that rgpt_cross_entropy takes from its caller (per-row losses and the
// {grad_scale/count, count} pair) lives instead in this file-scope array, which every
// GPU that loads the library holds until the process exits (1 MiB + 256 B).
#define RGPT_CE_NOALLOC_MAX_ROWS 262144
static __device__ __align__(256) float g_ce_noalloc_scratch[RGPT_CE_NOALLOC_MAX_ROWS + 64];

// Device address of the scratch array for `dev`, resolved once per device with that device
// current. (In host code the array's name only stands in for the symbol.) The cache is atomic, so
// threads making their first call on one device at the same time are safe (both store the same
// address). It belongs to the device context that resolved it: after cudaDeviceReset the cached
// address is stale, so a process that resets a device must not call this entry point on it again.
static float* ce_noalloc_scratch(int dev, int* status) {
  static std::atomic<float*> addr[64];
  if (dev < 0 || dev >= 64) {
    *status = rgpt_set_error(RGPT_ERR_INTERNAL, "device index %d out of range", dev);
    return nullptr;
  }
  float* a = addr[dev].load(std::memory_order_acquire);
  if (a == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ce_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = rgpt_set_error(RGPT_ERR_INTERNAL, "cudaGetSymbolAddress(cross-entropy scratch) failed: %s",
                               cudaGetErrorString(e));
      return nullptr;
    }
    a = reinterpret_cast<float*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

extern "C" int rgpt_cross_entropy_noalloc(void* logits, long long ld, int M, int V, const long long* labels,
                                          int ignore_index, float grad_scale, float* loss_out, int* argmax,
                                          int write_grad, void* stream) {
  if (M < 1 || M > RGPT_CE_NOALLOC_MAX_ROWS)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE,
                          "rgpt_cross_entropy_noalloc handles 1..%d rows (got %d); use rgpt_cross_entropy for more",
                          RGPT_CE_NOALLOC_MAX_ROWS, M);
  if (loss_out == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "loss_out is required");
  if ((reinterpret_cast<uintptr_t>(logits) & 15) || (ld % 8))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "logits must be 16-byte aligned with ld %% 8 == 0");
  int dev = 0;
  cudaGetDevice(&dev);
  int st = RGPT_OK;
  float* scratch = ce_noalloc_scratch(dev, &st);
  if (scratch == nullptr) return st;
  float* loss_rows = scratch;                           // M floats, every one rewritten by this call
  float* scale_buf = scratch + RGPT_CE_NOALLOC_MAX_ROWS;  // {grad_scale/count, count}, rewritten by this call
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_pdl(ce_count_kernel, dim3(1), dim3(1024), 0, s, 1, labels, M, ignore_index, grad_scale, scale_buf, scale_buf + 1);
  if ((st = launch_cross_entropy_rows(reinterpret_cast<__nv_bfloat16*>(logits), ld, M, V, labels, ignore_index,
                                      loss_rows, argmax, scale_buf, write_grad, s)))
    return st;
  launch_pdl(ce_finalize_kernel, dim3(1), dim3(1024), 0, s, 1, loss_rows, M, scale_buf + 1, loss_out);
  return rgpt_check_launch("cross_entropy_noalloc");
}

extern "C" int rgpt_drop_mask(unsigned* mask, long long ldm, const unsigned long long* seed, unsigned site, float p,
                              int M, int N, void* stream) {
  if (mask == nullptr || seed == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout mask and seed needed");
  if (!(p >= 0.0f && p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout p must be in [0, 1), got %g", p);
  const int words = (N + 31) / 32;
  if (M < 1 || N < 1 || ldm < words) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout mask: bad shape");
  const long long n = (long long)M * words;
  launch_pdl(drop_mask_rows_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
             reinterpret_cast<cudaStream_t>(stream), 1, reinterpret_cast<uint32_t*>(mask), ldm, seed, (uint32_t)site,
             (uint32_t)lrintf(p * 65536.0f), M, words);
  return rgpt_check_launch("drop_mask_rows_kernel");
}
