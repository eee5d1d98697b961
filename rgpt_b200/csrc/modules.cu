// Kernels behind the reference's submodules when they are called on their own, outside GPT's fused
// engine (which runs the norms, RoPE and QK norms inside its own kernels):
//
//   rownorm_any_fwd/bwd  every norm kind of model/norm.py:8-162 over rows of ANY length d (the QK norms'
//                        d_head = 64 included); fp32 in and out. One warp per row.
//   rope                 RotaryEmbedding.forward, model/rope.py:38-57: rotate-half RoPE of a [B, H, T, D]
//                        tensor (any strides, unit stride on D), angles t * inv_freq[j] in fp32; the
//                        backward applies the transposed rotation.
#include <math.h>

#include "common.cuh"
#include "norm.cuh"
#include "rgpt.h"

namespace rgpt {

// per-column affine factor: RMSNorm (1 + w[c]), L2Norm's learned temperature w[0] (read on the device)
__device__ __forceinline__ float row_affine(int kind, const float* w, int c) {
  if (kind == RGPT_NORM_RMS_AFFINE) return 1.0f + w[c];
  if (kind == RGPT_NORM_L2_TEMP) return w ? w[0] : 1.0f;
  return 1.0f;
}

__global__ void rownorm_any_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, const float* __restrict__ w,
                                       int kind, float eps, float alpha, long long M, int d) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const float* xr = x + row * d;
  float S = 0.f;
  for (int c = lane; c < d; c += 32) S += xr[c] * xr[c];
  S = warp_sum(S);
  const NS2 ns = norm_scale(kind, S, d, eps, alpha);
  float* yr = y + row * d;
  // x * s first, then the affine factor: the reference's order (model/norm.py:27-34, :50-51)
  for (int c = lane; c < d; c += 32) yr[c] = __fmul_rn(__fmul_rn(xr[c], ns.s), row_affine(kind, w, c));
}

// dx = s a dy + 2 s'(S) (sum a dy x) x;  dw[c] += dy x s (RMSNorm);  dtemp += sum dy x s (L2Norm).
// Grid-stride over rows; the column partials of dw / dtemp gather in shared memory, one global atomic
// per column and CTA.
__global__ void rownorm_any_bwd_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                       const float* __restrict__ w, int kind, float eps, float alpha, long long M,
                                       int d, float* __restrict__ dx, float* __restrict__ dw,
                                       float* __restrict__ dtemp) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float red[];  // [d] weight partials, [1] temperature partial
  const bool want_dw = dw != nullptr && kind == RGPT_NORM_RMS_AFFINE;
  const bool want_dt = dtemp != nullptr && kind == RGPT_NORM_L2_TEMP;
  for (int i = threadIdx.x; i <= d; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5); row < M;
       row += (long long)gridDim.x * warps) {
    const float* xr = x + row * d;
    const float* gr = dy + row * d;
    float S = 0.f, c = 0.f, xdy = 0.f;
    for (int j = lane; j < d; j += 32) {
      const float xv = xr[j], gv = gr[j];
      S += xv * xv;
      c += row_affine(kind, w, j) * gv * xv;
      xdy += gv * xv;
    }
    S = warp_sum(S);
    c = warp_sum(c);
    const NS2 ns = norm_scale(kind, S, d, eps, alpha);
    const float k2 = 2.0f * ns.ds * c;
    float* dr = dx + row * d;
    for (int j = lane; j < d; j += 32) {
      const float xv = xr[j], gv = gr[j];
      dr[j] = ns.s * row_affine(kind, w, j) * gv + k2 * xv;
      if (want_dw) atomicAdd(&red[j], gv * xv * ns.s);
    }
    if (want_dt) {
      xdy = warp_sum(xdy);
      if (lane == 0) atomicAdd(&red[d], xdy * ns.s);
    }
  }
  __syncthreads();
  if (want_dw)
    for (int j = threadIdx.x; j < d; j += blockDim.x) atomicAdd(&dw[j], red[j]);
  if (want_dt && threadIdx.x == 0) atomicAdd(dtemp, red[d]);
}

// One thread per (b, h, t, j < D/2): the pair (j, j + D/2) rotates by the angle t * inv_freq[j].
// forward:  y1 = x1 cos - x2 sin,  y2 = x2 cos + x1 sin   (q * cos + rotate_half(q) * sin)
// backward: the transpose, i.e. the same with sin negated (dir = -1).
// Products and the sum are rounded one by one, as torch evaluates q*cos + rotate_half(q)*sin.
__global__ void rope_kernel(const float* __restrict__ in, long long sb, long long sh, long long st,
                            float* __restrict__ out, const float* __restrict__ inv_freq, int B, int H, int T, int D,
                            float dir) {
  griddep_wait();
  griddep_launch();
  const int half = D >> 1;
  const long long total = (long long)B * H * T * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    long long r = i / half;
    const int t = (int)(r % T);
    r /= T;
    const int h = (int)(r % H);
    const int b = (int)(r / H);
    const float* p = in + b * sb + h * sh + t * st;
    const float x1 = p[j], x2 = p[j + half];
    float sn, cs;
    sincosf(__fmul_rn((float)t, inv_freq[j]), &sn, &cs);
    sn *= dir;
    float* o = out + (((long long)b * H + h) * T + t) * D;
    o[j] = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(-x2, sn));
    o[j + half] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
  }
}

}  // namespace rgpt

using namespace rgpt;

extern "C" int rgpt_rownorm_any_fwd(const float* x, float* y, const float* w, int kind, float eps, float alpha,
                                    long long M, int d, void* stream) {
  if (M < 0 || d < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm_any needs M >= 0, d >= 1 (M=%lld d=%d)", M, d);
  if (kind < RGPT_NORM_IDENTITY || kind > RGPT_NORM_HYPERBALL)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown norm kind %d", kind);
  if (kind == RGPT_NORM_RMS_AFFINE && w == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rmsnorm needs w");
  if (M == 0) return RGPT_OK;
  const int block = 256;
  const long long grid = (M + 7) / 8;
  if (grid > 0x7fffffffLL) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm_any: too many rows (%lld)", M);
  launch_pdl(rownorm_any_fwd_kernel, dim3((unsigned)grid), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1,
             x, y, w, kind, eps, alpha, M, d);
  return rgpt_check_launch("rownorm_any_fwd_kernel");
}

extern "C" int rgpt_rownorm_any_bwd(const float* x, const float* dy, const float* w, int kind, float eps, float alpha,
                                    long long M, int d, float* dx, float* dw, float* dtemp, void* stream) {
  if (M < 0 || d < 1 || d > 16384)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rownorm_any_bwd needs M >= 0, 1 <= d <= 16384 (M=%lld d=%d)", M, d);
  if (kind < RGPT_NORM_IDENTITY || kind > RGPT_NORM_HYPERBALL)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown norm kind %d", kind);
  if (kind == RGPT_NORM_RMS_AFFINE && w == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rmsnorm needs w");
  if (M == 0) return RGPT_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int block = 256;
  long long grid = (M + 7) / 8;
  const long long cap = 4LL * rgpt_num_sms(dev);
  if (grid > cap) grid = cap;
  const size_t smem = (size_t)(d + 1) * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(rownorm_any_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(rownorm_any_bwd_kernel, dim3((unsigned)grid), dim3(block), smem, s, 1, x, dy, w, kind, eps, alpha, M, d,
             dx, dw, dtemp);
  return rgpt_check_launch("rownorm_any_bwd_kernel");
}

extern "C" int rgpt_rope(const float* in, long long sb, long long sh, long long st, float* out, const float* inv_freq,
                         int B, int H, int T, int D, int backward, void* stream) {
  if (B < 0 || H < 0 || T < 0 || D < 2 || (D & 1))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "rope needs B, H, T >= 0 and an even D >= 2 (D=%d)", D);
  const long long total = (long long)B * H * T * (D / 2);
  if (total == 0) return RGPT_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int block = 256;
  long long grid = (total + block - 1) / block;
  const long long cap = 16LL * rgpt_num_sms(dev);
  if (grid > cap) grid = cap;
  launch_pdl(rope_kernel, dim3((unsigned)grid), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1, in, sb, sh,
             st, out, inv_freq, B, H, T, D, backward ? -1.0f : 1.0f);
  return rgpt_check_launch("rope_kernel");
}
