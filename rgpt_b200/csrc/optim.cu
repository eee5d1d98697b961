// Optimizer kernels: multi-tensor AdamW and the Muon update around Newton-Schulz.
//
// AdamW (optimizer.py:80-116), one launch for every tensor of a param group:
//   p *= 1 - lr*wd;  m = lerp(m, g, 1-b1);  v = lerp(v, g*g, 1-b2)
//   p -= lr * (m / bc1) / (sqrt(v) / sqrt(bc2) + eps)
// and, when a bf16 shadow pointer is given, shadow = bf16(p) (the GEMM operand copy).
//
// Muon (optimizer.py:51-74, :199-227), per shape class of matrices [R, C]:
//   muon_prep   g_b = bf16(grad); m = lerp(m, g_b, 1-beta) (bf16); g = lerp(g_b, m, beta) (Nesterov);
//               X = g (transposed when R > C) into a zero-padded bf16 stack; ||X||_F^2 per matrix
//   ns_scale    X = bf16(X / max(||X||_F, 1e-7))
//   (5 iterations of three batched tcgen05 GEMMs: A = X X^T; B = b*A + c*A*A; X = a*X + B*X)
//   muon_apply  p = p * (1 - lr*wd) - muon_lr * bf16(X * scale) (transposed back); shadow = bf16(p)
// Tensors are addressed through small device-resident descriptor tables built once by the host.
#include "common.cuh"
#include "rgpt.h"

namespace rgpt {

// ---------------------------------------------------------------------------- AdamW
__device__ __forceinline__ float lerpf_torch(float a, float b, float w) {
  // torch's lerp: a + w (b - a) for w < 0.5, else b - (b - a)(1 - w)
  return (w < 0.5f) ? a + w * (b - a) : b - (b - a) * (1.0f - w);
}

__global__ void adamw_kernel(const RgptAdamwTensor* __restrict__ tab, const int* __restrict__ chunk_tensor,
                             const long long* __restrict__ chunk_start, int chunk_elems, float lr, float wd,
                             float beta1, float beta2, float eps, float inv_bc1, float inv_sqrt_bc2) {
  const int c = blockIdx.x;
  const RgptAdamwTensor t = tab[chunk_tensor[c]];
  const long long start = chunk_start[c];
  const long long end = min(start + (long long)chunk_elems, t.n);
  const float decay = 1.0f - lr * wd;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    float p = t.p[i];
    const float g = t.g[i];
    if (wd != 0.f) p *= decay;
    const float m = lerpf_torch(t.m[i], g, 1.0f - beta1);
    const float v = lerpf_torch(t.v[i], g * g, 1.0f - beta2);
    t.m[i] = m;
    t.v[i] = v;
    const float denom = sqrtf(v) * inv_sqrt_bc2 + eps;
    p = p - lr * ((m / denom) * inv_bc1);
    t.p[i] = p;
    if (t.shadow) t.shadow[i] = __bfloat16_as_ushort(__float2bfloat16(p));
  }
}

// ---------------------------------------------------------------------------- Muon
// One CTA per 32x32 tile of one matrix. grid = (tiles_c, tiles_r, n_matrices).
__global__ void muon_prep_kernel(const RgptMuonTensor* __restrict__ tab, int R, int C, int transpose,
                                 __nv_bfloat16* __restrict__ X, long long x_bstride, int ldx, float beta,
                                 int nesterov, float* __restrict__ sumsq) {
  __shared__ float tile[32][33];
  const RgptMuonTensor t = tab[blockIdx.z];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  float ss = 0.f;
  for (int rr = ty; rr < 32; rr += 8) {
    const int r = r0 + rr, c = c0 + tx;
    float x = 0.f;
    if (r < R && c < C) {
      const long long i = (long long)r * C + c;
      const float gb = __bfloat162float(__float2bfloat16(t.grad[i]));  // grad.to(bf16)
      const float m_old = __bfloat162float(__ushort_as_bfloat16(t.mom[i]));
      const float m_new = __bfloat162float(__float2bfloat16(lerpf_torch(m_old, gb, 1.0f - beta)));
      t.mom[i] = __bfloat16_as_ushort(__float2bfloat16(m_new));
      x = nesterov ? __bfloat162float(__float2bfloat16(lerpf_torch(gb, m_new, beta))) : m_new;
      ss += x * x;
    }
    tile[rr][tx] = x;
  }
  __syncthreads();
  __nv_bfloat16* Xb = X + (long long)blockIdx.z * x_bstride;
  for (int rr = ty; rr < 32; rr += 8) {
    if (!transpose) {
      const int r = r0 + rr, c = c0 + tx;
      if (r < R && c < C) Xb[(long long)r * ldx + c] = __float2bfloat16(tile[rr][tx]);
    } else {
      // X[c][r] = g[r][c]: thread tx walks r (contiguous in X's row c)
      const int c = c0 + rr, r = r0 + tx;
      if (r < R && c < C) Xb[(long long)c * ldx + r] = __float2bfloat16(tile[tx][rr]);
    }
  }
  ss = warp_sum(ss);
  __shared__ float red[8];
  if (tx == 0) red[ty] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    atomicAdd(&sumsq[blockIdx.z], s);
  }
}

// X = bf16(X / max(sqrt(sumsq), 1e-7)) over the valid [rows, cols] block of each matrix.
__global__ void ns_scale_kernel(__nv_bfloat16* __restrict__ X, long long x_bstride, int ldx, int rows, int cols,
                                const float* __restrict__ sumsq) {
  const int b = blockIdx.y;
  const float inv = 1.0f / fmaxf(sqrtf(sumsq[b]), 1e-7f);
  __nv_bfloat16* Xb = X + (long long)b * x_bstride;
  const int pairs = cols / 2;  // cols is even (the stacks are padded to multiples of 8)
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    __nv_bfloat162* row = reinterpret_cast<__nv_bfloat162*>(Xb + (long long)r * ldx);
    for (int c = threadIdx.x; c < pairs; c += blockDim.x) {
      float2 v = __bfloat1622float2(row[c]);
      row[c] = __floats2bfloat162_rn(v.x * inv, v.y * inv);
    }
  }
}

__global__ void muon_apply_kernel(const RgptMuonTensor* __restrict__ tab, int R, int C, int transpose,
                                  const __nv_bfloat16* __restrict__ X, long long x_bstride, int ldx, float decay,
                                  float neg_lr, float scale) {
  __shared__ float tile[32][33];
  const RgptMuonTensor t = tab[blockIdx.z];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const __nv_bfloat16* Xb = X + (long long)blockIdx.z * x_bstride;
  for (int rr = ty; rr < 32; rr += 8) {
    if (!transpose) {
      const int r = r0 + rr, c = c0 + tx;
      tile[rr][tx] = (r < R && c < C) ? __bfloat162float(Xb[(long long)r * ldx + c]) : 0.f;
    } else {
      const int c = c0 + rr, r = r0 + tx;
      tile[tx][rr] = (r < R && c < C) ? __bfloat162float(Xb[(long long)c * ldx + r]) : 0.f;
    }
  }
  __syncthreads();
  for (int rr = ty; rr < 32; rr += 8) {
    const int r = r0 + rr, c = c0 + tx;
    if (r < R && c < C) {
      const long long i = (long long)r * C + c;
      const float u = __bfloat162float(__float2bfloat16(tile[rr][tx] * scale));  // upd.mul_(scale) in bf16
      float p = t.param[i];
      if (decay != 1.0f) p *= decay;
      p += neg_lr * u;
      t.param[i] = p;
      if (t.shadow) t.shadow[i] = __bfloat16_as_ushort(__float2bfloat16(p));
    }
  }
}

}  // namespace rgpt

using namespace rgpt;

extern "C" int rgpt_adamw(const RgptAdamwTensor* table, const int* chunk_tensor, const long long* chunk_start,
                          int n_chunks, int chunk_elems, float lr, float wd, float beta1, float beta2, float eps,
                          int step, void* stream) {
  if (n_chunks <= 0) return RGPT_OK;
  if (step < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "adamw step must be >= 1");
  const double bc1 = 1.0 - pow((double)beta1, (double)step);
  const double bc2 = 1.0 - pow((double)beta2, (double)step);
  adamw_kernel<<<n_chunks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      table, chunk_tensor, chunk_start, chunk_elems, lr, wd, beta1, beta2, eps, (float)(1.0 / bc1),
      (float)(1.0 / sqrt(bc2)));
  return rgpt_check_launch("adamw_kernel");
}

extern "C" int rgpt_muon_prep(const RgptMuonTensor* table, int n, int R, int C, void* X, long long x_bstride, int ldx,
                              float beta, int nesterov, float* sumsq, void* stream) {
  const int transpose = R > C ? 1 : 0;
  const int xr = transpose ? C : R, xc = transpose ? R : C;
  if (ldx < xc) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "NS stack too narrow (ldx %d < %d)", ldx, xc);
  (void)xr;
  dim3 grid((C + 31) / 32, (R + 31) / 32, n);
  muon_prep_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      table, R, C, transpose, reinterpret_cast<__nv_bfloat16*>(X), x_bstride, ldx, beta, nesterov, sumsq);
  return rgpt_check_launch("muon_prep_kernel");
}

extern "C" int rgpt_ns_scale(void* X, long long x_bstride, int ldx, int rows, int cols, int n, const float* sumsq,
                             void* stream) {
  if (cols % 2 != 0 || ldx % 2 != 0) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_scale needs even cols and ldx");
  const int gx = rows < 256 ? rows : 256;
  ns_scale_kernel<<<dim3(gx, n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(X), x_bstride, ldx, rows, cols, sumsq);
  return rgpt_check_launch("ns_scale_kernel");
}

extern "C" int rgpt_muon_apply(const RgptMuonTensor* table, int n, int R, int C, const void* X, long long x_bstride,
                               int ldx, float lr, float wd, float muon_lr, float scale, void* stream) {
  const int transpose = R > C ? 1 : 0;
  dim3 grid((C + 31) / 32, (R + 31) / 32, n);
  muon_apply_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      table, R, C, transpose, reinterpret_cast<const __nv_bfloat16*>(X), x_bstride, ldx, 1.0f - lr * wd, -muon_lr,
      scale);
  return rgpt_check_launch("muon_apply_kernel");
}
