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
//
// fp32 Newton-Schulz (zeropower_via_newtonschulz5 with X = G.float(), optimizer.py:8-45):
//   ns_sumsq    ||X||_F^2 per matrix, reading the unit-stride dimension fastest
//   ns_split    X / max(||X||_F, 1e-7) (optional), an fp32 copy, and bf16 hi/lo blocks for the GEMMs
// Tensors are addressed through small device-resident descriptor tables built once by the host.
#include "common.cuh"
#include "rgpt.h"

namespace rgpt {

// ---------------------------------------------------------------------------- AdamW
__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float lerpf_torch(float a, float b, float w) {
  // torch's lerp: a + w (b - a) for w < 0.5, else b - (b - a)(1 - w), each as one fused step
  const float d = b - a;
  return (w < 0.5f) ? fmaf(w, d, a) : fmaf(-d, 1.0f - w, b);
}

__global__ void adamw_kernel(const RgptAdamwTensor* __restrict__ tab, const int* __restrict__ chunk_tensor,
                             const long long* __restrict__ chunk_start, int chunk_elems, float lr, float wd,
                             float beta1, float beta2, float eps, float inv_bc1, float inv_sqrt_bc2,
                             const float* __restrict__ hp) {
  griddep_wait();
  griddep_launch();
  if (hp != nullptr) {  // this step's scalars from the device block (layout in rgpt.h)
    lr = hp[0], wd = hp[1], beta1 = hp[2], beta2 = hp[3], eps = hp[4], inv_bc1 = hp[5], inv_sqrt_bc2 = hp[6];
  }
  const int c = blockIdx.x;
  const RgptAdamwTensor t = tab[chunk_tensor[c]];
  const long long start = chunk_start[c];
  const long long end = min(start + (long long)chunk_elems, t.n);
  const float decay = 1.0f - lr * wd;
  // Every rounding spelled out (torch's op order: p*decay, lerps, sqrt(v)*c + eps, m/denom*c,
  // p - lr*u as one fused step), so no expression has two products the compiler could pick
  // between for contraction: the vector and scalar paths give identical bits.
  auto update = [&](float& p, float g, float& m, float& v) {
    if (wd != 0.f) p = __fmul_rn(p, decay);
    m = lerpf_torch(m, g, 1.0f - beta1);
    v = lerpf_torch(v, __fmul_rn(g, g), 1.0f - beta2);
    const float denom = __fadd_rn(__fmul_rn(sqrtf(v), inv_sqrt_bc2), eps);
    p = fmaf(-lr, __fmul_rn(__fdiv_rn(m, denom), inv_bc1), p);
  };
  long long i = start;
  // 16-byte accesses over the aligned body of the chunk (chunk starts are multiples of 4)
  if (aligned16(t.p) && aligned16(t.g) && aligned16(t.m) && aligned16(t.v) &&
      (reinterpret_cast<uintptr_t>(t.shadow) & 7) == 0 && (start & 3) == 0) {
    const long long end4 = start + ((end - start) & ~3ll);
    for (long long j = start + 4ll * threadIdx.x; j < end4; j += 4ll * blockDim.x) {
      float4 p = *reinterpret_cast<const float4*>(t.p + j);
      const float4 g = *reinterpret_cast<const float4*>(t.g + j);
      float4 m = *reinterpret_cast<const float4*>(t.m + j);
      float4 v = *reinterpret_cast<const float4*>(t.v + j);
      update(p.x, g.x, m.x, v.x);
      update(p.y, g.y, m.y, v.y);
      update(p.z, g.z, m.z, v.z);
      update(p.w, g.w, m.w, v.w);
      *reinterpret_cast<float4*>(t.m + j) = m;
      *reinterpret_cast<float4*>(t.v + j) = v;
      *reinterpret_cast<float4*>(t.p + j) = p;
      if (t.shadow) *reinterpret_cast<uint2*>(t.shadow + j) = make_uint2(pack_bf16x2(p.x, p.y), pack_bf16x2(p.z, p.w));
    }
    i = end4;
  }
  for (i += threadIdx.x; i < end; i += blockDim.x) {
    float p = t.p[i], m = t.m[i], v = t.v[i];
    update(p, t.g[i], m, v);
    t.m[i] = m;
    t.v[i] = v;
    t.p[i] = p;
    if (t.shadow) t.shadow[i] = __bfloat16_as_ushort(__float2bfloat16(p));
  }
}

// ---------------------------------------------------------------------------- Muon
// One CTA per 64x64 tile of one matrix; grid = (tiles_c, tiles_r, n_matrices). Each thread owns
// groups of 8 consecutive columns of one row (16-byte bf16 / 2x16-byte fp32 accesses). The
// transposed NS stack (R > C) is written through a shared tile of bf16 pairs: a thread then owns
// 8 consecutive rows of two columns, i.e. 16 contiguous bytes of two rows of X. Groups that run
// past the matrix edge, or tensors that are not 16-byte aligned, take the same path with scalar
// accesses, so the arithmetic (and the result) does not depend on alignment.
constexpr int MUON_TILE = 64;
constexpr int MUON_LDW = MUON_TILE / 2 + 1;  // 32-bit words per shared row: 32 bf16 pairs + 1 pad


__device__ __forceinline__ void load8_f32(const float* p, bool vec, int n, float* v) {
  if (vec) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = k < n ? p[k] : 0.f;
  }
}
__device__ __forceinline__ void store8_f32(float* p, bool vec, int n, const float* v) {
  if (vec) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < n) p[k] = v[k];
  }
}
__device__ __forceinline__ void load8_bf16(const unsigned short* p, bool vec, int n, float* v) {
  if (vec) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w4[j]);
      v[2 * j] = f.x, v[2 * j + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = k < n ? __bfloat162float(__ushort_as_bfloat16(p[k])) : 0.f;
  }
}
__device__ __forceinline__ void store8_bf16(unsigned short* p, bool vec, int n, const float* v) {
  if (vec) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                              pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < n) p[k] = __bfloat16_as_ushort(__float2bfloat16(v[k]));
  }
}

__global__ void __launch_bounds__(256) muon_prep_kernel(const RgptMuonTensor* __restrict__ tab, int R, int C,
                                                        int transpose, unsigned short* __restrict__ X,
                                                        long long x_bstride, int ldx, float beta, int nesterov,
                                                        float* __restrict__ sumsq, const float* __restrict__ hp) {
  griddep_wait();
  griddep_launch();
  if (hp != nullptr) beta = hp[0];
  __shared__ uint32_t tile[MUON_TILE][MUON_LDW];
  __shared__ float red[8];
  const RgptMuonTensor t = tab[blockIdx.z];
  const int r0 = blockIdx.y * MUON_TILE, c0 = blockIdx.x * MUON_TILE;
  unsigned short* Xb = X + (long long)blockIdx.z * x_bstride;
  const bool src_vec = (C % 8 == 0) && aligned16(t.grad) && aligned16(t.mom);
  const bool x_vec = (ldx % 8 == 0) && (x_bstride % 8 == 0) && aligned16(X);
  const int cg = threadIdx.x & 7;
  float ss = 0.f;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int rr = pass * 32 + (threadIdx.x >> 3);
    const int r = r0 + rr, c = c0 + cg * 8;
    const int n = r < R ? min(8, C - c) : 0;  // valid elements of this group (<= 0: none)
    float x[8];
    if (n > 0) {
      const long long i = (long long)r * C + c;
      const bool vec = src_vec && n == 8;
      float g[8], m[8];
      load8_f32(t.grad + i, vec, n, g);
      load8_bf16(t.mom + i, vec, n, m);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gb = __bfloat162float(__float2bfloat16(g[k]));  // grad.to(bf16)
        const float m_new = __bfloat162float(__float2bfloat16(lerpf_torch(m[k], gb, 1.0f - beta)));
        m[k] = m_new;
        x[k] = k < n ? (nesterov ? __bfloat162float(__float2bfloat16(lerpf_torch(gb, m_new, beta))) : m_new) : 0.f;
        ss += x[k] * x[k];
      }
      store8_bf16(t.mom + i, vec, n, m);
      if (!transpose) store8_bf16(Xb + (long long)r * ldx + c, x_vec && n == 8, n, x);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = 0.f;
    }
    if (transpose) {
#pragma unroll
      for (int j = 0; j < 4; ++j) tile[rr][cg * 4 + j] = pack_bf16x2(x[2 * j], x[2 * j + 1]);
    }
  }
  if (transpose) {
    __syncthreads();
    // X[c][r] = g[r][c]: this thread writes rows r0+8rg..+7 of columns c0+2cp and c0+2cp+1
    const int rg = threadIdx.x & 7, cp = threadIdx.x >> 3;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = tile[rg * 8 + k][cp];
    const int r = r0 + rg * 8;
    const int n = min(8, R - r);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + 2 * cp + h;
      if (c < C && n > 0) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 f = unpack_bf16x2(w[k]);
          v[k] = h ? f.y : f.x;
        }
        store8_bf16(Xb + (long long)c * ldx + r, x_vec && n == 8, n, v);
      }
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
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
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const float inv = 1.0f / fmaxf(sqrtf(sumsq[b]), 1e-7f);
  __nv_bfloat16* Xb = X + (long long)b * x_bstride;
  const bool vec = (cols % 8 == 0) && (ldx % 8 == 0) && (x_bstride % 8 == 0) && aligned16(X);
  if (vec) {
    const int octs = cols / 8;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      uint4* row = reinterpret_cast<uint4*>(Xb + (long long)r * ldx);
      for (int c = threadIdx.x; c < octs; c += blockDim.x) {
        uint4 w = row[c];
        uint32_t* w4 = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 v = unpack_bf16x2(w4[j]);
          w4[j] = pack_bf16x2(v.x * inv, v.y * inv);
        }
        row[c] = w;
      }
    }
    return;
  }
  // any width, stride or alignment: one 2-byte element per access
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    __nv_bfloat16* row = Xb + (long long)r * ldx;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) row[c] = __float2bfloat16(__bfloat162float(row[c]) * inv);
  }
}

__global__ void __launch_bounds__(256) muon_apply_kernel(const RgptMuonTensor* __restrict__ tab, int R, int C,
                                                         int transpose, const unsigned short* __restrict__ X,
                                                         long long x_bstride, int ldx, float decay, float neg_lr,
                                                         float scale, const float* __restrict__ hp) {
  griddep_wait();
  griddep_launch();
  if (hp != nullptr) decay = hp[1], neg_lr = hp[2];
  __shared__ uint32_t tile[MUON_TILE][MUON_LDW];
  const RgptMuonTensor t = tab[blockIdx.z];
  const int r0 = blockIdx.y * MUON_TILE, c0 = blockIdx.x * MUON_TILE;
  const unsigned short* Xb = X + (long long)blockIdx.z * x_bstride;
  const bool x_vec = (ldx % 8 == 0) && (x_bstride % 8 == 0) && aligned16(X);
  const bool dst_vec = (C % 8 == 0) && aligned16(t.param) && (t.shadow == nullptr || aligned16(t.shadow));
  if (transpose) {
    // gather X[c][r0+8rg..+7] for columns c0+2cp, c0+2cp+1 into the shared [r][c] tile
    const int rg = threadIdx.x & 7, cp = threadIdx.x >> 3;
    const int r = r0 + rg * 8;
    const int n = min(8, R - r);
    float v[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + 2 * cp + h;
      if (c < C && n > 0) {
        load8_bf16(Xb + (long long)c * ldx + r, x_vec && n == 8, n, v[h]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[h][k] = 0.f;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[rg * 8 + k][cp] = pack_bf16x2(v[0][k], v[1][k]);
    __syncthreads();
  }
  const int cg = threadIdx.x & 7;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int rr = pass * 32 + (threadIdx.x >> 3);
    const int r = r0 + rr, c = c0 + cg * 8;
    const int n = r < R ? min(8, C - c) : 0;
    if (n <= 0) continue;
    float u[8];
    if (transpose) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(tile[rr][cg * 4 + j]);
        u[2 * j] = f.x, u[2 * j + 1] = f.y;
      }
    } else {
      load8_bf16(Xb + (long long)r * ldx + c, x_vec && n == 8, n, u);
    }
    const long long i = (long long)r * C + c;
    const bool vec = dst_vec && n == 8;
    float p[8];
    load8_f32(t.param + i, vec, n, p);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float uk = __bfloat162float(__float2bfloat16(u[k] * scale));  // upd.mul_(scale) in bf16
      float pk = p[k];
      if (decay != 1.0f) pk = __fmul_rn(pk, decay);
      p[k] = fmaf(neg_lr, uk, pk);
    }
    store8_f32(t.param + i, vec, n, p);
    if (t.shadow) store8_bf16(t.shadow + i, vec, n, p);
  }
}

// ---------------------------------------------------------------------------- fp32 Newton-Schulz
// Each fp32 value v is carried to the bf16 tensor cores as hi = bf16(v), lo = bf16(v - hi): v - hi is
// exact in fp32 and |v - hi - lo| <= 2^-18 |v|. A product X Y is hi*hi + hi*lo + lo*hi (the dropped lo*lo
// is ~2^-18 relative), summed in one GEMM whose K runs over the three stacked operand blocks.
constexpr int NS_TILE = 32;

__device__ __forceinline__ float ns_load(const void* src, int src_bf16, long long off) {
  return src_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[off])
                  : reinterpret_cast<const float*>(src)[off];
}

// sumsq[b] += sum of squares of matrix b; the unit-stride dimension is walked by consecutive threads.
__global__ void __launch_bounds__(256) ns_sumsq_kernel(const void* __restrict__ src, int src_bf16, long long s_b,
                                                       long long s_i, long long s_j, int rows, int cols,
                                                       float* __restrict__ sumsq) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[8];
  const int b = blockIdx.y;
  const bool j_fast = s_j == 1;
  const int inner = j_fast ? cols : rows, outer = j_fast ? rows : cols;
  const long long s_in = j_fast ? s_j : s_i, s_out = j_fast ? s_i : s_j;
  float ss = 0.f;
  for (int o = blockIdx.x; o < outer; o += gridDim.x) {
    const long long base = (long long)b * s_b + (long long)o * s_out;
    for (int in = threadIdx.x; in < inner; in += blockDim.x) {
      const float v = ns_load(src, src_bf16, base + (long long)in * s_in);
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    atomicAdd(&sumsq[b], t);
  }
}

// One 32 x 32 tile of matrix blockIdx.z per block of 32 x 8 threads. The tile is read along the
// source's unit-stride dimension (so a transposed view reads coalesced), turned in shared memory,
// and written along rows: the fp32 copy and the nblk hi/lo blocks.
__global__ void __launch_bounds__(256) ns_split_kernel(const void* __restrict__ src, int src_bf16, long long s_b,
                                                       long long s_i, long long s_j, int rows, int cols,
                                                       const float* __restrict__ sumsq, float* __restrict__ xout,
                                                       long long o_bstride, long long ldo,
                                                       __nv_bfloat16* __restrict__ dst, long long d_bstride,
                                                       long long ldd, int nblk, long long blk_off,
                                                       unsigned lo_mask) {
  griddep_wait();
  griddep_launch();
  __shared__ float tile[NS_TILE][NS_TILE + 1];
  const int b = blockIdx.z, i0 = blockIdx.y * NS_TILE, j0 = blockIdx.x * NS_TILE;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long sb = (long long)b * s_b;
  if (s_i == 1 && s_j != 1) {  // column-major source: consecutive threads walk i
    for (int c = ty; c < NS_TILE; c += 8) {
      const int i = i0 + tx, j = j0 + c;
      tile[tx][c] = (i < rows && j < cols) ? ns_load(src, src_bf16, sb + i + (long long)j * s_j) : 0.f;
    }
  } else {
    for (int r = ty; r < NS_TILE; r += 8) {
      const int i = i0 + r, j = j0 + tx;
      tile[r][tx] = (i < rows && j < cols) ? ns_load(src, src_bf16, sb + (long long)i * s_i + (long long)j * s_j)
                                           : 0.f;
    }
  }
  __syncthreads();
  const float den = sumsq != nullptr ? fmaxf(sqrtf(sumsq[b]), 1e-7f) : 1.0f;
  for (int r = ty; r < NS_TILE; r += 8) {
    const int i = i0 + r, j = j0 + tx;
    if (i >= rows || j >= cols) continue;
    const float v = sumsq != nullptr ? __fdiv_rn(tile[r][tx], den) : tile[r][tx];
    if (xout != nullptr) xout[(long long)b * o_bstride + (long long)i * ldo + j] = v;
    if (dst != nullptr) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
      __nv_bfloat16* d = dst + (long long)b * d_bstride + (long long)i * ldd + j;
      for (int k = 0; k < nblk; ++k) d[(long long)k * blk_off] = ((lo_mask >> k) & 1u) ? lo : hi;
    }
  }
}

// ============================================================================ data-parallel staging
// Copies between per-segment tensors and one packed buffer: the staging of the sharded data-parallel
// optimizer step (gradients packed owner-major for a reduce-scatter, averaged gradients unpacked into
// the owner's gradient slots, updated parameters packed for an all-gather and unpacked everywhere).
// One block per chunk of `chunk_elems` elements of one segment; the cast and the scale are the only
// arithmetic. Pack: buf[off + i] = cast(scale * t[i]). Unpack: t[i] = cast(scale * buf[off + i]) and,
// when the segment has one, t2[i] = bf16(t[i]) (the parameter's bf16 GEMM copy).
__device__ __forceinline__ float seg_load(const void* p, long long i, int bf) {
  return bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void seg_store(void* p, long long i, int bf, float v) {
  if (bf)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__global__ void segment_copy_kernel(const RgptSegment* __restrict__ tab, const int* __restrict__ chunk_seg,
                                    const long long* __restrict__ chunk_start, int n_chunks, int chunk_elems,
                                    void* __restrict__ buf, int buf_bf16, int tensor_bf16, float scale, int unpack) {
  griddep_wait();
  griddep_launch();
  for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const RgptSegment sg = tab[chunk_seg[c]];
    const long long start = chunk_start[c];
    const long long end = min(start + (long long)chunk_elems, sg.n);
    for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
      if (unpack) {
        const float v = scale * seg_load(buf, sg.buf_off + i, buf_bf16);
        seg_store(sg.t, i, tensor_bf16, v);
        if (sg.t2) reinterpret_cast<__nv_bfloat16*>(sg.t2)[i] = __float2bfloat16_rn(v);
      } else {
        seg_store(buf, sg.buf_off + i, buf_bf16, scale * seg_load(sg.t, i, tensor_bf16));
      }
    }
  }
}

}  // namespace rgpt

using namespace rgpt;

extern "C" int rgpt_adamw(const RgptAdamwTensor* table, const int* chunk_tensor, const long long* chunk_start,
                          int n_chunks, int chunk_elems, float lr, float wd, float beta1, float beta2, float eps,
                          int step, const float* hp, void* stream) {
  if (n_chunks <= 0) return RGPT_OK;
  float inv_bc1 = 0.f, inv_sqrt_bc2 = 0.f;
  if (hp == nullptr) {  // else the bias corrections come from the device block
    if (step < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "adamw step must be >= 1");
    const double bc1 = 1.0 - pow((double)beta1, (double)step);
    const double bc2 = 1.0 - pow((double)beta2, (double)step);
    inv_bc1 = (float)(1.0 / bc1);
    inv_sqrt_bc2 = (float)(1.0 / sqrt(bc2));
  }
  launch_pdl(adamw_kernel, dim3(n_chunks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      table, chunk_tensor, chunk_start, chunk_elems, lr, wd, beta1, beta2, eps, inv_bc1, inv_sqrt_bc2, hp);
  return rgpt_check_launch("adamw_kernel");
}

extern "C" int rgpt_muon_prep(const RgptMuonTensor* table, int n, int R, int C, void* X, long long x_bstride, int ldx,
                              float beta, int nesterov, float* sumsq, const float* hp, void* stream) {
  const int transpose = R > C ? 1 : 0;
  const int xc = transpose ? R : C;
  if (ldx < xc) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "NS stack too narrow (ldx %d < %d)", ldx, xc);
  dim3 grid((C + MUON_TILE - 1) / MUON_TILE, (R + MUON_TILE - 1) / MUON_TILE, n);
  launch_pdl(muon_prep_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      table, R, C, transpose, reinterpret_cast<unsigned short*>(X), x_bstride, ldx, beta, nesterov, sumsq, hp);
  return rgpt_check_launch("muon_prep_kernel");
}

extern "C" int rgpt_ns_scale(void* X, long long x_bstride, int ldx, int rows, int cols, int n, const float* sumsq,
                             void* stream) {
  if (ldx < cols) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_scale: ldx %d < cols %d", ldx, cols);
  const int gx = rows < 256 ? rows : 256;
  launch_pdl(ns_scale_kernel, dim3(dim3(gx, n)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      reinterpret_cast<__nv_bfloat16*>(X), x_bstride, ldx, rows, cols, sumsq);
  return rgpt_check_launch("ns_scale_kernel");
}

extern "C" int rgpt_muon_apply(const RgptMuonTensor* table, int n, int R, int C, const void* X, long long x_bstride,
                               int ldx, float lr, float wd, float muon_lr, float scale, const float* hp,
                               void* stream) {
  const int transpose = R > C ? 1 : 0;
  dim3 grid((C + MUON_TILE - 1) / MUON_TILE, (R + MUON_TILE - 1) / MUON_TILE, n);
  launch_pdl(muon_apply_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      table, R, C, transpose, reinterpret_cast<const unsigned short*>(X), x_bstride, ldx, 1.0f - lr * wd, -muon_lr,
      scale, hp);
  return rgpt_check_launch("muon_apply_kernel");
}

extern "C" int rgpt_ns_sumsq(const void* src, int src_bf16, long long s_b, long long s_i, long long s_j, int rows,
                             int cols, int n, float* sumsq, void* stream) {
  if (rows < 1 || cols < 1 || n < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_sumsq: empty matrix stack");
  if (s_i != 1 && s_j != 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_sumsq: source needs a unit stride");
  if (src == nullptr || sumsq == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_sumsq: null pointer");
  const int outer = s_j == 1 ? rows : cols;
  const int gx = outer < 128 ? outer : 128;
  launch_pdl(ns_sumsq_kernel, dim3(gx, n), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, src, src_bf16,
             s_b, s_i, s_j, rows, cols, sumsq);
  return rgpt_check_launch("ns_sumsq_kernel");
}

extern "C" int rgpt_ns_split(const void* src, int src_bf16, long long s_b, long long s_i, long long s_j, int rows,
                             int cols, int n, const float* sumsq, float* xout, long long o_bstride, long long ldo,
                             void* dst, long long d_bstride, long long ldd, int nblk, long long blk_off,
                             unsigned lo_mask, void* stream) {
  if (rows < 1 || cols < 1 || n < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: empty matrix stack");
  if (src == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: null source");
  if (s_i != 1 && s_j != 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: source needs a unit stride");
  if (xout != nullptr && ldo < cols) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: ldo %lld < cols %d", ldo, cols);
  if (dst != nullptr && (ldd < cols || nblk < 1 || nblk > 32))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: ldd %lld / nblk %d invalid", ldd, nblk);
  if (rows > 65535 * NS_TILE) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_split: %d rows", rows);
  dim3 grid((cols + NS_TILE - 1) / NS_TILE, (rows + NS_TILE - 1) / NS_TILE, n);
  launch_pdl(ns_split_kernel, grid, dim3(NS_TILE, 8), 0, reinterpret_cast<cudaStream_t>(stream), 1, src, src_bf16,
             s_b, s_i, s_j, rows, cols, sumsq, xout, o_bstride, ldo, reinterpret_cast<__nv_bfloat16*>(dst),
             d_bstride, ldd, dst != nullptr ? nblk : 0, blk_off, lo_mask);
  return rgpt_check_launch("ns_split_kernel");
}

extern "C" int rgpt_segment_copy(const RgptSegment* table, const int* chunk_seg, const long long* chunk_start,
                                 int n_chunks, int chunk_elems, void* buf, int buf_bf16, int tensor_bf16, float scale,
                                 int unpack, void* stream) {
  if (n_chunks <= 0) return RGPT_OK;
  if (chunk_elems < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "segment_copy: chunk_elems must be >= 1");
  int dev = 0;
  cudaGetDevice(&dev);
  const int cap = 8 * rgpt_num_sms(dev);
  launch_pdl(segment_copy_kernel, dim3(n_chunks < cap ? n_chunks : cap), dim3(256), 0,
             reinterpret_cast<cudaStream_t>(stream), 1, table, chunk_seg, chunk_start, n_chunks, chunk_elems, buf,
             buf_bf16 ? 1 : 0, tensor_bf16 ? 1 : 0, scale, unpack ? 1 : 0);
  return rgpt_check_launch("segment_copy_kernel");
}
