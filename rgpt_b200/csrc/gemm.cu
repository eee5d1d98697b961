// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   D[b][m, n] = epilogue( sum_k A[b](m, k) * B[b](n, k) )
//
// A(m, k) is stored K-major (A[m*lda + k]) or MN-major (A[k*lda + m]); the same
// for B(n, k). Every GEMM of the rGPT training step maps onto this one kernel:
// forward projections are K-major/K-major, dX = dY*W uses an MN-major B, and
// dW = dY^T*X uses MN-major A and B, so no operand is ever transposed in HBM.
//
// CTA layout (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128-byte-swizzled tiles into a STAGES-deep smem ring
//   warp 1      allocates TMEM, issues tcgen05.mma (one elected thread), commits
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator (each thread owns one
//               row), apply the fused epilogue, store to HBM
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of
// tile i overlaps the main loop of tile i+1.
//
// Epilogues fuse what the reference runs as separate torch ops:
//   ACT_FWD   pre = acc, post = act(acc)          (model/kernels.py:127-200)
//   ACT_BWD   dpre = acc * act'(pre)              (model/kernels.py:207-281)
//   RESID_F32 x_out = x_in + acc * layer_scale    (model/transformer_block.py:43-57)
//   POLY_BF16 beta*C + alpha*acc                  (optimizer.py:36-41, Newton-Schulz)
//   ACCUM_F32 grad += acc (split-K via fp32 vector atomics)
#include <cudaTypedefs.h>
#include <stdio.h>

#include "act.cuh"
#include "common.cuh"
#include "rgpt.h"

namespace rgpt {

struct GemmShape {
  int M, N, K, batch;
  int m_tiles, n_tiles, splitk, kb_per_split, num_kb;
  int num_units;
};

struct EpiParams {
  int kind, act;
  float alpha, beta;
  void* d;
  long long ldd, d_bstride;
  void* d2;
  long long ldd2, d2_bstride;
  const void* c;
  long long ldc, c_bstride;
  const float* colscale;
  const float* alpha_dev;  // optional device scalar multiplying alpha (loss-gradient scale)
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr uint32_t B_BYTES = BN * GEMM_BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t BAR_BYTES = 256;
  static constexpr uint32_t TOTAL = STAGES * STAGE_BYTES + BAR_BYTES + 1024;  // +1024 alignment slack
};

__device__ __forceinline__ void decode_unit(int u, const GemmShape& sh, int& b, int& mt, int& nt, int& ks) {
  ks = u % sh.splitk;
  u /= sh.splitk;
  mt = u % sh.m_tiles;
  u /= sh.m_tiles;
  nt = u % sh.n_tiles;
  b = u / sh.n_tiles;
}

// Apply the epilogue to 32 consecutive accumulator columns of one row.
__device__ __forceinline__ void epilogue_chunk(const EpiParams& ep, const GemmShape& sh, int b, int gm, int gn0,
                                               const uint32_t (&r)[32]) {
  float v[32];
  const float alpha = ep.alpha_dev ? ep.alpha * __ldg(ep.alpha_dev) : ep.alpha;
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * alpha;
  const bool full = (gn0 + 32 <= sh.N);
  const int ncols = full ? 32 : (sh.N - gn0);

  switch (ep.kind) {
    case RGPT_EPI_STORE_BF16: {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (full) {
        uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 o;
          o.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
          o.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
          o.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
          o.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
          d4[q] = o;
        }
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = __float2bfloat16(v[j]);
      }
      break;
    }
    case RGPT_EPI_STORE_F32: {
      float* d = reinterpret_cast<float*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (full) {
        float4* d4 = reinterpret_cast<float4*>(d);
#pragma unroll
        for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = v[j];
      }
      break;
    }
    case RGPT_EPI_ACCUM_F32: {
      float* d = reinterpret_cast<float*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (sh.splitk > 1) {
        if (full) {
          float4* d4 = reinterpret_cast<float4*>(d);
#pragma unroll
          for (int q = 0; q < 8; ++q) atomicAdd(d4 + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
        } else {
          for (int j = 0; j < ncols; ++j) atomicAdd(d + j, v[j]);
        }
      } else {
        if (full) {
          float4* d4 = reinterpret_cast<float4*>(d);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 o = d4[q];
            o.x += v[4 * q];
            o.y += v[4 * q + 1];
            o.z += v[4 * q + 2];
            o.w += v[4 * q + 3];
            d4[q] = o;
          }
        } else {
          for (int j = 0; j < ncols; ++j) d[j] += v[j];
        }
      }
      break;
    }
    case RGPT_EPI_ACT_FWD: {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      __nv_bfloat16* d2 =
          reinterpret_cast<__nv_bfloat16*>(ep.d2) + b * ep.d2_bstride + (long long)gm * ep.ldd2 + gn0;
      if (full) {
        uint4* p4 = reinterpret_cast<uint4*>(d);
        uint4* q4 = reinterpret_cast<uint4*>(d2);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 o, a;
          o.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
          o.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
          o.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
          o.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
          a.x = pack_bf16x2(act_fwd(ep.act, v[8 * q + 0]), act_fwd(ep.act, v[8 * q + 1]));
          a.y = pack_bf16x2(act_fwd(ep.act, v[8 * q + 2]), act_fwd(ep.act, v[8 * q + 3]));
          a.z = pack_bf16x2(act_fwd(ep.act, v[8 * q + 4]), act_fwd(ep.act, v[8 * q + 5]));
          a.w = pack_bf16x2(act_fwd(ep.act, v[8 * q + 6]), act_fwd(ep.act, v[8 * q + 7]));
          p4[q] = o;
          q4[q] = a;
        }
      } else {
        for (int j = 0; j < ncols; ++j) {
          d[j] = __float2bfloat16(v[j]);
          d2[j] = __float2bfloat16(act_fwd(ep.act, v[j]));
        }
      }
      break;
    }
    case RGPT_EPI_ACT_BWD: {
      const __nv_bfloat16* c =
          reinterpret_cast<const __nv_bfloat16*>(ep.c) + b * ep.c_bstride + (long long)gm * ep.ldc + gn0;
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (full) {
        const uint4* c4 = reinterpret_cast<const uint4*>(c);
        uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pc = c4[q];
          uint32_t pw[4] = {pc.x, pc.y, pc.z, pc.w};
          uint32_t ow[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float2 pre = unpack_bf16x2(pw[h]);
            ow[h] = pack_bf16x2(v[8 * q + 2 * h] * act_grad(ep.act, pre.x),
                                v[8 * q + 2 * h + 1] * act_grad(ep.act, pre.y));
          }
          d4[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = __float2bfloat16(v[j] * act_grad(ep.act, __bfloat162float(c[j])));
      }
      break;
    }
    case RGPT_EPI_RESID_F32: {
      const float* c = reinterpret_cast<const float*>(ep.c) + b * ep.c_bstride + (long long)gm * ep.ldc + gn0;
      float* d = reinterpret_cast<float*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (ep.d2 != nullptr) {  // raw branch output (before scale and residual), for the layer-scale gradient
        float* d2 = reinterpret_cast<float*>(ep.d2) + b * ep.d2_bstride + (long long)gm * ep.ldd2 + gn0;
        if (full) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(d2)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
          for (int j = 0; j < ncols; ++j) d2[j] = v[j];
        }
      }
      if (full) {
        const float4* c4 = reinterpret_cast<const float4*>(c);
        float4* d4 = reinterpret_cast<float4*>(d);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 x = c4[q];
          float4 s = ep.colscale ? reinterpret_cast<const float4*>(ep.colscale + gn0)[q] : make_float4(1.f, 1.f, 1.f, 1.f);
          x.x += v[4 * q] * s.x;
          x.y += v[4 * q + 1] * s.y;
          x.z += v[4 * q + 2] * s.z;
          x.w += v[4 * q + 3] * s.w;
          d4[q] = x;
        }
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = c[j] + v[j] * (ep.colscale ? ep.colscale[gn0 + j] : 1.0f);
      }
      break;
    }
    case RGPT_EPI_POLY_BF16: {
      const __nv_bfloat16* c =
          reinterpret_cast<const __nv_bfloat16*>(ep.c) + b * ep.c_bstride + (long long)gm * ep.ldc + gn0;
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      if (full) {
        const uint4* c4 = reinterpret_cast<const uint4*>(c);
        uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pc = c4[q];
          uint32_t pw[4] = {pc.x, pc.y, pc.z, pc.w};
          uint32_t ow[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float2 cv = unpack_bf16x2(pw[h]);
            ow[h] = pack_bf16x2(ep.beta * cv.x + v[8 * q + 2 * h], ep.beta * cv.y + v[8 * q + 2 * h + 1]);
          }
          d4[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = __float2bfloat16(ep.beta * __bfloat162float(c[j]) + v[j]);
      }
      break;
    }
    case RGPT_EPI_BIAS_SIGMOID_BF16: {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + b * ep.d_bstride + (long long)gm * ep.ldd + gn0;
      const float* bias = ep.colscale + gn0;
      if (full) {
        uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] = 1.0f / (1.0f + expf(-(v[8 * q + e] + bias[8 * q + e])));
          d4[q] = make_uint4(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]), pack_bf16x2(g[4], g[5]),
                             pack_bf16x2(g[6], g[7]));
        }
      } else {
        for (int j = 0; j < ncols; ++j) d[j] = __float2bfloat16(1.0f / (1.0f + expf(-(v[j] + bias[j]))));
      }
      break;
    }
    default:
      break;
  }
}

template <int BN, int STAGES, int A_MN, int B_MN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmShape sh, EpiParams ep) {
  using L = GemmSmem<BN, STAGES>;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = make_idesc_bf16(GEMM_BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + STAGES * L::B_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < sh.num_units && ok; u += gridDim.x) {
        int b, mt, nt, ks;
        decode_unit(u, sh, b, mt, nt, ks);
        const int kb0 = ks * sh.kb_per_split;
        const int kb1 = min(kb0 + sh.kb_per_split, sh.num_kb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // MN-major operands arrive as 64-wide sub-boxes; a sub-box lying wholly past M (or N)
          // is not loaded: its smem only feeds output rows/columns the epilogue never stores.
          const int a_sub = A_MN ? min(GEMM_BM / 64, (sh.M - mt * GEMM_BM + 63) / 64) : 1;
          const int b_sub = B_MN ? min(BN / 64, (sh.N - nt * BN + 63) / 64) : 1;
          const uint32_t bytes = (A_MN ? a_sub * (64 * GEMM_BK * 2) : L::A_BYTES) +
                                 (B_MN ? b_sub * (64 * GEMM_BK * 2) : L::B_BYTES);
          mbar_arrive_expect_tx(&full_bar[stage], bytes);
          const int k0 = kb * GEMM_BK;
          uint8_t* a_dst = sA + stage * L::A_BYTES;
          uint8_t* b_dst = sB + stage * L::B_BYTES;
          if (A_MN) {
            for (int i = 0; i < a_sub; ++i)
              tma_load_3d(a_dst + i * (64 * GEMM_BK * 2), &tmA, &full_bar[stage], mt * GEMM_BM + i * 64, k0, b);
          } else {
            tma_load_3d(a_dst, &tmA, &full_bar[stage], k0, mt * GEMM_BM, b);
          }
          if (B_MN) {
            for (int i = 0; i < b_sub; ++i)
              tma_load_3d(b_dst + i * (64 * GEMM_BK * 2), &tmB, &full_bar[stage], nt * BN + i * 64, k0, b);
          } else {
            tma_load_3d(b_dst, &tmB, &full_bar[stage], k0, nt * BN, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for every load already issued into the ring.
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full_bar[s], phase, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < sh.num_units && ok; u += gridDim.x) {
        int b, mt, nt, ks;
        decode_unit(u, sh, b, mt, nt, ks);
        const int kb0 = ks * sh.kb_per_split;
        const int kb1 = min(kb0 + sh.kb_per_split, sh.num_kb);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * L::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * L::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            const uint64_t adesc = A_MN ? make_sw128_desc(a_addr + kk * 2048, 64 * GEMM_BK * 2, 1024)
                                        : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sw128_desc(b_addr + kk * 2048, 64 * GEMM_BK * 2, 1024)
                                        : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            umma_bf16(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int quarter = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < sh.num_units; u += gridDim.x) {
      int b, mt, nt, ks;
      decode_unit(u, sh, b, mt, nt, ks);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int gm = mt * GEMM_BM + row;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(t_row + c0, r);
        tmem_wait_ld();
        const int gn0 = nt * BN + c0;
        if (gm < sh.M && gn0 < sh.N) epilogue_chunk(ep, sh, b, gm, gn0, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D bf16 tensor map (inner, outer, batch) with a 128-byte swizzle.
int make_tmap_bf16_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch,
                      uint64_t ld_elems, uint64_t bstride_elems, uint32_t box_inner, uint32_t box_outer) {
  auto enc = get_encode_fn();
  if (enc == nullptr) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "TMA base pointer %p is not 16-byte aligned", ptr);
  if (batch <= 1) bstride_elems = ld_elems * outer;
  if ((ld_elems * 2) % 16 != 0 || (bstride_elems * 2) % 16 != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "TMA strides must be multiples of 16 bytes (ld=%llu, bstride=%llu)",
                          (unsigned long long)ld_elems, (unsigned long long)bstride_elems);
  cuuint64_t dims[3] = {inner, outer, batch < 1 ? 1 : batch};
  cuuint64_t strides[2] = {ld_elems * 2, bstride_elems * 2};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return RGPT_OK;
}

template <int BN, int STAGES, int A_MN, int B_MN>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmShape& sh, const EpiParams& ep,
                       int grid, cudaStream_t stream) {
  auto kern = gemm_bf16_tc_kernel<BN, STAGES, A_MN, B_MN>;
  constexpr uint32_t smem = GemmSmem<BN, STAGES>::TOTAL;
  static bool attr_set = false;  // per process; attribute applies to every device context
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return rgpt_check_launch("gemm set smem attribute");
    attr_set = true;
  }
  kern<<<grid, GEMM_THREADS, smem, stream>>>(ta, tb, sh, ep);
  return rgpt_check_launch("gemm_bf16_tc_kernel");
}

}  // namespace rgpt

using namespace rgpt;

extern "C" int rgpt_gemm_bf16(const void* A, int a_mn_major, long long lda, long long a_bstride, const void* B,
                              int b_mn_major, long long ldb, long long b_bstride, int M, int N, int K, int batch,
                              int epi, int act, float alpha, float beta, void* D, long long ldd, long long d_bstride,
                              void* D2, long long ldd2, long long d2_bstride, const void* C, long long ldc,
                              long long c_bstride, const float* colscale, int splitk, const float* alpha_dev, void* stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int st = rgpt_check_device(dev);
  if (st) return st;
  if (batch < 1) batch = 1;
  if (M < 1 || N < 1 || K < 1)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "gemm needs M, N, K >= 1 (got M=%d N=%d K=%d)", M, N, K);
  if (epi < RGPT_EPI_STORE_BF16 || epi > RGPT_EPI_BIAS_SIGMOID_BF16)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown epilogue %d", epi);
  if (D == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "gemm output pointer is null");
  const bool out_f32 = (epi == RGPT_EPI_STORE_F32 || epi == RGPT_EPI_ACCUM_F32 || epi == RGPT_EPI_RESID_F32);
  const int vec = out_f32 ? 4 : 8;
  if (ldd % vec != 0 || (reinterpret_cast<uintptr_t>(D) & 15) != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "output leading dim / pointer not 16-byte aligned");
  if (epi == RGPT_EPI_ACT_FWD && (D2 == nullptr || ldd2 % 8 != 0 || (reinterpret_cast<uintptr_t>(D2) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "ACT_FWD needs an aligned second output");
  if (epi == RGPT_EPI_RESID_F32 && D2 != nullptr && (ldd2 % 4 != 0 || (reinterpret_cast<uintptr_t>(D2) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "RESID_F32 raw output must be 16-byte aligned");
  if ((epi == RGPT_EPI_ACT_BWD || epi == RGPT_EPI_RESID_F32 || epi == RGPT_EPI_POLY_BF16) &&
      (C == nullptr || ldc % vec != 0 || (reinterpret_cast<uintptr_t>(C) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "epilogue input C missing or not 16-byte aligned");
  if (epi == RGPT_EPI_BIAS_SIGMOID_BF16 && colscale == nullptr)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "BIAS_SIGMOID needs the bias vector (colscale)");
  if (colscale != nullptr && (reinterpret_cast<uintptr_t>(colscale) & 15) != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "colscale must be 16-byte aligned");

  const int BN = (N > 128) ? 256 : 128;
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K = K;
  sh.batch = batch;
  sh.m_tiles = (M + GEMM_BM - 1) / GEMM_BM;
  sh.n_tiles = (N + BN - 1) / BN;
  sh.num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  const int nsm = rgpt_num_sms(dev);
  const int tiles = batch * sh.m_tiles * sh.n_tiles;
  if (splitk <= 0) {
    splitk = 1;
    if (epi == RGPT_EPI_ACCUM_F32 && tiles < nsm) {
      splitk = (nsm + tiles - 1) / tiles;
      int max_split = sh.num_kb / 4 > 0 ? sh.num_kb / 4 : 1;  // keep >= 4 k-blocks per split
      if (splitk > max_split) splitk = max_split;
    }
  }
  if (splitk > 1 && epi != RGPT_EPI_ACCUM_F32)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "split-K is only valid with the ACCUM_F32 epilogue");
  if (splitk > sh.num_kb) splitk = sh.num_kb;
  sh.kb_per_split = (sh.num_kb + splitk - 1) / splitk;
  sh.splitk = (sh.num_kb + sh.kb_per_split - 1) / sh.kb_per_split;  // no empty splits
  sh.num_units = tiles * sh.splitk;

  // Tensor maps. K-major: (inner=K, outer=rows); MN-major: (inner=rows, outer=K).
  CUtensorMap ta, tb;
  if (a_mn_major)
    st = make_tmap_bf16_3d(&ta, A, M, K, batch, lda, a_bstride, 64, GEMM_BK);
  else
    st = make_tmap_bf16_3d(&ta, A, K, M, batch, lda, a_bstride, GEMM_BK, GEMM_BM);
  if (st) return st;
  if (b_mn_major)
    st = make_tmap_bf16_3d(&tb, B, N, K, batch, ldb, b_bstride, 64, GEMM_BK);
  else
    st = make_tmap_bf16_3d(&tb, B, K, N, batch, ldb, b_bstride, GEMM_BK, BN);
  if (st) return st;

  EpiParams ep;
  ep.kind = epi;
  ep.act = act;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.d = D;
  ep.ldd = ldd;
  ep.d_bstride = d_bstride;
  ep.d2 = D2;
  ep.ldd2 = ldd2;
  ep.d2_bstride = d2_bstride;
  ep.c = C;
  ep.ldc = ldc;
  ep.c_bstride = c_bstride;
  ep.colscale = colscale;
  ep.alpha_dev = alpha_dev;

  const int grid = sh.num_units < nsm ? sh.num_units : nsm;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int key = (BN == 256 ? 4 : 0) | (a_mn_major ? 2 : 0) | (b_mn_major ? 1 : 0);
  switch (key) {
    case 0: return launch_gemm<128, 6, 0, 0>(ta, tb, sh, ep, grid, s);
    case 1: return launch_gemm<128, 6, 0, 1>(ta, tb, sh, ep, grid, s);
    case 2: return launch_gemm<128, 6, 1, 0>(ta, tb, sh, ep, grid, s);
    case 3: return launch_gemm<128, 6, 1, 1>(ta, tb, sh, ep, grid, s);
    case 4: return launch_gemm<256, 4, 0, 0>(ta, tb, sh, ep, grid, s);
    case 5: return launch_gemm<256, 4, 0, 1>(ta, tb, sh, ep, grid, s);
    case 6: return launch_gemm<256, 4, 1, 0>(ta, tb, sh, ep, grid, s);
    default: return launch_gemm<256, 4, 1, 1>(ta, tb, sh, ep, grid, s);
  }
}
