// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   D[b][m, n] = epilogue( sum_k A[b](m, k) * B[b](n, k) )
//
// A(m, k) is stored K-major (A[m*lda + k]) or MN-major (A[k*lda + m]); the same
// for B(n, k). Every GEMM of the rGPT training step maps onto this one kernel:
// forward projections are K-major/K-major, dX = dY*W uses an MN-major B, and
// dW = dY^T*X uses MN-major A and B, so no operand is ever transposed in HBM.
//
// CTA layout (64 + 32 * EW threads, EW = 4 or 8 epilogue warps; one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: 128-byte-swizzled tiles into a STAGES-deep smem ring
//   warp 1      allocates TMEM, issues tcgen05.mma (one elected thread), commits
//   warps 2..   epilogue: warp w owns TMEM lane quadrant w % 4 (32 accumulator rows) and,
//               with 8 epilogue warps, half of the tile's columns; per column chunk it
//               tcgen05.ld's the fp32 accumulator, applies the fused epilogue (an input C
//               is read by each thread for its own row with 16-byte loads, one chunk ahead),
//               stages the result in swizzled smem and writes it with a TMA bulk store (or a
//               TMA bulk reduce-add for accumulating outputs)
// Large GEMMs run on CTA pairs (a cluster of two SMs): one cta_group::2 MMA computes a
// 256 x 256 tile from 128 rows of A and 128 rows of B staged in each SM's shared memory,
// which halves the B operand's shared-memory and L2 traffic per SM.
// The accumulator is multi-buffered in TMEM (512 / BN buffers of BN columns) so the
// epilogue of tile i overlaps the main loops of the tiles after it. Tiles are visited in groups of
// GROUP_M row tiles so that consecutive CTAs share A and B panels in L2.
//
// Epilogues fuse what the reference runs as separate torch ops:
//   ACT_FWD      pre = acc, post = act(acc)          (model/kernels.py:127-200); post only for ACT_SQRELU_POST
//   ACT_BWD      dpre = acc * act'(pre)              (model/kernels.py:207-281)
//   RESID_F32    x_out = x_in + acc * layer_scale    (model/transformer_block.py:43-57)
//   POLY_BF16    beta*C + alpha*acc                  (optimizer.py:36-41, Newton-Schulz)
//   POLY_F32     the same in fp32 (C and D fp32)     (fp32 Newton-Schulz on split bf16 operands)
//   ARGMAX_BF16  per row and column tile: the first maximum of bf16(acc) and its column; no output
//                matrix (the rGPT per-step lm_head argmax, model/gpt.py:119-120)
//   BIAS_SIGMOID sigmoid(acc + bias)                 (model/attention.py:45-48, G1 gate)
//   ACCUM_F32    grad += acc (bulk reduce-add, so split-K needs no separate reduction)
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
  int group_m;  // row tiles per visiting group (see decode_unit)
};

struct EpiParams {
  int kind, act;
  float alpha, beta;
  const void* c;
  long long ldc, c_bstride;
  const float* colscale;
  const float* alpha_dev;  // optional device scalar multiplying alpha (loss-gradient scale)
  int has_d2;
  // RESID_F32 only: dropout of the branch output (nn.Dropout, model/transformer_block.py:45,52).
  // Null mask = no dropout; else the keep bit of (row, column) is bit column % 32 of
  // drop_mask[row * drop_ldm + column / 32] (filled beforehand by rgpt_drop_mask).
  const uint32_t* drop_mask;
  long long drop_ldm;
  float drop_scale;
  // ARGMAX_BF16 only: per (row, column tile) maximum and its column, [M, amax_ld]
  float* amax_val;
  int* amax_idx;
  long long amax_ld;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
// Epilogue warps per CTA (EW): 4 = one per TMEM lane quadrant; 8 = two per quadrant, each taking half
// of the tile's columns, for the epilogues that read an input C (their per-chunk work is the longest),
// so that two warps per SM sub-partition hide each other's latency (measured 2-5 % faster there;
// the two-output activation forward measured slower with 8).
__host__ __device__ constexpr int gemm_epi_warps(int epi) {
  return (epi == RGPT_EPI_ACT_BWD || epi == RGPT_EPI_POLY_BF16 || epi == RGPT_EPI_RESID_F32 ||
          epi == RGPT_EPI_POLY_F32) ? 8 : 4;
}
__host__ __device__ constexpr int gemm_threads(int ew) { return 64 + 32 * ew; }
constexpr int GROUP_M = 8;
constexpr uint32_t EPI_STAGE_BYTES = 4096;  // one warp's 32 rows x 128 bytes

__host__ __device__ constexpr bool epi_reads_c(int epi) {
  return epi == RGPT_EPI_ACT_BWD || epi == RGPT_EPI_POLY_BF16 || epi == RGPT_EPI_RESID_F32 ||
         epi == RGPT_EPI_POLY_F32;
}
// bytes per element of the epilogue input C: bf16 for ACT_BWD / POLY_BF16, fp32 for RESID / POLY_F32
__host__ __device__ constexpr int epi_c_bytes(int epi) {
  return (epi == RGPT_EPI_RESID_F32 || epi == RGPT_EPI_POLY_F32) ? 4 : 2;
}

template <int BN, int STAGES, bool PAIR, int EW>
struct GemmSmem {
  static constexpr uint32_t A_BYTES = GEMM_BM * GEMM_BK * 2;              // this CTA's 128 rows of A
  static constexpr uint32_t B_BYTES = (PAIR ? BN / 2 : BN) * GEMM_BK * 2;  // a CTA pair splits B's rows
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t EPI_BYTES = EW * 2 * EPI_STAGE_BYTES;  // 2 staging buffers per epilogue warp
  static constexpr uint32_t BAR_BYTES = 512;
  static constexpr uint32_t TOTAL = STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES + 1024;  // +1024 alignment slack
};

// 16 bytes of global memory through L1 (the epilogue's C rows: a row's 128-byte chunk is read
// as 8 such loads, so the line's later 16-byte pieces hit L1).
__device__ __forceinline__ uint4 ld_global_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void decode_unit(int u, const GemmShape& sh, int& b, int& mt, int& nt, int& ks) {
  ks = u % sh.splitk;
  int t = u / sh.splitk;
  const int per_batch = sh.m_tiles * sh.n_tiles;
  b = t / per_batch;
  t %= per_batch;
  const int group_span = sh.group_m * sh.n_tiles;
  const int first_m = (t / group_span) * sh.group_m;
  const int gsize = min(sh.m_tiles - first_m, sh.group_m);
  const int r = t % group_span;
  mt = first_m + r % gsize;
  nt = r / gsize;
}

// ------------------------------------------------------------------ bulk stores
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_g() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Row `lane` of a 32-row x 128-byte staging tile, 16-byte chunk j, 128-byte swizzle.
__device__ __forceinline__ uint8_t* stage_ptr(uint8_t* buf, int lane, int j) {
  return buf + lane * 128 + ((j ^ (lane & 7)) << 4);
}
__device__ __forceinline__ void stage_f32x32(uint8_t* buf, int lane, const float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(stage_ptr(buf, lane, j)) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
__device__ __forceinline__ void stage_bf16x64(uint8_t* buf, int lane, const float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(stage_ptr(buf, lane, j)) =
        make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                   pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

// Activation applied to 32 values: forward (ACT_FWD) or derivative times v (ACT_BWD, c = pre).
template <int ACT>
__device__ __forceinline__ void act_fwd32(float* v) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = act_fwd_t<ACT>(v[j]);
}
template <int ACT>
__device__ __forceinline__ void act_bwd32(float* v, const uint4* c) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t w4[4] = {c[q].x, c[q].y, c[q].z, c[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 cv = unpack_bf16x2(w4[e]);
      v[8 * q + 2 * e] *= act_grad_t<ACT>(cv.x);
      v[8 * q + 2 * e + 1] *= act_grad_t<ACT>(cv.y);
    }
  }
}
template <int BN, int STAGES, int A_MN, int B_MN, int EPI, bool PAIR, int ACT>
__global__ void __launch_bounds__(gemm_threads(gemm_epi_warps(EPI)), 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD2,
                        GemmShape sh, EpiParams ep) {
  constexpr bool reads_c = epi_reads_c(EPI);
  constexpr int EW = gemm_epi_warps(EPI);
  using L = GemmSmem<BN, STAGES, PAIR, EW>;
  constexpr int NUM_ACC = 512 / BN;  // TMEM accumulator buffers (2 for 256-wide tiles, 4 for 128-wide)
  constexpr uint32_t TMEM_COLS = NUM_ACC * BN;
  constexpr int TILE_M = PAIR ? 2 * GEMM_BM : GEMM_BM;
  constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B this CTA loads
  constexpr uint32_t IDESC = make_idesc_bf16(TILE_M, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::A_BYTES;
  uint8_t* sEpi = sB + STAGES * L::B_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sEpi + L::EPI_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + NUM_ACC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;  // 0 = the CTA that issues the pair's MMAs
  const int first_unit = PAIR ? (int)cluster_id_x() : (int)blockIdx.x;
  const int unit_step = PAIR ? (int)cluster_count_x() : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], PAIR ? 2 * EW : EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // operands, C and the output come from / go to the previous kernels' memory
  // barriers of the pair's MMA-issuing CTA, as shared::cluster addresses
  const uint32_t full_bar0 = PAIR ? mapa_shared(smem_u32(full_bar), 0) : smem_u32(full_bar);
  const uint32_t tempty_bar0 = PAIR ? mapa_shared(smem_u32(tempty_bar), 0) : smem_u32(tempty_bar);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = first_unit; u < sh.num_units && ok; u += unit_step) {
        int b, mt, nt, ks;
        decode_unit(u, sh, b, mt, nt, ks);
        const int kb0 = ks * sh.kb_per_split;
        const int kb1 = min(kb0 + sh.kb_per_split, sh.num_kb);
        // MN-major operands arrive as 64-wide sub-boxes; a sub-box lying wholly past M (or N)
        // is not loaded: its smem only feeds output rows/columns the epilogue never stores.
        auto a_subs = [&](int rk) {
          return A_MN ? max(0, min(GEMM_BM / 64, (sh.M - mt * TILE_M - rk * GEMM_BM + 63) / 64)) : 1;
        };
        auto b_subs = [&](int rk) {
          return B_MN ? max(0, min(B_ROWS / 64, (sh.N - nt * BN - rk * B_ROWS + 63) / 64)) : 1;
        };
        auto stage_bytes = [&](int rk) -> uint32_t {
          return (A_MN ? a_subs(rk) * (64 * GEMM_BK * 2) : L::A_BYTES) +
                 (B_MN ? b_subs(rk) * (64 * GEMM_BK * 2) : L::B_BYTES);
        };
        const int a_sub = a_subs(rank), b_sub = b_subs(rank);
        const int a_row = mt * TILE_M + rank * GEMM_BM, b_row = nt * BN + rank * B_ROWS;
        const uint32_t expect = PAIR ? stage_bytes(0) + stage_bytes(1) : stage_bytes(0);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // the pair's barrier lives in CTA 0, which posts the byte count of both CTAs' loads
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], expect);
          const int k0 = kb * GEMM_BK;
          uint8_t* a_dst = sA + stage * L::A_BYTES;
          uint8_t* b_dst = sB + stage * L::B_BYTES;
          const uint32_t fb = full_bar0 + stage * 8;
          auto load = [&](uint8_t* dst, const CUtensorMap* map, int c0, int c1) {
            if constexpr (PAIR) tma_load_3d_pair(dst, map, fb, c0, c1, b);
            else tma_load_3d(dst, map, &full_bar[stage], c0, c1, b);
          };
          if (A_MN) {
            for (int i = 0; i < a_sub; ++i) load(a_dst + i * (64 * GEMM_BK * 2), &tmA, a_row + i * 64, k0);
          } else {
            load(a_dst, &tmA, k0, a_row);
          }
          if (B_MN) {
            for (int i = 0; i < b_sub; ++i) load(b_dst + i * (64 * GEMM_BK * 2), &tmB, b_row + i * 64, k0);
          } else {
            load(b_dst, &tmB, k0, b_row);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      griddep_launch();  // every load of this CTA is issued: the next kernel may start filling SMs
      if (!ok && rank == 0) {
        // Drain: wait (bounded) for every load already issued into the ring (the pair's loads
        // all complete on CTA 0's barriers; the final cluster barrier keeps CTA 1 alive meanwhile).
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full_bar[s], phase, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      // completion signals go to both CTAs of a pair (same smem offsets)
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(bar), 0));
          umma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          umma_commit(bar);
        }
      };
      for (int u = first_unit; u < sh.num_units && ok; u += unit_step) {
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
            if constexpr (PAIR) umma_bf16_pair(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            else umma_bf16(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        commit(&tfull_bar[acc]);
        if (++acc == NUM_ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int quarter = warp & 3;          // TMEM lane quadrant this warp may access
    const int col_half = (warp - 2) >> 2;  // which part of the tile's columns this warp writes
    constexpr int COLS = BN * 4 / EW;
    uint8_t* buf0 = sEpi + (warp - 2) * 2 * EPI_STAGE_BYTES;
    uint8_t* buf1 = buf0 + EPI_STAGE_BYTES;
    int which = 0;
    constexpr bool bf16_out = (EPI == RGPT_EPI_STORE_BF16 || EPI == RGPT_EPI_ACT_FWD || EPI == RGPT_EPI_ACT_BWD ||
                               EPI == RGPT_EPI_POLY_BF16 || EPI == RGPT_EPI_BIAS_SIGMOID_BF16);
    constexpr bool act_two_out = EPI == RGPT_EPI_ACT_FWD && ACT != ACT_SQRELU_POST;  // pre and post
    const bool dual = act_two_out || (EPI == RGPT_EPI_RESID_F32 && ep.has_d2);
    const float alpha = ep.alpha_dev ? ep.alpha * __ldg(ep.alpha_dev) : ep.alpha;
    const bool scaled = alpha != 1.0f;

    int acc = 0;
    uint32_t acc_phase = 0;
    // Epilogue input C (bf16 for ACT_BWD / POLY, fp32 for RESID): each thread reads its own output
    // row's 128 bytes of every column chunk straight from global memory as eight 16-byte loads
    // (the line's later pieces hit L1). The next chunk's loads are issued before the current chunk
    // is processed, and a tile's first chunk before the wait for the tile's accumulator, so the
    // load latency hides behind the MMAs and the previous chunk's math.
    constexpr int CW = bf16_out ? 64 : 32;  // columns per chunk
    constexpr int CE = epi_c_bytes(EPI);   // bytes per C element
    constexpr int EPV = 16 / CE;           // C elements per 16-byte load
    auto c_load = [&](int b_, int row, int col, uint4 (&cc)[8]) {
      const uint8_t* base = reinterpret_cast<const uint8_t*>(ep.c) + ((long long)b_ * ep.c_bstride +
                                                                     (long long)row * ep.ldc) * CE;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = col + j * EPV;
        if (row < sh.M && c + EPV <= sh.N) {
          cc[j] = ld_global_v4(base + (long long)c * CE);
        } else {
          // ragged edge (past N inside the last vector, or rows/columns outside the matrix): zeros
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (row < sh.M) {
#pragma unroll
            for (int i = 0; i < EPV; ++i) {
              if (c + i < sh.N) {
                if constexpr (CE == 2)
                  w[i >> 1] |= (uint32_t)(*reinterpret_cast<const unsigned short*>(base + (long long)(c + i) * 2))
                               << (16 * (i & 1));
                else
                  w[i] = *reinterpret_cast<const uint32_t*>(base + (long long)(c + i) * 4);
              }
            }
          }
          cc[j] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    };
    for (int u = first_unit; u < sh.num_units; u += unit_step) {
      int b, mt, nt, ks;
      decode_unit(u, sh, b, mt, nt, ks);
      const int row0 = mt * TILE_M + rank * GEMM_BM + quarter * 32;  // first output row of this warp
      const bool rows_live = row0 < sh.M;
      const int cbeg = col_half * COLS, cend = cbeg + COLS;  // this warp's columns of the tile
      uint4 cnext[8];
      if constexpr (reads_c) c_load(b, row0 + lane, nt * BN + cbeg, cnext);  // ahead of the accumulator
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if constexpr (EPI == RGPT_EPI_ARGMAX_BF16) {
        // this thread's row over the tile's columns, in increasing order: a strict > keeps the first
        // maximum of the bf16-rounded values (the order a row argmax over stored bf16 logits sees)
        float best = -INFINITY;
        int besti = 0x7fffffff;
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += 64) {
          uint32_t rr[2][32];
          tmem_ld32(t_row + c0, rr[0]);
          tmem_ld32(t_row + c0 + 32, rr[1]);
          tmem_wait_ld();
          const int gn0 = nt * BN + c0;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = gn0 + hf * 32 + j;
              const float v = bf16_round(__uint_as_float(rr[hf][j]) * alpha);
              if (col < sh.N && v > best) {
                best = v;
                besti = col;
              }
            }
        }
        const int row = row0 + lane;
        if (row < sh.M) {
          ep.amax_val[(long long)row * ep.amax_ld + nt] = best;
          ep.amax_idx[(long long)row * ep.amax_ld + nt] = besti;
        }
      } else if constexpr (bf16_out) {
        auto chunk_bf16 = [&](int c0, const uint4 (&cc)[8]) {
          const int gn0 = nt * BN + c0;
          const bool live = rows_live && gn0 < sh.N;  // warp-uniform
          uint8_t* s0 = which ? buf1 : buf0;
          uint8_t* s1 = which ? buf0 : buf1;
          if (live) {
            if (lane == 0) {
              if (dual) bulk_wait_read_0();
              else bulk_wait_read_1();  // the store issued from this buffer two chunks ago has read it
            }
            __syncwarp();
          }
          uint32_t rr[2][32];
          tmem_ld32(t_row + c0, rr[0]);  // both 32-column halves in flight, one wait
          tmem_ld32(t_row + c0 + 32, rr[1]);
          tmem_wait_ld();
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {  // two 32-column halves of the 64-column box
            if (!live) continue;
            float v[32];
            if (scaled) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rr[hf][j]) * alpha;
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rr[hf][j]);
            }
            if constexpr (EPI == RGPT_EPI_ACT_BWD) {
              act_bwd32<ACT>(v, &cc[hf * 4]);
            } else if constexpr (EPI == RGPT_EPI_POLY_BF16) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 cq = cc[hf * 4 + q];
                const uint32_t w4[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 cv = unpack_bf16x2(w4[e]);
                  v[8 * q + 2 * e] += ep.beta * cv.x;
                  v[8 * q + 2 * e + 1] += ep.beta * cv.y;
                }
              }
            } else if constexpr (EPI == RGPT_EPI_BIAS_SIGMOID_BF16) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int col = gn0 + hf * 32 + j;
                const float bias = (col < sh.N) ? __ldg(ep.colscale + col) : 0.f;
                v[j] = rcp_approx(1.0f + ex2_approx(-(v[j] + bias) * 1.4426950408889634f));
              }
            } else if constexpr (EPI == RGPT_EPI_ACT_FWD && !act_two_out) {
              act_fwd32<ACT>(v);  // the post-activation is the only output
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<uint4*>(stage_ptr(s0, lane, hf * 4 + j)) =
                  make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                             pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
            if constexpr (act_two_out) {
              act_fwd32<ACT>(v);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(stage_ptr(s1, lane, hf * 4 + j)) =
                    make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                               pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
            }
          }
          if (!live) return;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmD, s0, gn0, row0, b);
            if constexpr (act_two_out) tma_store_3d(&tmD2, s1, gn0, row0, b);
            bulk_commit_g();
          }
          if (!dual) which ^= 1;
        };
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += CW) {
          uint4 cc[8];
          if constexpr (reads_c) {
#pragma unroll
            for (int j = 0; j < 8; ++j) cc[j] = cnext[j];
            if (c0 + CW < cend) c_load(b, row0 + lane, nt * BN + c0 + CW, cnext);
          }
          chunk_bf16(c0, cc);
        }
      } else {
        constexpr bool resid = EPI == RGPT_EPI_RESID_F32;
        auto chunk_f32 = [&](int c0, const uint4 (&cc)[8]) {
          const int gn0 = nt * BN + c0;
          const bool live = rows_live && gn0 < sh.N;
          uint32_t r[32];
          tmem_ld32(t_row + c0, r);
          tmem_wait_ld();
          if (!live) return;
          float v[32];
          if (scaled) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * alpha;
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          }
          uint8_t* s0 = which ? buf1 : buf0;
          uint8_t* s1 = which ? buf0 : buf1;
          if (lane == 0) {
            if (dual) bulk_wait_read_0();
            else bulk_wait_read_1();
          }
          __syncwarp();
          if constexpr (resid) {
            if (ep.drop_mask != nullptr) {  // dropout of the branch output (warp-uniform branch)
              const int row = row0 + lane;
              const uint32_t keep = row < sh.M ? __ldg(ep.drop_mask + (long long)row * ep.drop_ldm + (gn0 >> 5)) : 0u;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = ((keep >> j) & 1u) ? v[j] * ep.drop_scale : 0.f;
            }
            if (ep.has_d2) stage_f32x32(s1, lane, v);  // raw (dropped) branch output
            const float* cs = reinterpret_cast<const float*>(cc);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float sc = (ep.colscale != nullptr && gn0 + j < sh.N) ? __ldg(ep.colscale + gn0 + j) : 1.0f;
              v[j] = cs[j] + v[j] * sc;
            }
          } else if constexpr (EPI == RGPT_EPI_POLY_F32) {
            const float* cs = reinterpret_cast<const float*>(cc);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(ep.beta, cs[j], v[j]);
          }
          stage_f32x32(s0, lane, v);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == RGPT_EPI_ACCUM_F32) {
              tma_reduce_add_3d(&tmD, s0, gn0, row0, b);
            } else {
              tma_store_3d(&tmD, s0, gn0, row0, b);
              if (resid && ep.has_d2) tma_store_3d(&tmD2, s1, gn0, row0, b);
            }
            bulk_commit_g();
          }
          if (!dual) which ^= 1;
        };
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += CW) {
          uint4 cc[8];
          if constexpr (reads_c) {
#pragma unroll
            for (int j = 0; j < 8; ++j) cc[j] = cnext[j];
            if (c0 + CW < cend) c_load(b, row0 + lane, nt * BN + c0 + CW, cnext);
          }
          chunk_f32(c0, cc);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(tempty_bar0 + acc * 8);
        else mbar_arrive(&tempty_bar[acc]);
      }
      if (++acc == NUM_ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();  // every bulk store has landed before the CTA retires
    __syncwarp();
  }

  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // neither CTA frees TMEM or exits while the pair still works
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
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

// 3-D tensor map (inner, outer, batch) with a 128-byte swizzle; elem_bytes 2 (bf16) or 4 (fp32).
static int make_tmap_3d(CUtensorMap* map, const void* ptr, int elem_bytes, uint64_t inner, uint64_t outer,
                        uint64_t batch, uint64_t ld_elems, uint64_t bstride_elems, uint32_t box_inner,
                        uint32_t box_outer) {
  auto enc = get_encode_fn();
  if (enc == nullptr) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "TMA base pointer %p is not 16-byte aligned", ptr);
  if (batch <= 1) bstride_elems = ld_elems * outer;
  if ((ld_elems * elem_bytes) % 16 != 0 || (bstride_elems * elem_bytes) % 16 != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "TMA strides must be multiples of 16 bytes (ld=%llu, bstride=%llu)",
                          (unsigned long long)ld_elems, (unsigned long long)bstride_elems);
  cuuint64_t dims[3] = {inner, outer, batch < 1 ? 1 : batch};
  cuuint64_t strides[2] = {ld_elems * elem_bytes, bstride_elems * elem_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return RGPT_OK;
}

int make_tmap_bf16_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch,
                      uint64_t ld_elems, uint64_t bstride_elems, uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_3d(map, ptr, 2, inner, outer, batch, ld_elems, bstride_elems, box_inner, box_outer);
}

// Operand stages that fit beside EW warps' staging buffers (at most `want`).
template <int BN, bool PAIR, int EW>
constexpr int gemm_fit_stages(int want) {
  using L1 = GemmSmem<BN, 1, PAIR, EW>;
  const int fit = (int)((232448u - L1::EPI_BYTES - L1::BAR_BYTES - 1024u) / L1::STAGE_BYTES);
  return fit < want ? fit : want;
}

template <int BN, int STAGES_IN, int A_MN, int B_MN, int EPI, bool PAIR, int ACT = ACT_NONE>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& td2,
                       const GemmShape& sh, const EpiParams& ep, cudaStream_t stream, int dev) {
  constexpr int EW = gemm_epi_warps(EPI);
  constexpr int STAGES = gemm_fit_stages<BN, PAIR, EW>(STAGES_IN);
  constexpr int THREADS = gemm_threads(EW);
  auto kern = gemm_bf16_tc_kernel<BN, STAGES, A_MN, B_MN, EPI, PAIR, ACT>;
  constexpr uint32_t smem = GemmSmem<BN, STAGES, PAIR, EW>::TOTAL;
  static_assert(smem <= 232448, "GEMM shared memory exceeds the per-CTA limit");
  static bool attr_set[64] = {false};
  static int max_clusters[64] = {0};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return rgpt_check_launch("gemm set smem attribute");
    if (PAIR) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * rgpt_num_sms(dev), 1, 1);
      q.blockDim = dim3(THREADS, 1, 1);
      q.dynamicSmemBytes = smem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1)
        return rgpt_set_error(RGPT_ERR_INTERNAL, "no CTA pair fits on this GPU (%s)",
                              cudaGetErrorString(cudaGetLastError()));
      max_clusters[dev] = n;
    }
    attr_set[dev] = true;
  }
  if constexpr (PAIR) {
    const int clusters = sh.num_units < max_clusters[dev] ? sh.num_units : max_clusters[dev];
    launch_pdl(kern, dim3(2 * clusters), dim3(THREADS), smem, stream, 2, ta, tb, td, td2, sh, ep);
  } else {
    const int nsm = rgpt_num_sms(dev);
    const int grid = sh.num_units < nsm ? sh.num_units : nsm;
    launch_pdl(kern, dim3(grid), dim3(THREADS), smem, stream, 1, ta, tb, td, td2, sh, ep);
  }
  return rgpt_check_launch("gemm_bf16_tc_kernel");
}

template <int BN, int STAGES, int A_MN, int B_MN, bool PAIR>
static int dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                        const CUtensorMap& td2, const GemmShape& sh, const EpiParams& ep,
                        cudaStream_t s, int dev) {
#define RGPT_GEMM_EPI_CASE(E) \
  case E: return launch_gemm<BN, STAGES, A_MN, B_MN, E, PAIR>(ta, tb, td, td2, sh, ep, s, dev);
  switch (epi) {
    RGPT_GEMM_EPI_CASE(RGPT_EPI_STORE_BF16)
    RGPT_GEMM_EPI_CASE(RGPT_EPI_STORE_F32)
    RGPT_GEMM_EPI_CASE(RGPT_EPI_ACCUM_F32)
    case RGPT_EPI_ACT_FWD:
    case RGPT_EPI_ACT_BWD: {
      // the activation is a compile-time parameter of the epilogue
      const bool fwd = epi == RGPT_EPI_ACT_FWD;
#define RGPT_GEMM_ACT_CASE(A)                                                                                      \
  case A:                                                                                                          \
    return fwd ? launch_gemm<BN, STAGES, A_MN, B_MN, RGPT_EPI_ACT_FWD, PAIR, A>(ta, tb, td, td2, sh, ep, s, dev) \
               : launch_gemm<BN, STAGES, A_MN, B_MN, RGPT_EPI_ACT_BWD, PAIR, A>(ta, tb, td, td2, sh, ep, s, dev);
      switch (ep.act) {
        RGPT_GEMM_ACT_CASE(ACT_SQRELU)
        RGPT_GEMM_ACT_CASE(ACT_GELU)
        RGPT_GEMM_ACT_CASE(ACT_SILU)
        RGPT_GEMM_ACT_CASE(ACT_MISH)
        RGPT_GEMM_ACT_CASE(ACT_SQRELU_POST)
        default:
          return fwd ? launch_gemm<BN, STAGES, A_MN, B_MN, RGPT_EPI_ACT_FWD, PAIR, ACT_NONE>(ta, tb, td, td2, sh,
                                                                                          ep, s, dev)
                     : launch_gemm<BN, STAGES, A_MN, B_MN, RGPT_EPI_ACT_BWD, PAIR, ACT_NONE>(ta, tb, td, td2, sh,
                                                                                          ep, s, dev);
      }
#undef RGPT_GEMM_ACT_CASE
    }
    RGPT_GEMM_EPI_CASE(RGPT_EPI_RESID_F32)
    RGPT_GEMM_EPI_CASE(RGPT_EPI_POLY_BF16)
    RGPT_GEMM_EPI_CASE(RGPT_EPI_POLY_F32)
    RGPT_GEMM_EPI_CASE(RGPT_EPI_ARGMAX_BF16)
    default: return launch_gemm<BN, STAGES, A_MN, B_MN, RGPT_EPI_BIAS_SIGMOID_BF16, PAIR>(ta, tb, td, td2, sh, ep, s, dev);
  }
#undef RGPT_GEMM_EPI_CASE
}

// Tile configurations: 128 x 128 (6 stages), 128 x 256 (4 stages), and the CTA pair's
// 256 x 256 (6 stages of 128 x 64 A + 128 x 64 B per CTA).
static int dispatch_gemm(int BN, bool pair, int a_mn, int b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                         const CUtensorMap& td, const CUtensorMap& td2, const GemmShape& sh,
                         const EpiParams& ep, cudaStream_t s, int dev) {
  const int key = (pair ? 8 : 0) | (BN == 256 ? 4 : 0) | (a_mn ? 2 : 0) | (b_mn ? 1 : 0);
  switch (key) {
    case 0: return dispatch_epi<128, 6, 0, 0, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 1: return dispatch_epi<128, 6, 0, 1, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 2: return dispatch_epi<128, 6, 1, 0, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 3: return dispatch_epi<128, 6, 1, 1, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 4: return dispatch_epi<256, 4, 0, 0, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 5: return dispatch_epi<256, 4, 0, 1, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 6: return dispatch_epi<256, 4, 1, 0, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 7: return dispatch_epi<256, 4, 1, 1, false>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 12: return dispatch_epi<256, 6, 0, 0, true>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 13: return dispatch_epi<256, 6, 0, 1, true>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 14: return dispatch_epi<256, 6, 1, 0, true>(epi, ta, tb, td, td2, sh, ep, s, dev);
    case 15: return dispatch_epi<256, 6, 1, 1, true>(epi, ta, tb, td, td2, sh, ep, s, dev);
    default: return rgpt_set_error(RGPT_ERR_INTERNAL, "no GEMM configuration for key %d", key);
  }
}

}  // namespace rgpt

using namespace rgpt;

// Row argmax from the ARGMAX_BF16 GEMM's per-tile results: one warp per row, the largest value and,
// among equal values, the smallest column (so the first maximum of the row, as torch.argmax).
__global__ void argmax_reduce_kernel(const float* __restrict__ val, const int* __restrict__ idx, long long ld,
                                     int n_tiles, int M, int* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int t = lane; t < n_tiles; t += 32) {
    const float v = val[(long long)row * ld + t];
    const int i = idx[(long long)row * ld + t];
    if (v > best || (v == best && i < besti)) {
      best = v;
      besti = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) {
      best = ov;
      besti = oi;
    }
  }
  if (lane == 0) out[row] = besti;
}

struct DropArgs {
  const void* mask;
  long long ldm;
  float p;
};

struct AmaxArgs {  // ARGMAX_BF16 partial results, [M, ld] each; n_tiles is set to the column tiles used
  float* val;
  int* idx;
  long long ld;
  int n_tiles;
};

static int gemm_entry(const void* A, int a_mn_major, long long lda, long long a_bstride, const void* B,
                      int b_mn_major, long long ldb, long long b_bstride, int M, int N, int K, int batch, int epi,
                      int act, float alpha, float beta, void* D, long long ldd, long long d_bstride, void* D2,
                      long long ldd2, long long d2_bstride, const void* C, long long ldc, long long c_bstride,
                      const float* colscale, int splitk, const float* alpha_dev, const DropArgs* drop,
                      void* stream, AmaxArgs* amax = nullptr) {
  int dev = 0;
  cudaGetDevice(&dev);
  int st = rgpt_check_device(dev);
  if (st) return st;
  if (dev >= 64) return rgpt_set_error(RGPT_ERR_INTERNAL, "device index %d", dev);
  if (batch < 1) batch = 1;
  if (M < 1 || N < 1 || K < 1)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "gemm needs M, N, K >= 1 (got M=%d N=%d K=%d)", M, N, K);
  if (epi < RGPT_EPI_STORE_BF16 || epi > RGPT_EPI_ARGMAX_BF16 || (epi == RGPT_EPI_ARGMAX_BF16 && amax == nullptr))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "unknown epilogue %d", epi);
  const bool amx = epi == RGPT_EPI_ARGMAX_BF16;  // no output matrix: per-tile row maxima instead
  if (amx && (batch != 1 || amax->val == nullptr || amax->idx == nullptr || amax->ld < (N + 127) / 128))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "argmax GEMM needs batch 1 and [M, >= %d] partial buffers",
                          (N + 127) / 128);
  if (D == nullptr && !amx) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "gemm output pointer is null");
  const bool out_f32 = (epi == RGPT_EPI_STORE_F32 || epi == RGPT_EPI_ACCUM_F32 || epi == RGPT_EPI_RESID_F32 ||
                        epi == RGPT_EPI_POLY_F32);
  const int vec = out_f32 ? 4 : 8;
  if (!amx && (ldd % vec != 0 || (reinterpret_cast<uintptr_t>(D) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "output leading dim / pointer not 16-byte aligned");
  if (epi == RGPT_EPI_ACT_FWD && act != ACT_SQRELU_POST &&
      (D2 == nullptr || ldd2 % 8 != 0 || (reinterpret_cast<uintptr_t>(D2) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "ACT_FWD needs an aligned second output");
  if (epi == RGPT_EPI_RESID_F32 && D2 != nullptr && (ldd2 % 4 != 0 || (reinterpret_cast<uintptr_t>(D2) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "RESID_F32 raw output must be 16-byte aligned");
  if (epi_reads_c(epi) &&
      (C == nullptr || ldc % vec != 0 || (reinterpret_cast<uintptr_t>(C) & 15) != 0))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "epilogue input C missing or not 16-byte aligned");
  if (epi == RGPT_EPI_BIAS_SIGMOID_BF16 && colscale == nullptr)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "BIAS_SIGMOID needs the bias vector (colscale)");

  const int nsm = rgpt_num_sms(dev);
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K = K;
  sh.batch = batch;
  // 256-wide tiles unless at most half the SMs would get one. Both widths run the tensor pipe at
  // full rate (a 128 x N x 16 MMA takes 64 SM cycles at N = 128 and 128 at N = 256; only N = 64
  // falls short at ~55), but a 128 x 128 tile moves 64 bytes of operands from L2 per 1024 FLOP
  // against 48 for 128 x 256, and measured 15-40 % slower on the step's GEMMs; halving the tile
  // only pays when both widths fit in one wave. Accumulating GEMMs keep the wide tile (fewer
  // operand re-reads) and split K instead.
  const int m128 = (M + GEMM_BM - 1) / GEMM_BM;
  int BN = (N > 128) ? 256 : 128;
  if (BN == 256 && epi != RGPT_EPI_ACCUM_F32 && 2LL * batch * m128 * ((N + 255) / 256) <= nsm) BN = 128;
  sh.num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  // CTA pairs (256 x 256 tiles, half the B traffic per SM) pay off once the main loop is long
  // (K >= 1024) and there is a wave of pair tiles, or for plain stores with very many tiles
  // (a vocabulary-sized output); long-K accumulating GEMMs split K to fill the GPU anyway.
  // Short-K GEMMs with few tiles stay on single-CTA tiles, whose shorter signalling chain
  // finishes each tile sooner.
  const long long pair_tiles = (long long)batch * ((M + 255) / 256) * ((N + 255) / 256);
  const bool plain_store = epi == RGPT_EPI_STORE_BF16 || epi == RGPT_EPI_STORE_F32 || amx;
  const bool pair = BN == 256 && M > GEMM_BM &&
                    ((pair_tiles >= nsm / 2 && (sh.num_kb >= 16 || (plain_store && pair_tiles >= 8LL * nsm))) ||
                     (epi == RGPT_EPI_ACCUM_F32 && sh.num_kb >= 32));
  const int units_per_wave = pair ? nsm / 2 : nsm;
  sh.m_tiles = pair ? (M + 255) / 256 : m128;
  sh.n_tiles = (N + BN - 1) / BN;
  const int tiles = batch * sh.m_tiles * sh.n_tiles;
  if (splitk <= 0) {
    // Split K (accumulating epilogue only) to minimise waves x (k-blocks per unit + the
    // tile's reduce-add epilogue, worth about 8 k-blocks), keeping >= 4 k-blocks per split;
    // fewer splits win ties (fewer reduce-adds).
    splitk = 1;
    if (epi == RGPT_EPI_ACCUM_F32) {
      long long best = -1;
      const int max_split = sh.num_kb / 4 > 0 ? (sh.num_kb / 4 < 64 ? sh.num_kb / 4 : 64) : 1;
      for (int s = 1; s <= max_split; ++s) {
        const long long waves = ((long long)tiles * s + units_per_wave - 1) / units_per_wave;
        const long long cost = waves * ((sh.num_kb + s - 1) / s + 8);
        if (best < 0 || cost < best) {
          best = cost;
          splitk = s;
        }
      }
    }
  }
  if (splitk > 1 && epi != RGPT_EPI_ACCUM_F32)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "split-K is only valid with the ACCUM_F32 epilogue");
  if (splitk > sh.num_kb) splitk = sh.num_kb;
  sh.kb_per_split = (sh.num_kb + splitk - 1) / splitk;
  sh.splitk = (sh.num_kb + sh.kb_per_split - 1) / sh.kb_per_split;  // no empty splits
  sh.num_units = tiles * sh.splitk;
  // Visiting order: groups of GROUP_M row tiles, each swept across all column tiles. A very wide
  // output (the vocabulary-sized lm_head logits, N / BN >= 64) with a small A (<= 32 MB) is swept
  // column by column over ALL row tiles instead: A stays in L2 and B streams through once, where
  // groups of 8 row tiles would read the 51 MB lm_head weight once per group (m_tiles / 8 times).
  sh.group_m = GROUP_M;
  if (sh.n_tiles >= 64 && (long long)M * K * 2 <= (32LL << 20)) sh.group_m = sh.m_tiles;

  // Operand maps. K-major: (inner=K, outer=rows); MN-major: (inner=rows, outer=K).
  CUtensorMap ta, tb, td, td2;
  if (a_mn_major)
    st = make_tmap_3d(&ta, A, 2, M, K, batch, lda, a_bstride, 64, GEMM_BK);
  else
    st = make_tmap_3d(&ta, A, 2, K, M, batch, lda, a_bstride, GEMM_BK, GEMM_BM);
  if (st) return st;
  if (b_mn_major)
    st = make_tmap_3d(&tb, B, 2, N, K, batch, ldb, b_bstride, 64, GEMM_BK);
  else
    st = make_tmap_3d(&tb, B, 2, K, N, batch, ldb, b_bstride, GEMM_BK, pair ? BN / 2 : BN);
  if (st) return st;
  // Output maps: one 32-row x 128-byte box per epilogue warp and chunk.
  const int ob = out_f32 ? 4 : 2;
  const uint32_t obox = out_f32 ? 32 : 64;
  if (amx)
    td = ta;  // never used by the argmax epilogue (only its descriptor is prefetched)
  else if ((st = make_tmap_3d(&td, D, ob, N, M, batch, ldd, d_bstride, obox, 32)))
    return st;
  const bool has_d2 = (epi == RGPT_EPI_ACT_FWD && act != ACT_SQRELU_POST) || (epi == RGPT_EPI_RESID_F32 && D2 != nullptr);
  if (has_d2) {
    if ((st = make_tmap_3d(&td2, D2, ob, N, M, batch, ldd2, d2_bstride, obox, 32))) return st;
  } else {
    td2 = td;
  }

  // epilogue input C (bf16 for ACT_BWD / POLY, fp32 for RESID) is read with 16-byte loads
  if (epi_reads_c(epi)) {
    const long long cb = epi_c_bytes(epi);
    if (C == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "epilogue %d needs its input C", epi);
    if (ldc < N) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ldc (%lld) < N (%d)", ldc, N);
    if ((reinterpret_cast<uintptr_t>(C) & 15) != 0 || (ldc * cb) % 16 != 0 || (batch > 1 && (c_bstride * cb) % 16 != 0))
      return rgpt_set_error(RGPT_ERR_MISALIGNED, "C must be 16-byte aligned with 16-byte row and batch strides");
  }

  EpiParams ep;
  ep.kind = epi;
  ep.act = act;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.c = C;
  ep.ldc = ldc;
  ep.c_bstride = c_bstride;
  ep.colscale = colscale;
  ep.alpha_dev = alpha_dev;
  ep.has_d2 = has_d2 ? 1 : 0;
  ep.drop_mask = nullptr;
  ep.drop_ldm = 0;
  ep.drop_scale = 1.0f;
  if (amx) amax->n_tiles = sh.n_tiles;
  ep.amax_val = amx ? amax->val : nullptr;
  ep.amax_idx = amx ? amax->idx : nullptr;
  ep.amax_ld = amx ? amax->ld : 0;
  if (drop != nullptr && drop->p > 0.0f) {
    if (epi != RGPT_EPI_RESID_F32)
      return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout is only fused into the RESID_F32 epilogue");
    if (!(drop->p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout p must be in [0, 1), got %g", drop->p);
    if (batch != 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout GEMMs are not batched");
    if (drop->mask == nullptr || drop->ldm < (N + 31) / 32)
      return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout needs a mask of >= %d words per row", (N + 31) / 32);
    ep.drop_mask = reinterpret_cast<const uint32_t*>(drop->mask);
    ep.drop_ldm = drop->ldm;
    ep.drop_scale = (float)(1.0 / (1.0 - (double)drop->p));
  }

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dispatch_gemm(BN, pair, a_mn_major, b_mn_major, epi, ta, tb, td, td2, sh, ep, s, dev);
}

extern "C" int rgpt_gemm_bf16(const void* A, int a_mn_major, long long lda, long long a_bstride, const void* B,
                              int b_mn_major, long long ldb, long long b_bstride, int M, int N, int K, int batch,
                              int epi, int act, float alpha, float beta, void* D, long long ldd, long long d_bstride,
                              void* D2, long long ldd2, long long d2_bstride, const void* C, long long ldc,
                              long long c_bstride, const float* colscale, int splitk, const float* alpha_dev,
                              void* stream) {
  return gemm_entry(A, a_mn_major, lda, a_bstride, B, b_mn_major, ldb, b_bstride, M, N, K, batch, epi, act, alpha,
                    beta, D, ldd, d_bstride, D2, ldd2, d2_bstride, C, ldc, c_bstride, colscale, splitk, alpha_dev,
                    nullptr, stream);
}

extern "C" int rgpt_gemm_bf16_dropout(const void* A, int a_mn_major, long long lda, long long a_bstride,
                                      const void* B, int b_mn_major, long long ldb, long long b_bstride, int M, int N,
                                      int K, int batch, int epi, int act, float alpha, float beta, void* D,
                                      long long ldd, long long d_bstride, void* D2, long long ldd2,
                                      long long d2_bstride, const void* C, long long ldc, long long c_bstride,
                                      const float* colscale, int splitk, const float* alpha_dev,
                                      const void* drop_mask, long long drop_ldm, float drop_p, void* stream) {
  const DropArgs d = {drop_mask, drop_ldm, drop_p};
  return gemm_entry(A, a_mn_major, lda, a_bstride, B, b_mn_major, ldb, b_bstride, M, N, K, batch, epi, act, alpha,
                    beta, D, ldd, d_bstride, D2, ldd2, d2_bstride, C, ldc, c_bstride, colscale, splitk, alpha_dev,
                    &d, stream);
}

extern "C" int rgpt_gemm_argmax(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                float* part_val, int* part_idx, long long ld_part, int* argmax, void* stream) {
  if (argmax == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "argmax output pointer is null");
  AmaxArgs a = {part_val, part_idx, ld_part, 0};
  int st = gemm_entry(A, 0, lda, 0, B, 0, ldb, 0, M, N, K, 1, RGPT_EPI_ARGMAX_BF16, 0, 1.0f, 0.0f, nullptr, 0, 0,
                      nullptr, 0, 0, nullptr, 0, 0, nullptr, 1, nullptr, nullptr, stream, &a);
  if (st) return st;
  // a.n_tiles: the column tiles of the width the GEMM chose (128 or 256), each written for every row
  launch_pdl(argmax_reduce_kernel, dim3((unsigned)((M + 7) / 8)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1,
             (const float*)part_val, (const int*)part_idx, ld_part, a.n_tiles, M, argmax);
  return rgpt_check_launch("argmax_reduce_kernel");
}
