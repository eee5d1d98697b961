// The whole quintic Newton-Schulz iteration of a batch of same-shape matrices in ONE persistent launch
// (zeropower_via_newtonschulz5, optimizer.py:18-45): `steps` x {A = X X^T; B = b A + c A A; X' = a X + B X}.
//
// The batched-GEMM path launches the 3 * steps GEMMs one after another; each is one or two waves of
// small tiles with its own pipeline fill and drain, and the chain is a string of dependent launches.
// Here the 3 * steps GEMMs are phases of one kernel. Every (phase, matrix, output tile) is a work unit
// (128 x 128 tiles on single CTAs, or 256 x 256 tiles on CTA pairs, see ns_chain_kernel); units are
// dealt round-robin to persistent CTAs or CTA pairs (at most one CTA per SM, all resident) in
// phase-major order, and a unit only waits for the previous phase of ITS OWN matrix: a per (matrix,
// phase) counter that the epilogue warps raise once their part of a tile has landed in global memory.
// So while some matrices are still in phase p, SMs already run phase p + 1 of others: no grid-wide
// barrier, no launch gaps, and the TMEM accumulator ring keeps the epilogue of one tile under the MMAs
// of the next. Dependencies only point to earlier units and each CTA visits its units in order, so
// the waits always end; every wait is still bounded (1 s), after which the kernel records a device
// error and stops.
//
// CTA: 320 threads. Warp 0 TMA producer (waits for the unit's dependency, then streams 64-deep
// k-blocks of A and B into a 5-stage ring), warp 1 TMEM allocation + tcgen05.mma issue (one elected
// thread), warps 2-9 epilogue, two per TMEM lane quadrant, each taking one half of the tile's columns
// (TMEM -> registers, + beta * C for B and X', bf16 -> swizzled smem -> TMA bulk store; then the
// completion counter). A warp publishes its part of a tile as soon as the store has landed: the phase
// chain is latency-bound, so a deferred publish (to keep the store in flight under the next tile's
// math) measured slower. A diagonal tile of A = X X^T or of A A reads the same panel as both MMA
// operands, so it is loaded once. Operands and outputs are bf16, accumulation fp32: the same
// roundings as the batched path (one per GEMM, the polynomial combine fused).
//
// Memory ordering between units of different CTAs: a tile's TMA stores complete (bulk wait_group 0),
// a proxy fence orders them before the generic-proxy release increment of the counter; the consumer
// acquires the counter, fences the async proxy and only then issues its TMA loads. The epilogue reads
// C (A or X) with L1-bypassing loads after its own acquire: a persistent CTA's L1 may hold lines of a
// buffer that an earlier phase rewrote.
#include <cudaTypedefs.h>
#include <stdlib.h>

#include "common.cuh"
#include "rgpt.h"

namespace rgpt {

int make_tmap_bf16_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch,
                      uint64_t ld_elems, uint64_t bstride_elems, uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int NS_BK = 64;       // k-block
constexpr int NS_PANEL = 128;   // rows of each operand panel one CTA stages per k-block (= the MMA M per CTA)
constexpr int NS_STAGES = 5;
constexpr int NS_EW = 8;        // epilogue warps: two per TMEM lane quadrant, each taking half of the tile's columns
constexpr int NS_THREADS = 64 + 32 * NS_EW;
constexpr uint32_t NS_PANEL_BYTES = NS_PANEL * NS_BK * 2;  // 16 KB
constexpr uint32_t NS_EPI_STAGE = 4096;                     // one warp's 32 rows x 128 bytes
// two staging buffers per epilogue warp (a warp stores two 64-column chunks of a 256-wide pair tile)
constexpr uint32_t NS_SMEM = NS_STAGES * 2 * NS_PANEL_BYTES + NS_EW * 2 * NS_EPI_STAGE + 512 + 1024;

struct NsMaps {
  CUtensorMap xk[2];   // X buffers as K-major operands: (inner xc, outer xr, batch), box (64, 128)
  CUtensorMap xmn[2];  // X buffers as the MN-major B operand of B X: box (64 along xc, 64 along xr)
  CUtensorMap ak;      // A [xr, xr], box (64, 128)
  CUtensorMap bk;      // B [xr, xr], box (64, 128)
  CUtensorMap da, db;  // output maps: box (64, 32)
  CUtensorMap dx[2];
};

struct NsParams {
  int n, xr, xc, steps;
  int mt, nt_r, nt_c;   // tile rows of xr; tile columns of xr and of xc (tiles of 128, or 256 for CTA pairs)
  int t01, t2;          // tiles of phases A/B and of X'
  long long units_per_step, num_units;
  float a, b, c;
  const __nv_bfloat16* x[2];
  const __nv_bfloat16* abuf;
  long long x_ld, x_bs, a_ld, a_bs;  // row / batch strides (elements) of the X and A/B buffers
  unsigned* ctr;                     // [n][3 * steps] completion counters, zero at launch
};

struct NsUnit {
  int kind, step, m, mt, nt, phase;
};

__device__ __forceinline__ NsUnit ns_decode(long long u, const NsParams& P) {
  NsUnit r;
  r.step = (int)(u / P.units_per_step);
  long long q = u % P.units_per_step;
  const long long na = (long long)P.n * P.t01;
  int t;
  if (q < na) {
    r.kind = 0;
  } else if (q < 2 * na) {
    r.kind = 1;
    q -= na;
  } else {
    r.kind = 2;
    q -= 2 * na;
  }
  const int tiles = r.kind == 2 ? P.t2 : P.t01;
  r.m = (int)(q / tiles);
  t = (int)(q % tiles);
  const int ncols = r.kind == 2 ? P.nt_c : P.nt_r;
  r.mt = t / ncols;
  r.nt = t % ncols;
  r.phase = 3 * r.step + r.kind;
  return r;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void ns_tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void ns_bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void ns_bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ uint8_t* ns_stage_ptr(uint8_t* buf, int lane, int j) {
  return buf + lane * 128 + ((j ^ (lane & 7)) << 4);
}

// Bounded wait until *ctr >= target (acquire). False on timeout or when another role gave up.
__device__ __forceinline__ bool dep_wait(const unsigned* ctr, unsigned target, volatile int* abort) {
  if (ld_acquire_u32(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_u32(ctr) >= target) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > RGPT_WAIT_LIMIT_NS) {
      record_device_error(RGPT_DEVERR_WAIT_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

}  // namespace

// PAIR = false: one CTA per 128 x 128 tile. PAIR = true: a cluster of two CTAs per 256 x 256 tile
// (tcgen05.mma.cta_group::2 issued by the even CTA): each CTA stages 128 rows of A and 128 rows (columns
// of the output) of B per k-block, so each SM moves 32 KB of operands per 256 x 256 x 64 step instead of
// per 128 x 128 x 64 step, and each CTA holds 128 rows x 256 columns of the accumulator in its TMEM.
template <bool PAIR>
__global__ void __launch_bounds__(NS_THREADS, 1)
    ns_chain_kernel(const __grid_constant__ NsMaps maps, const NsParams P) {
  constexpr int TILE = PAIR ? 2 * NS_PANEL : NS_PANEL;  // output tile edge
  constexpr int NUM_ACC = 512 / TILE;                   // TMEM accumulators of TILE columns
  constexpr int COLS = TILE / 2;                        // columns of a tile one epilogue warp writes
  constexpr uint32_t IDESC_KK = make_idesc_bf16(TILE, TILE, 0, 0);
  constexpr uint32_t IDESC_KM = make_idesc_bf16(TILE, TILE, 0, 1);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + NS_STAGES * NS_PANEL_BYTES;
  uint8_t* sEpi = sB + NS_STAGES * NS_PANEL_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sEpi + NS_EW * 2 * NS_EPI_STAGE);
  uint64_t* empty_bar = full_bar + NS_STAGES;
  uint64_t* tfull_bar = empty_bar + NS_STAGES;
  uint64_t* tempty_bar = tfull_bar + NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + NUM_ACC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P3 = 3 * P.steps;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;  // 0 = the CTA that issues the pair's MMAs
  const long long first_unit = PAIR ? (long long)cluster_id_x() : (long long)blockIdx.x;
  const long long unit_step = PAIR ? (long long)cluster_count_x() : (long long)gridDim.x;
  // every epilogue warp of every CTA working on a tile raises the tile's phase counter once
  constexpr unsigned PUBS = PAIR ? 2 * NS_EW : NS_EW;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], PUBS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      tma_prefetch_desc(&maps.xk[i]);
      tma_prefetch_desc(&maps.xmn[i]);
      tma_prefetch_desc(&maps.dx[i]);
    }
    tma_prefetch_desc(&maps.ak);
    tma_prefetch_desc(&maps.bk);
    tma_prefetch_desc(&maps.da);
    tma_prefetch_desc(&maps.db);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, NUM_ACC * TILE);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, NUM_ACC * TILE);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // the normalised X comes from the previous kernel; the counters were zeroed before
  // the pair's shared barriers live in the even CTA (shared::cluster addresses)
  const uint32_t full_bar0 = PAIR ? mapa_shared(smem_u32(full_bar), 0) : smem_u32(full_bar);
  const uint32_t tempty_bar0 = PAIR ? mapa_shared(smem_u32(tempty_bar), 0) : smem_u32(tempty_bar);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs of a pair)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (long long u = first_unit; u < P.num_units && ok; u += unit_step) {
        const NsUnit U = ns_decode(u, P);
        if (U.phase > 0) {
          const int prev_kind = (U.kind + 2) % 3;
          const unsigned target = (unsigned)((prev_kind == 2 ? P.t2 : P.t01) * PUBS);
          if (!dep_wait(P.ctr + (long long)U.m * P3 + U.phase - 1, target, abort_flag)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();  // the acquired writes are visible to the TMA loads below
        }
        const int xin = U.step & 1;
        const CUtensorMap* mA = U.kind == 0 ? &maps.xk[xin] : (U.kind == 1 ? &maps.ak : &maps.bk);
        const CUtensorMap* mB = U.kind == 0 ? &maps.xk[xin] : (U.kind == 1 ? &maps.ak : &maps.xmn[xin]);
        const int K = U.kind == 0 ? P.xc : P.xr;
        const int N = U.kind == 2 ? P.xc : P.xr;
        const int num_kb = (K + NS_BK - 1) / NS_BK;
        const int a_row = U.mt * TILE + rank * NS_PANEL, b_row = U.nt * TILE + rank * NS_PANEL;
        // A diagonal tile of A or B has the same rows as both operands: its one panel is loaded once and
        // the MMA reads it as both. The MN-major B of X' arrives as 64-column sub-boxes; those wholly
        // past N are not loaded.
        const bool diag = U.kind != 2 && U.mt == U.nt;
        auto b_subs = [&](int rk) {
          return U.kind == 2 ? max(0, min(2, (N - (U.nt * TILE + rk * NS_PANEL) + 63) / 64)) : (diag ? 0 : 2);
        };
        const int b_sub = b_subs(rank);
        const uint32_t expect = PAIR ? 2 * NS_PANEL_BYTES + (uint32_t)(b_subs(0) + b_subs(1)) * (64 * NS_BK * 2)
                                     : NS_PANEL_BYTES + (uint32_t)b_sub * (64 * NS_BK * 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // the pair's barrier lives in the even CTA, which posts the byte count of both CTAs' loads
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], expect);
          const int k0 = kb * NS_BK;
          uint8_t* a_dst = sA + stage * NS_PANEL_BYTES;
          uint8_t* b_dst = sB + stage * NS_PANEL_BYTES;
          auto load = [&](uint8_t* dst, const CUtensorMap* map, int c0, int c1) {
            if constexpr (PAIR) tma_load_3d_pair(dst, map, full_bar0 + stage * 8, c0, c1, U.m);
            else tma_load_3d(dst, map, &full_bar[stage], c0, c1, U.m);
          };
          load(a_dst, mA, k0, a_row);
          if (U.kind == 2) {
            for (int i = 0; i < b_sub; ++i) load(b_dst + i * (64 * NS_BK * 2), mB, b_row + i * 64, k0);
          } else if (!diag) {
            load(b_dst, mB, k0, b_row);
          }
          if (++stage == NS_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      griddep_launch();
      if (!ok && rank == 0) {
        // bounded drain of the loads already issued (a pair's loads all complete on the even CTA's
        // barriers; the final cluster barrier keeps the odd CTA alive meanwhile)
        for (int s = 0; s < NS_STAGES; ++s) mbar_wait(&full_bar[s], phase, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the even CTA of a pair)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      auto commit = [&](uint64_t* bar) {  // completion signals go to both CTAs of a pair (same offsets)
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(bar), 0));
          umma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          umma_commit(bar);
        }
      };
      for (long long u = first_unit; u < P.num_units && ok; u += unit_step) {
        const NsUnit U = ns_decode(u, P);
        const int K = U.kind == 0 ? P.xc : P.xr;
        const int num_kb = (K + NS_BK - 1) / NS_BK;
        const bool bmn = U.kind == 2;
        const bool diag = !bmn && U.mt == U.nt;  // B operand = the A stage
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * TILE;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * NS_PANEL_BYTES);
          const uint32_t b_addr = diag ? a_addr : smem_u32(sB + stage * NS_PANEL_BYTES);
#pragma unroll
          for (int kk = 0; kk < NS_BK / 16; ++kk) {
            const uint64_t adesc = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = bmn ? make_sw128_desc(b_addr + kk * 2048, 64 * NS_BK * 2, 1024)
                                       : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            const uint32_t idesc = bmn ? IDESC_KM : IDESC_KK;
            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
            if constexpr (PAIR) umma_bf16_pair(d_tmem, adesc, bdesc, idesc, accum);
            else umma_bf16(d_tmem, adesc, bdesc, idesc, accum);
          }
          commit(&empty_bar[stage]);
          if (++stage == NS_STAGES) {
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
    const int quarter = warp & 3;                // TMEM lane quadrant: rows quarter*32 .. +31 of this CTA's half
    const int c0 = ((warp - 2) >> 2) * COLS;     // this warp's columns of the tile
    uint8_t* sbuf = sEpi + (warp - 2) * 2 * NS_EPI_STAGE;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (long long u = first_unit; u < P.num_units; u += unit_step) {
      const NsUnit U = ns_decode(u, P);
      const int M = P.xr, N = U.kind == 2 ? P.xc : P.xr;
      const int row0 = U.mt * TILE + rank * NS_PANEL + quarter * 32;
      const int row = row0 + lane;
      const int gn0 = U.nt * TILE + c0;
      // C of the polynomial: A (for B = b A + c A A) or the current X (for X' = a X + B X)
      const bool reads_c = U.kind != 0;
      const float alpha = U.kind == 1 ? P.c : 1.0f;
      const float beta = U.kind == 1 ? P.b : P.a;
      bool ok = true;
      if (reads_c && U.phase > 0) {
        const int prev_kind = (U.kind + 2) % 3;
        const unsigned* dctr = P.ctr + (long long)U.m * P3 + U.phase - 1;
        ok = dep_wait(dctr, (unsigned)((prev_kind == 2 ? P.t2 : P.t01) * PUBS), abort_flag);
      }
      const __nv_bfloat16* cbase = U.kind == 1 ? P.abuf : P.x[U.step & 1];
      const long long c_ld = U.kind == 1 ? P.a_ld : P.x_ld;
      const long long c_bs = U.kind == 1 ? P.a_bs : P.x_bs;
      const uint8_t* crow = reinterpret_cast<const uint8_t*>(cbase) + ((long long)U.m * c_bs + (long long)row * c_ld) * 2;
      // this row's C for a 64-column chunk: L1-bypassing 16-byte loads (bounds-checked at the edges)
      auto c_load = [&](int gc, uint4 (&cc)[8]) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = gc + 8 * j;
          if (row < M && c + 8 <= N) {
            cc[j] = ld_cg_v4(crow + (long long)c * 2);
          } else {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (row < M)
              for (int i = 0; i < 8; ++i)
                if (c + i < N)
                  w[i >> 1] |= (uint32_t)(*reinterpret_cast<const volatile unsigned short*>(crow + (long long)(c + i) * 2))
                               << (16 * (i & 1));
            cc[j] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      };
      uint4 cc[8];
      if (reads_c && ok && row0 < M && gn0 < N) c_load(gn0, cc);  // the first chunk's C, ahead of the accumulator
      int okw = ok ? 1 : 0;
      if (lane == 0 && okw) okw = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0) & (ok ? 1 : 0);
      if (!__all_sync(0xffffffffu, okw)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * TILE + c0;
      const CUtensorMap* dmap = U.kind == 0 ? &maps.da : (U.kind == 1 ? &maps.db : &maps.dx[(U.step + 1) & 1]);
      bool stored = false;
#pragma unroll
      for (int ch = 0; ch < COLS / 64; ++ch) {
        const int gc = gn0 + ch * 64;
        const bool live = row0 < M && gc < N;  // warp-uniform: this warp stores something of this chunk
        uint4 cn[8];
        if (reads_c && live && ch + 1 < COLS / 64 && gc + 64 < N) c_load(gc + 64, cn);  // the next chunk's C
        uint8_t* buf = sbuf + ch * NS_EPI_STAGE;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {  // two 32-column halves of the 64-column chunk
          uint32_t r[32];
          tmem_ld32(t_row + ch * 64 + hf * 32, r);
          tmem_wait_ld();
          if (ch == COLS / 64 - 1 && hf == 1) {
            // every TMEM read of this warp is done: the accumulator is free for the next tile's MMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (PAIR) mbar_arrive_cluster(tempty_bar0 + acc * 8);
              else mbar_arrive(&tempty_bar[acc]);
            }
          }
          if (!live) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * alpha;
          if (reads_c) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 cq = cc[hf * 4 + q];
              const uint32_t w4[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 cv = unpack_bf16x2(w4[e]);
                v[8 * q + 2 * e] += beta * cv.x;
                v[8 * q + 2 * e + 1] += beta * cv.y;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(ns_stage_ptr(buf, lane, hf * 4 + j)) =
                make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                           pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
        }
        if (live) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ns_tma_store_3d(dmap, buf, gc, row0, U.m);
            ns_bulk_commit();
          }
          stored = true;
        }
        if (ch + 1 < COLS / 64) {
#pragma unroll
          for (int j = 0; j < 8; ++j) cc[j] = cn[j];
        }
      }
      if (++acc == NUM_ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // this warp's part of the tile is complete once its stores have landed (ordered before the release)
      unsigned* my_ctr = P.ctr + (long long)U.m * P3 + U.phase;
      if (lane == 0) {
        if (stored) {
          ns_bulk_wait_all();
          fence_proxy_async_global();
        }
        red_release_add(my_ctr, 1u);
      }
      __syncwarp();
    }
    if (lane == 0) ns_bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // neither CTA frees TMEM or exits while the pair still works
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, NUM_ACC * TILE);
    else tmem_dealloc(tmem_base, NUM_ACC * TILE);
  }
}

}  // namespace rgpt

using namespace rgpt;

// One persistent launch of ns_chain_kernel<PAIR>. Its CTAs wait on one another, so the launch is
// cooperative: all of them are resident at once (one CTA per SM at this shared-memory size), whatever
// else runs on the GPU. Grid: one CTA (or CTA pair) per SM (pair of SMs), at most one per unit.
template <bool PAIR>
static int launch_ns_chain(const NsMaps& maps, const NsParams& P, cudaStream_t s, int dev) {
  auto kern = ns_chain_kernel<PAIR>;
  static bool attr_set[64] = {false};
  static int max_groups[64] = {0};  // co-resident CTAs (CTA pairs)
  const int d = dev < 64 ? dev : 63;
  if (!attr_set[d]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)NS_SMEM) != cudaSuccess)
      return rgpt_check_launch("ns_chain smem attribute");
    if constexpr (PAIR) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * rgpt_num_sms(dev), 1, 1);
      q.blockDim = dim3(NS_THREADS, 1, 1);
      q.dynamicSmemBytes = NS_SMEM;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1)
        return rgpt_set_error(RGPT_ERR_INTERNAL, "no ns_chain CTA pair fits on this GPU (%s)",
                              cudaGetErrorString(cudaGetLastError()));
      max_groups[d] = n;
    } else {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NS_THREADS, NS_SMEM) != cudaSuccess ||
          per_sm < 1)
        return rgpt_set_error(RGPT_ERR_INTERNAL, "ns_chain_kernel does not fit on an SM");
      max_groups[d] = per_sm * rgpt_num_sms(dev);
    }
    attr_set[d] = true;
  }
  const int groups = P.num_units < max_groups[d] ? (int)P.num_units : max_groups[d];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(PAIR ? 2 * groups : groups);
  cfg.blockDim = dim3(NS_THREADS);
  cfg.dynamicSmemBytes = NS_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = PAIR ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, maps, P);
  return rgpt_check_launch(PAIR ? "ns_chain_kernel (CTA pairs)" : "ns_chain_kernel");
}

extern "C" int rgpt_ns_chain(void* X, void* X2, void* A, void* B, int n, int xr, int xc, long long x_ld,
                             long long x_bstride, long long a_ld, long long a_bstride, int steps, float a, float b,
                             float c, unsigned* counters, void* stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int st = rgpt_check_device(dev);
  if (st) return st;
  if (n < 1 || xr < 1 || xc < xr || steps < 1)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_chain needs n >= 1, 1 <= xr <= xc, steps >= 1 (n=%d xr=%d xc=%d)",
                          n, xr, xc);
  if (counters == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_chain needs its counters buffer");
  if (x_ld < xc || a_ld < xr || x_bstride < x_ld * xr || a_bstride < a_ld * xr)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "ns_chain: strides too small");
  // Batches of matrices taller than one 128-row panel run on CTA pairs (256 x 256 tiles: half the operand
  // bytes per SM and MMA); a few matrices (fewer than 32 pair tiles in the A = X X^T phase, e.g. the
  // single-matrix step) keep single-CTA 128 x 128 tiles, whose 4x more units per phase spread each
  // phase over more SMs (measured: 16 x [512, 2048] 303 -> 281 us and 32 x [512, 512] 209 -> 199 us on
  // pairs, but 1 x [512, 2048] 154 -> 197 us).
  const long long pair_tiles = (long long)n * ((xr + 2 * NS_PANEL - 1) / (2 * NS_PANEL)) *
                               ((xr + 2 * NS_PANEL - 1) / (2 * NS_PANEL));
  // RGPT_NS_PAIRS=0 in the environment keeps every class on single-CTA tiles (ncu, for one, cannot replay
  // the cooperative cluster launch of the pair kernel)
  static const bool pairs_allowed = [] {
    const char* v = getenv("RGPT_NS_PAIRS");
    return !(v != nullptr && v[0] == '0');
  }();
  const bool pair = pairs_allowed && xr > NS_PANEL && pair_tiles >= 32;
  const int tile = pair ? 2 * NS_PANEL : NS_PANEL;
  NsMaps maps;
  const void* xs[2] = {X, X2};
  for (int i = 0; i < 2; ++i) {
    if ((st = make_tmap_bf16_3d(&maps.xk[i], xs[i], xc, xr, n, x_ld, x_bstride, NS_BK, NS_PANEL))) return st;
    if ((st = make_tmap_bf16_3d(&maps.xmn[i], xs[i], xc, xr, n, x_ld, x_bstride, 64, NS_BK))) return st;
    if ((st = make_tmap_bf16_3d(&maps.dx[i], xs[i], xc, xr, n, x_ld, x_bstride, 64, 32))) return st;
  }
  if ((st = make_tmap_bf16_3d(&maps.ak, A, xr, xr, n, a_ld, a_bstride, NS_BK, NS_PANEL))) return st;
  if ((st = make_tmap_bf16_3d(&maps.bk, B, xr, xr, n, a_ld, a_bstride, NS_BK, NS_PANEL))) return st;
  if ((st = make_tmap_bf16_3d(&maps.da, A, xr, xr, n, a_ld, a_bstride, 64, 32))) return st;
  if ((st = make_tmap_bf16_3d(&maps.db, B, xr, xr, n, a_ld, a_bstride, 64, 32))) return st;
  NsParams P;
  P.n = n;
  P.xr = xr;
  P.xc = xc;
  P.steps = steps;
  P.mt = (xr + tile - 1) / tile;
  P.nt_r = P.mt;
  P.nt_c = (xc + tile - 1) / tile;
  P.t01 = P.mt * P.nt_r;
  P.t2 = P.mt * P.nt_c;
  P.units_per_step = (long long)n * (2LL * P.t01 + P.t2);
  P.num_units = P.units_per_step * steps;
  P.a = a;
  P.b = b;
  P.c = c;
  P.x[0] = reinterpret_cast<const __nv_bfloat16*>(X);
  P.x[1] = reinterpret_cast<const __nv_bfloat16*>(X2);
  P.abuf = reinterpret_cast<const __nv_bfloat16*>(A);
  P.x_ld = x_ld;
  P.x_bs = x_bstride;
  P.a_ld = a_ld;
  P.a_bs = a_bstride;
  P.ctr = counters;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // counters start at zero (a memset node when captured)
  if (cudaMemsetAsync(counters, 0, sizeof(unsigned) * (size_t)n * 3 * steps, s) != cudaSuccess)
    return rgpt_check_launch("ns_chain counter reset");
  return pair ? launch_ns_chain<true>(maps, P, s, dev) : launch_ns_chain<false>(maps, P, s, dev);
}
