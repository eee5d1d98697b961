// Causal flash attention (head_dim 64) on tcgen05 tensor cores, with the G1
// output gate fused in.
//
// Reference semantics (model/attention.py:52-61):
//   o  = softmax(q k^T / sqrt(64) + causal mask) v       (F.scaled_dot_product_attention)
//   og = o * gate                                        (G1 gate, gate = sigmoid(...))
//
// HBM layouts (token-major, no transposes anywhere):
//   q, k : qk [B*T, 2*d]   columns [0, d) = q heads, [d, 2d) = k heads (post QK-norm + RoPE)
//   v    : qkv[B*T, 3*d]   columns [2d, 3d)  (read in place from the QKV projection output)
//   o, og, gate, do : [B*T, d]
//   lse, D : [B, H, T] fp32
// A 4-D TMA map (64, H, T, B) per operand fetches one 128-row x 64-column tile of
// one head, with rows past T zero-filled.
//
// Forward CTA (192 threads) = one 128-query tile of one (b, h):
//   warp 0 TMA (Q once, then 64-key K and V tiles in separate 3-deep rings)
//   warp 1 TMEM alloc + tcgen05.mma: S = Q K^T into a double-buffered TMEM S, one
//          tile ahead; O += P_j V_j accumulated in TMEM
//   warps 2-5: one thread per query row: online softmax on S (tcgen05.ld), P as
//          bf16 into 128B-swizzled smem for the P V MMA; O rescaled in TMEM only
//          when a row max grows by more than 2^8.
// Backward CTA = one 128-key tile of one (b, h), looping over query tiles in 64-query
//   halves: S^T = K Q^T, dP^T = V dO^T (TMEM, K and V read from TMEM); P^T and dS^T into TMEM
//   (dS^T also into smem); then dV += P^T dO, dK += dS^T Q (TMEM-resident, A from TMEM),
//   dQ = dS K (TMEM -> TMA bulk reduce-add).
//   Two softmax warpgroups take alternate halves, overlapping the MMAs of the other half.
#include <cudaTypedefs.h>
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "rgpt.h"

namespace rgpt {

constexpr int ATT_TILE = 128;   // query rows / keys per tile
constexpr int ATT_D = 64;       // head dim
constexpr int ATT_THREADS = 192;
constexpr uint32_t TILE_BYTES = ATT_TILE * ATT_D * 2;  // 16 KB, one 128x64 bf16 tile

int make_tmap_bf16_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch,
                      uint64_t ld_elems, uint64_t bstride_elems, uint32_t box_inner, uint32_t box_outer);

static PFN_cuTensorMapEncodeTiled_v12000 att_encode_fn() {
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

// (64, H, T, B) view of a token-major [B*T, row_stride] bf16 matrix starting at `base`;
// one box = `box_rows` rows x 64 columns of one head (128-byte swizzle).
static int make_head_map(CUtensorMap* map, const void* base, int H, int T, int B, long long row_stride,
                         int box_rows = ATT_TILE) {
  auto enc = att_encode_fn();
  if (enc == nullptr) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride * 2) % 16 != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "attention operand base/row stride not 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)ATT_D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ATT_D * 2, (cuuint64_t)row_stride * 2, (cuuint64_t)T * row_stride * 2};
  cuuint32_t box[4] = {ATT_D, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return rgpt_set_error(RGPT_ERR_INTERNAL, "attention tensor map encode failed (%d)", (int)r);
  return RGPT_OK;
}

// fp32 (64, H, T, B) view of a token-major [B*T, d] fp32 matrix, 32 x 32 boxes (128-byte swizzle):
// the target of the per-warp dQ bulk reduce-adds.
static int make_head_map_f32(CUtensorMap* map, const float* base, int H, int T, int B, long long row_stride) {
  auto enc = att_encode_fn();
  if (enc == nullptr) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride * 4) % 16 != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "dq base/row stride not 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)ATT_D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ATT_D * 4, (cuuint64_t)row_stride * 4, (cuuint64_t)T * row_stride * 4};
  cuuint32_t box[4] = {32, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return rgpt_set_error(RGPT_ERR_INTERNAL, "dq tensor map encode failed (%d)", (int)r);
  return RGPT_OK;
}

// bf16 (64, H, T, B) view with 32-row x 32-column boxes and no swizzle (64-byte smem rows): the
// target of the per-warp dV bulk stores.
static int make_head_map_bf16_32(CUtensorMap* map, const void* base, int H, int T, int B, long long row_stride) {
  auto enc = att_encode_fn();
  if (enc == nullptr) return rgpt_set_error(RGPT_ERR_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride * 2) % 16 != 0)
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "dv base/row stride not 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)ATT_D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ATT_D * 2, (cuuint64_t)row_stride * 2, (cuuint64_t)T * row_stride * 2};
  cuuint32_t box[4] = {32, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return rgpt_set_error(RGPT_ERR_INTERNAL, "dv tensor map encode failed (%d)", (int)r);
  return RGPT_OK;
}

// Bulk add of a 32 x 32 fp32 smem tile into global memory through a tensor map (rows past the
// tensor's extent are skipped by the hardware). Coordinates are never negative here.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2,
                                                  int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Store 8 fp32 values of row `r` (as bf16) into 16-byte chunk `chunk` of a
// 128-row x 64-column K-major SW128 tile.
__device__ __forceinline__ void st_sw128_chunk(uint8_t* tile, int r, int chunk, const float* v) {
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(tile + r * 128 + ((chunk ^ (r & 7)) << 4)) = o;
}

// ============================================================================ forward
struct AttnFwdParams {
  int B, T, H, d;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;  // [B*T, d]
  __nv_bfloat16* og; // [B*T, d] (gated) or null
  const __nv_bfloat16* gate;  // [B*T, d] or null
  float* lse;        // [B, H, T] natural-log LSE of the scaled scores
  // dropout of the attention probabilities (SDPA dropout_p, model/attention.py:57), DROP kernels only:
  // the keep bit of (query q, key k) of head bh is bit q % 32 of drop_mask[(bh * ceil(T/32) + q / 32) * T
  // + k], filled beforehand by attn_drop_mask_kernel (one word per key and 32 queries)
  const uint32_t* drop_mask;
  float drop_scale;
};

constexpr int FWD_KT = 64;                                  // keys per tile in the forward
constexpr int FWD_KV_STAGES = 3;                            // K and V rings (separate barriers)
constexpr uint32_t KV_TILE_BYTES = FWD_KT * ATT_D * 2;      // 8 KB
constexpr uint32_t P_TILE_BYTES = ATT_TILE * FWD_KT * 2;    // 16 KB: [128 queries x 64 keys] bf16
constexpr float FWD_RESCALE_LOG2 = 8.0f;                    // rescale O only when a row max grows by > 2^8

// Forward CTA: 128 queries of one (b, h), 64-key tiles, two CTAs per SM (256 TMEM columns and
// ~97 KB of smem each) so one CTA's softmax overlaps the other's tensor-core work.
// MMA order: S(0), then per tile j: S(j+1), O += P(j) V(j); the softmax of tile j+1 thus
// overlaps P(j) V(j). O accumulates in TMEM. The running row max used for P is only raised
// when the tile max exceeds it by more than 2^8 (P then stays below 2^8, well inside bf16);
// that rare rescale multiplies O in TMEM after the previous P V has landed.
template <bool DROP>
__global__ void __launch_bounds__(ATT_THREADS, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmG,
                    const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmOG,
                    AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                    // 16 KB
  uint8_t* sK = sQ + TILE_BYTES;                         // FWD_KV_STAGES x 8 KB
  uint8_t* sV = sK + FWD_KV_STAGES * KV_TILE_BYTES;      // FWD_KV_STAGES x 8 KB
  uint8_t* sP = sV + FWD_KV_STAGES * KV_TILE_BYTES;      // 2 x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                        // [FWD_KV_STAGES]
  uint64_t* k_empty = k_full + FWD_KV_STAGES;         // [FWD_KV_STAGES]
  uint64_t* v_full = k_empty + FWD_KV_STAGES;         // [FWD_KV_STAGES]
  uint64_t* v_empty = v_full + FWD_KV_STAGES;         // [FWD_KV_STAGES]
  uint64_t* s_full = v_empty + FWD_KV_STAGES;         // [2]
  uint64_t* s_empty = s_full + 2;                     // [2]
  uint64_t* p_full = s_empty + 2;                     // [2]
  uint64_t* pv_done = p_full + 2;                     // [2] P V of the tile using P buffer i has landed
  uint64_t* g_full = pv_done + 2;                     // gate tile landed in sQ (after the last S)
  uint64_t* q_free = g_full + 1;                      // the last S MMA (last reader of Q) has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + ATT_TILE - 1) / ATT_TILE;
  // one linear grid, heaviest query tiles (longest causal rows) of every (b, h) first, so the
  // last CTAs to start are the shortest ones
  const int bh = blockIdx.x % (p.H * p.B);
  const int qt = n_qt - 1 - (int)(blockIdx.x / (p.H * p.B));
  const int h = bh % p.H, b = bh / p.H;
  const int q0 = qt * ATT_TILE;
  const int last_key = min(q0 + ATT_TILE - 1, p.T - 1);
  const int nkv = last_key / FWD_KT + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < FWD_KV_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(g_full, 1);
    mbar_init(q_free, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // every operand and output lives in memory the previous kernels use
  griddep_launch();
  constexpr uint32_t O_COL = 128;  // TMEM columns: S0 [0,64) S1 [64,128) O [128,192)

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_4d(sQ, &tmQ, q_full, 0, h, q0, b);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j % FWD_KV_STAGES;
        const uint32_t ph = ((j / FWD_KV_STAGES) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], ph, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], KV_TILE_BYTES);
        tma_load_4d(sK + st * KV_TILE_BYTES, &tmK, &k_full[st], 0, h, j * FWD_KT, b);
        ++issued_k;
        if (!mbar_wait(&v_empty[st], ph, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], KV_TILE_BYTES);
        tma_load_4d(sV + st * KV_TILE_BYTES, &tmV, &v_full[st], 0, h, j * FWD_KT, b);
        ++issued_v;
      }
      // the gate tile reuses sQ once the last S MMA (the last reader of Q) has completed
      if (ok && p.og != nullptr) {
        if (mbar_wait(q_free, 0, abort_flag)) {
          mbar_arrive_expect_tx(g_full, TILE_BYTES);
          tma_load_4d(sQ, &tmG, g_full, 0, h, q0, b);
          mbar_wait(g_full, 0, nullptr);  // the copy lands before this thread moves on
        } else {
          ok = false;
        }
      }
      if (!ok) {  // let the copies already issued land before the CTA retires
        mbar_wait(q_full, 0, nullptr);
        for (int j = max(0, issued_k - FWD_KV_STAGES); j < issued_k; ++j)
          mbar_wait(&k_full[j % FWD_KV_STAGES], (j / FWD_KV_STAGES) & 1, nullptr);
        for (int j = max(0, issued_v - FWD_KV_STAGES); j < issued_v; ++j)
          mbar_wait(&v_full[j % FWD_KV_STAGES], (j / FWD_KV_STAGES) & 1, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = make_idesc_bf16(128, FWD_KT, 0, 0);
      constexpr uint32_t IDESC_O = make_idesc_bf16(128, 64, 0, 1);
      bool ok = mbar_wait(q_full, 0, abort_flag);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j % FWD_KV_STAGES, sb = j & 1;
        if (!mbar_wait(&k_full[st], (j / FWD_KV_STAGES) & 1, abort_flag)) return false;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * KV_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < ATT_D / 16; ++kk)
          umma_bf16(tmem + sb * 64, make_sw128_desc(q_addr + kk * 32, 16, 1024),
                    make_sw128_desc(k_addr + kk * 32, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j % FWD_KV_STAGES, pb = j & 1;
        if (!mbar_wait(&p_full[pb], (j >> 1) & 1, abort_flag)) return false;
        if (!mbar_wait(&v_full[st], (j / FWD_KV_STAGES) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + pb * P_TILE_BYTES);
        const uint32_t v_addr = smem_u32(sV + st * KV_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < FWD_KT / 16; ++kk)
          umma_bf16(tmem + O_COL, make_sw128_desc(p_addr + kk * 32, 16, 1024),
                    make_sw128_desc(v_addr + kk * 2048, KV_TILE_BYTES, 1024), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[pb]);
        umma_commit(&v_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !issue_s(j + 1)) ok = false;
        if (ok && j + 1 == nkv - 1) umma_commit(q_free);  // after the last S
        if (ok && !issue_pv(j)) ok = false;
      }
      if (ok && nkv == 1) umma_commit(q_free);
    }
    __syncwarp();
  } else {
    // softmax / epilogue: one thread per query row
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qrow = q0 + r;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    const int drop_qb = (q0 >> 5) + quarter;  // this warp's 32-query block of the dropout mask

    auto wait_all = [&](uint64_t* bar, uint32_t ph) -> bool {
      int v = 1;
      if (lane == 0) v = mbar_wait(bar, ph, abort_flag) ? 1 : 0;
      return __shfl_sync(0xffffffffu, v, 0) != 0;
    };

    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      uint32_t mw[2] = {0u, 0u};  // dropout words of keys j*64 + c*32 + lane over this warp's queries
      if constexpr (DROP) {
        const int nqb = (p.T + 31) >> 5;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int key = j * FWD_KT + c * 32 + lane;
          if (key < p.T && drop_qb < nqb) mw[c] = __ldg(p.drop_mask + ((long long)bh * nqb + drop_qb) * p.T + key);
        }
      }
      if (!wait_all(&s_full[sb], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kbase = j * FWD_KT;
      const bool masked = (kbase + FWD_KT > q0) || (kbase + FWD_KT > p.T);  // tiles on the diagonal / past T
      uint32_t v[2][32];
      tmem_ld32(t_lane + sb * 64, v[0]);
      tmem_ld32(t_lane + sb * 64 + 32, v[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);  // S is in registers now; the TMEM buffer can be refilled
      if (masked) {  // causal mask and keys past T (warp-uniform branch)
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int key = kbase + c * 32 + t;
            if (key > qrow || key >= p.T) v[c][t] = __float_as_uint(-INFINITY);
          }
      }
      // row max of the raw scores (the scale is positive), four independent chains of 3-input max
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int t = 0; t < 32; t += 2)
          mx4[(t >> 1) & 3] = fmax3(mx4[(t >> 1) & 3], __uint_as_float(v[c][t]), __uint_as_float(v[c][t + 1]));
      const float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      // raise the running max only when P would otherwise exceed 2^8 (always on the first tile)
      const bool raise = mt > m_run + FWD_RESCALE_LOG2;
      float alpha = 1.f;
      if (raise) {
        alpha = ex2_approx(m_run - mt);  // 0 on the first tile
        m_run = mt;
        l_run *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        // O holds P V of tiles < j: wait for the last of them, then scale the raised rows
        if (!wait_all(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(t_lane + O_COL + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st32(t_lane + O_COL + c * 32, o);
        }
        tmem_wait_st();
      }
      // the P buffer was last read by P V of tile j - 2
      if (j >= 2 && !wait_all(&pv_done[sb], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      // P = exp2(s * scale_log2 - m) with the FMAs and the row-sum adds on packed fp32 pairs
      float2 sum_a = make_float2(0.f, 0.f), sum_b = sum_a;
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_run, -m_run);
      uint8_t* pbuf = sP + sb * P_TILE_BYTES;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float pv[32];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const float2 x = ffma2(make_float2(__uint_as_float(v[c][t]), __uint_as_float(v[c][t + 1])), sc2, nm2);
          pv[t] = ex2_approx(x.x);
          pv[t + 1] = ex2_approx(x.y);
        }
#pragma unroll
        for (int t = 0; t < 32; t += 4) {
          sum_a = fadd2(sum_a, make_float2(pv[t], pv[t + 1]));
          sum_b = fadd2(sum_b, make_float2(pv[t + 2], pv[t + 3]));
        }
        if constexpr (DROP) {
          // the row sum keeps every probability; P V sees only the kept ones (1/(1-p) is applied to O).
          // The loaded words hold one key's bits over the warp's 32 queries; transposed, lane t holds
          // its own query's bits over the chunk's 32 keys.
          const uint32_t keep = warp_transpose_bits(mw[c], lane);
#pragma unroll
          for (int t = 0; t < 32; ++t) pv[t] = ((keep >> t) & 1u) ? pv[t] : 0.f;
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) st_sw128_chunk(pbuf, r, c * 4 + t, pv + 8 * t);
      }
      l_run += (sum_a.x + sum_a.y) + (sum_b.x + sum_b.y);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // every P V has landed once the last one has (in-order tensor pipe)
    if (ok) ok = wait_all(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1);
    if (ok) {
      // O / l as bf16 (and og = bf16(o) * gate) staged in the free P buffers as 128B-swizzled rows,
      // then written by TMA bulk stores, one 32-row box per warp (rows past T are clipped)
      tc_fence_after();
      uint32_t o[2][32];
      tmem_ld32(t_lane + O_COL, o[0]);
      tmem_ld32(t_lane + O_COL + 32, o[1]);
      tmem_wait_ld();
      const float inv_l = (DROP ? p.drop_scale : 1.0f) / l_run;
      float ov[ATT_D];
#pragma unroll
      for (int i = 0; i < ATT_D; ++i) ov[i] = __uint_as_float(o[i >> 5][i & 31]) * inv_l;
      uint8_t* so = sP;                 // o tile  [128 x 64] bf16
      uint8_t* sog = sP + P_TILE_BYTES;  // og tile [128 x 64] bf16
#pragma unroll
      for (int c = 0; c < 8; ++c) st_sw128_chunk(so, r, c, ov + 8 * c);
      const bool gated = p.og != nullptr;
      if (gated) {
        if (!wait_all(g_full, 0)) ok = false;
        if (ok) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 g = *reinterpret_cast<const uint4*>(sQ + r * 128 + ((c ^ (r & 7)) << 4));
            const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
            float gv[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 gf = unpack_bf16x2(gw[e]);
              // gate the bf16-rounded o, as the reference multiplies the stored attention output
              gv[2 * e] = bf16_round(ov[8 * c + 2 * e]) * gf.x;
              gv[2 * e + 1] = bf16_round(ov[8 * c + 2 * e + 1]) * gf.y;
            }
            st_sw128_chunk(sog, r, c, gv);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (ok && lane == 0 && q0 + quarter * 32 < p.T) {
        tma_store_4d(&tmO, so + quarter * 32 * 128, 0, h, q0 + quarter * 32, b);
        if (gated) tma_store_4d(&tmOG, sog + quarter * 32 * 128, 0, h, q0 + quarter * 32, b);
        bulk_commit();
      }
      // natural-log LSE of the scaled scores
      if (qrow < p.T) p.lse[((long long)b * p.H + h) * p.T + qrow] = (m_run + log2f(l_run)) * 0.69314718055994531f;
      if (lane == 0) bulk_wait0();  // the stores have read the staging tiles before the CTA retires
      __syncwarp();
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ============================================================================ dropout mask
// Keep bits of the attention probabilities for every causal (query, key) pair: the bit of (q, k) of head
// bh comes from Philox4x32-10 block (k / 8, q, site, bh) under key (seed low, high 32 bits) -- the 16-bit
// uniform (k % 8) -> word (k % 8) / 2, half k % 2 -- kept iff >= thresh. A warp draws 32 keys for its 32
// queries (one row of bits per lane), transposes them and stores one coalesced word per key:
// mask[(bh * ceil(T/32) + q / 32) * T + k] bit q % 32. Block = one (bh, 32-query block), its 4 warps
// stride over the key chunks that any of the block's queries can see.
__global__ void __launch_bounds__(128) attn_drop_mask_kernel(uint32_t* __restrict__ mask,
                                                             const unsigned long long* __restrict__ seed,
                                                             uint32_t site, uint32_t thresh, int BH, int T) {
  griddep_wait();
  griddep_launch();
  const int nqb = (T + 31) >> 5;
  const int bh = blockIdx.x / nqb, qb = blockIdx.x % nqb;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned long long sd = *seed;
  const uint32_t k0 = (uint32_t)sd, k1 = (uint32_t)(sd >> 32);
  const int q = qb * 32 + lane;
  uint32_t* row = mask + ((long long)bh * nqb + qb) * T;
  for (int c = warp; c <= qb; c += 4) {  // keys [32c, 32c + 32) reach the block's last query
    const uint32_t keep = keep32((uint32_t)(c * 32), (uint32_t)q, site, (uint32_t)bh, k0, k1, thresh);
    const uint32_t kw = warp_transpose_bits(keep, lane);
    if (c * 32 + lane < T) row[c * 32 + lane] = kw;
  }
}

// ============================================================================ backward prep
// do = dog * gate; dgate_pre = dog * o * gate * (1 - gate); D = rowsum(do * o)   (8 threads per (token, head))
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ dog, const __nv_bfloat16* __restrict__ o,
                                     const __nv_bfloat16* __restrict__ gate, __nv_bfloat16* __restrict__ dout,
                                     __nv_bfloat16* __restrict__ dgate_pre, float* __restrict__ Dvec,
                                     float* __restrict__ dq_zero, int B, int T, int H, int d) {
  griddep_wait();
  griddep_launch();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long rowhead = gid >> 3;  // (token, head) index
  const int part = gid & 7;
  const long long total = (long long)B * T * H;
  const bool valid = rowhead < total;
  const long long tok = valid ? rowhead / H : 0;
  const int h = valid ? (int)(rowhead % H) : 0;
  const long long off = tok * d + h * ATT_D + part * 8;
  float dsum = 0.f;
  if (valid) {
    uint4 vg = *reinterpret_cast<const uint4*>(dog + off);
    uint4 vo = *reinterpret_cast<const uint4*>(o + off);
    uint32_t g4[4] = {vg.x, vg.y, vg.z, vg.w}, o4[4] = {vo.x, vo.y, vo.z, vo.w};
    uint32_t do4[4], dg4[4];
    uint4 vgate = gate ? *reinterpret_cast<const uint4*>(gate + off) : make_uint4(0, 0, 0, 0);
    uint32_t gt4[4] = {vgate.x, vgate.y, vgate.z, vgate.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 gg = unpack_bf16x2(g4[e]);
      float2 oo = unpack_bf16x2(o4[e]);
      float2 gt = gate ? unpack_bf16x2(gt4[e]) : make_float2(1.f, 1.f);
      float d0 = gg.x * gt.x, d1 = gg.y * gt.y;
      do4[e] = pack_bf16x2(d0, d1);
      float2 dr = unpack_bf16x2(do4[e]);  // D uses the rounded dO that the MMAs see
      dsum += dr.x * oo.x + dr.y * oo.y;
      dg4[e] = pack_bf16x2(gg.x * oo.x * gt.x * (1.f - gt.x), gg.y * oo.y * gt.y * (1.f - gt.y));
    }
    *reinterpret_cast<uint4*>(dout + off) = make_uint4(do4[0], do4[1], do4[2], do4[3]);
    if (gate) *reinterpret_cast<uint4*>(dgate_pre + off) = make_uint4(dg4[0], dg4[1], dg4[2], dg4[3]);
    if (dq_zero) {  // the attention backward accumulates dQ into this [B*T, d] fp32 buffer
      float4* z = reinterpret_cast<float4*>(dq_zero + off);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
  dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
  dsum += __shfl_xor_sync(0xffffffffu, dsum, 4);
  if (valid && part == 0) {
    const long long b = tok / T, t = tok % T;
    Dvec[(b * H + h) * T + t] = dsum;
  }
}

// ============================================================================ backward
struct AttnBwdParams {
  int B, T, H, d;
  float scale;       // softmax scale (1/sqrt(64))
  float scale_log2;  // scale * log2(e)
  const float* lse;  // [B, H, T] natural log
  const float* Dvec; // [B, H, T]
  float* dk;         // [B*T, dk_stride] fp32
  long long dk_stride;
  __nv_bfloat16* dv; // [B*T, dv_stride] bf16
  long long dv_stride;
  const uint32_t* drop_mask;  // DROP kernels: the forward's attention-probability keep bits
  float drop_scale;           // 1 / (1 - p)
};

constexpr int ATT_BWD_THREADS = 320;  // TMA warp, MMA warp, 8 softmax/epilogue warps
constexpr uint32_t DQ_STAGE_BYTES = 32 * 32 * 4;  // one warp's 32 x 32 fp32 dQ tile
constexpr int BWD_STAT_FLOATS = 128;              // one warp's 64 query LSEs (log2 units) + 64 D values

// Backward CTA = one 128-key tile of one (b, h), looping over the query tiles that see
// these keys, each split into two 64-query halves. Softmax warpgroup g (warps 2-5: g = 0,
// warps 6-9: g = 1) handles half g of every query tile, so the two halves are computed
// concurrently, and the MMA warp issues the next tile's S/dP half as soon as a warpgroup has
// handed over this tile's P/dS half:
//   tensor pipe: SD(0,0) SD(0,1) VK(0,0) SD(1,0) VK(0,1) SD(1,1) Q(0) VK(1,0) SD(2,0) ...
//   SD(t,g): S^T and dP^T of half g (TMEM buffer g), VK(t,g): dV += P^T dO, dK += dS^T Q on
//   half g, Q(t): dQ = dS K for the whole tile (reads both halves' dS).
// A warpgroup stores its next P/dS half only after Q of the previous tile has completed (it
// reads both dS halves), and writes that tile's dQ (TMEM -> TMA bulk reduce-add) right after.
template <bool DROP>
__global__ void __launch_bounds__(ATT_BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmDK,
                    const __grid_constant__ CUtensorMap tmDV, AttnBwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;                     // 16 KB
  uint8_t* sV = sK + TILE_BYTES;          // 16 KB
  uint8_t* sQ = sV + TILE_BYTES;          // 2 x 16 KB (query-tile ring)
  uint8_t* sDO = sQ + 2 * TILE_BYTES;     // 2 x 16 KB
  uint8_t* sDS = sDO + 2 * TILE_BYTES;    // dS^T: 2 atoms (query half 0, 1) x 16 KB (P^T lives in TMEM)
  uint8_t* sDQ = sDS + 2 * TILE_BYTES;    // 8 x 4 KB dQ staging (one per softmax warp)
  float* sStat = reinterpret_cast<float*>(sDQ + 8 * DQ_STAGE_BYTES);  // 8 warps x [64 lse*log2(e) | 64 D]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStat + 8 * BWD_STAT_FLOATS);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;   // [2] query-tile ring
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* sdp_full = bars + 5;  // [2] S^T/dP^T of half g in TMEM buffer g
  uint64_t* ds_ready = bars + 7;  // [2] P^T/dS^T of half g in smem (and its S/dP read)
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_empty = bars + 10;
  uint64_t* kv_tmem = bars + 11;  // K and V copied into TMEM (the A operands of S^T / dP^T)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // one linear grid, heaviest key tiles (most query tiles: lowest index) of every (b, h) first
  const int bh = blockIdx.x % (p.H * p.B);
  const int kt = (int)(blockIdx.x / (p.H * p.B));
  const int h = bh % p.H, b = bh / p.H;
  const int k0 = kt * ATT_TILE;
  const int n_qt = (p.T + ATT_TILE - 1) / ATT_TILE;
  const int qt0 = kt;  // query tiles qt >= kt see these keys
  const int nq = n_qt - qt0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&sdp_full[i], 1);
      mbar_init(&ds_ready[i], 128);
    }
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 256);
    mbar_init(kv_tmem, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmDQ);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // every operand and output lives in memory the previous kernels use
  griddep_launch();
  // TMEM columns: half g: S^T [128g, 128g+64) dP^T [128g+64, 128g+128), overwritten after the softmax by
  // P^T [128g, 128g+32) and dS^T [128g+32, 128g+64) as packed bf16 pairs; dV [256,320) dK [320,384)
  // dQ [384,448); K [448,480) and V [480,512) as packed bf16 pairs (A operands read from TMEM).
  constexpr uint32_t KA_COL = 448, VA_COL = 480;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_4d(sK, &tmK, kv_full, 0, h, k0, b);
      tma_load_4d(sV, &tmV, kv_full, 0, h, k0, b);
      for (int i = 0; i < nq && ok; ++i) {
        const int s = i & 1;
        if (!mbar_wait(&qd_empty[s], ((i >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const int qrow0 = (qt0 + i) * ATT_TILE;
        mbar_arrive_expect_tx(&qd_full[s], 2 * TILE_BYTES);
        tma_load_4d(sQ + s * TILE_BYTES, &tmQ, &qd_full[s], 0, h, qrow0, b);
        tma_load_4d(sDO + s * TILE_BYTES, &tmDO, &qd_full[s], 0, h, qrow0, b);
      }
      if (!ok) {
        mbar_wait(kv_full, 0, nullptr);
        for (int s = 0; s < 2; ++s) mbar_wait(&qd_full[s], 0, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = make_idesc_bf16(128, 64, 0, 0);    // K Q_g^T, V dO_g^T (64 queries)
      constexpr uint32_t IDESC_KV = make_idesc_bf16(128, 64, 0, 1);   // P_g^T dO_g, dS_g^T Q_g (B MN-major)
      constexpr uint32_t IDESC_Q = make_idesc_bf16(128, 64, 1, 1);    // dS K (A, B MN-major)
      bool ok = mbar_wait(kv_full, 0, abort_flag) && mbar_wait(kv_tmem, 0, abort_flag);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t ds_addr = smem_u32(sDS);
      // S^T and dP^T of half g of query tile t into TMEM buffer g
      auto issue_sd = [&](int t, int g) {
        const int s = t & 1;
        const uint32_t q_addr = smem_u32(sQ + s * TILE_BYTES) + g * 8192;
        const uint32_t do_addr = smem_u32(sDO + s * TILE_BYTES) + g * 8192;
#pragma unroll
        for (int kk = 0; kk < ATT_D / 16; ++kk) {  // A = K / V rows from TMEM, 8 columns per 16 head dims
          umma_bf16_ts(tmem + g * 128, tmem + KA_COL + kk * 8, make_sw128_desc(q_addr + kk * 32, 16, 1024), IDESC_S,
                       kk > 0 ? 1u : 0u);
          umma_bf16_ts(tmem + g * 128 + 64, tmem + VA_COL + kk * 8, make_sw128_desc(do_addr + kk * 32, 16, 1024),
                       IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sdp_full[g]);
      };
      // dV += P_g^T dO_g ; dK += dS_g^T Q_g  (64 queries of half g as the K dimension)
      auto issue_vk = [&](int t, int g) {
        const int s = t & 1;
        const uint32_t q_addr = smem_u32(sQ + s * TILE_BYTES) + g * 8192;
        const uint32_t do_addr = smem_u32(sDO + s * TILE_BYTES) + g * 8192;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // A = P^T / dS^T of half g from TMEM, 8 columns per 16 queries
          const uint32_t acc = (t > 0 || g > 0 || kk > 0) ? 1u : 0u;
          umma_bf16_ts(tmem + 256, tmem + g * 128 + kk * 8, make_sw128_desc(do_addr + kk * 2048, TILE_BYTES, 1024),
                       IDESC_KV, acc);
          umma_bf16_ts(tmem + 320, tmem + g * 128 + 32 + kk * 8,
                       make_sw128_desc(q_addr + kk * 2048, TILE_BYTES, 1024), IDESC_KV, acc);
        }
      };
      // dQ = dS K over the whole tile: A = dS^T atoms read MN-major (rows = keys), B = K MN-major
      auto issue_q = [&]() {
#pragma unroll
        for (int kk = 0; kk < ATT_TILE / 16; ++kk)
          umma_bf16(tmem + 384, make_sw128_desc(ds_addr + kk * 2048, TILE_BYTES, 1024),
                    make_sw128_desc(k_addr + kk * 2048, TILE_BYTES, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
      };
      if (ok && nq > 0) {
        ok = mbar_wait(&qd_full[0], 0, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_sd(0, 0);
          issue_sd(0, 1);
        }
      }
      for (int t = 0; t < nq && ok; ++t) {
        for (int g = 0; g < 2 && ok; ++g) {
          if (!mbar_wait(&ds_ready[g], t & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_vk(t, g);
          if (g == 1) umma_commit(&qd_empty[t & 1]);  // the last reader of this tile's Q / dO
          if (t + 1 < nq) {
            if (g == 0 && !mbar_wait(&qd_full[(t + 1) & 1], ((t + 1) >> 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_sd(t + 1, g);  // buffer g was read before ds_ready[g] arrived
          }
        }
        if (!ok) break;
        if (t > 0 && !mbar_wait(dq_empty, (t - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_q();
      }
    }
    __syncwarp();
  } else {
    const int sw = warp - 2;            // 0..7
    const int quarter = warp & 3;       // TMEM lane quadrant
    const int g = sw >> 2;              // softmax warpgroup = query half it handles
    const int r = quarter * 32 + lane;  // key row (S^T / dP^T / dV / dK) and query row (dQ)
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* stage = sDQ + sw * DQ_STAGE_BYTES;
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t ph) -> bool {
      int v = 1;
      if (lane == 0) v = mbar_wait(bar, ph, abort_flag) ? 1 : 0;
      return __shfl_sync(0xffffffffu, v, 0) != 0;
    };
    const float* lse_bh = p.lse + ((long long)b * p.H + h) * p.T;
    const float* D_bh = p.Dvec + ((long long)b * p.H + h) * p.T;
    float* wstat = sStat + sw * BWD_STAT_FLOATS;
    uint8_t* datom = sDS + g * TILE_BYTES;
    if (g == 0) {  // K and V rows (this thread's key row r) into TMEM as packed bf16 pairs
      ok = wait_all(kv_full, 0);
      if (ok) {
        uint32_t w[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 v4 = *reinterpret_cast<const uint4*>(sK + r * 128 + ((j ^ (r & 7)) << 4));
          w[4 * j] = v4.x, w[4 * j + 1] = v4.y, w[4 * j + 2] = v4.z, w[4 * j + 3] = v4.w;
        }
        tmem_st32(t_lane + KA_COL, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 v4 = *reinterpret_cast<const uint4*>(sV + r * 128 + ((j ^ (r & 7)) << 4));
          w[4 * j] = v4.x, w[4 * j + 1] = v4.y, w[4 * j + 2] = v4.z, w[4 * j + 3] = v4.w;
        }
        tmem_st32(t_lane + VA_COL, w);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(kv_tmem);
    }
    // P^T = exp2(S^T * scale*log2(e) - lse*log2(e)) and dS^T/scale = P^T (dP^T - D) for 32
    // queries (chunk cc of this half) of this thread's key row, in registers. Queries past T
    // carry lse = +inf (P = 0); keys past T need no mask (their K/V rows are zero and their
    // dK/dV rows are never stored).
    // With dropout (keep bits kw over the chunk's 32 queries, z = kept / (1-p)): P~ = P z feeds dV and
    // dS = P (z dP~ - D), dP~ = dO V^T being what the dP^T MMA computed.
    auto softmax_chunk = [&](auto mask_tag, int cc, uint4 (&pk)[4], uint4 (&dk)[4], uint32_t kw) {
      constexpr bool MASK = decltype(mask_tag)::value;
      uint32_t sv[32], dv[32];
      tmem_ld32(t_lane + g * 128 + cc * 32, sv);
      tmem_ld32(t_lane + g * 128 + 64 + cc * 32, dv);
      tmem_wait_ld();
      const float4* l4 = reinterpret_cast<const float4*>(wstat + cc * 32);
      const float4* d4 = reinterpret_cast<const float4*>(wstat + 64 + cc * 32);
      float pr[8], ds[8];
#pragma unroll
      for (int t4 = 0; t4 < 8; ++t4) {
        const float4 l = l4[t4], dd = d4[t4];
        const float la[4] = {l.x, l.y, l.z, l.w}, da[4] = {dd.x, dd.y, dd.z, dd.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t_ = 4 * t4 + e;
          float pv = ex2_approx(fmaf(__uint_as_float(sv[t_]), p.scale_log2, -la[e]));
          if constexpr (MASK) pv = (g * 64 + cc * 32 + t_ < r) ? 0.f : pv;  // causal: query before key
          if constexpr (DROP) {
            const float z = ((kw >> t_) & 1u) ? p.drop_scale : 0.f;
            pr[t_ & 7] = pv * z;
            ds[t_ & 7] = pv * fmaf(__uint_as_float(dv[t_]), z, -da[e]);
          } else {
            pr[t_ & 7] = pv;
            ds[t_ & 7] = pv * (__uint_as_float(dv[t_]) - da[e]);
          }
        }
        if (t4 & 1) {  // 8 values -> one 16-byte chunk of bf16
          pk[t4 >> 1] = make_uint4(pack_bf16x2(pr[0], pr[1]), pack_bf16x2(pr[2], pr[3]), pack_bf16x2(pr[4], pr[5]),
                                   pack_bf16x2(pr[6], pr[7]));
          dk[t4 >> 1] = make_uint4(pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]), pack_bf16x2(ds[4], ds[5]),
                                   pack_bf16x2(ds[6], ds[7]));
        }
      }
    };
    // dQ rows of tile i (TMEM lane = query row), this warp's 32 of the 64 head columns
    auto dq_out = [&](int i) -> bool {
      if (!wait_all(dq_full, i & 1)) return false;
      tc_fence_after();
      const int qrow0 = (qt0 + i) * ATT_TILE;
      uint32_t v[32];
      tmem_ld32(t_lane + 384 + g * 32, v);
      tmem_wait_ld();
      if (lane == 0) bulk_wait_read0();  // the previous bulk reduce has finished reading the stage
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_float4(__uint_as_float(v[4 * j]) * p.scale, __uint_as_float(v[4 * j + 1]) * p.scale,
                        __uint_as_float(v[4 * j + 2]) * p.scale, __uint_as_float(v[4 * j + 3]) * p.scale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && qrow0 + quarter * 32 < p.T) {  // boxes wholly past T carry only zeros
        tma_reduce_add_4d(&tmDQ, stage, g * 32, h, qrow0 + quarter * 32, b);
        bulk_commit();
      }
      tc_fence_before();
      mbar_arrive(dq_empty);
      return true;
    };
    const int key = k0 + r;
    for (int i = 0; i < nq && ok; ++i) {
      const int qrow0 = (qt0 + i) * ATT_TILE;
      uint32_t kw0 = 0, kw1 = 0;  // dropout keep bits of this key over the half's two 32-query chunks
      if constexpr (DROP) {
        const int qb = (qrow0 + g * 64) >> 5, nqb = (p.T + 31) >> 5;
        const uint32_t* mrow = p.drop_mask + ((long long)bh * nqb + qb) * p.T + key;
        if (key < p.T && qb < nqb) kw0 = __ldg(mrow);
        if (key < p.T && qb + 1 < nqb) kw1 = __ldg(mrow + p.T);
      }
      {  // this warp's 64 queries: LSE in log2 units and D, staged for broadcast reads
        const int qa = qrow0 + g * 64 + lane, qb = qa + 32;
        const float la = qa < p.T ? __ldg(lse_bh + qa) * 1.4426950408889634f : INFINITY;
        const float lb = qb < p.T ? __ldg(lse_bh + qb) * 1.4426950408889634f : INFINITY;
        const float da = qa < p.T ? __ldg(D_bh + qa) : 0.f;
        const float db = qb < p.T ? __ldg(D_bh + qb) : 0.f;
        __syncwarp();
        wstat[lane] = la;
        wstat[32 + lane] = lb;
        wstat[64 + lane] = da;
        wstat[96 + lane] = db;
        __syncwarp();
      }
      if (!wait_all(&sdp_full[g], i & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint4 pk[2][4], dk[2][4];  // P^T / dS^T as bf16, 16-byte chunks of this key row
      if (i == 0) {  // the diagonal tile (query tile == key tile)
        softmax_chunk(std::true_type{}, 0, pk[0], dk[0], kw0);
        softmax_chunk(std::true_type{}, 1, pk[1], dk[1], kw1);
      } else {
        softmax_chunk(std::false_type{}, 0, pk[0], dk[0], kw0);
        softmax_chunk(std::false_type{}, 1, pk[1], dk[1], kw1);
      }
      // dQ of the previous tile reads both dS halves: it must have completed before we overwrite
      if (i > 0 && !dq_out(i - 1)) {
        ok = false;
        break;
      }
      // P^T and dS^T of this key row into TMEM (A operands of dV / dK); dS^T also into smem for dQ
      {
        uint32_t pw[32], dw[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint4 a = pk[cc][t], d4 = dk[cc][t];
            const int o = cc * 16 + t * 4;
            pw[o] = a.x, pw[o + 1] = a.y, pw[o + 2] = a.z, pw[o + 3] = a.w;
            dw[o] = d4.x, dw[o + 1] = d4.y, dw[o + 2] = d4.z, dw[o + 3] = d4.w;
          }
        tmem_st32(t_lane + g * 128, pw);
        tmem_st32(t_lane + g * 128 + 32, dw);
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int ch = cc * 4 + t;
          *reinterpret_cast<uint4*>(datom + r * 128 + ((ch ^ (r & 7)) << 4)) = dk[cc][t];
        }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&ds_ready[g]);
    }
    if (ok && nq > 0) ok = dq_out(nq - 1);
    if (lane == 0) bulk_wait0();  // every dQ reduce has landed before the CTA retires
    __syncwarp();
    // dK, dV (key-major) once every query tile has been folded in: dq_full of the last tile means
    // every earlier MMA (in-order tensor pipe) has completed. This warp's 32 key rows x 32 head
    // columns are staged (dK fp32 in its dQ stage, dV bf16 in the now idle dS area) and written by
    // TMA bulk stores; rows past T are clipped by the hardware.
    if (ok) {
      uint32_t v[32];
      tmem_ld32(t_lane + 320 + g * 32, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_float4(__uint_as_float(v[4 * j]) * p.scale, __uint_as_float(v[4 * j + 1]) * p.scale,
                        __uint_as_float(v[4 * j + 2]) * p.scale, __uint_as_float(v[4 * j + 3]) * p.scale);
      tmem_ld32(t_lane + 256 + g * 32, v);
      tmem_wait_ld();
      uint8_t* dv_stage = sDS + sw * 2048;  // 32 rows x 64 bytes, unswizzled
#pragma unroll
      for (int t = 0; t < 4; ++t)
        *reinterpret_cast<uint4*>(dv_stage + lane * 64 + t * 16) =
            make_uint4(pack_bf16x2(__uint_as_float(v[8 * t]), __uint_as_float(v[8 * t + 1])),
                       pack_bf16x2(__uint_as_float(v[8 * t + 2]), __uint_as_float(v[8 * t + 3])),
                       pack_bf16x2(__uint_as_float(v[8 * t + 4]), __uint_as_float(v[8 * t + 5])),
                       pack_bf16x2(__uint_as_float(v[8 * t + 6]), __uint_as_float(v[8 * t + 7])));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && k0 + quarter * 32 < p.T) {
        tma_store_4d(&tmDK, stage, g * 32, h, k0 + quarter * 32, b);
        tma_store_4d(&tmDV, dv_stage, g * 32, h, k0 + quarter * 32, b);
        bulk_commit();
        bulk_wait0();
      }
      __syncwarp();
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

constexpr uint32_t FWD_SMEM = TILE_BYTES + 2 * FWD_KV_STAGES * KV_TILE_BYTES + 2 * P_TILE_BYTES + 256 + 1024;
constexpr uint32_t BWD_SMEM = 8 * TILE_BYTES + 8 * DQ_STAGE_BYTES + 8 * BWD_STAT_FLOATS * 4 + 256 + 1024;

}  // namespace rgpt

using namespace rgpt;

static int check_attn_args(int B, int T, int H, int d) {
  if (B < 1 || T < 1 || H < 1 || d != H * ATT_D)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention needs head_dim 64 and d == H*64 (B=%d T=%d H=%d d=%d)", B, T,
                          H, d);
  return RGPT_OK;
}

extern "C" int rgpt_attn_fwd(const void* qk, const void* qkv, const void* gate, void* o, void* og, float* lse, int B,
                             int T, int H, int d, const unsigned* drop_mask, float drop_p, void* stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int st = rgpt_check_device(dev);
  if (st) return st;
  if ((st = check_attn_args(B, T, H, d))) return st;
  if (o == nullptr || lse == nullptr || (og != nullptr && gate == nullptr))
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention outputs missing (og needs gate)");
  CUtensorMap tq, tk, tv;
  const __nv_bfloat16* qkb = reinterpret_cast<const __nv_bfloat16*>(qk);
  const __nv_bfloat16* qkvb = reinterpret_cast<const __nv_bfloat16*>(qkv);
  if ((st = make_head_map(&tq, qkb, H, T, B, 2LL * d))) return st;
  if ((st = make_head_map(&tk, qkb + d, H, T, B, 2LL * d, FWD_KT))) return st;
  if ((st = make_head_map(&tv, qkvb + 2 * d, H, T, B, 3LL * d, FWD_KT))) return st;
  // gate (read) and the outputs o / og (written): 4-D maps with 128-row (gate) / 32-row (stores) boxes
  CUtensorMap tg, to, tog;
  if ((st = make_head_map(&to, o, H, T, B, (long long)d, 32))) return st;
  tog = to;
  tg = to;
  if (og != nullptr) {
    if ((st = make_head_map(&tog, og, H, T, B, (long long)d, 32))) return st;
    if ((st = make_head_map(&tg, gate, H, T, B, (long long)d))) return st;
  }
  AttnFwdParams p;
  p.B = B;
  p.T = T;
  p.H = H;
  p.d = d;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.og = reinterpret_cast<__nv_bfloat16*>(og);
  p.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  p.lse = lse;
  const bool drop = drop_mask != nullptr && drop_p > 0.0f;
  if (drop && !(drop_p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention dropout needs p in [0, 1)");
  p.drop_mask = drop ? reinterpret_cast<const uint32_t*>(drop_mask) : nullptr;
  p.drop_scale = drop ? (float)(1.0 / (1.0 - (double)drop_p)) : 1.0f;
  static bool attr[2][64] = {{false}};
  if (!attr[drop][dev]) {
    const cudaError_t e =
        drop ? cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM)
             : cudaFuncSetAttribute(attn_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM);
    if (e != cudaSuccess) return rgpt_check_launch("attn_fwd set smem");
    attr[drop][dev] = true;
  }
  const dim3 grid((unsigned)(((T + ATT_TILE - 1) / ATT_TILE) * H * B));
  cudaStream_t st_ = reinterpret_cast<cudaStream_t>(stream);
  if (drop)
    launch_pdl(attn_fwd_kernel<true>, dim3(grid), dim3(ATT_THREADS), FWD_SMEM, st_, 1, tq, tk, tv, tg, to, tog, p);
  else
    launch_pdl(attn_fwd_kernel<false>, dim3(grid), dim3(ATT_THREADS), FWD_SMEM, st_, 1, tq, tk, tv, tg, to, tog, p);
  return rgpt_check_launch("attn_fwd_kernel");
}

extern "C" int rgpt_attn_bwd_prep(const void* dog, const void* o, const void* gate, void* dout, void* dgate_pre,
                                  float* Dvec, float* dq_zero, int B, int T, int H, int d, void* stream) {
  int st = check_attn_args(B, T, H, d);
  if (st) return st;
  if (reinterpret_cast<uintptr_t>(dq_zero) & 15)
    return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dq_zero must be 16-byte aligned");
  if (gate != nullptr && dgate_pre == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "gate needs dgate_pre");
  const long long threads = (long long)B * T * H * 8;
  const int block = 256;
  const long long grid = (threads + block - 1) / block;
  launch_pdl(attn_bwd_prep_kernel, dim3((unsigned)grid), dim3(block), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      reinterpret_cast<const __nv_bfloat16*>(dog), reinterpret_cast<const __nv_bfloat16*>(o),
      reinterpret_cast<const __nv_bfloat16*>(gate), reinterpret_cast<__nv_bfloat16*>(dout),
      reinterpret_cast<__nv_bfloat16*>(dgate_pre), Dvec, dq_zero, B, T, H, d);
  return rgpt_check_launch("attn_bwd_prep_kernel");
}

extern "C" int rgpt_attn_bwd(const void* qk, const void* qkv, const void* dout, const float* lse, const float* Dvec,
                             float* dq, float* dk, long long dk_stride, void* dv, long long dv_stride, int B, int T,
                             int H, int d, const unsigned* drop_mask, float drop_p, void* stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int st = rgpt_check_device(dev);
  if (st) return st;
  if ((st = check_attn_args(B, T, H, d))) return st;
  if ((reinterpret_cast<uintptr_t>(dq) & 15) || (reinterpret_cast<uintptr_t>(dk) & 15) ||
      (reinterpret_cast<uintptr_t>(dv) & 15) || (dk_stride % 4) || (dv_stride % 8))
    return rgpt_set_error(RGPT_ERR_MISALIGNED, "attention gradient buffers must be 16-byte aligned");
  CUtensorMap tq, tk, tv, tdo, tdq;
  const __nv_bfloat16* qkb = reinterpret_cast<const __nv_bfloat16*>(qk);
  const __nv_bfloat16* qkvb = reinterpret_cast<const __nv_bfloat16*>(qkv);
  if ((st = make_head_map(&tq, qkb, H, T, B, 2LL * d))) return st;
  if ((st = make_head_map(&tk, qkb + d, H, T, B, 2LL * d))) return st;
  if ((st = make_head_map(&tv, qkvb + 2 * d, H, T, B, 3LL * d))) return st;
  if ((st = make_head_map(&tdo, dout, H, T, B, (long long)d))) return st;
  if ((st = make_head_map_f32(&tdq, dq, H, T, B, (long long)d))) return st;
  CUtensorMap tdk, tdv;
  if ((st = make_head_map_f32(&tdk, dk, H, T, B, dk_stride))) return st;
  if ((st = make_head_map_bf16_32(&tdv, dv, H, T, B, dv_stride))) return st;
  AttnBwdParams p;
  p.B = B;
  p.T = T;
  p.H = H;
  p.d = d;
  p.scale = 0.125f;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  p.lse = lse;
  p.Dvec = Dvec;
  p.dk = dk;
  p.dk_stride = dk_stride;
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.dv_stride = dv_stride;
  const bool drop = drop_mask != nullptr && drop_p > 0.0f;
  if (drop && !(drop_p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention dropout needs p in [0, 1)");
  p.drop_mask = drop ? reinterpret_cast<const uint32_t*>(drop_mask) : nullptr;
  p.drop_scale = drop ? (float)(1.0 / (1.0 - (double)drop_p)) : 1.0f;
  static bool attr[2][64] = {{false}};
  if (!attr[drop][dev]) {
    const cudaError_t e =
        drop ? cudaFuncSetAttribute(attn_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM)
             : cudaFuncSetAttribute(attn_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM);
    if (e != cudaSuccess) return rgpt_check_launch("attn_bwd set smem");
    attr[drop][dev] = true;
  }
  const dim3 grid((unsigned)(((T + ATT_TILE - 1) / ATT_TILE) * H * B));
  cudaStream_t st_ = reinterpret_cast<cudaStream_t>(stream);
  if (drop)
    launch_pdl(attn_bwd_kernel<true>, dim3(grid), dim3(ATT_BWD_THREADS), BWD_SMEM, st_, 1, tq, tk, tv, tdo, tdq, tdk,
               tdv, p);
  else
    launch_pdl(attn_bwd_kernel<false>, dim3(grid), dim3(ATT_BWD_THREADS), BWD_SMEM, st_, 1, tq, tk, tv, tdo, tdq,
               tdk, tdv, p);
  return rgpt_check_launch("attn_bwd_kernel");
}

extern "C" int rgpt_attn_drop_mask(unsigned* mask, const unsigned long long* seed, unsigned site, float p, int B,
                                   int T, int H, void* stream) {
  if (mask == nullptr || seed == nullptr) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout mask and seed needed");
  if (!(p >= 0.0f && p < 1.0f)) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "dropout p must be in [0, 1), got %g", p);
  if (B < 1 || T < 1 || H < 1) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention dropout mask: empty shape");
  const long long blocks = (long long)B * H * ((T + 31) / 32);
  if (blocks > 0x7fffffffLL) return rgpt_set_error(RGPT_ERR_BAD_SHAPE, "attention dropout mask too large");
  // 4-warp blocks: small enough to run beside the resident CTAs of the kernels they overlap
  launch_pdl(attn_drop_mask_kernel, dim3((unsigned)blocks), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), 1,
             reinterpret_cast<uint32_t*>(mask), seed, (uint32_t)site, (uint32_t)lrintf(p * 65536.0f), B * H, T);
  return rgpt_check_launch("attn_drop_mask_kernel");
}
