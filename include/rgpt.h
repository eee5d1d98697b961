/*
 * rgpt.h — C ABI of librgpt_kernels.so, the B200 (sm_100a) kernels behind the
 * rGPT training step.
 *
 * Conventions (every entry point):
 *   - Pointers are device pointers allocated by the caller; nothing here allocates
 *     device memory except the lazily created per-device state noted below.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it with no
 *     implicit device synchronisation.
 *   - Return 0 on success, otherwise an RgptStatus code; rgpt_last_error() gives
 *     the message for the calling thread. Nothing aborts or traps.
 *   - Matrices are row-major with explicit leading dimensions (in elements).
 *   - bf16 = IEEE bfloat16 stored as uint16; f32 = float.
 *
 * Each declaration names the reference interface it replaces
 * (newbee1905/rgpt, file:line).
 */
#ifndef RGPT_H_
#define RGPT_H_

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
/* Copies the calling thread's last error message into buf (NUL-terminated). */
int rgpt_last_error(char* buf, unsigned long long buflen);
/* Reads and clears the device-side error word (bounded-wait timeouts etc.).
 * Synchronises the current device. Returns 0 when no device error was recorded. */
int rgpt_device_error(void);
/* Library ABI version (major*100 + minor). */
int rgpt_version(void);

/* ------------------------------------------------------------------ GEMM
 * D[b](m,n) = epilogue( sum_k A[b](m,k) * B[b](n,k) ), bf16 inputs, fp32 accumulate
 * on tcgen05 tensor cores.
 *   A(m,k) = A[m*lda + k] if a_mn_major == 0 else A[k*lda + m]
 *   B(n,k) = B[n*ldb + k] if b_mn_major == 0 else B[k*ldb + n]
 * Replaces: the nn.Linear/torch.matmul GEMMs of model/attention.py:38-40,63-64,
 * model/gpt.py:112,130, model/kernels.py:327,340,371-372 and the fused Triton
 * kernels model/kernels.py:127-200 (ACT_FWD) and :207-281 (ACT_BWD), and the
 * Newton-Schulz matmuls of optimizer.py:36-41 (POLY_BF16).
 */
enum RgptEpilogue {
  RGPT_EPI_STORE_BF16 = 0, /* D bf16 = alpha*acc                                    */
  RGPT_EPI_STORE_F32 = 1,  /* D f32  = alpha*acc                                    */
  RGPT_EPI_ACCUM_F32 = 2,  /* D f32 += alpha*acc (split-K allowed: fp32 atomics)    */
  RGPT_EPI_ACT_FWD = 3,    /* D bf16 = alpha*acc (pre), D2 bf16 = act(alpha*acc)    */
  RGPT_EPI_ACT_BWD = 4,    /* D bf16 = alpha*acc * act'(C), C bf16 (pre)            */
  RGPT_EPI_RESID_F32 = 5,  /* D f32 = C f32 + alpha*acc*colscale[n] (colscale opt.);
                              D2 f32 (optional) = alpha*acc, the unscaled branch output */
  RGPT_EPI_POLY_BF16 = 6,  /* D bf16 = beta*C + alpha*acc, C bf16                   */
  RGPT_EPI_BIAS_SIGMOID_BF16 = 7, /* D bf16 = sigmoid(alpha*acc + colscale[n]) (G1 gate)  */
  RGPT_EPI_POLY_F32 = 8,   /* D f32  = beta*C + alpha*acc, C f32 (fp32 Newton-Schulz)  */
  RGPT_EPI_ARGMAX_BF16 = 9 /* no D: per row and column tile, the first maximum of bf16(alpha*acc) and its
                              column (rgpt_gemm_argmax only)                          */
};
enum RgptActivation { RGPT_ACT_NONE = 0, RGPT_ACT_SQUARED_RELU = 1, RGPT_ACT_GELU = 2, RGPT_ACT_SILU = 3, RGPT_ACT_MISH = 4,
                      /* squared ReLU, post-activation only: ACT_FWD writes D = relu(acc)^2 and no D2 (pass
                         D2 = NULL); ACT_BWD takes C = that post-activation and forms act' = 2 sqrt(C) */
                      RGPT_ACT_SQUARED_RELU_POST = 5 };

/* Requirements: M, N, K >= 1 (tiles past the edges are zero-filled / masked); 16-byte aligned base pointers;
 * leading dimensions and batch strides multiples of 8 elements (16 bytes).
 * splitk: 0 = automatic (only for ACCUM_F32), 1 = none, >1 = explicit (ACCUM_F32 only).
 * alpha_dev: optional device scalar; the effective alpha is alpha * (*alpha_dev). */
int rgpt_gemm_bf16(const void* A, int a_mn_major, long long lda, long long a_bstride,
                   const void* B, int b_mn_major, long long ldb, long long b_bstride,
                   int M, int N, int K, int batch,
                   int epi, int act, float alpha, float beta,
                   void* D, long long ldd, long long d_bstride,
                   void* D2, long long ldd2, long long d2_bstride,
                   const void* C, long long ldc, long long c_bstride,
                   const float* colscale, int splitk, const float* alpha_dev, void* stream);
/* Row argmax of bf16(A @ B^T) without writing the product: the rGPT per-recurrence lm_head whose logits
 * only feed argmax (model/gpt.py:112-120). A [M, K] and B [N, K] bf16, K-major. The GEMM epilogue keeps,
 * per row and column tile, the first maximum of the bf16-rounded values (part_val / part_idx, [M, ld_part]
 * with ld_part >= ceil(N/128)); a second kernel combines the tiles into argmax[M] (int32): the first
 * index of the row maximum, as torch.argmax over the stored bf16 logits. */
int rgpt_gemm_argmax(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K, float* part_val,
                     int* part_idx, long long ld_part, int* argmax, void* stream);
/* RGPT_DROPOUT. rgpt_gemm_bf16 with the residual-branch dropout of model/transformer_block.py:45,52 fused
 * into the RESID_F32 epilogue (batch 1 only): the branch output alpha*acc becomes alpha*acc*keep/(1-drop_p)
 * (D2 stores that dropped branch output), keep = bit column%32 of drop_mask[row*drop_ldm + column/32]. */
int rgpt_gemm_bf16_dropout(const void* A, int a_mn_major, long long lda, long long a_bstride,
                           const void* B, int b_mn_major, long long ldb, long long b_bstride,
                           int M, int N, int K, int batch, int epi, int act, float alpha, float beta,
                           void* D, long long ldd, long long d_bstride, void* D2, long long ldd2, long long d2_bstride,
                           const void* C, long long ldc, long long c_bstride, const float* colscale, int splitk,
                           const float* alpha_dev, const void* drop_mask, long long drop_ldm, float drop_p,
                           void* stream);
/* Row-layout keep bits [M, N] for the residual-branch dropout: bit column%32 of mask[row*ldm + column/32]
 * from Philox4x32-10 block (column/8, row, drop_site, 0) under key (*drop_seed low, high 32 bits), element
 * column%8 = 16-bit half (column%2) of word (column%8)/2, kept iff >= round(drop_p*65536). No counterpart
 * in the reference (nn.Dropout draws its mask internally). */
int rgpt_drop_mask(unsigned* mask, long long ldm, const unsigned long long* drop_seed, unsigned drop_site,
                   float drop_p, int M, int N, void* stream);


/* ------------------------------------------------------------------ attention
 * Causal softmax attention, head_dim 64, scale 1/8, token-major operands:
 *   qk  [B*T, 2d] bf16 (q heads | k heads, after QK norm + RoPE), qkv [B*T, 3d] bf16 (v = cols [2d,3d)),
 *   gate/o/og/dout/dgate_pre [B*T, d] bf16, lse/Dvec [B, H, T] fp32.
 * Replaces F.scaled_dot_product_attention(is_causal=True, dropout_p) and the G1 gate multiply,
 * model/attention.py:56-61 (forward) and their autograd backward.
 * Dropout (drop_mask != null and drop_p > 0): the keep bit of (query q, key k) of head bh = b*H + h is
 * bit q%32 of drop_mask[(bh*ceil(T/32) + q/32)*T + k], filled by rgpt_attn_drop_mask from Philox4x32-10
 * block (k/8, q, drop_site, bh) under key (*drop_seed low, high 32 bits) -- 16-bit uniform (k%8 picks
 * word (k%8)/2, half k%2) >= round(p*65536). The forward scales the kept probabilities by 1/(1-p) (the
 * softmax normaliser keeps all of them); the backward applies the same bits. See RGPT_DROPOUT below for
 * the other sites. */
int rgpt_attn_fwd(const void* qk, const void* qkv, const void* gate, void* o, void* og, float* lse,
                  int B, int T, int H, int d, const unsigned* drop_mask, float drop_p, void* stream);
/* Keep bits of the attention-probability dropout for rgpt_attn_fwd / rgpt_attn_bwd, drawn for every causal
 * (query, key) pair into drop_mask [B*H][ceil(T/32)][T] (see above); no counterpart in the reference, whose
 * SDPA draws them internally. */
int rgpt_attn_drop_mask(unsigned* drop_mask, const unsigned long long* drop_seed, unsigned drop_site, float drop_p,
                        int B, int T, int H, void* stream);
/* dout = dog*gate; dgate_pre = dog*o*gate*(1-gate); Dvec = rowsum(dout*o). gate may be null (ungated).
 * dq_zero (optional, [B*T, d] fp32, 16-byte aligned) is zeroed: the dq accumulator of rgpt_attn_bwd. */
int rgpt_attn_bwd_prep(const void* dog, const void* o, const void* gate, void* dout, void* dgate_pre,
                       float* Dvec, float* dq_zero, int B, int T, int H, int d, void* stream);
/* dq [B*T, d] fp32 is ACCUMULATED (caller zeroes it); dk fp32 and dv bf16 are written with row strides. */
int rgpt_attn_bwd(const void* qk, const void* qkv, const void* dout, const float* lse, const float* Dvec,
                  float* dq, float* dk, long long dk_stride, void* dv, long long dv_stride,
                  int B, int T, int H, int d, const unsigned* drop_mask, float drop_p, void* stream);

/* ------------------------------------------------------------------ norms
 * y = x * s(sum x^2) * affine over rows of length d. Kinds follow model/norm.py. */
enum RgptNormKind {
  RGPT_NORM_IDENTITY = 0,
  RGPT_NORM_RMS_AFFINE = 1, /* RMSNorm (Gemma, (1+w)), model/norm.py:8-34          */
  RGPT_NORM_RMS = 2,        /* functional_rms_norm (eps = FLT_EPSILON), :37-38     */
  RGPT_NORM_L2_TEMP = 3,    /* L2Norm (learned temp), :44-51                       */
  RGPT_NORM_L2 = 4,         /* functional_l2_norm, :54-55                          */
  RGPT_NORM_ELASTIC = 5,    /* HybridElasticNorm, :58-95                           */
  RGPT_NORM_ELASTICBALL = 6,/* ElasticBallNorm / DualElasticBallNorm, :97-141      */
  RGPT_NORM_HYPERBALL = 7   /* HyperballNorm / functional_hyperball_norm, :40-42,156-162 */
};
/* Residual-stream norm: x fp32 [M, d] -> y bf16 [M, d]; stat[M] = s (optional).
 * With qout != null also computes the 2-way q_head, qout[M,2] = y @ qw^T + qb (model/gpt.py:107-109).
 * d in {128, 256, 512, 1024, 2048}. Replaces RMSNorm.forward & co (model/norm.py).
 * w: RMS_AFFINE's weight [d]; for L2_TEMP, when w is not null, the learned temperature is read from w[0]
 * on the device (L2Norm.temp, model/norm.py:48) and the by-value temp is ignored. */
int rgpt_rownorm_fwd(const float* x, void* y, float* stat, const float* w, float temp, int kind, float eps,
                     float alpha, int M, int d, const float* qw, const float* qb, float* qout, void* stream);
/* Norm backward fused with the residual-gradient add (model/transformer_block.py:43-57):
 *   g_out = g_in + dx; g_bf16 = bf16(g_out * ls * z); dls += sum_rows g_out*raw; dw += sum_rows dy*x*s,
 *   z = keep/(1-drop_p) from the branch's dropout mask [M, d/32] (drop_mask null: z = 1).
 * q_head mode (dq != null): dy = dq @ qw, plus dqw += dq^T h, dqb += sum dq. Optional pointers may be null. */
int rgpt_rownorm_bwd(const float* x, const float* dy, const float* w, float temp, int kind, float eps, float alpha,
                     int M, int d, const float* g_in, float* g_out, void* g_bf16, const float* ls,
                     const float* raw, float* dls, float* dw, float* dtemp, const float* dq, const float* qw,
                     const void* h, float* dqw, float* dqb, const unsigned* drop_mask, float drop_p, void* stream);

/* ------------------------------------------------------------------ QKV prep
 * Per (token, head): QK norm (QKNorm, model/norm.py:182-204) and RoPE (model/rope.py:38-57).
 * qkv [M, 3d] bf16 -> qk [M, 2d] bf16 (roped normalised q | k), qn [M, d] bf16 (normalised q before
 * RoPE, the input of the G1 gate GEMM sigmoid(qn Wg^T + bg), model/attention.py:45-48; may be null).
 * inv_freq[32] as model/rope.py:11. sq/sk: constant post-scales (asymmetric hyperball 1.0/1.1, else 1). */
int rgpt_qkv_prep_fwd(const void* qkv, void* qk, void* qn, const float* inv_freq, int qk_kind, float eps,
                      float alpha, const float* wq, const float* wk, float tq, float tk, float sq, float sk,
                      int M, int T, int H, void* stream);
/* wq/wk: RMS_AFFINE's q/k weights [64]; for L2_TEMP, when not null, the learned q/k temperatures are read
 * from wq[0]/wk[0] on the device and tq/tk are ignored.
 * Backward: dq, dk fp32 [M, d] (grads of the roped q, k) and dqn_gate fp32 [M, d] (= dgp Wg from the
 * gate GEMM, may be null) -> the q/k column blocks of dqkv (bf16). dbg += column sums of dgp (bf16
 * [M, d]); dwq/dwk (RMS_AFFINE QK norms) and dtq/dtk (L2_TEMP) are ACCUMULATED. */
int rgpt_qkv_prep_bwd(const void* qkv, const float* dq, const float* dk, const float* dqn_gate, const void* dgp,
                      void* dqkv, float* dbg, float* dwq, float* dwk, float* dtq, float* dtk, const float* inv_freq,
                      int qk_kind, float eps, float alpha, const float* wq, const float* wk, float tq, float tk,
                      float sq, float sk, int M, int T, int H, void* stream);

/* ------------------------------------------------------------------ standalone modules
 * The reference's submodules called on their own, outside GPT's engine (which fuses them into its
 * kernels). Row norm of any kind over rows of ANY length d (1..16384; the QK norms' d_head = 64 too),
 * x fp32 [M, d] -> y fp32 [M, d]; w as rgpt_rownorm_fwd (RMS_AFFINE weight, or the L2_TEMP temperature
 * read from w[0]). Replaces RMSNorm / L2Norm / HybridElasticNorm / ElasticBallNorm / HyperballNorm and
 * the functional norms, model/norm.py:8-162, as QKNorm.forward (:200-204) calls them. */
int rgpt_rownorm_any_fwd(const float* x, float* y, const float* w, int kind, float eps, float alpha, long long M, int d,
                         void* stream);
/* dx fp32 [M, d] (written); dw [d] (RMS_AFFINE) and dtemp [1] (L2_TEMP) ACCUMULATED, each optional. */
int rgpt_rownorm_any_bwd(const float* x, const float* dy, const float* w, int kind, float eps, float alpha,
                         long long M, int d, float* dx, float* dw, float* dtemp, void* stream);
/* RotaryEmbedding.forward (model/rope.py:38-57) on one [B, H, T, D] fp32 tensor: in at element strides
 * (sb, sh, st, 1), out contiguous [B, H, T, D]; angle t * inv_freq[j] (inv_freq [D/2], model/rope.py:11),
 * y = x cos + rotate_half(x) sin. backward != 0 applies the transposed rotation (the gradient). */
int rgpt_rope(const float* in, long long sb, long long sh, long long st, float* out, const float* inv_freq, int B,
              int H, int T, int D, int backward, void* stream);

/* ------------------------------------------------------------------ embedding / loss
 * nn.Embedding forward (model/gpt.py:95) and its backward (dx rows ACCUMULATED into demb), with the
 * embedding dropout of model/gpt.py:96 when drop_mask != null (d % 128 == 0): keep bits of (row, column)
 * from Philox block (column/8, row, drop_site, 0), stored in drop_mask [M, d/32] and read back by the
 * backward. */
int rgpt_embedding_fwd(const long long* ids, const float* emb, float* x, int M, int d, int V, unsigned* drop_mask,
                       const unsigned long long* drop_seed, unsigned drop_site, float drop_p, void* stream);
int rgpt_embedding_bwd(const long long* ids, const float* dx, float* demb, int M, int d, int V,
                       const unsigned* drop_mask, float drop_p, void* stream);
/* Cross entropy over bf16 logits rows (F.cross_entropy with ignore_index, trainer.py:148) plus the
 * row argmax (model/gpt.py:119-120). scale_buf[2] = {grad_scale/count, count}; loss_out = mean loss.
 * write_grad: logits are overwritten in place by bf16 (softmax - onehot) * grad_scale / count. */
int rgpt_cross_entropy(void* logits, long long ld, int M, int V, const long long* labels, int ignore_index,
                       float grad_scale, float* loss_rows, int* argmax, float* scale_buf, float* loss_out,
                       int write_grad, void* stream);
/* Allocation-free variant of rgpt_cross_entropy (no counterpart in the reference). For callers that
 * cannot allocate device memory (plugin hosts that hand over only input/output buffers, processes whose
 * device memory is fully reserved by another allocator): the per-row losses and the scale/count pair live
 * in a static device array inside this library (1 MiB, held by every GPU that loads it until exit).
 * Same outputs as rgpt_cross_entropy: loss_out[0] = mean loss, argmax (optional), in-place dlogits when
 * write_grad. M is limited to 262144 rows; larger M is rejected with RGPT_ERR_BAD_SHAPE. The first call on
 * a device resolves the array's device address, so make that first call before any stream capture.
 * Calls share the array: calls that overlap on the GPU (e.g. on two streams) race. Nothing in it needs to
 * start at zero; each call rewrites what it reads. No cudaMalloc/cudaFree is made. */
int rgpt_cross_entropy_noalloc(void* logits, long long ld, int M, int V, const long long* labels, int ignore_index,
                               float grad_scale, float* loss_out, int* argmax, int write_grad, void* stream);
/* rGPT halting losses (model/gpt.py:105-141, trainer.py:150-162): q [R, M, 2], argmax [R, M].
 * losses[0] += halt BCE mean, losses[1] += q_continue BCE mean; dq = grad_scale * d(total)/dq. */
int rgpt_halt_losses(const float* q, const int* argmax, const long long* labels, int R, int M, float grad_scale,
                     float* dq, float* losses, void* stream);

/* ------------------------------------------------------------------ optimizer */
typedef struct RgptAdamwTensor {
  float* p; const float* g; float* m; float* v; unsigned short* shadow; long long n;
} RgptAdamwTensor;
typedef struct RgptMuonTensor {
  float* param; const float* grad; unsigned short* mom; unsigned short* shadow;
} RgptMuonTensor;
/* One segment of the data-parallel staging copies (rgpt_segment_copy): tensor t (and t2, a bf16 copy written on
 * unpack, or 0), its element count n and its element offset in the packed buffer. */
typedef struct RgptSegment {
  void* t;
  void* t2;
  long long buf_off;
  long long n;
} RgptSegment;
/* The whole quintic Newton-Schulz iteration (zeropower_via_newtonschulz5, optimizer.py:18-45) of n same-shape
 * matrices in ONE persistent, cooperative launch: `steps` x {A = X X^T; B = b A + c A A; X' = a X + B X}, bf16
 * operands and results, fp32 accumulation, the polynomial combines fused into the GEMM epilogues (the same
 * roundings as the batched GEMM path). X, X2: [n][rows >= xr][x_ld] bf16 (batch stride x_bstride), X holding the
 * normalised input (rows <= cols: 1 <= xr <= xc); the result lands in X2 for odd `steps`, else in X. A, B:
 * [n][>= xr][a_ld] bf16 scratch. counters: n * 3 * steps unsigned ints, zeroed by this call (a memset on the
 * stream): each work unit waits (bounded, 1 s) only for the previous phase of its own matrix. Row strides are
 * multiples of 8 elements, base pointers 16-byte aligned. */
int rgpt_ns_chain(void* X, void* X2, void* A, void* B, int n, int xr, int xc, long long x_ld, long long x_bstride,
                  long long a_ld, long long a_bstride, int steps, float a, float b, float c, unsigned* counters,
                  void* stream);

/* Staging copies of the sharded data-parallel optimizer step (no kernel in the reference, whose DDP
 * all-reduces every gradient and whose DistMuon repeats the whole update on every rank, trainer.py:47-53,
 * optimizer.py:317-415): pack (unpack == 0) buf[off + i] = scale * t[i] for every segment, or unpack
 * t[i] = scale * buf[off + i] (and t2[i] = bf16 of it when t2 != 0). buf_bf16 / tensor_bf16 select bf16
 * instead of fp32 storage. Work items: n_chunks (segment index, start element) pairs of up to chunk_elems
 * elements each. */
int rgpt_segment_copy(const RgptSegment* table, const int* chunk_seg, const long long* chunk_start, int n_chunks,
                      int chunk_elems, void* buf, int buf_bf16, int tensor_bf16, float scale, int unpack,
                      void* stream);
/* Per-step scalars read from DEVICE memory instead of the by-value arguments when the `hp` pointer
 * of an optimizer entry point is non-null (so that a captured CUDA graph of the step sees each
 * step's learning rate and bias corrections). Layout, 8 floats per parameter group:
 *   AdamW group: {lr, wd, beta1, beta2, eps, 1/(1-beta1^step), 1/sqrt(1-beta2^step), 0}
 *   Muon group:  {beta, 1 - lr*wd, -muon_lr, 0, ...}                                        */
#define RGPT_HP_FLOATS 8
/* foreach_adamw_step (optimizer.py:80-116) over a device table of tensors split into chunks
 * (chunk_tensor[i], chunk_start[i]); shadow (bf16 copy of p) optional per tensor. */
int rgpt_adamw(const RgptAdamwTensor* table, const int* chunk_tensor, const long long* chunk_start, int n_chunks,
               int chunk_elems, float lr, float wd, float beta1, float beta2, float eps, int step, const float* hp,
               void* stream);
/* muon_update's momentum/Nesterov/transposition (optimizer.py:51-69, :23-26) for n same-shape [R, C]
 * matrices into the bf16 NS stack X (zero-padded, leading dim ldx); sumsq[n] ACCUMULATES ||X||_F^2. */
int rgpt_muon_prep(const RgptMuonTensor* table, int n, int R, int C, void* X, long long x_bstride, int ldx,
                   float beta, int nesterov, float* sumsq, const float* hp, void* stream);
/* X /= max(||X||_F, 1e-7) per matrix (optimizer.py:31-32). */
int rgpt_ns_scale(void* X, long long x_bstride, int ldx, int rows, int cols, int n, const float* sumsq, void* stream);
/* Newton-Schulz at fp32 accuracy on the bf16 tensor cores (the fp32 form of
 * zeropower_via_newtonschulz5, optimizer.py:8-45, with X = G.float()). Each fp32 value x is split as
 * hi = bf16(x), lo = bf16(x - hi); a product X*Y is then hi*hi + hi*lo + lo*hi (relative error ~2^-17),
 * computed as ONE bf16 GEMM over K tripled by stacking the operand blocks along K.
 * Logical source matrix b, element (i, j) = src[b*s_b + i*s_i + j*s_j], rows x cols, fp32 (bf16 if
 * src_bf16), one of s_i / s_j equal to 1 (so a transposed view reads coalesced).
 * rgpt_ns_sumsq: sumsq[b] += sum of squares of matrix b (caller zeroes sumsq).
 * rgpt_ns_split: v = x * s with s = 1/max(sqrt(sumsq[b]), 1e-7) if sumsq != null, else 1;
 *   xout (optional, fp32, row stride ldo, batch stride o_bstride) = v;
 *   dst (optional, bf16, row stride ldd, batch stride d_bstride): nblk copies, block k at dst + k*blk_off
 *   (elements), holding lo(v) if bit k of lo_mask is set, else hi(v). Padding outside rows x cols is
 *   never written. */
int rgpt_ns_sumsq(const void* src, int src_bf16, long long s_b, long long s_i, long long s_j, int rows, int cols,
                  int n, float* sumsq, void* stream);
int rgpt_ns_split(const void* src, int src_bf16, long long s_b, long long s_i, long long s_j, int rows, int cols,
                  int n, const float* sumsq, float* xout, long long o_bstride, long long ldo, void* dst,
                  long long d_bstride, long long ldd, int nblk, long long blk_off, unsigned lo_mask, void* stream);
/* p = p*(1 - lr*wd) - muon_lr * bf16(X*scale) (optimizer.py:209-227); shadow = bf16(p). */
int rgpt_muon_apply(const RgptMuonTensor* table, int n, int R, int C, const void* X, long long x_bstride, int ldx,
                    float lr, float wd, float muon_lr, float scale, const float* hp, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RGPT_H_ */
