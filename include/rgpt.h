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
  RGPT_EPI_RESID_F32 = 5,  /* D f32 = C f32 + alpha*acc*colscale[n] (colscale opt.) */
  RGPT_EPI_POLY_BF16 = 6   /* D bf16 = beta*C + alpha*acc, C bf16                   */
};
enum RgptActivation { RGPT_ACT_NONE = 0, RGPT_ACT_SQUARED_RELU = 1, RGPT_ACT_GELU = 2, RGPT_ACT_SILU = 3, RGPT_ACT_MISH = 4 };

/* Requirements: M >= 128, N >= 128, K >= 64; 16-byte aligned base pointers;
 * leading dimensions and batch strides multiples of 8 elements (16 bytes).
 * splitk: 0 = automatic (only for ACCUM_F32), 1 = none, >1 = explicit (ACCUM_F32 only). */
int rgpt_gemm_bf16(const void* A, int a_mn_major, long long lda, long long a_bstride,
                   const void* B, int b_mn_major, long long ldb, long long b_bstride,
                   int M, int N, int K, int batch,
                   int epi, int act, float alpha, float beta,
                   void* D, long long ldd, long long d_bstride,
                   void* D2, long long ldd2, long long d2_bstride,
                   const void* C, long long ldc, long long c_bstride,
                   const float* colscale, int splitk, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RGPT_H_ */
