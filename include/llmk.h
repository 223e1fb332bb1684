/*
 * llmk.h — C ABI of the B200-native (sm_100a) GPT-2 training hot path.
 *
 * Every entry point takes raw device pointers, plain sizes and a CUDA stream
 * passed as `void*` (a cudaStream_t; NULL = legacy default stream). Nothing is
 * allocated on the device by the op-level entry points: scratch memory is
 * passed in by the caller, sized by the matching *_workspace() query.
 * All device work is asynchronous on the given stream; no entry point
 * synchronises unless its comment says so.
 *
 * Return value: 0 (LLMK_OK) or an llmk_status code. llmk_status_string()
 * names it; llmk_last_error() gives the detail of the last failure on the
 * calling thread.
 *
 * Each entry point names the reference interface it replaces as
 * path:line inside the llm.cpp project tree.
 */
#ifndef LLMK_H_
#define LLMK_H_

#include <stddef.h>
#include <stdint.h>

#include "llmk_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum llmk_dtype { LLMK_F32 = 0, LLMK_BF16 = 1 } llmk_dtype;

/* Operand precision of the tensor-core contractions.
 *   LLMK_MATH_BF16: A/B operands are bf16 in memory, fp32 accumulation.
 *   LLMK_MATH_TF32: A/B operands are fp32 in memory, multiplied as tf32,
 *                   fp32 accumulation (the precision of the reference's
 *                   CUTLASS Sm80 GEMMs, gpt2/cuda/matmul.cu:195-220). */
typedef enum llmk_math { LLMK_MATH_BF16 = 1, LLMK_MATH_TF32 = 2 } llmk_math;

/* ------------------------------------------------------------------ misc */
const char* llmk_status_string(int status);
const char* llmk_last_error(void);
const char* llmk_version(void);
/* Reads and (if reset != 0) clears the device status word of the current
 * device: bit LLMK_DEV_TIMEOUT is set by a kernel whose bounded wait expired.
 * Synchronises the device. */
int llmk_device_status(unsigned int* out, int reset);
/* Number of kernels this library launched on the calling process (host-side
 * counter; every launch of every entry point increments it). */
unsigned long long llmk_launch_count(void);

/* ------------------------------------------------------------ GEMM core */
/* Epilogue applied to the fp32 accumulator of D[M,N] = A[M,K] * B[N,K]^T,
 * in this order: + bias[n]; + residual[m,n]; GELU (pre-activation stored to
 * aux as bf16 when aux != NULL); * gelu'(aux[m,n]) (GELU_BWD, aux = bf16
 * pre-activation); + D_old[m,n] (ACCUMULATE). */
#define LLMK_EPI_ACCUMULATE 1
#define LLMK_EPI_GELU 2
#define LLMK_EPI_GELU_BWD 4
typedef struct llmk_epilogue {
  const float* bias;     /* [N] fp32 or NULL */
  const float* residual; /* fp32 [M, ldr] or NULL */
  long long ldr;
  void* aux;             /* bf16 [M, ldaux] (see flags) or NULL */
  long long ldaux;
  int flags;
} llmk_epilogue;

/* D = epilogue(A * B^T) on the tcgen05 tensor cores.
 *   a_trans = 0: A is stored [M][lda] (K contiguous); 1: stored [K][lda] (M contiguous).
 *   b_trans = 0: B is stored [N][ldb] (K contiguous); 1: stored [K][ldb] (N contiguous).
 * Constraints (else LLMK_ERR_UNSUPPORTED): row strides of A, B, D, residual
 * and aux are multiples of 16 bytes, base pointers 16-byte aligned, N % 8 == 0.
 * workspace (optional, >= llmk_gemm_workspace(M,N,K,math) bytes) enables
 * split-K for output grids too small to fill the GPU; without it the GEMM
 * runs unsplit. Results are deterministic either way.
 * New entry point: the engine behind llmk_matmul_forward/backward. */
size_t llmk_gemm_workspace(int M, int N, int K, llmk_math math);
int llmk_gemm(void* D, llmk_dtype d_dtype, long long ldd, const void* A, int a_trans, long long lda,
              const void* B, int b_trans, long long ldb, llmk_math math, int M, int N, int K,
              const llmk_epilogue* epi, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------- matmul */
/* out[BT,OC] = inp[BT,C] * weight[OC,C]^T (+ bias[OC]); bias may be NULL
 * (the tied lm_head). inp/weight are bf16 (LLMK_MATH_BF16) or fp32
 * (LLMK_MATH_TF32); out is fp32 or bf16.
 * Replaces gpt2cuda::BatchMatmulNTForward, gpt2/cuda/matmul.cu:653-661
 * (kernel::BatchMatmulForward<RowMajor,ColumnMajor>, matmul.cu:223-324). */
int llmk_matmul_forward(void* out, llmk_dtype out_dtype, const void* inp, const void* weight, const float* bias,
                        int BT, int C, int OC, llmk_math math, void* stream);

/* Backward of llmk_matmul_forward:
 *   dinp[BT,C]   (+)= dout[BT,OC] * weight[OC,C]
 *   dweight[OC,C] (+)= dout^T * inp          (fp32, one K = BT reduction)
 *   dbias[OC]    (+)= column sums of dout   (fp32; skipped when NULL)
 * flags: LLMK_ACCUM_DINP / LLMK_ACCUM_DWEIGHT / LLMK_ACCUM_DBIAS select "+="
 * (the reference accumulates dinp and dweight, matmul.cu:337,395, and
 * overwrites dbias, matmul.cu:446-448); without a flag the output is
 * overwritten. dinp may be NULL (skipped). dout/inp/weight in the math dtype.
 * workspace: >= llmk_matmul_backward_workspace(BT, C, OC, math) bytes of
 * device memory (dbias partial sums, split-K partial tiles of dweight); may
 * be NULL when dbias is NULL (dweight then runs unsplit).
 * Replaces gpt2cuda::BatchMatmulNTBackward, gpt2/cuda/matmul.cu:663-669
 * (kernel::BatchMatmulBackward, matmul.cu:327-449, and MatrixColSumKernel,
 * matmul.cu:26-187). */
#define LLMK_ACCUM_DINP 1
#define LLMK_ACCUM_DWEIGHT 2
#define LLMK_ACCUM_DBIAS 4
size_t llmk_matmul_backward_workspace(int BT, int C, int OC, llmk_math math);
int llmk_matmul_backward(void* dinp, llmk_dtype dinp_dtype, float* dweight, float* dbias, const void* dout,
                         const void* inp, const void* weight, int BT, int C, int OC, llmk_math math, int flags,
                         void* workspace, size_t workspace_bytes, void* stream);

/* dbias[N] (+)= sum over M rows of x[M,N] (x fp32 or bf16), deterministic
 * two-pass reduction through `workspace`.
 * Replaces kernel::MatrixColSumCUDA, gpt2/cuda/matmul.cu:180-187. */
size_t llmk_colsum_workspace(int M, int N);
int llmk_colsum(float* dbias, const void* x, llmk_dtype x_dtype, int M, int N, int accumulate, void* workspace,
                size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLMK_H_ */
