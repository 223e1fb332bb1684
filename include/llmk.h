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

typedef enum llmk_dtype { LLMK_F32 = 0, LLMK_BF16 = 1, LLMK_F16 = 2 } llmk_dtype;

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
 * aux when aux != NULL); * gelu'(aux[m,n]) (GELU_BWD, aux = pre-activation);
 * + D_old[m,n] (ACCUMULATE). aux is bf16, or fp32 with LLMK_EPI_AUX_F32. */
#define LLMK_EPI_ACCUMULATE 1
#define LLMK_EPI_GELU 2
#define LLMK_EPI_GELU_BWD 4
#define LLMK_EPI_AUX_F32 8 /* aux is fp32 instead of bf16 */
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

/* dbias[N] (+)= sum over M rows of x[M,N] (x fp32 or bf16; other dtypes are
 * rejected with LLMK_ERR_UNSUPPORTED), deterministic two-pass reduction
 * through `workspace`.
 * Replaces kernel::MatrixColSumCUDA, gpt2/cuda/matmul.cu:180-187. */
size_t llmk_colsum_workspace(int M, int N);
int llmk_colsum(float* dbias, const void* x, llmk_dtype x_dtype, int M, int N, int accumulate, void* workspace,
                size_t workspace_bytes, void* stream);

/* llmk_colsum for callers that cannot allocate device memory when they call
 * it: code that runs inside another framework's memory pool or under a fixed
 * memory budget where cudaMalloc after start-up is not allowed, or that must
 * not stall its stream (cudaMalloc can synchronise the device). It takes no
 * workspace: its partial sums live in a fixed array inside the library (1 MiB,
 * held by every GPU that loads the library until the process exits), so it
 * calls no cudaMalloc / cudaFree and allocates nothing.
 * Limit: N <= 262144 columns (one row chunk holds N partial sums); larger N
 * is rejected with LLMK_ERR_UNSUPPORTED (use llmk_colsum). Any M is
 * accepted: the rows are split into min(llmk_colsum's chunk count,
 * 262144 / N) chunks, where llmk_colsum uses about 8 x SMs / ceil(N / 256)
 * chunks of at least 64 rows. x must be fp32 or bf16.
 * Results match llmk_colsum's to fp32 rounding; they are bitwise equal when
 * the chunk count is not capped by the array (both sum the same chunks in the
 * same order).
 * The first call on a device looks up the array's device address with that
 * device current (again after a device reset gave the device a new context);
 * make that first call before any stream capture. All calls share the array:
 * calls that can overlap on the GPU (different streams, or different host
 * threads on one device) race and must be serialised by the caller.
 * No counterpart in the reference: its column sum takes no scratch
 * (gpt2/cuda/matmul.cu:26-187). */
int llmk_colsum_noalloc(float* dbias, const void* x, llmk_dtype x_dtype, int M, int N, int accumulate, void* stream);

/* ------------------------------------------------------------ attention */
/* Causal multi-head attention, head size 64, 16-bit tensor-core operands
 * (qkv_dtype: LLMK_BF16, or LLMK_F16 for 3 more mantissa bits where values
 * stay inside fp16 range), fp32 softmax and accumulation. qkv: (B, T, C3),
 * Q|K|V blocks of C = C3/3 columns, head h at columns h*64 of each block.
 * out: (B, T, C) in out_dtype (qkv_dtype, or fp32 to skip the output
 * rounding). lse: (B, NH, T) fp32 natural-log logsumexp of the scaled scores
 * (scale 1/8). Any T >= 1.
 * Replaces gpt2cuda::BatchCausalAttentionForward, gpt2/cuda/attention.cu:119-133
 * (AttentionForwardCUDA, kernel/flash_attn/flash_fwd_launch.cuh:18-68, which
 * requires T % 128 == 0). */
int llmk_attention_forward(void* out, llmk_dtype out_dtype, float* lse, const void* qkv, llmk_dtype qkv_dtype, int B,
                           int T, int C3, int NH, void* stream);

/* Gradient of llmk_attention_forward. dout, out (B, T, C) and dqkv (B, T, C3)
 * are in io_dtype (qkv_dtype, or fp32: D = rowsum(dO * O) and the dQ/dK/dV
 * stores then skip the 16-bit rounding; dO still enters the MMAs in
 * qkv_dtype). qkv is in qkv_dtype (LLMK_BF16 or LLMK_F16), as in the forward.
 * dqkv is OVERWRITTEN (dQ, dK and dV); the reference accumulates dQ and
 * overwrites dK/dV (flash_bwd_kernel.cuh:377-472) on buffers its callers zero
 * first. workspace >= llmk_attention_backward_workspace(): D, an fp32 dQ
 * accumulator and a 16-bit copy of dO.
 * Replaces gpt2cuda::BatchCausalAttentionBackward, gpt2/cuda/attention.cu:135-148. */
size_t llmk_attention_backward_workspace(int B, int T, int C3, int NH);
int llmk_attention_backward(void* dqkv, const void* dout, const void* out, llmk_dtype io_dtype, const void* qkv,
                            llmk_dtype qkv_dtype, const float* lse, int B, int T, int C3, int NH, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ layernorm */
/* out = (inp - mean) * rstd * gamma + beta over rows of C (eps 1e-5, two-pass
 * variance as the reference CPU path gpt2/layernorm.cpp:16-23). inp fp32,
 * out fp32 or bf16; mean/rstd (N) may be NULL.
 * Replaces gpt2cuda::BatchLayerNormForward, gpt2/cuda/layernorm.cu:348-350. */
int llmk_layernorm_forward(void* out, llmk_dtype out_dtype, float* mean, float* rstd, const float* inp,
                           const float* gamma, const float* beta, int N, int C, void* stream);

/* dinp (+)= LN backward (LLMK_ACCUM_DINP selects +=); dgamma, dbeta (+)=
 * (LLMK_ACCUM_DPARAM selects +=, as the reference). dinp_bf16 (optional)
 * receives a bf16 copy of the final dinp; dinp_colsum (optional, [C]) the
 * column sums of the final dinp (overwritten) — the bias gradient of a linear
 * layer whose output gradient is dinp, fused here instead of a separate pass.
 * dout fp32 or bf16. workspace >= llmk_layernorm_backward_workspace(N, C)
 * (per-block partials, reduced in a fixed order: deterministic).
 * Replaces gpt2cuda::BatchLayerNormBackward, gpt2/cuda/layernorm.cu:351-353. */
#define LLMK_ACCUM_DPARAM 8
size_t llmk_layernorm_backward_workspace(int N, int C);
int llmk_layernorm_backward(float* dinp, void* dinp_bf16, float* dgamma, float* dbeta, float* dinp_colsum,
                            const void* dout, llmk_dtype dout_dtype, const float* inp, const float* gamma,
                            const float* mean, const float* rstd, int N, int C, int flags, void* workspace,
                            size_t workspace_bytes, void* stream);

/* --------------------------------------------------- elementwise helpers */
/* GELU (tanh form, gpt2/gelu.h:7-8) forward / backward over n elements
 * (n % 4 == 0). Replaces gpt2cuda::BatchGeluForward/Backward, gpt2/cuda/gelu.cu:85-90. */
int llmk_gelu_forward(void* out, const void* inp, llmk_dtype dtype, long long n, void* stream);
int llmk_gelu_backward(void* dinp, const void* dout, const void* inp, llmk_dtype dtype, long long n, int accumulate,
                       void* stream);
/* out = a + b; backward da (+)= dy, db (+)= dy.
 * Replaces gpt2cuda::BatchResidualForward/Backward, gpt2/cuda/residual.cu:74-81. */
int llmk_residual_forward(void* out, const void* a, const void* b, llmk_dtype dtype, long long n, void* stream);
int llmk_residual_backward(void* da, void* db, const void* dy, llmk_dtype dtype, long long n, int accumulate,
                           void* stream);
/* dtype conversion (f32 <-> bf16), n % 4 == 0. New helper. */
int llmk_cast(void* out, llmk_dtype out_dtype, const void* in, llmk_dtype in_dtype, long long n, void* stream);

/* --------------------------------------------------------------- encoder */
/* out[b,t,:] = wte[tokens[b,t],:] + wpe[t,:] (fp32).
 * Replaces gpt2cuda::BatchEncoderForward, gpt2/cuda/encoder.cu:92-99. */
int llmk_encoder_forward(float* out, const int* tokens, const float* wte, const float* wpe, int B, int T, int C,
                         void* stream);
/* dwte[tokens[b,t],:] += dout[b,t,:]; dwpe[t,:] += sum_b dout[b,t,:]. Summed
 * in position order (deterministic; the reference scatters with float
 * atomicAdd, encoder.cu:17-25): positions are sorted by token in one CTA when
 * B*T <= 32768 and V < 2^17, and linked by a scan otherwise. V = rows of dwte.
 * workspace >= llmk_encoder_backward_workspace(B,T). */
size_t llmk_encoder_backward_workspace(int B, int T);
int llmk_encoder_backward(float* dwte, float* dwpe, const float* dout, const int* tokens, int B, int T, int C, int V,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------ softmax + cross-entropy */
/* Per row of logits (BT, Vp) over the first V columns: losses[row] =
 * logsumexp - logit[target]; when dlogits != NULL it receives
 * (softmax - onehot(target)) * dscale on columns < V and 0 on [V, Vp)
 * (dlogits may alias logits). Fuses the reference's BatchSoftmaxForward +
 * BatchCrossEntropyForward + BatchCrossEntropySoftmaxBackward
 * (gpt2/cuda/softmax.cu:13-91, cross_entropy.cu:7-32; call sites
 * gpt2/cuda/gpt2cuda.cu:325,342,398). */
int llmk_softmax_crossentropy(float* losses, void* dlogits, const void* logits, llmk_dtype dtype, const int* targets,
                              int BT, int V, int Vp, float dscale, void* stream);
/* The three ops of the reference's unfused lm_head tail, one each (rows =
 * B*T, row stride ld = Vp, first V columns live; fp32 or bf16):
 * llmk_softmax_forward: probs[row, :V] = softmax(logits[row, :V]); columns
 * [V, ld) are left untouched. Replaces gpt2cuda::BatchSoftmaxForward
 * (gpt2/cuda/softmax.cu:13-91, softmax.cuh:8). */
int llmk_softmax_forward(void* probs, const void* logits, llmk_dtype dtype, int rows, int V, int ld, void* stream);
/* llmk_crossentropy_forward: losses[row] (+)= -log(probs[row, target[row]])
 * (accumulate != 0 adds, as the reference does; a target outside [0, ld)
 * gives NaN). Replaces gpt2cuda::BatchCrossEntropyForward
 * (gpt2/cuda/cross_entropy.cu:24-29, cross_entropy.cuh:9). */
int llmk_crossentropy_forward(float* losses, const void* probs, llmk_dtype dtype, const int* targets, int rows, int ld,
                              int accumulate, void* stream);
/* llmk_crossentropy_softmax_backward: dlogits[row, c] (+)= (probs[row, c] -
 * [c == target[row]]) * scale for c < V; [V, ld) untouched. Replaces
 * gpt2cuda::BatchCrossEntropySoftmaxBackward (gpt2/cuda/cross_entropy.cu:7-21,
 * cross_entropy.cuh:8), whose kernel computes (2 * dlogits + probs - onehot)
 * * scale: the same values on the zeroed buffer its caller passes
 * (gpt2cuda.cu ZeroGrad); accumulate = 0 overwrites. */
int llmk_crossentropy_softmax_backward(void* dlogits, const void* probs, llmk_dtype dtype, const int* targets,
                                       int rows, int V, int ld, float scale, int accumulate, void* stream);
/* ------------------------------- fused lm_head + softmax / cross-entropy */
/* logits[BT, Vp] = inp[BT, C] * W[Vp, C]^T (+ bias) on the tensor cores
 * (inp and W in the math mode's operand type: bf16, or fp32 for TF32), with
 * the epilogue folding each row into per-64-column (max, sum exp) statistics
 * in `workspace` (llmk_matmul_softmax_workspace bytes), then one pass per row.
 * llmk_matmul_softmax_forward: probs = softmax over the first V columns of each
 * row, 0 on [V, Vp); probs may alias logits. Replaces
 * gpt2cuda::BatchMatmulNTSoftmaxForward (gpt2/cuda/matmul_softmax.cu:9-110,
 * B*T rows flattened; the reference's weight is the same (Vp, C) row-major
 * buffer). */
size_t llmk_matmul_softmax_workspace(int BT, int Vp);
int llmk_matmul_softmax_forward(void* probs, void* logits, llmk_dtype dtype, const void* inp, const void* W,
                                const float* bias, int BT, int C, int Vp, int V, llmk_math math, void* workspace,
                                size_t workspace_bytes, void* stream);
/* The training step's lm_head + softmax + cross-entropy (+ its backward):
 * losses[row] = logsumexp(logits[row, :V]) - logits[row, target] (NaN for a
 * target outside [0, V)); with backward != 0 the logits buffer is then
 * overwritten by dlogits = (softmax - onehot(target)) * dscale, 0 on
 * [V, Vp). Replaces the reference step's lm_head matmul + Softmax +
 * CrossEntropy + CrossEntropySoftmaxBackward (gpt2/cuda/gpt2cuda.cu:323-325,
 * 398), in one GEMM and one pass over the logits. */
int llmk_matmul_crossentropy_forward(float* losses, void* logits, llmk_dtype dtype, const void* inp, const void* W,
                                     const float* bias, const int* targets, int BT, int C, int Vp, int V,
                                     float dscale, int backward, llmk_math math, void* workspace,
                                     size_t workspace_bytes, void* stream);
/* *out = mean(x[0..n)) on the device, fixed reduction order. */
int llmk_mean(float* out, const float* x, int n, void* stream);

/* ----------------------------------------------------------------- AdamW */
/* One launch over a flat parameter buffer: g' = g * grad_scale,
 * m = b1 m + (1-b1) g', v = b2 v + (1-b2) g'^2,
 * p -= lr (m/(1-b1^t) / (sqrt(v/(1-b2^t)) + eps) + wd p); params_bf16
 * (optional) receives bf16(p). n % 4 == 0.
 * Replaces gpt2cuda::AdamW (gpt2/cuda/adamw.cu:66-69), launched once per
 * parameter tensor by GPT2::Update (gpt2/cuda/gpt2cuda.cu:434-441). */
int llmk_adamw(float* params, void* params_bf16, const float* grads, float* m, float* v, long long n, float lr,
               float beta1, float beta2, float eps, float weight_decay, int t, float grad_scale, void* stream);

/* AdamW reading its hyperparameters from device memory: hparams = 8 floats
 * {lr, beta1, beta2, eps, weight_decay, 1/(1-beta1^t), 1/(1-beta2^t),
 * grad_scale} (16-byte aligned), filled on the host by llmk_adamw_hparams.
 * The reference has no counterpart (its AdamW takes host scalars,
 * gpt2/cuda/adamw.cu:33-44); this form lets a captured CUDA graph replay the
 * update with per-step values (llmk_gpt2_use_graph). */
void llmk_adamw_hparams(float* out8, float lr, float beta1, float beta2, float eps, float weight_decay, int t,
                        float grad_scale);
int llmk_adamw_device_hparams(float* params, void* params_bf16, const float* grads, float* m, float* v, long long n,
                              const float* hparams, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLMK_H_ */
