/* llmk_status.h — status codes shared by the C ABI and the device code. */
#ifndef LLMK_STATUS_H_
#define LLMK_STATUS_H_

/* Host return codes. The reference reports the same conditions by throwing
 * (CUDA_CHECK, gpt2/cuda/error.cuh:5-7; std::invalid_argument,
 * gpt2/cuda/kernel/flash_attn/flash_fwd_launch.cuh:21-31) or exit(1)
 * (gpt2/cuda/matmul.cu:383-386, gpt2/cuda/attention.cu:130-132). */
#define LLMK_OK 0
#define LLMK_ERR_INVALID_ARG 1   /* bad shape / null pointer / inconsistent sizes */
#define LLMK_ERR_UNSUPPORTED 2   /* valid but not supported (alignment, head size) */
#define LLMK_ERR_CUDA 3          /* a CUDA runtime / driver call failed */
#define LLMK_ERR_DEVICE_TIMEOUT 4 /* a kernel's bounded wait expired */
#define LLMK_ERR_WORKSPACE 5     /* workspace missing or too small */
#define LLMK_ERR_NCCL 6          /* an NCCL call failed */
#define LLMK_ERR_NO_DEVICE 7     /* no CUDA device / not sm_100 */

/* Bits of the per-device status word written by kernels. */
#define LLMK_DEV_TIMEOUT 1u
/* a kernel found its dynamic shared memory less aligned than it declared
 * (it returned without doing any work) */
#define LLMK_DEV_SMEM_ALIGN 2u

#endif /* LLMK_STATUS_H_ */
