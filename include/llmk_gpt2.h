/*
 * llmk_gpt2.h — C ABI of the native GPT-2 trainer built on the llmk ops.
 *
 * The model owns its device buffers (like the reference's gpt2cuda::GPT2,
 * which holds every weight, gradient and activation in DevVecf members,
 * gpt2/cuda/gpt2cuda.h:90-147). Parameters cross the host boundary in llm.c
 * v3 checkpoint order (gpt2/gpt2.cpp:112-230): wte, wpe, ln1w, ln1b, qkvw,
 * qkvb, attprojw, attprojb, ln2w, ln2b, fcw, fcb, fcprojw, fcprojb, lnfw,
 * lnfb. All calls are asynchronous on the model's stream unless noted.
 */
#ifndef LLMK_GPT2_H_
#define LLMK_GPT2_H_

#include <stddef.h>

#include "llmk_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct llmk_gpt2_config {
  int max_seq_len;       /* e.g. 1024 */
  int vocab_size;        /* e.g. 50257 */
  int padded_vocab_size; /* e.g. 50304 */
  int num_layers;
  int num_heads;
  int channels;
} llmk_gpt2_config; /* mirrors GPT2Config, gpt2/gpt2.h:16-26 */

typedef struct llmk_gpt2 llmk_gpt2;

/* Number of parameters of a configuration (padded vocabulary included). */
size_t llmk_gpt2_num_parameters(const llmk_gpt2_config* cfg);
size_t llmk_gpt2_parameter_count(const llmk_gpt2* model);
/* The configuration the model was created with. */
int llmk_gpt2_get_config(const llmk_gpt2* model, llmk_gpt2_config* cfg);

/* Allocates a model for micro-batch B x T on the current device. math:
 * LLMK_MATH_BF16 (bf16 GEMM operands and activations, fp32 residual stream,
 * master weights and optimizer: the throughput mode) or LLMK_MATH_TF32 (fp32
 * activations, TF32 GEMMs, the reference GPU path's precision; attention
 * still runs on bf16 copies). stream: the cudaStream_t to run on, or NULL
 * for a private one. Head size must be 64.
 * Replaces gpt2cuda::GPT2 construction + Init (gpt2/cuda/gpt2cuda.cu:168-302). */
int llmk_gpt2_create(llmk_gpt2** out, const llmk_gpt2_config* cfg, int B, int T, int math, void* stream);
int llmk_gpt2_destroy(llmk_gpt2* model);
int llmk_gpt2_stream(llmk_gpt2* model, void** stream);
/* Device token buffers the model reads (B*T int32 each). */
int llmk_gpt2_buffers(llmk_gpt2* model, int** d_inputs, int** d_targets);

/* Parameters in llm.c order, host fp32; resets the AdamW state. Synchronous.
 * (The reference loads them from a checkpoint file, gpt2/cuda/gpt2cuda.cu:33-166.) */
int llmk_gpt2_load_parameters(llmk_gpt2* model, const float* host_params, size_t n);
int llmk_gpt2_read_parameters(llmk_gpt2* model, float* host_out, size_t n);
int llmk_gpt2_read_gradients(llmk_gpt2* model, float* host_out, size_t n);
/* AdamW first and second moments in llm.c order, host fp32 (new: the
 * reference keeps them only in device memory, gpt2/cuda/gpt2cuda.h:137-140).
 * Synchronous. */
int llmk_gpt2_read_optimizer_state(llmk_gpt2* model, float* host_m, float* host_v, size_t n);
int llmk_gpt2_load_optimizer_state(llmk_gpt2* model, const float* host_m, const float* host_v, size_t n);

/* ------------------------------------------------ checkpoint files */
/* llm.c v3 model file: 256 int32 header words ([0] = 20240326, [1] = 3,
 * [2] max_seq_len, [3] vocab_size, [4] num_layers, [5] num_heads,
 * [6] channels, [7] padded_vocab_size) followed by every parameter as fp32
 * in llm.c order — the file the reference's GPT2 constructors read
 * (gpt2/cuda/gpt2cuda.cu:33-166, gpt2/gpt2.cpp:112-230). Host only: reads
 * the header into *cfg, and checks the file holds exactly that model's
 * parameters. Bad magic / version / size -> LLMK_ERR_INVALID_ARG (the
 * reference prints and exit()s). */
int llmk_gpt2_checkpoint_config(const char* path, llmk_gpt2_config* cfg);
/* Loads a model file into a model of the same configuration (parameters,
 * bf16 copies; AdamW state reset). Synchronous. */
int llmk_gpt2_load_checkpoint(llmk_gpt2* model, const char* path);
/* Writes the model's parameters as a model file (new: the reference only
 * reads them). Written to path + ".tmp" and renamed, so an interrupted save
 * leaves the old file. Synchronous. */
int llmk_gpt2_save_checkpoint(llmk_gpt2* model, const char* path);

/* Training state (new; the reference has no resume path): the model file's
 * header words and parameters, then the AdamW moments m and v (fp32, llm.c
 * order), with header [0] = 20241202 (state magic), [1] = 1,
 * [2..7] = the configuration as above, [8] = optimizer steps taken,
 * [9] = world size that wrote it, [10..11] / [12..13] = data-loader shard and
 * sample position (int64, low word first). Replicated data parallelism keeps
 * the full state on every rank, so one rank saves and every rank loads. */
typedef struct llmk_train_state {
  int step;              /* AdamW steps done: the next update uses t = step + 1 */
  int world;             /* ranks of the run that saved it (informational) */
  long long shard_idx;   /* llmk_loader_position() of the next batch */
  long long sample_idx;
} llmk_train_state;
int llmk_gpt2_save_state(llmk_gpt2* model, const char* path, const llmk_train_state* state);
/* Restores parameters and AdamW moments and fills *state. Synchronous. */
int llmk_gpt2_load_state(llmk_gpt2* model, const char* path, llmk_train_state* state);

/* Copies B*T input (and target) tokens from host memory to the device,
 * through pinned staging. Replaces GPT2::SetTrainData (gpt2cuda.cu:350-367). */
int llmk_gpt2_set_train_data(llmk_gpt2* model, const int* host_inputs, const int* host_targets);
/* Forward over device tokens; with targets also computes the mean loss and
 * leaves dlogits ready for llmk_gpt2_backward.
 * Replaces GPT2::Forward (gpt2cuda.cu:338-345). */
int llmk_gpt2_forward(llmk_gpt2* model, const int* d_inputs, const int* d_targets);
/* Zeroes the gradients the backward accumulates into (GPT2::ZeroGrad, gpt2cuda.cu:548). */
int llmk_gpt2_zero_grad(llmk_gpt2* model);
/* Backward of the last forward; with data parallelism enabled, also the
 * gradient all-reduce (overlapped per layer). Replaces GPT2::Backward (gpt2cuda.cu:388-418). */
int llmk_gpt2_backward(llmk_gpt2* model);
/* AdamW over all parameters (gradients averaged over ranks).
 * Replaces GPT2::Update (gpt2cuda.cu:420-459). */
int llmk_gpt2_update(llmk_gpt2* model, float lr, float beta1, float beta2, float eps, float weight_decay, int t);
/* Mean loss of the last forward: host copy (synchronises the model stream)
 * or the device address. */
int llmk_gpt2_loss(llmk_gpt2* model, float* host_loss);
int llmk_gpt2_device_loss(llmk_gpt2* model, const float** d_loss);
/* forward + backward + update over device tokens. */
int llmk_gpt2_step_device(llmk_gpt2* model, const int* d_inputs, const int* d_targets, float lr, float beta1,
                          float beta2, float eps, float weight_decay, int t);
/* One full training step from host tokens to host loss (the loop body of
 * traincuda.cpp:286-323). host_loss may be NULL (no device->host copy). */
int llmk_gpt2_train_step(llmk_gpt2* model, const int* host_inputs, const int* host_targets, float lr, float beta1,
                         float beta2, float eps, float weight_decay, int t, float* host_loss);

/* ------------------------------------------------ data parallelism (new) */
/* Host-only, no device needed. Gradient buckets of the data-parallel
 * all-reduce as [begin, end) element ranges of the layer-major parameter
 * buffer, in issue order (layers L-1..0, then wte+wpe, then lnf). Writes
 * 2*count values when max_buckets >= count; returns count (L + 2). */
int llmk_gpt2_dp_buckets(const llmk_gpt2_config* cfg, size_t* ranges, int max_buckets);
/* Permutes a flat parameter (or gradient) vector between llm.c order and the
 * trainer's layer-major order (reverse = 0: llm.c -> layer-major). */
int llmk_gpt2_to_layer_major(const llmk_gpt2_config* cfg, const float* src, float* dst, int reverse);
/* 128-byte NCCL unique id, created on one rank and shared by the caller. */
int llmk_nccl_unique_id(void* out, size_t bytes);
/* Joins the model to a world of `world` replicas (one per GPU). */
int llmk_gpt2_enable_dp(llmk_gpt2* model, const void* unique_id, size_t bytes, int rank, int world);
/* Copies root's parameters to every rank (synchronous). */
int llmk_gpt2_broadcast_parameters(llmk_gpt2* model, int root);
/* Host-side bounded wait for the model's queued work, polling NCCL for
 * asynchronous errors; on error or after timeout_ms (>0) aborts the
 * communicator and returns LLMK_ERR_NCCL / LLMK_ERR_DEVICE_TIMEOUT. */
int llmk_gpt2_synchronize(llmk_gpt2* model, int timeout_ms);

/* CUDA-graph mode (enable != 0): llmk_gpt2_step_device (and so
 * llmk_gpt2_train_step) captures forward + backward + AdamW once into a CUDA
 * graph and then replays it, with the per-step AdamW values copied to device
 * memory before each replay; a call with other device token buffers captures
 * again. The reference launches every kernel each step
 * (gpt2/cuda/gpt2cuda.cu:304-459). Steps run eagerly while step timing is on. */
int llmk_gpt2_use_graph(llmk_gpt2* model, int enable);

/* ------------------------------------------------------- step timing */
/* Per-kernel-class device time of the training step. The reference has no
 * counterpart (its trainers time whole steps only, gpt2/traincuda.cpp). While
 * timing is on, every library call llmk_gpt2_forward / _backward / _update
 * makes is bracketed by two CUDA events on the model stream (a few
 * microseconds of device time per call); llmk_gpt2_set_timing also clears the
 * records. The report synchronises the model stream and sums, per class, the
 * calls, the kernel launches they made, their device time and their
 * algorithmic work: FLOPs (unit 0) for gemm / attention_fwd /
 * attention_bwd, HBM bytes with each operand read once and each result
 * written once (unit 1) for the bandwidth-bound classes. */
typedef struct llmk_kernel_stat {
  char name[24];
  long long calls;
  long long launches;
  double ms;
  double work;
  int unit;
} llmk_kernel_stat;
int llmk_gpt2_set_timing(llmk_gpt2* model, int enable);
/* Writes min(max, *count) records; *count = number of classes. */
int llmk_gpt2_timing_report(llmk_gpt2* model, llmk_kernel_stat* out, int max, int* count);

#ifdef __cplusplus
}
#endif

#endif /* LLMK_GPT2_H_ */
