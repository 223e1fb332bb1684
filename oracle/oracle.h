/*
 * oracle.h — CPU fp32 restatement of llm.cpp's GPT-2 training path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared
 * against; it is never linked into, called by or shipped with the product
 * library (libllmk.so). Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it.
 *
 * Every function restates the reference CPU algorithm of the cited
 * gpt2/*.cpp lines (Eigen, column-major VecBTC) in plain C over row-major
 * buffers. Parity pins: tests/golden/reference_unit_vectors.json (the
 * literal PyTorch vectors of the reference's gtest suite) and the reference's
 * own CPU code compiled by oracle/Makefile into oracle/_ref/.
 */
#ifndef LLMK_ORACLE_H_
#define LLMK_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------- seeded data */
/* SplitMix64-seeded xoshiro256**; normals by Box-Muller in double (first
 * output of each pair), cast to fp32. stream separates independent uses of
 * one seed (0 = parameters, 1 = tokens, 2.. = test tensors). */
typedef struct orc_rng { uint64_t s[4]; } orc_rng;
void orc_rng_seed(orc_rng* r, uint64_t seed, uint64_t stream);
uint64_t orc_rng_next(orc_rng* r);
double orc_rng_uniform(orc_rng* r); /* (0, 1] */
void orc_fill_normal(float* out, size_t n, float stddev, uint64_t seed, uint64_t stream);
void orc_fill_tokens(int* out, size_t n, int vocab, uint64_t seed, uint64_t stream);

/* -------------------------------------------------------------- ops */
/* out[BT,OC] = inp[BT,C] * W[OC,C]^T + bias (bias may be NULL). gpt2/matmul.cpp:15-37 */
void orc_matmul_forward(float* out, const float* inp, const float* W, const float* bias, int BT, int C, int OC);
/* dinp += dout*W; dW += dout^T*inp; dbias += colsum(dout) (dbias may be NULL).
 * gpt2/matmul.cpp:40-71 (trans=false), :60-71 (trans=true: same math with
 * OC = the live vocabulary rows of wte). */
void orc_matmul_backward(float* dinp, float* dW, float* dbias, const float* dout, const float* inp, const float* W,
                         int BT, int C, int OC);
/* Causal attention over qkv (B,T,3C) -> out (B,T,C), att (B,NH,T,T) probabilities
 * (row t zero beyond t), lse (B,NH,T) = log sum_t1<=t exp(scale*q.k).
 * gpt2/attention.cpp:5-50,136-163; LSE as tests/gpt2/cuda/test_cuda_attention.cpp:46-54. */
void orc_attention_forward(float* out, float* att, float* lse, const float* qkv, int B, int T, int C, int NH);
/* dqkv += gradient of out given dout and the forward's att.
 * gpt2/attention.cpp:54-133,165-187 (d_pre_att restated in O(T^2) form:
 * att*(d_att - sum_t1 att*d_att), the same sum the reference's triple loop forms). */
void orc_attention_backward(float* dqkv, const float* dout, const float* qkv, const float* att, int B, int T, int C,
                            int NH);
/* gpt2/layernorm.cpp:7-35 (two-pass mean/variance, eps 1e-5) */
void orc_layernorm_forward(float* out, float* mean, float* rstd, const float* inp, const float* gamma,
                           const float* beta, int N, int C);
/* dinp = LN backward (overwrites); dgamma/dbeta accumulate. gpt2/layernorm.cpp:37-73 */
void orc_layernorm_backward(float* dinp, float* dgamma, float* dbeta, const float* dout, const float* inp,
                            const float* gamma, const float* mean, const float* rstd, int N, int C);
/* gpt2/gelu.cpp:5-18 and :20-37 (dinp = dout * gelu'(x), overwrites) */
void orc_gelu_forward(float* out, const float* inp, size_t n);
void orc_gelu_backward(float* dinp, const float* dout, const float* inp, size_t n);
/* gpt2/residual.cpp:5-25 */
void orc_residual_forward(float* out, const float* a, const float* b, size_t n);
/* probs[BT,V] = row softmax of logits[BT, ld] over the first V columns. gpt2/softmax.cpp:20-31 */
void orc_softmax(float* probs, const float* logits, int BT, int V, int ld);
/* mean NLL; losses[BT] per position. gpt2/cross_entropy.cpp:20-34 */
float orc_cross_entropy(float* losses, const float* probs, const int* targets, int BT, int V);
/* dlogits[BT, ld] += (probs - onehot) then /= BT (columns < V). gpt2/cross_entropy.cpp:6-18 */
void orc_cross_entropy_softmax_backward(float* dlogits, const float* probs, const int* targets, int BT, int V,
                                        int ld);
/* gpt2/encoder.cpp:5-20 and :22-40 */
void orc_encoder_forward(float* out, const int* tokens, const float* wte, const float* wpe, int B, int T, int C);
void orc_encoder_backward(float* dwte, float* dwpe, const float* dout, const int* tokens, int B, int T, int C);
/* gpt2/adamw.cpp:3-20 */
void orc_adamw(float* p, const float* g, float* m, float* v, size_t n, float lr, float beta1, float beta2, float eps,
               float weight_decay, int t);

/* --------------------------------------------------------------- model */
typedef struct orc_config {
  int max_seq_len, vocab_size, padded_vocab_size, num_layers, num_heads, channels;
} orc_config;
/* The 16 parameter tensors in llm.c v3 checkpoint order (gpt2/gpt2.cpp:112-230):
 * wte, wpe, ln1w, ln1b, qkvw, qkvb, attprojw, attprojb, ln2w, ln2b, fcw, fcb,
 * fcprojw, fcprojb, lnfw, lnfb. Returns the total. */
size_t orc_gpt2_param_sizes(const orc_config* cfg, size_t sizes[16]);
/* Seeded init: weights ~ N(0, 0.02) (attprojw, fcprojw scaled by
 * 1/sqrt(2L)), biases 0, LayerNorm gamma 1 / beta 0, wte rows >= V zero. */
void orc_gpt2_init_params(float* params, const orc_config* cfg, uint64_t seed);

typedef struct orc_gpt2 orc_gpt2;
orc_gpt2* orc_gpt2_create(const orc_config* cfg, const float* params, int B, int T);
void orc_gpt2_free(orc_gpt2* m);
/* gpt2/gpt2.cpp:232-279; returns the mean loss */
float orc_gpt2_forward(orc_gpt2* m, const int* inputs, const int* targets);
void orc_gpt2_zero_grad(orc_gpt2* m);                                /* gpt2.cpp:380-388 */
void orc_gpt2_backward(orc_gpt2* m);                                 /* gpt2.cpp:281-317 */
void orc_gpt2_update(orc_gpt2* m, float lr, float b1, float b2, float eps, float wd, int t); /* gpt2.cpp:390-409 */
float* orc_gpt2_params(orc_gpt2* m);
float* orc_gpt2_grads(orc_gpt2* m);
size_t orc_gpt2_num_params(orc_gpt2* m);
/* Activation probe for tests: name in {"logits","lnf","encoded"}; NULL if unknown. */
const float* orc_gpt2_activation(orc_gpt2* m, const char* name);

#ifdef __cplusplus
}
#endif

#endif /* LLMK_ORACLE_H_ */
