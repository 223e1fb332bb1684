// llmk_gpt2cuda.hpp — the reference's gpt2cuda:: op API over the llmk C ABI.
//
// Header-only adapter: a maintainer includes this instead of the reference's
// gpt2/cuda/{matmul,attention,layernorm,gelu,residual,adamw,encoder}.cuh and
// the layer/model code (gpt2/cuda/layer.cu, gpt2cuda.cu) compiles unchanged.
// Every function is a template over the caller's device-vector type (the
// reference's DevVecf / DevVeci, gpt2/cuda/devvector.cuh:8-131, or anything
// with .data() and .size()), keeps the reference's argument order and
// semantics, and throws on failure as the reference does (CUDA_CHECK ->
// exception, gpt2/cuda/error.cuh:5-7; bad shapes -> std::invalid_argument,
// kernel/flash_attn/flash_fwd_launch.cuh:21-31).
//
// Precision: the reference's fp32 GEMMs run as TF32 on the tensor cores
// (its CUTLASS Sm80 kernels are TF32, gpt2/cuda/matmul.cu:195-220); attention
// runs the tcgen05 kernels on fp16 copies of its fp32 operands (the
// reference's FA-2 rounds to tf32/fp16/bf16 internally, config.cuh:56,163-165).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <stdexcept>
#include <string>

#include "llmk.h"

namespace gpt2cuda {

namespace llmk_detail {

inline void check(int rc, const char* what) {
  if (rc == LLMK_OK) return;
  std::string msg = std::string(what) + ": " + llmk_status_string(rc) + " (" + llmk_last_error() + ")";
  if (rc == LLMK_ERR_INVALID_ARG || rc == LLMK_ERR_UNSUPPORTED) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

// Grow-only scratch owned by the adapter (one per host thread and device);
// the C ABI itself never allocates.
inline void* scratch(size_t bytes, int slot = 0) {
  struct Buf {
    void* p = nullptr;
    size_t n = 0;
    int dev = -1;
  };
  thread_local Buf bufs[4];
  int dev = 0;
  cudaGetDevice(&dev);
  Buf& b = bufs[slot];
  if (b.n < bytes || b.dev != dev) {
    if (b.p && b.dev == dev) cudaFree(b.p);
    if (cudaMalloc(&b.p, bytes) != cudaSuccess) throw std::runtime_error("llmk adapter: cudaMalloc failed");
    b.n = bytes;
    b.dev = dev;
  }
  return b.p;
}

template <class V>
inline const float* fptr(const V& v) {
  return v.size() ? reinterpret_cast<const float*>(v.data()) : nullptr;
}
template <class V>
inline float* fptr(V& v) {
  return v.size() ? reinterpret_cast<float*>(v.data()) : nullptr;
}

}  // namespace llmk_detail

// gpt2/cuda/matmul.cu:653-661. out[B*T,Oc] = in[B*T,C] * W[Oc,C]^T (+ bias).
template <class Vec>
void BatchMatmulNTForward(Vec& outputs, const Vec& inputs, const Vec& weight, const Vec& bias, int B, int T, int C,
                          int Oc, cudaStream_t stream) {
  llmk_detail::check(llmk_matmul_forward(outputs.data(), LLMK_F32, inputs.data(), weight.data(),
                                         llmk_detail::fptr(bias), B * T, C, Oc, LLMK_MATH_TF32, stream),
                     "BatchMatmulNTForward");
}

// gpt2/cuda/matmul.cu:663-669. dinp += dout*W; dW += dout^T*in; dbias = colsum(dout).
template <class Vec>
void BatchMatmulNTBackward(Vec& d_inputs, Vec& d_weight, Vec& d_bias, const Vec& d_outputs, const Vec& inputs,
                           const Vec& weight, int B, int T, int C, int Oc, cudaStream_t stream) {
  const size_t ws = llmk_matmul_backward_workspace(B * T, C, Oc, LLMK_MATH_TF32);
  llmk_detail::check(llmk_matmul_backward(d_inputs.data(), LLMK_F32, d_weight.data(), llmk_detail::fptr(d_bias),
                                          d_outputs.data(), inputs.data(), weight.data(), B * T, C, Oc,
                                          LLMK_MATH_TF32, LLMK_ACCUM_DINP | LLMK_ACCUM_DWEIGHT,
                                          llmk_detail::scratch(ws), ws, stream),
                     "BatchMatmulNTBackward");
}

// gpt2/cuda/attention.cu:119-133. logsumexp (B, NH, T).
template <class Vec>
void BatchCausalAttentionForward(Vec& outputs, Vec& logsumexp, const Vec& inputs, int B, int T, int C3, int NH,
                                 cudaStream_t stream) {
  const long long n_in = 1LL * B * T * C3;
  void* qkv = llmk_detail::scratch(n_in * 2, 1);
  llmk_detail::check(llmk_cast(qkv, LLMK_F16, inputs.data(), LLMK_F32, n_in, stream), "BatchCausalAttentionForward");
  llmk_detail::check(
      llmk_attention_forward(outputs.data(), LLMK_F32, logsumexp.data(), qkv, LLMK_F16, B, T, C3, NH, stream),
      "BatchCausalAttentionForward");
}

// gpt2/cuda/attention.cu:135-148. d_inputs (B,T,3C) accumulates dQ, dK, dV;
// att_D is unused (the D vector lives in the C ABI's workspace).
template <class Vec>
void BatchCausalAttentionBackward(Vec& d_inputs, Vec& att_D, const Vec& d_outputs, const Vec& outputs,
                                  const Vec& inputs, const Vec& logsumexp, int B, int T, int C3, int NH,
                                  cudaStream_t stream) {
  (void)att_D;
  const long long n_in = 1LL * B * T * C3;
  const size_t ws = llmk_attention_backward_workspace(B, T, C3, NH);
  char* base = static_cast<char*>(llmk_detail::scratch(ws + n_in * 6 + 1024, 3));
  void* qkv = base;
  float* dq32 = reinterpret_cast<float*>(base + n_in * 2);
  void* work = base + n_in * 6;
  const char* w = "BatchCausalAttentionBackward";
  llmk_detail::check(llmk_cast(qkv, LLMK_F16, inputs.data(), LLMK_F32, n_in, stream), w);
  llmk_detail::check(llmk_attention_backward(dq32, d_outputs.data(), outputs.data(), LLMK_F32, qkv, LLMK_F16,
                                             logsumexp.data(), B, T, C3, NH, work, ws, stream),
                     w);
  llmk_detail::check(llmk_residual_forward(d_inputs.data(), d_inputs.data(), dq32, LLMK_F32, n_in, stream), w);
}

// gpt2/cuda/layernorm.cu:348-353
template <class Vec>
void BatchLayerNormForward(Vec& outputs, Vec& means, Vec& rstds, const Vec& inputs, const Vec& gamma, const Vec& beta,
                           int B, int T, int C, cudaStream_t stream) {
  llmk_detail::check(llmk_layernorm_forward(outputs.data(), LLMK_F32, means.data(), rstds.data(), inputs.data(),
                                            gamma.data(), beta.data(), B * T, C, stream),
                     "BatchLayerNormForward");
}
template <class Vec>
void BatchLayerNormBackward(Vec& d_inputs, Vec& d_gamma, Vec& d_beta, const Vec& d_outputs, const Vec& inputs,
                            const Vec& gamma, const Vec& means, const Vec& rstds, int B, int T, int C,
                            cudaStream_t stream) {
  const size_t ws = llmk_layernorm_backward_workspace(B * T, C);
  llmk_detail::check(llmk_layernorm_backward(d_inputs.data(), nullptr, d_gamma.data(), d_beta.data(), nullptr,
                                             d_outputs.data(), LLMK_F32, inputs.data(), gamma.data(), means.data(),
                                             rstds.data(), B * T, C, LLMK_ACCUM_DINP | LLMK_ACCUM_DPARAM,
                                             llmk_detail::scratch(ws), ws, stream),
                     "BatchLayerNormBackward");
}

// gpt2/cuda/gelu.cu:85-90 (backward accumulates into d_inputs)
template <class Vec>
void BatchGeluForward(Vec& outputs, const Vec& inputs, int B, int T, int C, cudaStream_t stream) {
  llmk_detail::check(llmk_gelu_forward(outputs.data(), inputs.data(), LLMK_F32, 1LL * B * T * C, stream),
                     "BatchGeluForward");
}
template <class Vec>
void BatchGeluBackward(Vec& d_inputs, const Vec& d_outputs, const Vec& inputs, int B, int T, int C,
                       cudaStream_t stream) {
  llmk_detail::check(
      llmk_gelu_backward(d_inputs.data(), d_outputs.data(), inputs.data(), LLMK_F32, 1LL * B * T * C, 1, stream),
      "BatchGeluBackward");
}

// gpt2/cuda/residual.cu:74-81 (backward accumulates into both inputs)
template <class Vec>
void BatchResidualForward(Vec& outputs, const Vec& inputs1, const Vec& inputs2, size_t B, size_t T, size_t C,
                          cudaStream_t stream) {
  llmk_detail::check(llmk_residual_forward(outputs.data(), inputs1.data(), inputs2.data(), LLMK_F32,
                                           static_cast<long long>(B * T * C), stream),
                     "BatchResidualForward");
}
template <class Vec>
void BatchResidualBackward(Vec& d_inputs1, Vec& d_inputs2, const Vec& d_outputs, size_t B, size_t T, size_t C,
                           cudaStream_t stream) {
  llmk_detail::check(llmk_residual_backward(d_inputs1.data(), d_inputs2.data(), d_outputs.data(), LLMK_F32,
                                            static_cast<long long>(B * T * C), 1, stream),
                     "BatchResidualBackward");
}

// gpt2/cuda/encoder.cu:92-99
template <class VecF, class VecI>
void BatchEncoderForward(VecF& outputs, const VecI& inputs, const VecF& wte, const VecF& wpe, int B, int T, int C,
                         int V, int MaxT, cudaStream_t stream) {
  (void)V;
  (void)MaxT;
  llmk_detail::check(llmk_encoder_forward(outputs.data(), inputs.data(), wte.data(), wpe.data(), B, T, C, stream),
                     "BatchEncoderForward");
}
template <class VecF, class VecI>
void BatchEncoderBackward(VecF& d_wte, VecF& d_wpe, const VecF& d_outputs, const VecI& inputs, int B, int T, int C,
                          int Vp, int MaxT, cudaStream_t stream) {
  (void)MaxT;
  const size_t ws = llmk_encoder_backward_workspace(B, T);
  llmk_detail::check(llmk_encoder_backward(d_wte.data(), d_wpe.data(), d_outputs.data(), inputs.data(), B, T, C, Vp,
                                           llmk_detail::scratch(ws), ws, stream),
                     "BatchEncoderBackward");
}

// gpt2/cuda/adamw.cuh:5-17
struct AdamWConfig {
  float lr;
  float beta1;
  float beta2;
  float eps;
  float weight_decay;
  int t;
};
template <class Vec>
void AdamW(Vec& data, const Vec& grad_data, Vec& m, Vec& v, std::size_t size, const AdamWConfig& c,
           cudaStream_t stream) {
  llmk_detail::check(llmk_adamw(data.data(), nullptr, grad_data.data(), m.data(), v.data(),
                                static_cast<long long>(size), c.lr, c.beta1, c.beta2, c.eps, c.weight_decay, c.t, 1.0f,
                                stream),
                     "AdamW");
}

}  // namespace gpt2cuda
