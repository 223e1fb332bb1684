// llmk_gpt2cuda.hpp — the reference's gpt2cuda:: op API over the llmk C ABI.
//
// Two ways to use it in the reference's CUDA trainer (gpt2/cuda/):
//  * header-only: include this instead of the reference's op headers
//    (gpt2/cuda/{matmul,attention,layernorm,gelu,residual,adamw,encoder,
//    softmax,cross_entropy,matmul_softmax}.cuh). Every op is a template over
//    the caller's device-vector type (the reference's DevVecf / DevVeci,
//    gpt2/cuda/devvector.cuh:8-131, or anything with .data() and .size()).
//  * link-level: keep the reference's headers and link
//    llm.cpp_b200/dropin/gpt2cuda_llmk.cu in place of the reference's op
//    sources (gpt2/cuda/{matmul,attention,layernorm,gelu,residual,adamw,
//    encoder,softmax,cross_entropy,matmul_softmax}.cu); it defines every
//    gpt2cuda:: op that gpt2cuda.cu and layer.cu call with the reference's
//    exact signatures, by instantiating the templates below.
// Either way each op keeps the reference's argument order and semantics and
// throws on failure as the reference does (CUDA_CHECK -> exception,
// gpt2/cuda/error.cuh:5-7; bad shapes -> std::invalid_argument,
// kernel/flash_attn/flash_fwd_launch.cuh:21-31).
//
// Scratch memory: the ops never allocate. The GEMM split-K partials, the
// attention's fp16 operand copy, D vector and dQ accumulator, and the
// LayerNorm / encoder partial sums come from ONE workspace per device that
// the caller registers once, before the first op (and before any stream
// capture): either its own device memory with LlmkSetWorkspace(ptr, bytes),
// sized by LlmkWorkspaceBytes(B, T, C, NH, Vp), or memory the adapter
// allocates then with LlmkReserveWorkspace(B, T, C, NH, Vp). An op called
// without one, or with one too small, throws std::runtime_error naming the
// size it needs. Ops on one device share the workspace: ops that can
// overlap on the GPU (different streams) must be ordered by the caller —
// the reference runs one step's ops on one stream.
//
// The host-pointer variants the reference's CUDA tests call (matmul.cuh:10,
// 16; attention.cuh:6-7) allocate, copy and synchronise per call, as the
// reference's own do (matmul.cu:513-651); they are test conveniences, not
// the training path.
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
#include <vector>

#include "llmk.h"

namespace gpt2cuda {

namespace llmk_detail {

inline void check(int rc, const char* what) {
  if (rc == LLMK_OK) return;
  std::string msg = std::string(what) + ": " + llmk_status_string(rc) + " (" + llmk_last_error() + ")";
  if (rc == LLMK_ERR_INVALID_ARG || rc == LLMK_ERR_UNSUPPORTED) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

inline void cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// The registered workspace of each device (one per process).
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool owned = false;
};
constexpr int kMaxDevices = 64;
inline Workspace& workspace_slot() {
  static Workspace slots[kMaxDevices];
  int dev = 0;
  cuda(cudaGetDevice(&dev), "llmk adapter: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("llmk adapter: device index out of range");
  return slots[dev];
}

// `bytes` of the current device's registered workspace; never allocates.
inline char* scratch(size_t bytes, const char* who) {
  Workspace& w = workspace_slot();
  if (!w.ptr || w.bytes < bytes)
    throw std::runtime_error(std::string(who) + ": llmk adapter workspace " +
                             (w.ptr ? "too small" : "not registered") + ": needs " + std::to_string(bytes) +
                             " bytes (LlmkSetWorkspace / LlmkReserveWorkspace before the first op)");
  return static_cast<char*>(w.ptr);
}

inline size_t round256(size_t n) { return (n + 255) / 256 * 256; }

template <class V>
inline const float* fptr(const V& v) {
  return v.size() ? reinterpret_cast<const float*>(v.data()) : nullptr;
}
template <class V>
inline float* fptr(V& v) {
  return v.size() ? reinterpret_cast<float*>(v.data()) : nullptr;
}

// Scratch of the attention ops: fp16 q/k/v copy | fp32 dqkv | the C ABI's workspace.
inline size_t attention_fwd_scratch(int B, int T, int C3) { return round256(2ull * B * T * C3); }
inline size_t attention_bwd_scratch(int B, int T, int C3, int NH) {
  return round256(2ull * B * T * C3) + round256(4ull * B * T * C3) + llmk_attention_backward_workspace(B, T, C3, NH);
}

}  // namespace llmk_detail

// Bytes of workspace the ops need for a GPT-2 step of B x T tokens, C
// channels, NH heads and a padded vocabulary of Vp: the largest single op.
inline size_t LlmkWorkspaceBytes(int B, int T, int C, int NH, int Vp) {
  using namespace llmk_detail;
  const int BT = B * T;
  size_t n = 0;
  auto take = [&](size_t x) { n = x > n ? x : n; };
  for (int oc : {3 * C, C, 4 * C, Vp}) take(llmk_matmul_backward_workspace(BT, C, oc, LLMK_MATH_TF32));
  take(llmk_matmul_backward_workspace(BT, 4 * C, C, LLMK_MATH_TF32));
  take(attention_fwd_scratch(B, T, 3 * C));
  take(attention_bwd_scratch(B, T, 3 * C, NH));
  take(llmk_layernorm_backward_workspace(BT, C));
  take(llmk_encoder_backward_workspace(B, T));
  return round256(n);
}

// Registers caller-owned device memory of the current device as the ops'
// workspace (replacing an earlier registration; memory the adapter reserved
// before is freed). ptr must stay valid while ops run.
inline void LlmkSetWorkspace(void* ptr, size_t bytes) {
  llmk_detail::Workspace& w = llmk_detail::workspace_slot();
  if (w.owned && w.ptr) llmk_detail::cuda(cudaFree(w.ptr), "LlmkSetWorkspace: cudaFree");
  w.ptr = ptr;
  w.bytes = bytes;
  w.owned = false;
}

// Allocates (once, at set-up) LlmkWorkspaceBytes(...) on the current device
// and registers it; a second call only grows it. Returns the bytes held.
inline size_t LlmkReserveWorkspace(int B, int T, int C, int NH, int Vp) {
  const size_t need = LlmkWorkspaceBytes(B, T, C, NH, Vp);
  llmk_detail::Workspace& w = llmk_detail::workspace_slot();
  if (w.ptr && w.bytes >= need) return w.bytes;
  void* p = nullptr;
  llmk_detail::cuda(cudaMalloc(&p, need), "LlmkReserveWorkspace: cudaMalloc");
  LlmkSetWorkspace(p, need);
  llmk_detail::workspace_slot().owned = true;
  return need;
}

// ------------------------------------------------------------------ matmul
// gpt2/cuda/matmul.cu:653-661. out[B*T,Oc] = in[B*T,C] * W[Oc,C]^T (+ bias);
// an empty bias means none (the lm_head, gpt2cuda.cu:323).
template <class Vec>
void BatchMatmulNTForward(Vec& outputs, const Vec& inputs, const Vec& weight, const Vec& bias, int B, int T, int C,
                          int Oc, cudaStream_t stream) {
  llmk_detail::check(llmk_matmul_forward(outputs.data(), LLMK_F32, inputs.data(), weight.data(),
                                         llmk_detail::fptr(bias), B * T, C, Oc, LLMK_MATH_TF32, stream),
                     "BatchMatmulNTForward");
}

// gpt2/cuda/matmul.cu:663-669. dinp += dout*W; dW += dout^T*in; dbias = colsum(dout)
// (an empty d_bias skips it).
template <class Vec>
void BatchMatmulNTBackward(Vec& d_inputs, Vec& d_weight, Vec& d_bias, const Vec& d_outputs, const Vec& inputs,
                           const Vec& weight, int B, int T, int C, int Oc, cudaStream_t stream) {
  const char* w = "BatchMatmulNTBackward";
  const size_t ws = llmk_matmul_backward_workspace(B * T, C, Oc, LLMK_MATH_TF32);
  llmk_detail::check(llmk_matmul_backward(d_inputs.data(), LLMK_F32, d_weight.data(), llmk_detail::fptr(d_bias),
                                          d_outputs.data(), inputs.data(), weight.data(), B * T, C, Oc,
                                          LLMK_MATH_TF32, LLMK_ACCUM_DINP | LLMK_ACCUM_DWEIGHT,
                                          llmk_detail::scratch(ws, w), ws, stream),
                     w);
}

// ---------------------------------------------------------------- attention
// gpt2/cuda/attention.cu:119-133. logsumexp (B, NH, T).
template <class Vec>
void BatchCausalAttentionForward(Vec& outputs, Vec& logsumexp, const Vec& inputs, int B, int T, int C3, int NH,
                                 cudaStream_t stream) {
  const char* w = "BatchCausalAttentionForward";
  const long long n_in = 1LL * B * T * C3;
  void* qkv = llmk_detail::scratch(llmk_detail::attention_fwd_scratch(B, T, C3), w);
  llmk_detail::check(llmk_cast(qkv, LLMK_F16, inputs.data(), LLMK_F32, n_in, stream), w);
  llmk_detail::check(
      llmk_attention_forward(outputs.data(), LLMK_F32, logsumexp.data(), qkv, LLMK_F16, B, T, C3, NH, stream), w);
}

// gpt2/cuda/attention.cu:135-148. d_inputs (B,T,3C) += dQ, dK, dV (the
// reference accumulates dQ and overwrites dK / dV: the same on the zeroed
// buffer its Layer passes, layer.cu:135, gpt2cuda.cu ZeroGrad); att_D is
// unused (the D vector lives in the workspace).
template <class Vec>
void BatchCausalAttentionBackward(Vec& d_inputs, Vec& att_D, const Vec& d_outputs, const Vec& outputs,
                                  const Vec& inputs, const Vec& logsumexp, int B, int T, int C3, int NH,
                                  cudaStream_t stream) {
  (void)att_D;
  const char* w = "BatchCausalAttentionBackward";
  const long long n_in = 1LL * B * T * C3;
  char* base = llmk_detail::scratch(llmk_detail::attention_bwd_scratch(B, T, C3, NH), w);
  void* qkv = base;
  float* dqkv32 = reinterpret_cast<float*>(base + llmk_detail::round256(2ull * n_in));
  void* work = base + llmk_detail::round256(2ull * n_in) + llmk_detail::round256(4ull * n_in);
  const size_t ws = llmk_attention_backward_workspace(B, T, C3, NH);
  llmk_detail::check(llmk_cast(qkv, LLMK_F16, inputs.data(), LLMK_F32, n_in, stream), w);
  llmk_detail::check(llmk_attention_backward(dqkv32, d_outputs.data(), outputs.data(), LLMK_F32, qkv, LLMK_F16,
                                             logsumexp.data(), B, T, C3, NH, work, ws, stream),
                     w);
  llmk_detail::check(llmk_residual_forward(d_inputs.data(), d_inputs.data(), dqkv32, LLMK_F32, n_in, stream), w);
}

// ---------------------------------------------------------------- layernorm
// gpt2/cuda/layernorm.cu:348-353 (backward accumulates d_inputs, d_gamma, d_beta)
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
  const char* w = "BatchLayerNormBackward";
  const size_t ws = llmk_layernorm_backward_workspace(B * T, C);
  llmk_detail::check(llmk_layernorm_backward(d_inputs.data(), nullptr, d_gamma.data(), d_beta.data(), nullptr,
                                             d_outputs.data(), LLMK_F32, inputs.data(), gamma.data(), means.data(),
                                             rstds.data(), B * T, C, LLMK_ACCUM_DINP | LLMK_ACCUM_DPARAM,
                                             llmk_detail::scratch(ws, w), ws, stream),
                     w);
}

// ------------------------------------------------------------ gelu, residual
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

// ------------------------------------------------------------------ encoder
// gpt2/cuda/encoder.cu:92-99 (backward accumulates into d_wte / d_wpe; V is
// the row count of wte, MaxT of wpe)
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
  const char* w = "BatchEncoderBackward";
  const size_t ws = llmk_encoder_backward_workspace(B, T);
  llmk_detail::check(llmk_encoder_backward(d_wte.data(), d_wpe.data(), d_outputs.data(), inputs.data(), B, T, C, Vp,
                                           llmk_detail::scratch(ws, w), ws, stream),
                     w);
}

// ------------------------------------------------- softmax + cross-entropy
// gpt2/cuda/softmax.cu (softmax.cuh:8): probs[:, :V] = softmax(logits[:, :V])
// per row of stride Vp; columns [V, Vp) untouched.
template <class Vec>
void BatchSoftmaxForward(Vec& outputs, const Vec& inputs, size_t B, size_t T, size_t V, size_t Vp,
                         cudaStream_t stream) {
  llmk_detail::check(llmk_softmax_forward(outputs.data(), inputs.data(), LLMK_F32, static_cast<int>(B * T),
                                          static_cast<int>(V), static_cast<int>(Vp), stream),
                     "BatchSoftmaxForward");
}
// softmax.cuh:9 — a no-op in the reference too (softmax.cu: empty body); the
// step's softmax gradient is fused into BatchCrossEntropySoftmaxBackward.
template <class Vec>
void BatchSoftmaxBackward(Vec& d_inputs, const Vec& d_outputs, const Vec& inputs, size_t B, size_t T, size_t V,
                          size_t Vp, cudaStream_t stream) {
  (void)d_inputs, (void)d_outputs, (void)inputs, (void)B, (void)T, (void)V, (void)Vp, (void)stream;
}

// cross_entropy.cu:24-29 (cross_entropy.cuh:9): losses[b*T+t] += -log(probs[.., target]).
template <class VecF, class VecI>
void BatchCrossEntropyForward(VecF& losses, const VecF& inputs, const VecI& targets, int B, int T, int Vp,
                              cudaStream_t stream) {
  llmk_detail::check(llmk_crossentropy_forward(losses.data(), inputs.data(), LLMK_F32, targets.data(), B * T, Vp, 1,
                                               stream),
                     "BatchCrossEntropyForward");
}

// cross_entropy.cu:7-21 (cross_entropy.cuh:8): dlogits[:, :V] = (probs -
// onehot) * scale. The reference kernel computes (2 * dlogits + probs -
// onehot) * scale, which is this on the zeroed dlogits its GPT2 passes
// (gpt2cuda.cu ZeroGrad memsets it); this one overwrites.
template <class VecF, class VecI>
void BatchCrossEntropySoftmaxBackward(VecF& d_logits, const VecF& probs, const VecI& targets, int B, int T, int V,
                                      int Vp, float scale, cudaStream_t stream) {
  llmk_detail::check(llmk_crossentropy_softmax_backward(d_logits.data(), probs.data(), LLMK_F32, targets.data(), B * T,
                                                        V, Vp, scale, 0, stream),
                     "BatchCrossEntropySoftmaxBackward");
}

namespace llmk_detail {
inline std::size_t matmul_softmax_workspace_floats(int B, int T, int Vp) {
  return (llmk_matmul_softmax_workspace(B * T, Vp) + sizeof(float) - 1) / sizeof(float);
}
}  // namespace llmk_detail
#ifndef LLMK_GPT2CUDA_LINK_LEVEL
// matmul_softmax.cuh:8: floats of the `workspace` BatchMatmulNTSoftmaxForward takes.
inline std::size_t GetMatmulSoftmaxWorkSpaceSize(int B, int T, int Vp) {
  return llmk_detail::matmul_softmax_workspace_floats(B, T, Vp);
}
#endif

// matmul_softmax.cu:9-110 (matmul_softmax.cuh:5): outputs = in * W^T (+ bias)
// (the logits, B*T x Vp) and soft_outputs = their softmax over the first V
// columns; workspace holds GetMatmulSoftmaxWorkSpaceSize(B, T, Vp) floats.
template <class Vec>
void BatchMatmulNTSoftmaxForward(Vec& soft_outputs, Vec& outputs, Vec& workspace, const Vec& inputs,
                                 const Vec& weight, const Vec& bias, int B, int T, int C, int Vp, int V,
                                 cudaStream_t stream) {
  const size_t ws = workspace.size() * sizeof(float);
  llmk_detail::check(llmk_matmul_softmax_forward(soft_outputs.data(), outputs.data(), LLMK_F32, inputs.data(),
                                                 weight.data(), llmk_detail::fptr(bias), B * T, C, Vp, V,
                                                 LLMK_MATH_TF32, workspace.data(), ws, stream),
                     "BatchMatmulNTSoftmaxForward");
}

// -------------------------------------------------------------------- AdamW
#ifndef LLMK_GPT2CUDA_LINK_LEVEL
// gpt2/cuda/adamw.cuh:5-17 (the link-level build takes the reference's own)
struct AdamWConfig {
  float lr;
  float beta1;
  float beta2;
  float eps;
  float weight_decay;
  int t;
};
#endif
template <class Vec, class Config>
void AdamW(Vec& data, const Vec& grad_data, Vec& m, Vec& v, std::size_t size, const Config& c, cudaStream_t stream) {
  llmk_detail::check(llmk_adamw(data.data(), nullptr, grad_data.data(), m.data(), v.data(),
                                static_cast<long long>(size), c.lr, c.beta1, c.beta2, c.eps, c.weight_decay, c.t, 1.0f,
                                stream),
                     "AdamW");
}

// ------------------------------------------------ host-pointer test variants
// matmul.cuh:10,16 and attention.cuh:6-7: host buffers in and out; device
// copies are allocated, filled and read back per call, synchronously (as the
// reference's own, matmul.cu:513-651). The workspace must be registered.
namespace llmk_detail {
struct DevBuf {
  float* p = nullptr;
  size_t n = 0;
  explicit DevBuf(size_t count, const float* host = nullptr) : n(count) {
    cuda(cudaMalloc(&p, (count ? count : 1) * sizeof(float)), "cudaMalloc");
    if (host && count) cuda(cudaMemcpy(p, host, count * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy");
  }
  ~DevBuf() { cudaFree(p); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  float* data() const { return p; }
  size_t size() const { return n; }
  void to_host(float* host) const {
    cuda(cudaMemcpy(host, p, n * sizeof(float), cudaMemcpyDeviceToHost), "cudaMemcpy");
  }
};

inline void host_matmul_nt_forward(float* outputs, float const* inputs, float const* weight, float const* bias, int B,
                                   int T, int C, int Oc) {
  DevBuf out(static_cast<size_t>(B) * T * Oc), in(static_cast<size_t>(B) * T * C, inputs),
      w(static_cast<size_t>(Oc) * C, weight), b(bias ? Oc : 0, bias);
  BatchMatmulNTForward<DevBuf>(out, in, w, b, B, T, C, Oc, nullptr);
  cuda(cudaDeviceSynchronize(), "BatchMatmulNTForward");
  out.to_host(outputs);
}

inline void host_matmul_nt_backward(float* d_inputs, float* d_weight, float* d_bias, float const* d_outputs,
                                    float const* inputs, float const* weight, int B, int T, int C, int Oc) {
  const size_t BT = static_cast<size_t>(B) * T;
  DevBuf di(BT * C, d_inputs), dw(static_cast<size_t>(Oc) * C, d_weight), db(d_bias ? Oc : 0, d_bias),
      dout(BT * Oc, d_outputs), in(BT * C, inputs), w(static_cast<size_t>(Oc) * C, weight);
  BatchMatmulNTBackward<DevBuf>(di, dw, db, dout, in, w, B, T, C, Oc, nullptr);
  cuda(cudaDeviceSynchronize(), "BatchMatmulNTBackward");
  di.to_host(d_inputs);
  dw.to_host(d_weight);
  if (d_bias) db.to_host(d_bias);
}

inline void host_causal_attention_forward(float* outputs, float* logsumexp, float const* inputs, int B, int T, int C3,
                                          int NH) {
  DevBuf out(static_cast<size_t>(B) * T * (C3 / 3)), lse(static_cast<size_t>(B) * NH * T),
      in(static_cast<size_t>(B) * T * C3, inputs);
  BatchCausalAttentionForward<DevBuf>(out, lse, in, B, T, C3, NH, nullptr);
  cuda(cudaDeviceSynchronize(), "BatchCausalAttentionForward");
  out.to_host(outputs);
  lse.to_host(logsumexp);
}

inline void host_causal_attention_backward(float* d_inputs, float const* d_outputs, float const* outputs,
                                           float const* inputs, float const* logsumexp, int B, int T, int C3,
                                           int NH) {
  const size_t n_in = static_cast<size_t>(B) * T * C3, n_out = n_in / 3;
  DevBuf din(n_in, d_inputs), D(static_cast<size_t>(B) * NH * T), dout(n_out, d_outputs), out(n_out, outputs),
      in(n_in, inputs), lse(static_cast<size_t>(B) * NH * T, logsumexp);
  BatchCausalAttentionBackward<DevBuf>(din, D, dout, out, in, lse, B, T, C3, NH, nullptr);
  cuda(cudaDeviceSynchronize(), "BatchCausalAttentionBackward");
  din.to_host(d_inputs);
}
}  // namespace llmk_detail

#ifndef LLMK_GPT2CUDA_LINK_LEVEL
// (the link-level build defines these out of line with the reference's declarations)
inline void BatchMatmulNTForward(float* outputs, float const* inputs, float const* weight, float const* bias, int B,
                                 int T, int C, int Oc) {
  llmk_detail::host_matmul_nt_forward(outputs, inputs, weight, bias, B, T, C, Oc);
}
inline void BatchMatmulNTBackward(float* d_inputs, float* d_weight, float* d_bias, float const* d_outputs,
                                  float const* inputs, float const* weight, int B, int T, int C, int Oc) {
  llmk_detail::host_matmul_nt_backward(d_inputs, d_weight, d_bias, d_outputs, inputs, weight, B, T, C, Oc);
}
inline void BatchCausalAttentionForward(float* outputs, float* logsumexp, float const* inputs, int B, int T, int C3,
                                        int NH) {
  llmk_detail::host_causal_attention_forward(outputs, logsumexp, inputs, B, T, C3, NH);
}
inline void BatchCausalAttentionBackward(float* d_inputs, float const* d_outputs, float const* outputs,
                                         float const* inputs, float const* logsumexp, int B, int T, int C3, int NH) {
  llmk_detail::host_causal_attention_backward(d_inputs, d_outputs, outputs, inputs, logsumexp, B, T, C3, NH);
}
#endif

}  // namespace gpt2cuda
