// Link-level drop-in for the reference's CUDA op sources.
//
// Build this file into the reference's CUDA trainer in place of
// gpt2/cuda/{matmul,attention,layernorm,gelu,residual,adamw,encoder,softmax,
// cross_entropy,matmul_softmax}.cu and link libllmk.so: the reference's own
// headers (its gpt2cuda:: declarations and DevVecf) stay, so gpt2cuda.cu,
// layer.cu and the tests compile unchanged and call the sm_100a kernels.
// Compile with the reference's include paths (gpt2/, gpt2/cuda/ and the
// CUTLASS util headers its devvector.cuh uses) plus this repository's
// include/. Before the first op, reserve or register the ops' workspace
// once per device (gpt2cuda::LlmkReserveWorkspace / LlmkSetWorkspace,
// include/llmk_gpt2cuda.hpp): the ops never allocate.
//
// Each definition below has the signature the reference declares (file:line
// of the declaration) and forwards to the adapter template of the same name.
#include "adamw.cuh"
#include "attention.cuh"
#include "cross_entropy.cuh"
#include "devvector.cuh"
#include "encoder.cuh"
#include "gelu.cuh"
#include "layernorm.cuh"
#include "matmul.cuh"
#include "matmul_softmax.cuh"
#include "residual.cuh"
#include "softmax.cuh"

#define LLMK_GPT2CUDA_LINK_LEVEL 1
#include "llmk_gpt2cuda.hpp"

namespace gpt2cuda {

// matmul.cuh:26
void BatchMatmulNTForward(DevVecf& outputs, const DevVecf& inputs, const DevVecf& weight, const DevVecf& bias, int B,
                          int T, int C, int Oc, cudaStream_t stream) {
  BatchMatmulNTForward<DevVecf>(outputs, inputs, weight, bias, B, T, C, Oc, stream);
}
// matmul.cuh:28
void BatchMatmulNTBackward(DevVecf& d_inputs, DevVecf& d_weight, DevVecf& d_bias, const DevVecf& d_outputs,
                           const DevVecf& inputs, const DevVecf& weight, int B, int T, int C, int Oc,
                           cudaStream_t stream) {
  BatchMatmulNTBackward<DevVecf>(d_inputs, d_weight, d_bias, d_outputs, inputs, weight, B, T, C, Oc, stream);
}
// matmul.cuh:10, 16 (host pointers)
void BatchMatmulNTForward(float* outputs, float const* inputs, float const* weight, float const* bias, int B, int T,
                          int C, int Oc) {
  llmk_detail::host_matmul_nt_forward(outputs, inputs, weight, bias, B, T, C, Oc);
}
void BatchMatmulNTBackward(float* d_inputs, float* d_weight, float* d_bias, float const* d_outputs,
                           float const* inputs, float const* weight, int B, int T, int C, int Oc) {
  llmk_detail::host_matmul_nt_backward(d_inputs, d_weight, d_bias, d_outputs, inputs, weight, B, T, C, Oc);
}

// attention.cuh:10-11
void BatchCausalAttentionForward(DevVecf& outputs, DevVecf& logsumexp, const DevVecf& inputs, int B, int T, int C3,
                                 int NH, cudaStream_t stream) {
  BatchCausalAttentionForward<DevVecf>(outputs, logsumexp, inputs, B, T, C3, NH, stream);
}
void BatchCausalAttentionBackward(DevVecf& d_inputs, DevVecf& att_D, const DevVecf& d_outputs, const DevVecf& outputs,
                                  const DevVecf& inputs, const DevVecf& logsumexp, int B, int T, int C3, int NH,
                                  cudaStream_t stream) {
  BatchCausalAttentionBackward<DevVecf>(d_inputs, att_D, d_outputs, outputs, inputs, logsumexp, B, T, C3, NH, stream);
}
// attention.cuh:6-7 (host pointers)
void BatchCausalAttentionForward(float* outputs, float* logsumexp, float const* inputs, int B, int T, int C3, int NH) {
  llmk_detail::host_causal_attention_forward(outputs, logsumexp, inputs, B, T, C3, NH);
}
void BatchCausalAttentionBackward(float* d_inputs, float const* d_outputs, float const* outputs, float const* inputs,
                                  float const* logsumexp, int B, int T, int C3, int NH) {
  llmk_detail::host_causal_attention_backward(d_inputs, d_outputs, outputs, inputs, logsumexp, B, T, C3, NH);
}

// layernorm.cuh:7-8
void BatchLayerNormForward(DevVecf& outputs, DevVecf& means, DevVecf& rstds, const DevVecf& inputs,
                           const DevVecf& gamma, const DevVecf& beta, int B, int T, int C, cudaStream_t stream) {
  BatchLayerNormForward<DevVecf>(outputs, means, rstds, inputs, gamma, beta, B, T, C, stream);
}
void BatchLayerNormBackward(DevVecf& d_inputs, DevVecf& d_gamma, DevVecf& d_beta, const DevVecf& d_outputs,
                            const DevVecf& inputs, const DevVecf& gamma, const DevVecf& means, const DevVecf& rstds,
                            int B, int T, int C, cudaStream_t stream) {
  BatchLayerNormBackward<DevVecf>(d_inputs, d_gamma, d_beta, d_outputs, inputs, gamma, means, rstds, B, T, C, stream);
}

// gelu.cuh:7-8
void BatchGeluForward(DevVecf& outputs, const DevVecf& inputs, int B, int T, int C, cudaStream_t stream) {
  BatchGeluForward<DevVecf>(outputs, inputs, B, T, C, stream);
}
void BatchGeluBackward(DevVecf& d_inputs, const DevVecf& d_outputs, const DevVecf& inputs, int B, int T, int C,
                       cudaStream_t stream) {
  BatchGeluBackward<DevVecf>(d_inputs, d_outputs, inputs, B, T, C, stream);
}

// residual.cuh:6-7
void BatchResidualForward(DevVecf& outputs, const DevVecf& inputs1, const DevVecf& inputs2, size_t B, size_t T,
                          size_t C, cudaStream_t stream) {
  BatchResidualForward<DevVecf>(outputs, inputs1, inputs2, B, T, C, stream);
}
void BatchResidualBackward(DevVecf& d_inputs1, DevVecf& d_inputs2, const DevVecf& d_outputs, size_t B, size_t T,
                           size_t C, cudaStream_t stream) {
  BatchResidualBackward<DevVecf>(d_inputs1, d_inputs2, d_outputs, B, T, C, stream);
}

// encoder.cuh:6-7
void BatchEncoderForward(DevVecf& outputs, const DevVeci& inputs, const DevVecf& wte, const DevVecf& wpe, int B, int T,
                         int C, int V, int MaxT, cudaStream_t stream) {
  BatchEncoderForward<DevVecf, DevVeci>(outputs, inputs, wte, wpe, B, T, C, V, MaxT, stream);
}
void BatchEncoderBackward(DevVecf& d_wte, DevVecf& d_wpe, const DevVecf& d_outputs, const DevVeci& inputs, int B,
                          int T, int C, int Vp, int MaxT, cudaStream_t stream) {
  BatchEncoderBackward<DevVecf, DevVeci>(d_wte, d_wpe, d_outputs, inputs, B, T, C, Vp, MaxT, stream);
}

// softmax.cuh:8-9
void BatchSoftmaxForward(DevVecf& outputs, const DevVecf& inputs, size_t B, size_t T, size_t V, size_t Vp,
                         cudaStream_t stream) {
  BatchSoftmaxForward<DevVecf>(outputs, inputs, B, T, V, Vp, stream);
}
void BatchSoftmaxBackward(DevVecf& d_inputs, const DevVecf& d_outputs, const DevVecf& inputs, size_t B, size_t T,
                          size_t V, size_t Vp, cudaStream_t stream) {
  BatchSoftmaxBackward<DevVecf>(d_inputs, d_outputs, inputs, B, T, V, Vp, stream);
}

// cross_entropy.cuh:8-9
void BatchCrossEntropySoftmaxBackward(DevVecf& d_logits, const DevVecf& probs, const DevVeci& targets, int B, int T,
                                      int V, int Vp, float scale, cudaStream_t stream) {
  BatchCrossEntropySoftmaxBackward<DevVecf, DevVeci>(d_logits, probs, targets, B, T, V, Vp, scale, stream);
}
void BatchCrossEntropyForward(DevVecf& losses, const DevVecf& inputs, const DevVeci& targets, int B, int T, int Vp,
                              cudaStream_t stream) {
  BatchCrossEntropyForward<DevVecf, DevVeci>(losses, inputs, targets, B, T, Vp, stream);
}

// matmul_softmax.cuh:8
std::size_t GetMatmulSoftmaxWorkSpaceSize(int B, int T, int Vp) {
  return llmk_detail::matmul_softmax_workspace_floats(B, T, Vp);
}
// matmul_softmax.cuh:5
void BatchMatmulNTSoftmaxForward(DevVecf& soft_outputs, DevVecf& outputs, DevVecf& workspace, const DevVecf& inputs,
                                 const DevVecf& weight, const DevVecf& bias, int B, int T, int C, int Vp, int V,
                                 cudaStream_t stream) {
  BatchMatmulNTSoftmaxForward<DevVecf>(soft_outputs, outputs, workspace, inputs, weight, bias, B, T, C, Vp, V,
                                       stream);
}

// adamw.cuh:16-17
void AdamW(DevVecf& data, const DevVecf& grad_data, DevVecf& m, DevVecf& v, std::size_t size,
           const AdamWConfig& config, cudaStream_t stream) {
  AdamW<DevVecf, AdamWConfig>(data, grad_data, m, v, size, config, stream);
}

}  // namespace gpt2cuda
