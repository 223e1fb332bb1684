// Drives the reference's own CUDA trainer (gpt2cuda::GPT2 from
// gpt2/cuda/gpt2cuda.cu, gpt2cuda::Layer from layer.cu, compiled unchanged
// from the reference tree) linked against llm.cpp_b200/dropin/gpt2cuda_llmk.cu
// and libllmk.so instead of the reference's op sources (TEST INFRASTRUCTURE:
// it checks the drop-in boundary; built by `make -C oracle dropin`).
//
// The loop is the reference's training step (traincuda.cpp:284-302):
// Forward(losses) -> ZeroGrad -> Backward -> Update(lr, .9, .999, 1e-8, 0, t).
#include <cstdio>
#include <cstring>
#include <exception>
#include <fstream>
#include <vector>

#include "attention.cuh"
#include "gpt2cuda.h"
#include "matmul.cuh"
#include "pinvector.cuh"

#define LLMK_GPT2CUDA_LINK_LEVEL 1
#include "llmk_gpt2cuda.hpp"

namespace {
thread_local char g_err[512];

int fail(const char* what) {
  std::snprintf(g_err, sizeof(g_err), "%s", what);
  return 1;
}

// Reads the llm.c v3 header fields the workspace size needs.
bool read_config(const char* path, int* maxT, int* V, int* L, int* NH, int* C, int* Vp) {
  std::ifstream f(path, std::ios::binary);
  int h[8];
  if (!f.read(reinterpret_cast<char*>(h), sizeof(h))) return false;
  *maxT = h[2];
  *V = h[3];
  *L = h[4];
  *NH = h[5];
  *C = h[6];
  *Vp = h[7];
  return h[0] == 20240326;
}
}  // namespace

extern "C" {

const char* gpt2cuda_harness_error(void) { return g_err; }

// Trains the reference's gpt2cuda::GPT2 loaded from an llm.c v3 file for
// `steps` steps on one batch; losses[s] = mean per-token loss of step s.
int gpt2cuda_harness_train(const char* checkpoint, int B, int T, const int* inputs, const int* targets, int steps,
                           float lr, float* losses) {
  try {
    int maxT, V, L, NH, C, Vp;
    if (!read_config(checkpoint, &maxT, &V, &L, &NH, &C, &Vp)) return fail("bad checkpoint header");
    gpt2cuda::LlmkReserveWorkspace(B, T, C, NH, Vp);
    gpt2cuda::GPT2 model(checkpoint, B, T);
    auto stream = model.CreateStream();
    const size_t BT = static_cast<size_t>(B) * T;
    gpt2cuda::PinVeci in(inputs, inputs + BT), tg(targets, targets + BT);
    model.SetTrainData(stream, in, tg);
    gpt2cuda::DevVecf dloss(BT);
    std::vector<float> h(BT);
    for (int s = 0; s < steps; ++s) {
      dloss.zero(stream.GetStream());
      model.Forward(dloss, stream);
      model.ZeroGrad(stream);
      model.Backward(stream);
      model.Update(lr, 0.9f, 0.999f, 1e-8f, 0.0f, s + 1, stream);
      if (cudaMemcpyAsync(h.data(), dloss.data(), BT * sizeof(float), cudaMemcpyDeviceToHost,
                          stream.GetStream()) != cudaSuccess ||
          cudaStreamSynchronize(stream.GetStream()) != cudaSuccess)
        return fail("copying the losses failed");
      double sum = 0;
      for (float x : h) sum += x;
      losses[s] = static_cast<float>(sum / BT);
    }
    return 0;
  } catch (const std::exception& e) {
    return fail(e.what());
  }
}

// The reference's host-pointer test entry points (matmul.cuh:10,16;
// attention.cuh:6-7) as its CUDA tests call them, after reserving the
// drop-in's workspace for the shape.
int gpt2cuda_harness_matmul_host(float* out, float* dinp, float* dW, float* dbias, const float* dout, const float* inp,
                                 const float* W, const float* bias, int B, int T, int C, int Oc) {
  try {
    gpt2cuda::LlmkReserveWorkspace(B, T, C, 1, Oc);
    gpt2cuda::BatchMatmulNTForward(out, inp, W, bias, B, T, C, Oc);
    gpt2cuda::BatchMatmulNTBackward(dinp, dW, dbias, dout, inp, W, B, T, C, Oc);
    return 0;
  } catch (const std::exception& e) {
    return fail(e.what());
  }
}

int gpt2cuda_harness_attention_host(float* out, float* lse, float* dqkv, const float* dout, const float* qkv, int B,
                                    int T, int C3, int NH) {
  try {
    gpt2cuda::LlmkReserveWorkspace(B, T, C3 / 3, NH, 8);
    gpt2cuda::BatchCausalAttentionForward(out, lse, qkv, B, T, C3, NH);
    gpt2cuda::BatchCausalAttentionBackward(dqkv, dout, out, qkv, lse, B, T, C3, NH);
    return 0;
  } catch (const std::exception& e) {
    return fail(e.what());
  }
}

}  // extern "C"
