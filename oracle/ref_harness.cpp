// ref_harness.cpp — C entry points over the REFERENCE's own CPU code.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles the reference sources
// gpt2/{matmul,attention,layernorm,gelu,residual,softmax,cross_entropy,
// encoder,adamw,global,layer,gpt2}.cpp and utils/dataloader.cpp where they lie
// (read-only) together with this file into oracle/_ref/libref.so. Tests use it to pin the C
// restatement (oracle.c) and tests/golden/make_fixtures.py uses it to record
// the reference's 20-step loss trajectory; bench.py's reference arm times
// its training step. Buffers cross this boundary row-major; the reference's
// column-major Eigen matrices are filled through row-major maps.
#include <chrono>
#include <cstring>
#include <vector>

#include "attention.h"
#include "dataloader.h"
#include "gelu.h"
#include "global.h"
#include "gpt2.h"
#include "layernorm.h"
#include "matmul.h"

using RowMat = Eigen::Matrix<float, Eigen::Dynamic, Eigen::Dynamic, Eigen::RowMajor>;

static VecBTC to_btc(const float* x, int B, int T, int C) {
  VecBTC v(B);
  for (int b = 0; b < B; ++b) v[b] = Eigen::Map<const RowMat>(x + (size_t)b * T * C, T, C);
  return v;
}
static void from_btc(float* out, const VecBTC& v) {
  for (size_t b = 0; b < v.size(); ++b) {
    const int T = (int)v[b].rows(), C = (int)v[b].cols();
    Eigen::Map<RowMat>(out + b * (size_t)T * C, T, C) = v[b];
  }
}
// Reference weights are Eigen (C, OC) column-major: byte-identical to a
// row-major (OC, C) buffer.
static Matf to_weight(const float* W, int C, int OC) {
  Matf w(C, OC);
  std::memcpy(w.data(), W, sizeof(float) * (size_t)C * OC);
  return w;
}

extern "C" {

void ref_matmul_forward(float* out, const float* inp, const float* W, const float* bias, int B, int T, int C, int OC) {
  VecBTC x = to_btc(inp, B, T, C);
  Matf w = to_weight(W, C, OC);
  VecBTC y = bias ? MatMulForward(x, w, Eigen::Map<const Vecf>(bias, OC)) : MatMulForward(x, w);
  from_btc(out, y);
}

void ref_matmul_backward(float* dinp, float* dW, float* dbias, const float* dout, const float* inp, const float* W,
                         int B, int T, int C, int OC) {
  MatMul mm(C, OC);
  mm.weight = to_weight(W, C, OC);
  VecBTC d = mm.Backward(to_btc(dout, B, T, OC), to_btc(inp, B, T, C));
  from_btc(dinp, d);
  std::memcpy(dW, mm.d_weight.data(), sizeof(float) * (size_t)C * OC);
  std::memcpy(dbias, mm.d_bias.data(), sizeof(float) * (size_t)OC);
}

void ref_attention_forward(float* out, float* att, const float* qkv, int B, int T, int C, int NH) {
  Attention a(B, T, C, NH);
  VecBTC y = a.Forward(to_btc(qkv, B, T, 3 * C));
  from_btc(out, y);
  if (att) {
    for (int b = 0; b < B; ++b)
      for (int h = 0; h < NH; ++h)
        Eigen::Map<RowMat>(att + ((size_t)b * NH + h) * T * T, T, T) = a.att[b][h];
  }
}

void ref_attention_backward(float* dqkv, const float* dout, const float* qkv, int B, int T, int C, int NH) {
  Attention a(B, T, C, NH);
  VecBTC x = to_btc(qkv, B, T, 3 * C);
  VecBTC y = a.Forward(x);
  VecBTC d = a.Backward(to_btc(dout, B, T, C), x);
  from_btc(dqkv, d);
}

void ref_layernorm_forward(float* out, float* mean, float* rstd, const float* inp, const float* gamma, const float* beta,
                           int B, int T, int C) {
  LayerNorm ln(B, T, C);
  ln.gamma = Eigen::Map<const Vecf>(gamma, C);
  ln.beta = Eigen::Map<const Vecf>(beta, C);
  from_btc(out, ln.Forward(to_btc(inp, B, T, C)));
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) {
      mean[b * T + t] = ln.mean[b](t);
      rstd[b * T + t] = ln.rstd[b](t);
    }
}

void ref_layernorm_backward(float* dinp, float* dgamma, float* dbeta, const float* dout, const float* inp,
                            const float* gamma, const float* beta, int B, int T, int C) {
  LayerNorm ln(B, T, C);
  ln.gamma = Eigen::Map<const Vecf>(gamma, C);
  ln.beta = Eigen::Map<const Vecf>(beta, C);
  VecBTC x = to_btc(inp, B, T, C);
  VecBTC y = ln.Forward(x);
  from_btc(dinp, ln.Backward(to_btc(dout, B, T, C), x));
  std::memcpy(dgamma, ln.d_gamma.data(), sizeof(float) * C);
  std::memcpy(dbeta, ln.d_beta.data(), sizeof(float) * C);
}

void ref_gelu_forward(float* out, const float* inp, int B, int T, int C) {
  GELU g;
  from_btc(out, g.Forward(to_btc(inp, B, T, C)));
}

void ref_gelu_backward(float* dinp, const float* dout, const float* inp, int B, int T, int C) {
  GELU g;
  from_btc(dinp, g.Backward(to_btc(dout, B, T, C), to_btc(inp, B, T, C)));
}

// Loads an llm.c v3 checkpoint with the reference loader (gpt2/gpt2.cpp:112-230)
// and runs `steps` training steps on one fixed batch (inputs/targets, B*T
// each) exactly as train.cpp:123-146 does: Forward, ZeroGrad, Backward,
// Update(lr, 0.9, 0.999, 1e-8, 0, step+1). losses[i] = mean loss of step i;
// step_ms[i] = wall time of step i (may be NULL).
int ref_gpt2_train(const char* checkpoint, int B, int T, const int* inputs, const int* targets, int steps, float lr,
                   float* losses, double* step_ms) {
  GPT2 model(std::filesystem::path(checkpoint), B, T);
  std::vector<int> in(inputs, inputs + (size_t)B * T), tg(targets, targets + (size_t)B * T);
  for (int s = 0; s < steps; ++s) {
    auto t0 = std::chrono::steady_clock::now();
    model.Forward(in, tg);
    model.ZeroGrad();
    model.Backward();
    model.Update(lr, 0.9f, 0.999f, 1e-8f, 0.0f, s + 1);
    auto t1 = std::chrono::steady_clock::now();
    losses[s] = model.mean_loss;
    if (step_ms) step_ms[s] = std::chrono::duration<double, std::milli>(t1 - t0).count();
  }
  return 0;
}

// DataLoader (utils/dataloader.cpp) behind opaque handles. The reference
// exit()s on a bad shard, so callers pass only well-formed shard files.
void* ref_loader_create(const char* path, int B, int T, int rank, int world, int shuffle) {
  return new DataLoader(std::filesystem::path(path), (size_t)B, (size_t)T, (unsigned)rank, (unsigned)world,
                        shuffle != 0);
}
void ref_loader_destroy(void* l) { delete static_cast<DataLoader*>(l); }
void ref_loader_next(void* l, int* inputs, int* targets) { static_cast<DataLoader*>(l)->NextBatch(inputs, targets); }
void ref_loader_reset(void* l) { static_cast<DataLoader*>(l)->Reset(); }
void ref_loader_resume(void* l, size_t shard, size_t sample) { static_cast<DataLoader*>(l)->Resume(shard, sample); }
long long ref_loader_num_tokens(void* l) { return (long long)static_cast<DataLoader*>(l)->num_tokens; }

}  // extern "C"
