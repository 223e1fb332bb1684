// Native GPT-2 trainer on the llmk ops: the B200 counterpart of the
// reference's gpt2cuda::GPT2 and gpt2cuda::Layer (gpt2/cuda/gpt2cuda.h:34-190,
// gpt2/cuda/layer.cuh:5-102) with replicated data parallelism over NCCL.
//
// Precision (bf16 mode): fp32 master parameters, gradients and AdamW state; a
// bf16 copy of the parameters feeds the tensor-core GEMMs; activations that
// feed GEMMs or attention are bf16, the residual stream and its gradient are
// fp32. TF32 mode keeps every activation fp32 (TF32 GEMMs) and gives the
// attention MMAs an fp16 copy of q, k, v.
//
// Memory layout (HBM): parameters live LAYER-MAJOR in one flat buffer —
// [wte | wpe | layer 0 {ln1w ln1b qkvw qkvb attprojw attprojb ln2w ln2b fcw
// fcb fcprojw fcprojb} | ... | layer L-1 {...} | lnfw lnfb] — so each layer's
// gradients are one contiguous bucket for the data-parallel all-reduce, which
// is issued on a communication stream as soon as that layer's backward is
// done and overlaps the backward of the layers below. The llm.c v3 checkpoint
// order (tensor-major) is used only at the host boundary
// (llmk_gpt2_{load,read}_parameters).
//
// Per-step data flow mirrors gpt2/cuda/gpt2cuda.cu:304-459 and
// gpt2/cuda/layer.cu:151-266, with bias, residual add, GELU and GELU-backward
// fused into the GEMM epilogues and softmax + cross-entropy fused into one
// pass that turns logits into dlogits in place.
#include <cuda_fp16.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "llmk.h"
#include "llmk_gpt2.h"
#include "runtime.h"

namespace llmk {
namespace {

enum Tensor { WTE = 0, WPE, LN1W, LN1B, QKVW, QKVB, ATTPROJW, ATTPROJB, LN2W, LN2B, FCW, FCB, FCPROJW, FCPROJB, LNFW, LNFB };

// Sizes of the 16 llm.c tensors (gpt2/gpt2.cpp:112-230 read order); per-layer
// tensors are L times the per-layer size.
void tensor_sizes(const llmk_gpt2_config& c, size_t s[16]) {
  const size_t C = c.channels, L = c.num_layers;
  s[WTE] = static_cast<size_t>(c.padded_vocab_size) * C;
  s[WPE] = static_cast<size_t>(c.max_seq_len) * C;
  s[LN1W] = s[LN1B] = L * C;
  s[QKVW] = L * 3 * C * C;
  s[QKVB] = L * 3 * C;
  s[ATTPROJW] = L * C * C;
  s[ATTPROJB] = L * C;
  s[LN2W] = s[LN2B] = L * C;
  s[FCW] = L * 4 * C * C;
  s[FCB] = L * 4 * C;
  s[FCPROJW] = L * 4 * C * C;
  s[FCPROJB] = L * C;
  s[LNFW] = s[LNFB] = C;
}

template <typename T>
int dalloc(T** p, size_t n) {
  static_assert(!std::is_void<T>::value, "dalloc counts elements of a typed pointer");
  return cuda_check(cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
}

}  // namespace
}  // namespace llmk

using llmk::fail;

struct LayerParams {
  // offsets (elements) into the flat layer-major parameter buffer
  size_t ln1w, ln1b, qkvw, qkvb, attprojw, attprojb, ln2w, ln2b, fcw, fcb, fcprojw, fcprojb, begin, end;
};

struct LayerActs {
  float *ln1_mean, *ln1_rstd, *ln2_mean, *ln2_rstd, *lse, *res2, *res3;
  // GEMM operands in the activation dtype (bf16, or fp32 in tf32 mode)
  void *ln1, *qkv, *atty, *ln2, *fch_pre, *fch_gelu;
  __half* qkv16;  // tf32 mode only: fp16 copy of q, k, v for the attention MMAs
};

struct llmk_gpt2 {
  llmk_gpt2_config cfg{};
  int B = 0, T = 0, device = 0;
  cudaStream_t stream = nullptr, comm_stream = nullptr;
  // backward: weight gradients and bias column sums run on aux_stream beside
  // the input-gradient chain on `stream` (own workspace), forked and joined
  // with events
  cudaStream_t aux_stream = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_j1 = nullptr, ev_j2 = nullptr, ev_j3 = nullptr;
  void* workspace2 = nullptr;
  size_t workspace2_bytes = 0;
  bool own_stream = false;
  size_t nparams = 0;
  size_t tsize[16] = {};
  size_t off_wte = 0, off_wpe = 0, off_lnfw = 0, off_lnfb = 0;
  std::vector<LayerParams> lp;
  llmk_math math = LLMK_MATH_BF16;
  llmk_dtype adt = LLMK_BF16;  // activation dtype of GEMM operands
  size_t ae = 2;               // its element size
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr;
  __nv_bfloat16* params_bf16 = nullptr;  // bf16 mode only
  // activations
  float* encoded = nullptr;
  std::vector<LayerActs> acts;
  float *lnf_mean = nullptr, *lnf_rstd = nullptr, *losses = nullptr, *loss = nullptr;
  void *lnf = nullptr, *logits = nullptr;
  // backward scratch
  float *dres = nullptr, *dln = nullptr;
  __nv_bfloat16* dres_bf16 = nullptr;  // bf16 mode: GEMM copy of dres
  void *datty = nullptr, *dqkv = nullptr, *dfch = nullptr;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  int *inputs = nullptr, *targets = nullptr;
  int *h_inputs = nullptr, *h_targets = nullptr;  // pinned staging
  float* h_loss = nullptr;
  bool have_targets = false;
  // data parallel
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  std::vector<cudaEvent_t> layer_done;
  cudaEvent_t embed_done = nullptr, comm_done = nullptr, h2d_done = nullptr;
  // data parallel: lnf bucket issued, every bucket but the embeddings reduced
  cudaEvent_t lnf_done = nullptr, layers_reduced = nullptr;
  unsigned long long steps = 0;
  // per-kernel-class timing (llmk_gpt2_set_timing): event pairs on `stream`
  struct Mark {
    int cls;
    double work;
    int e0, e1;
    unsigned long long launches;
  };
  bool timing = false;
  std::vector<cudaEvent_t> tev;
  size_t tev_used = 0;
  std::vector<Mark> marks;
  // CUDA-graph mode (llmk_gpt2_use_graph)
  bool use_graph = false;
  cudaGraphExec_t graph_exec = nullptr;
  const int *graph_in = nullptr, *graph_tg = nullptr;
  unsigned long long graph_launches = 0;  // kernels one replay runs
  float* hp_dev = nullptr;  // AdamW hyperparameters read by the captured update
};

namespace {

int ensure_device(llmk_gpt2* g) { return llmk::cuda_check(cudaSetDevice(g->device), "cudaSetDevice"); }

// ------------------------------------------------------- step timing
// Kernel classes of one training step; work is algorithmic FLOPs for the
// tensor-core classes and algorithmic HBM bytes (each operand read once,
// each result written once) for the bandwidth classes.
// The GEMM classes split the tensor-core work by form: layer forward, layer
// input gradient, layer weight gradient, and all three forms of the tied
// lm_head.
enum KClass { KC_GEMM_FWD = 0, KC_GEMM_DINP, KC_GEMM_DW, KC_GEMM_LMHEAD, KC_ATTN_FWD, KC_ATTN_BWD, KC_LN_FWD,
              KC_LN_BWD, KC_XENT, KC_COLSUM, KC_ADAMW, KC_ENCODER, KC_CAST, KC_OTHER, KC_COUNT };
const char* const kClassName[KC_COUNT] = {"gemm_fwd", "gemm_dinp", "gemm_dweight", "gemm_lm_head", "attention_fwd",
                                          "attention_bwd", "layernorm_fwd", "layernorm_bwd", "softmax_xent", "colsum",
                                          "adamw", "encoder", "cast", "other"};
const int kClassUnit[KC_COUNT] = {0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1};  // 0 flop, 1 byte

int timing_event(llmk_gpt2* g) {
  if (g->tev_used == g->tev.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return -1;
    g->tev.push_back(e);
  }
  return static_cast<int>(g->tev_used++);
}

// Brackets the launches of one library call with two events on the model
// stream while timing is on; a no-op otherwise.
struct TimedScope {
  llmk_gpt2* g;
  cudaStream_t st;
  int idx = -1;
  TimedScope(llmk_gpt2* model, int cls, double work, cudaStream_t stream = nullptr)
      : g(model), st(stream ? stream : model->stream) {
    if (!g->timing) return;
    const int e0 = timing_event(g);
    if (e0 < 0 || cudaEventRecord(g->tev[e0], st) != cudaSuccess) return;
    idx = static_cast<int>(g->marks.size());
    g->marks.push_back({cls, work, e0, -1, llmk_launch_count()});
  }
  ~TimedScope() {
    if (idx < 0) return;
    const int e1 = timing_event(g);
    if (e1 < 0 || cudaEventRecord(g->tev[e1], st) != cudaSuccess) {
      g->marks.resize(idx);
      return;
    }
    g->marks[idx].e1 = e1;
    g->marks[idx].launches = llmk_launch_count() - g->marks[idx].launches;
  }
  TimedScope(const TimedScope&) = delete;
  TimedScope& operator=(const TimedScope&) = delete;
};

double causal_pairs(int T) { return 0.5 * static_cast<double>(T) * (T + 1); }

int nccl_check(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return LLMK_OK;
  return fail(LLMK_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

void layout(llmk_gpt2* g) {
  const size_t C = g->cfg.channels, L = g->cfg.num_layers;
  llmk::tensor_sizes(g->cfg, g->tsize);
  size_t o = 0;
  g->off_wte = o;
  o += g->tsize[llmk::WTE];
  g->off_wpe = o;
  o += g->tsize[llmk::WPE];
  g->lp.resize(L);
  for (size_t l = 0; l < L; ++l) {
    LayerParams& p = g->lp[l];
    p.begin = o;
    p.ln1w = o; o += C;
    p.ln1b = o; o += C;
    p.qkvw = o; o += 3 * C * C;
    p.qkvb = o; o += 3 * C;
    p.attprojw = o; o += C * C;
    p.attprojb = o; o += C;
    p.ln2w = o; o += C;
    p.ln2b = o; o += C;
    p.fcw = o; o += 4 * C * C;
    p.fcb = o; o += 4 * C;
    p.fcprojw = o; o += 4 * C * C;
    p.fcprojb = o; o += C;
    p.end = o;
  }
  g->off_lnfw = o;
  o += C;
  g->off_lnfb = o;
  o += C;
  g->nparams = o;
}

// Maps llm.c tensor-major order <-> layer-major order on the host.
// dir = 0: src is llm.c order, dst layer-major; dir = 1: the reverse.
void permute_params(const llmk_gpt2* g, const float* src, float* dst, int dir) {
  const size_t C = g->cfg.channels, L = g->cfg.num_layers;
  const size_t per[12] = {C, C, 3 * C * C, 3 * C, C * C, C, C, C, 4 * C * C, 4 * C, 4 * C * C, C};
  size_t llmc_off[16];
  size_t o = 0;
  for (int i = 0; i < 16; ++i) {
    llmc_off[i] = o;
    o += g->tsize[i];
  }
  auto copy = [&](size_t lm, size_t lay, size_t n) {
    if (dir == 0) std::memcpy(dst + lay, src + lm, n * sizeof(float));
    else std::memcpy(dst + lm, src + lay, n * sizeof(float));
  };
  copy(llmc_off[llmk::WTE], g->off_wte, g->tsize[llmk::WTE]);
  copy(llmc_off[llmk::WPE], g->off_wpe, g->tsize[llmk::WPE]);
  for (size_t l = 0; l < L; ++l) {
    const LayerParams& p = g->lp[l];
    const size_t lay[12] = {p.ln1w, p.ln1b, p.qkvw, p.qkvb, p.attprojw, p.attprojb,
                            p.ln2w, p.ln2b, p.fcw, p.fcb, p.fcprojw, p.fcprojb};
    for (int t = 0; t < 12; ++t) copy(llmc_off[2 + t] + l * per[t], lay[t], per[t]);
  }
  copy(llmc_off[llmk::LNFW], g->off_lnfw, C);
  copy(llmc_off[llmk::LNFB], g->off_lnfb, C);
}

void free_all(llmk_gpt2* g) {
  auto f = [](void* p) {
    if (p) cudaFree(p);
  };
  f(g->params); f(g->grads); f(g->m); f(g->v); f(g->params_bf16); f(g->encoded);
  for (auto& a : g->acts) {
    f(a.ln1_mean); f(a.ln1_rstd); f(a.ln2_mean); f(a.ln2_rstd); f(a.lse); f(a.res2); f(a.res3);
    f(a.ln1); f(a.qkv); f(a.atty); f(a.ln2); f(a.fch_pre); f(a.fch_gelu); f(a.qkv16);
  }
  f(g->lnf_mean); f(g->lnf_rstd); f(g->losses); f(g->loss); f(g->lnf); f(g->logits);
  f(g->dres); f(g->dln); f(g->dres_bf16); f(g->datty); f(g->dqkv); f(g->dfch); f(g->workspace);
  f(g->inputs); f(g->targets);
  if (g->h_inputs) cudaFreeHost(g->h_inputs);
  if (g->h_targets) cudaFreeHost(g->h_targets);
  if (g->h_loss) cudaFreeHost(g->h_loss);
  for (auto e : g->layer_done) cudaEventDestroy(e);
  if (g->embed_done) cudaEventDestroy(g->embed_done);
  if (g->comm_done) cudaEventDestroy(g->comm_done);
  if (g->lnf_done) cudaEventDestroy(g->lnf_done);
  if (g->layers_reduced) cudaEventDestroy(g->layers_reduced);
  if (g->h2d_done) cudaEventDestroy(g->h2d_done);
  for (auto e : g->tev) cudaEventDestroy(e);
  if (g->graph_exec) cudaGraphExecDestroy(g->graph_exec);
  f(g->hp_dev);
  if (g->comm) ncclCommDestroy(g->comm);
  if (g->comm_stream) cudaStreamDestroy(g->comm_stream);
  if (g->aux_stream) cudaStreamDestroy(g->aux_stream);
  for (cudaEvent_t e : {g->ev_fork, g->ev_j1, g->ev_j2, g->ev_j3})
    if (e) cudaEventDestroy(e);
  f(g->workspace2);
  if (g->own_stream && g->stream) cudaStreamDestroy(g->stream);
}

int alloc_all(llmk_gpt2* g) {
  using llmk::dalloc;
  const size_t B = g->B, T = g->T, C = g->cfg.channels, L = g->cfg.num_layers, NH = g->cfg.num_heads;
  const size_t BT = B * T, Vp = g->cfg.padded_vocab_size;
  LLMK_TRY(dalloc(&g->params, g->nparams));
  LLMK_TRY(dalloc(&g->grads, g->nparams));
  LLMK_TRY(dalloc(&g->m, g->nparams));
  LLMK_TRY(dalloc(&g->v, g->nparams));
  const bool bf = g->math == LLMK_MATH_BF16;
  const size_t ae = g->ae;
  auto aalloc = [&](void** p, size_t n) {
    return llmk::cuda_check(cudaMalloc(p, std::max<size_t>(n, 1) * ae), "cudaMalloc");
  };
  if (bf) LLMK_TRY(dalloc(&g->params_bf16, g->nparams));
  LLMK_CUDA(cudaMemset(g->m, 0, g->nparams * sizeof(float)));
  LLMK_CUDA(cudaMemset(g->v, 0, g->nparams * sizeof(float)));
  LLMK_CUDA(cudaMemset(g->grads, 0, g->nparams * sizeof(float)));
  LLMK_TRY(dalloc(&g->encoded, BT * C));
  g->acts.resize(L);
  for (auto& a : g->acts) {
    LLMK_TRY(dalloc(&a.ln1_mean, BT)); LLMK_TRY(dalloc(&a.ln1_rstd, BT));
    LLMK_TRY(dalloc(&a.ln2_mean, BT)); LLMK_TRY(dalloc(&a.ln2_rstd, BT));
    LLMK_TRY(dalloc(&a.lse, B * NH * T));
    LLMK_TRY(dalloc(&a.res2, BT * C)); LLMK_TRY(dalloc(&a.res3, BT * C));
    a.qkv16 = nullptr;
    LLMK_TRY(aalloc(&a.ln1, BT * C)); LLMK_TRY(aalloc(&a.qkv, BT * 3 * C)); LLMK_TRY(aalloc(&a.atty, BT * C));
    LLMK_TRY(aalloc(&a.ln2, BT * C)); LLMK_TRY(aalloc(&a.fch_pre, BT * 4 * C)); LLMK_TRY(aalloc(&a.fch_gelu, BT * 4 * C));
    if (!bf) LLMK_TRY(dalloc(&a.qkv16, BT * 3 * C));
  }
  LLMK_TRY(dalloc(&g->lnf_mean, BT)); LLMK_TRY(dalloc(&g->lnf_rstd, BT));
  LLMK_TRY(dalloc(&g->losses, BT)); LLMK_TRY(dalloc(&g->loss, 1));
  LLMK_TRY(aalloc(&g->lnf, BT * C)); LLMK_TRY(aalloc(&g->logits, BT * Vp));
  LLMK_TRY(dalloc(&g->dres, BT * C)); LLMK_TRY(dalloc(&g->dln, BT * C));
  if (bf) LLMK_TRY(dalloc(&g->dres_bf16, BT * C));
  LLMK_TRY(aalloc(&g->datty, BT * C)); LLMK_TRY(aalloc(&g->dqkv, BT * 3 * C)); LLMK_TRY(aalloc(&g->dfch, BT * 4 * C));
  LLMK_TRY(dalloc(&g->inputs, BT)); LLMK_TRY(dalloc(&g->targets, BT));
  LLMK_TRY(dalloc(&g->hp_dev, 8));
  LLMK_CUDA(cudaMallocHost(reinterpret_cast<void**>(&g->h_inputs), BT * sizeof(int)));
  LLMK_CUDA(cudaMallocHost(reinterpret_cast<void**>(&g->h_targets), BT * sizeof(int)));
  LLMK_CUDA(cudaMallocHost(reinterpret_cast<void**>(&g->h_loss), sizeof(float)));
  // one workspace, sized for the largest consumer
  const int iC = static_cast<int>(C), iBT = static_cast<int>(BT), iVp = static_cast<int>(Vp);
  size_t ws = 0;
  for (int oc : {3 * iC, iC, 4 * iC}) ws = std::max(ws, llmk_matmul_backward_workspace(iBT, iC, oc, g->math));
  ws = std::max(ws, llmk_matmul_backward_workspace(iBT, 4 * iC, iC, g->math));
  ws = std::max(ws, llmk_gemm_workspace(iVp, iC, iBT, g->math));
  ws = std::max(ws, llmk_layernorm_backward_workspace(iBT, iC));
  ws = std::max(ws, llmk_attention_backward_workspace(g->B, g->T, 3 * iC, static_cast<int>(NH)));
  ws = std::max(ws, llmk::rowstats_bytes(iBT, iVp));
  ws = std::max(ws, llmk_encoder_backward_workspace(g->B, g->T));
  g->workspace_bytes = ws;
  LLMK_CUDA(cudaMalloc(&g->workspace, std::max<size_t>(ws, 256)));
  g->layer_done.resize(L);
  for (auto& e : g->layer_done) LLMK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  LLMK_CUDA(cudaEventCreateWithFlags(&g->embed_done, cudaEventDisableTiming));
  LLMK_CUDA(cudaEventCreateWithFlags(&g->comm_done, cudaEventDisableTiming));
  LLMK_CUDA(cudaEventCreateWithFlags(&g->lnf_done, cudaEventDisableTiming));
  for (cudaEvent_t* e : {&g->ev_fork, &g->ev_j1, &g->ev_j2, &g->ev_j3})
    LLMK_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  // the side stream's workspace: split-K partials of every weight gradient and the column sums
  size_t ws2 = 0;
  for (int oc : {3 * iC, iC, 4 * iC}) ws2 = std::max(ws2, llmk_gemm_workspace(oc, iC, iBT, g->math));
  ws2 = std::max(ws2, llmk_gemm_workspace(iC, 4 * iC, iBT, g->math));
  ws2 = std::max(ws2, llmk_gemm_workspace(iVp, iC, iBT, g->math));
  ws2 = std::max(ws2, llmk_colsum_workspace(iBT, 4 * iC));
  g->workspace2_bytes = ws2;
  LLMK_CUDA(cudaMalloc(&g->workspace2, std::max<size_t>(ws2, 256)));
  LLMK_CUDA(cudaEventCreateWithFlags(&g->layers_reduced, cudaEventDisableTiming));
  LLMK_CUDA(cudaEventCreateWithFlags(&g->h2d_done, cudaEventDisableTiming));
  return LLMK_OK;
}

llmk_epilogue epi(const float* bias = nullptr, const float* residual = nullptr, long long ldr = 0, void* aux = nullptr,
                  long long ldaux = 0, int flags = 0) {
  llmk_epilogue e{};
  e.bias = bias;
  e.residual = residual;
  e.ldr = ldr;
  e.aux = aux;
  e.ldaux = ldaux;
  e.flags = flags;
  return e;
}

// Gradient all-reduce of one contiguous bucket on the comm stream, after `ev`
// (recorded on the model stream) and, when given, `aux_ev` (already recorded
// on the side stream).
int allreduce_bucket(llmk_gpt2* g, cudaEvent_t ev, size_t begin, size_t end, cudaEvent_t aux_ev = nullptr) {
  if (g->world <= 1) return LLMK_OK;
  LLMK_CUDA(cudaEventRecord(ev, g->stream));
  LLMK_CUDA(cudaStreamWaitEvent(g->comm_stream, ev, 0));
  if (aux_ev) LLMK_CUDA(cudaStreamWaitEvent(g->comm_stream, aux_ev, 0));
  return nccl_check(ncclAllReduce(g->grads + begin, g->grads + begin, end - begin, ncclFloat, ncclSum, g->comm,
                                  g->comm_stream),
                    "ncclAllReduce");
}

}  // namespace

extern "C" {

size_t llmk_gpt2_num_parameters(const llmk_gpt2_config* cfg) {
  if (!cfg) return 0;
  size_t s[16];
  llmk::tensor_sizes(*cfg, s);
  size_t n = 0;
  for (size_t x : s) n += x;
  return n;
}

int llmk_gpt2_create(llmk_gpt2** out, const llmk_gpt2_config* cfg, int B, int T, int math_mode, void* stream) {
  if (!out || !cfg || B <= 0 || T <= 0) return fail(LLMK_ERR_INVALID_ARG, "gpt2_create: bad arguments");
  if (math_mode != LLMK_MATH_BF16 && math_mode != LLMK_MATH_TF32)
    return fail(LLMK_ERR_INVALID_ARG, "gpt2_create: math mode");
  const llmk_math math = static_cast<llmk_math>(math_mode);
  if (T > cfg->max_seq_len || cfg->channels % cfg->num_heads || cfg->channels / cfg->num_heads != 64 ||
      cfg->padded_vocab_size < cfg->vocab_size || cfg->padded_vocab_size % 8 || cfg->channels % 64)
    return fail(LLMK_ERR_UNSUPPORTED, "gpt2_create: needs head size 64, C % 64 == 0, Vp % 8 == 0, T <= maxT");
  auto* g = new llmk_gpt2();
  g->cfg = *cfg;
  g->math = math;
  g->adt = math == LLMK_MATH_BF16 ? LLMK_BF16 : LLMK_F32;
  g->ae = math == LLMK_MATH_BF16 ? 2 : 4;
  g->B = B;
  g->T = T;
  int rc = llmk::cuda_check(cudaGetDevice(&g->device), "cudaGetDevice");
  if (rc == LLMK_OK) {
    if (stream) {
      g->stream = static_cast<cudaStream_t>(stream);
    } else {
      rc = llmk::cuda_check(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "cudaStreamCreate");
      g->own_stream = true;
    }
  }
  if (rc == LLMK_OK)
    rc = llmk::cuda_check(cudaStreamCreateWithFlags(&g->comm_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc == LLMK_OK)
    rc = llmk::cuda_check(cudaStreamCreateWithFlags(&g->aux_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc == LLMK_OK) {
    layout(g);
    rc = alloc_all(g);
  }
  if (rc != LLMK_OK) {
    free_all(g);
    delete g;
    return rc;
  }
  *out = g;
  return LLMK_OK;
}

int llmk_gpt2_destroy(llmk_gpt2* g) {
  if (!g) return LLMK_OK;
  cudaSetDevice(g->device);
  cudaStreamSynchronize(g->stream);
  cudaStreamSynchronize(g->comm_stream);
  free_all(g);
  delete g;
  return LLMK_OK;
}

size_t llmk_gpt2_parameter_count(const llmk_gpt2* g) { return g ? g->nparams : 0; }

int llmk_gpt2_get_config(const llmk_gpt2* g, llmk_gpt2_config* cfg) {
  if (!g || !cfg) return fail(LLMK_ERR_INVALID_ARG, "gpt2_get_config: null argument");
  *cfg = g->cfg;
  return LLMK_OK;
}

int llmk_gpt2_load_parameters(llmk_gpt2* g, const float* host_params, size_t n) {
  if (!g || !host_params || n != g->nparams) return fail(LLMK_ERR_INVALID_ARG, "gpt2_load_parameters: size mismatch");
  LLMK_TRY(ensure_device(g));
  std::vector<float> tmp(n);
  permute_params(g, host_params, tmp.data(), 0);
  // On the model's stream: a plain cudaMemcpy from pageable memory runs on the
  // legacy stream and may return before its DMA lands, which a kernel on the
  // model's non-blocking stream would not wait for.
  LLMK_CUDA(cudaMemcpyAsync(g->params, tmp.data(), n * sizeof(float), cudaMemcpyHostToDevice, g->stream));
  if (g->params_bf16)
    LLMK_TRY(llmk_cast(g->params_bf16, LLMK_BF16, g->params, LLMK_F32, static_cast<long long>(n), g->stream));
  LLMK_CUDA(cudaMemsetAsync(g->m, 0, n * sizeof(float), g->stream));
  LLMK_CUDA(cudaMemsetAsync(g->v, 0, n * sizeof(float), g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  return LLMK_OK;
}

static int read_flat(llmk_gpt2* g, const float* dev, float* host_out, size_t n) {
  if (!g || !host_out || n != g->nparams) return fail(LLMK_ERR_INVALID_ARG, "gpt2_read: size mismatch");
  LLMK_TRY(ensure_device(g));
  std::vector<float> tmp(n);
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->comm_stream));
  LLMK_CUDA(cudaMemcpy(tmp.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost));
  permute_params(g, tmp.data(), host_out, 1);
  return LLMK_OK;
}

int llmk_gpt2_read_parameters(llmk_gpt2* g, float* host_out, size_t n) { return read_flat(g, g ? g->params : nullptr, host_out, n); }
int llmk_gpt2_read_gradients(llmk_gpt2* g, float* host_out, size_t n) { return read_flat(g, g ? g->grads : nullptr, host_out, n); }

int llmk_gpt2_read_optimizer_state(llmk_gpt2* g, float* host_m, float* host_v, size_t n) {
  LLMK_TRY(read_flat(g, g ? g->m : nullptr, host_m, n));
  return read_flat(g, g->v, host_v, n);
}

int llmk_gpt2_load_optimizer_state(llmk_gpt2* g, const float* host_m, const float* host_v, size_t n) {
  if (!g || !host_m || !host_v || n != g->nparams)
    return fail(LLMK_ERR_INVALID_ARG, "gpt2_load_optimizer_state: size mismatch");
  LLMK_TRY(ensure_device(g));
  std::vector<float> tmp(n);
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  permute_params(g, host_m, tmp.data(), 0);
  LLMK_CUDA(cudaMemcpyAsync(g->m, tmp.data(), n * sizeof(float), cudaMemcpyHostToDevice, g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  permute_params(g, host_v, tmp.data(), 0);
  LLMK_CUDA(cudaMemcpyAsync(g->v, tmp.data(), n * sizeof(float), cudaMemcpyHostToDevice, g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  return LLMK_OK;
}

// Timed wrappers of the library calls the step makes (work = algorithmic
// FLOPs or HBM bytes of the call, for the per-class step report).
namespace {
struct StepOps {
  llmk_gpt2* g;
  cudaStream_t s;
  llmk_math mm;
  double ae;  // activation element size
  int gemm(int cls, void* D, llmk_dtype dt, long long ldd, const void* A, int at, long long lda, const void* Bm,
           int bt, long long ldb, int M, int N, int K, const llmk_epilogue* e, void* w, size_t wb) const {
    TimedScope ts(g, cls, 2.0 * M * N * K, s);
    return llmk_gemm(D, dt, ldd, A, at, lda, Bm, bt, ldb, mm, M, N, K, e, w, wb, s);
  }
  int ln_fwd(void* out, llmk_dtype dt, float* mean, float* rstd, const float* x, const float* w, const float* b,
             int N, int C) const {
    TimedScope ts(g, KC_LN_FWD, static_cast<double>(N) * C * (4.0 + ae) + 8.0 * N + 8.0 * C, s);
    return llmk_layernorm_forward(out, dt, mean, rstd, x, w, b, N, C, s);
  }
  int ln_bwd(float* dinp, void* mirror, float* dw, float* db, float* colsum, const float* dout, const float* x,
             const float* w, const float* mean, const float* rstd, int N, int C, int flags, void* ws,
             size_t wsb) const {
    const double dres = (flags & LLMK_ACCUM_DINP) ? 8.0 : 4.0;
    TimedScope ts(g, KC_LN_BWD,
                  static_cast<double>(N) * C * (4.0 + 4.0 + dres + (mirror ? 2.0 : 0.0)) + 8.0 * N + 16.0 * C, s);
    return llmk_layernorm_backward(dinp, mirror, dw, db, colsum, dout, LLMK_F32, x, w, mean, rstd, N, C, flags, ws,
                                   wsb, s);
  }
  int colsum(float* db, const void* x, llmk_dtype dt, int M, int N, void* ws, size_t wsb) const {
    TimedScope ts(g, KC_COLSUM, static_cast<double>(M) * N * ae + 4.0 * N, s);
    return llmk_colsum(db, x, dt, M, N, 0, ws, wsb, s);
  }
};
}  // namespace

int llmk_gpt2_forward(llmk_gpt2* g, const int* d_inputs, const int* d_targets) {
  if (!g || !d_inputs) return fail(LLMK_ERR_INVALID_ARG, "gpt2_forward: null argument");
  const int B = g->B, T = g->T, C = g->cfg.channels, NH = g->cfg.num_heads, L = g->cfg.num_layers;
  const int V = g->cfg.vocab_size, Vp = g->cfg.padded_vocab_size, BT = B * T;
  cudaStream_t s = g->stream;
  const float* P = g->params;
  const llmk_math mm = g->math;
  const llmk_dtype adt = g->adt;
  const bool bf = mm == LLMK_MATH_BF16;
  const StepOps op{g, s, mm, static_cast<double>(g->ae)};
  const double bt_c = static_cast<double>(BT) * C;
  // GEMM weights: the bf16 mirror in bf16 mode, the fp32 master in tf32 mode
  auto W = [&](size_t off) -> const void* {
    return bf ? static_cast<const void*>(g->params_bf16 + off) : static_cast<const void*>(P + off);
  };
  const int aux_f32 = bf ? 0 : LLMK_EPI_AUX_F32;
  if (d_inputs != g->inputs) LLMK_CUDA(cudaMemcpyAsync(g->inputs, d_inputs, BT * sizeof(int), cudaMemcpyDeviceToDevice, s));
  g->have_targets = d_targets != nullptr;
  if (d_targets && d_targets != g->targets)
    LLMK_CUDA(cudaMemcpyAsync(g->targets, d_targets, BT * sizeof(int), cudaMemcpyDeviceToDevice, s));
  // encoder (gpt2cuda.cu:313)
  {
    TimedScope ts(g, KC_ENCODER, bt_c * 12.0 + 4.0 * BT);
    LLMK_TRY(llmk_encoder_forward(g->encoded, g->inputs, P + g->off_wte, P + g->off_wpe, B, T, C, s));
  }
  const float* x = g->encoded;
  const double attn_flop = 4.0 * B * NH * (C / NH) * causal_pairs(T);
  for (int l = 0; l < L; ++l) {
    // Layer::Forward (gpt2/cuda/layer.cu:151-177)
    const LayerParams& p = g->lp[l];
    LayerActs& a = g->acts[l];
    LLMK_TRY(op.ln_fwd(a.ln1, adt, a.ln1_mean, a.ln1_rstd, x, P + p.ln1w, P + p.ln1b, BT, C));
    llmk_epilogue e1 = epi(P + p.qkvb);
    LLMK_TRY(op.gemm(KC_GEMM_FWD, a.qkv, adt, 3 * C, a.ln1, 0, C, W(p.qkvw), 0, C, BT, 3 * C, C, &e1, nullptr, 0));
    if (bf) {
      TimedScope ts(g, KC_ATTN_FWD, attn_flop);
      LLMK_TRY(llmk_attention_forward(a.atty, LLMK_BF16, a.lse, a.qkv, LLMK_BF16, B, T, 3 * C, NH, s));
    } else {
      // the attention MMAs take bf16 operands: round q, k, v once; the output
      // leaves the kernel in fp32
      {
        TimedScope ts(g, KC_CAST, bt_c * 3.0 * 6.0);
        LLMK_TRY(llmk_cast(a.qkv16, LLMK_F16, a.qkv, LLMK_F32, static_cast<long long>(BT) * 3 * C, s));
      }
      TimedScope ts(g, KC_ATTN_FWD, attn_flop);
      LLMK_TRY(llmk_attention_forward(a.atty, LLMK_F32, a.lse, a.qkv16, LLMK_F16, B, T, 3 * C, NH, s));
    }
    llmk_epilogue e2 = epi(P + p.attprojb, x, C);  // residual add fused
    LLMK_TRY(op.gemm(KC_GEMM_FWD, a.res2, LLMK_F32, C, a.atty, 0, C, W(p.attprojw), 0, C, BT, C, C, &e2, nullptr, 0));
    LLMK_TRY(op.ln_fwd(a.ln2, adt, a.ln2_mean, a.ln2_rstd, a.res2, P + p.ln2w, P + p.ln2b, BT, C));
    // GELU fused, pre-activation kept for the backward
    llmk_epilogue e3 = epi(P + p.fcb, nullptr, 0, a.fch_pre, 4 * C, LLMK_EPI_GELU | aux_f32);
    LLMK_TRY(op.gemm(KC_GEMM_FWD, a.fch_gelu, adt, 4 * C, a.ln2, 0, C, W(p.fcw), 0, C, BT, 4 * C, C, &e3, nullptr, 0));
    llmk_epilogue e4 = epi(P + p.fcprojb, a.res2, C);
    LLMK_TRY(op.gemm(KC_GEMM_FWD, a.res3, LLMK_F32, C, a.fch_gelu, 0, 4 * C, W(p.fcprojw), 0, 4 * C, BT, C, 4 * C, &e4, nullptr,
                     0));
    x = a.res3;
  }
  LLMK_TRY(op.ln_fwd(g->lnf, adt, g->lnf_mean, g->lnf_rstd, x, P + g->off_lnfw, P + g->off_lnfb, BT, C));
  // tied lm_head (gpt2cuda.cu:323): logits[BT, Vp] = lnf * wte^T, no bias
  if (!g->have_targets) {
    LLMK_TRY(op.gemm(KC_GEMM_LMHEAD, g->logits, adt, Vp, g->lnf, 0, C, W(g->off_wte), 0, C, BT, Vp, C, nullptr, nullptr, 0));
    return LLMK_OK;
  }
  // With targets, the lm_head GEMM's epilogue also reduces each row to
  // per-slot softmax statistics (in the workspace, free during the forward),
  // and one pass over the logits gives the losses and overwrites the logits
  // with dlogits = (softmax - onehot) / (B*T) (gpt2cuda.cu:325,398).
  auto* stats = static_cast<float2*>(g->workspace);
  {
    TimedScope ts(g, KC_GEMM_LMHEAD, 2.0 * BT * static_cast<double>(Vp) * C);
    LLMK_TRY(llmk::gemm_rowstats(g->logits, adt, Vp, g->lnf, C, W(g->off_wte), C, g->math, BT, Vp, C, nullptr, stats,
                                 V, s));
  }
  {
    TimedScope ts(g, KC_XENT, 2.0 * BT * static_cast<double>(Vp) * g->ae + llmk::rowstats_bytes(BT, Vp) + 8.0 * BT);
    LLMK_TRY(llmk::rowstats_finish(0, g->losses, g->logits, g->logits, adt, stats, g->targets, BT, V, Vp,
                                   1.0f / static_cast<float>(BT), 1, s));
  }
  TimedScope ts(g, KC_OTHER, 4.0 * BT);
  LLMK_TRY(llmk_mean(g->loss, g->losses, BT, s));
  return LLMK_OK;
}

int llmk_gpt2_zero_grad(llmk_gpt2* g) {
  // Every gradient is overwritten by its producer in llmk_gpt2_backward except
  // dwpe (accumulated by the encoder backward); the reference memsets all of
  // them (gpt2cuda.cu:514-565).
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_zero_grad");
  LLMK_CUDA(cudaMemsetAsync(g->grads + g->off_wpe, 0, g->tsize[llmk::WPE] * sizeof(float), g->stream));
  return LLMK_OK;
}

int llmk_gpt2_backward(llmk_gpt2* g) {
  if (!g || !g->have_targets) return fail(LLMK_ERR_INVALID_ARG, "gpt2_backward: forward with targets first");
  const int B = g->B, T = g->T, C = g->cfg.channels, NH = g->cfg.num_heads, L = g->cfg.num_layers;
  const int Vp = g->cfg.padded_vocab_size, BT = B * T;
  cudaStream_t s = g->stream;
  const float* P = g->params;
  const llmk_math mm = g->math;
  const llmk_dtype adt = g->adt;
  const bool bf = mm == LLMK_MATH_BF16;
  auto W = [&](size_t off) -> const void* {
    return bf ? static_cast<const void*>(g->params_bf16 + off) : static_cast<const void*>(P + off);
  };
  // the residual gradient as a GEMM operand: its bf16 mirror, or itself in tf32 mode
  const void* dres_op = bf ? static_cast<const void*>(g->dres_bf16) : static_cast<const void*>(g->dres);
  void* dres_mirror = bf ? g->dres_bf16 : nullptr;
  const int aux_f32 = bf ? 0 : LLMK_EPI_AUX_F32;
  float* G = g->grads;
  void* ws = g->workspace;
  const size_t wsb = g->workspace_bytes;
  const StepOps op{g, s, mm, static_cast<double>(g->ae)};
  const double bt_c = static_cast<double>(BT) * C;
  const double attn_flop = 10.0 * B * NH * (C / NH) * causal_pairs(T);
  {
    TimedScope ts(g, KC_OTHER, static_cast<double>(g->tsize[llmk::WPE]) * 4.0);
    LLMK_TRY(llmk_gpt2_zero_grad(g));
  }
  // Two streams: the input-gradient chain (dinp GEMMs, LayerNorm and
  // attention backward) on `s`; every weight gradient and bias column sum on
  // the side stream `a` with its own workspace, so they fill the gaps and
  // tails of the chain. fork: `a` waits for `s` to reach this point. A join
  // event marks where `a` is done reading something `s` overwrites next: the
  // bf16 residual gradient (dres_op) is rewritten by each LayerNorm backward.
  // With per-kernel-class timing on, everything runs on `s`: the events then
  // time each library call alone, not two overlapping ones (the step
  // without timing is what runs concurrently).
  cudaStream_t a = g->timing ? s : g->aux_stream;
  const StepOps opa{g, a, mm, static_cast<double>(g->ae)};
  void* ws2 = g->workspace2;
  const size_t wsb2 = g->workspace2_bytes;
  auto fork = [&]() -> int {
    if (a == s) return LLMK_OK;
    LLMK_CUDA(cudaEventRecord(g->ev_fork, s));
    LLMK_CUDA(cudaStreamWaitEvent(a, g->ev_fork, 0));
    return LLMK_OK;
  };
  auto mark = [&](cudaEvent_t ev) -> int { return llmk::cuda_check(cudaEventRecord(ev, a), "cudaEventRecord"); };
  auto wait_mark = [&](cudaEvent_t ev) -> int { return llmk::cuda_check(cudaStreamWaitEvent(s, ev, 0), "cudaStreamWaitEvent"); };
  // lm_head backward (gpt2cuda.cu:402): dlnf = dlogits * wte on s; dwte = dlogits^T * lnf on a
  LLMK_TRY(fork());
  LLMK_TRY(opa.gemm(KC_GEMM_LMHEAD, G + g->off_wte, LLMK_F32, C, g->logits, 1, Vp, g->lnf, 1, C, Vp, C, BT, nullptr,
                    ws2, wsb2));
  LLMK_TRY(op.gemm(KC_GEMM_LMHEAD, g->dln, LLMK_F32, C, g->logits, 0, Vp, W(g->off_wte), 1, C, BT, C, Vp, nullptr, nullptr, 0));
  const float* xL = L > 0 ? g->acts[L - 1].res3 : g->encoded;
  // the column sums of the new dres are the last layer's fcproj bias gradient
  LLMK_TRY(op.ln_bwd(g->dres, dres_mirror, G + g->off_lnfw, G + g->off_lnfb, L > 0 ? G + g->lp[L - 1].fcprojb : nullptr,
                     g->dln, xL, P + g->off_lnfw, g->lnf_mean, g->lnf_rstd, BT, C, 0, ws, wsb));
  // the final LayerNorm's gradients are final now: reduce them first
  LLMK_TRY(allreduce_bucket(g, g->lnf_done, g->off_lnfw, g->off_lnfw + 2 * static_cast<size_t>(C)));
  for (int l = L - 1; l >= 0; --l) {
    // Layer::Backward (gpt2/cuda/layer.cu:180-266); dres = d(layer output)
    const LayerParams& p = g->lp[l];
    LayerActs& a_ = g->acts[l];
    const float* x = l > 0 ? g->acts[l - 1].res3 : g->encoded;
    // fcproj: dW = dres^T fch_gelu (a), dfch = (dres Wfcproj) * gelu'(fch_pre) (s); its bias
    // gradient colsum(dres) came out of the LayerNorm backward that produced dres
    LLMK_TRY(fork());
    LLMK_TRY(opa.gemm(KC_GEMM_DW, G + p.fcprojw, LLMK_F32, 4 * C, dres_op, 1, C, a_.fch_gelu, 1, 4 * C, C, 4 * C, BT,
                      nullptr, ws2, wsb2));
    LLMK_TRY(mark(g->ev_j1));  // dres_op read
    llmk_epilogue eg = epi(nullptr, nullptr, 0, a_.fch_pre, 4 * C, LLMK_EPI_GELU_BWD | aux_f32);
    LLMK_TRY(op.gemm(KC_GEMM_DINP, g->dfch, adt, 4 * C, dres_op, 0, C, W(p.fcprojw), 1, 4 * C, BT, 4 * C, C, &eg, nullptr, 0));
    // fc: dW = dfch^T ln2, db = colsum(dfch) (a); dln2 = dfch Wfc (s)
    LLMK_TRY(fork());
    LLMK_TRY(opa.gemm(KC_GEMM_DW, G + p.fcw, LLMK_F32, C, g->dfch, 1, 4 * C, a_.ln2, 1, C, 4 * C, C, BT, nullptr, ws2,
                      wsb2));
    LLMK_TRY(opa.colsum(G + p.fcb, g->dfch, adt, BT, 4 * C, ws2, wsb2));
    LLMK_TRY(op.gemm(KC_GEMM_DINP, g->dln, LLMK_F32, C, g->dfch, 0, 4 * C, W(p.fcw), 1, C, BT, C, 4 * C, nullptr, nullptr, 0));
    // ln2: dres += LN2 backward (dres becomes d(res2)); its column sums are the
    // attproj bias gradient
    LLMK_TRY(wait_mark(g->ev_j1));
    LLMK_TRY(op.ln_bwd(g->dres, dres_mirror, G + p.ln2w, G + p.ln2b, G + p.attprojb, g->dln, a_.res2, P + p.ln2w,
                       a_.ln2_mean, a_.ln2_rstd, BT, C, LLMK_ACCUM_DINP, ws, wsb));
    // attproj: dW = dres^T atty (a), datty = dres Wproj (s)
    LLMK_TRY(fork());
    LLMK_TRY(opa.gemm(KC_GEMM_DW, G + p.attprojw, LLMK_F32, C, dres_op, 1, C, a_.atty, 1, C, C, C, BT, nullptr, ws2,
                      wsb2));
    LLMK_TRY(mark(g->ev_j2));  // dres_op read
    LLMK_TRY(op.gemm(KC_GEMM_DINP, g->datty, adt, C, dres_op, 0, C, W(p.attprojw), 1, C, BT, C, C, nullptr, nullptr, 0));
    // attention
    // (tf32 mode: fp32 dO, O and dqkv; q, k, v from the fp16 copy the forward made)
    {
      TimedScope ts(g, KC_ATTN_BWD, attn_flop);
      LLMK_TRY(llmk_attention_backward(g->dqkv, g->datty, a_.atty, adt, bf ? static_cast<const void*>(a_.qkv) : a_.qkv16,
                                       bf ? LLMK_BF16 : LLMK_F16, a_.lse, B, T, 3 * C, NH,
                                       ws, wsb, s));
    }
    // qkv: dW = dqkv^T ln1, db = colsum(dqkv) (a); dln1 = dqkv Wqkv (s)
    LLMK_TRY(fork());
    LLMK_TRY(opa.gemm(KC_GEMM_DW, G + p.qkvw, LLMK_F32, C, g->dqkv, 1, 3 * C, a_.ln1, 1, C, 3 * C, C, BT, nullptr, ws2,
                      wsb2));
    LLMK_TRY(opa.colsum(G + p.qkvb, g->dqkv, adt, BT, 3 * C, ws2, wsb2));
    LLMK_TRY(mark(g->ev_j3));  // this layer's weight and bias gradients are final
    LLMK_TRY(op.gemm(KC_GEMM_DINP, g->dln, LLMK_F32, C, g->dqkv, 0, 3 * C, W(p.qkvw), 1, C, BT, C, 3 * C, nullptr, nullptr, 0));
    // ln1: dres += LN1 backward (dres becomes d(layer input)); its column sums are
    // the previous layer's fcproj bias gradient
    LLMK_TRY(wait_mark(g->ev_j2));
    LLMK_TRY(op.ln_bwd(g->dres, dres_mirror, G + p.ln1w, G + p.ln1b, l > 0 ? G + g->lp[l - 1].fcprojb : nullptr, g->dln,
                       x, P + p.ln1w, a_.ln1_mean, a_.ln1_rstd, BT, C, LLMK_ACCUM_DINP, ws, wsb));
    // this layer's gradients are final: reduce them while the layers below run
    LLMK_TRY(allreduce_bucket(g, g->layer_done[l], p.begin, p.end, g->ev_j3));
  }
  // the side stream rejoins before the encoder adds into dwte (the lm_head's
  // weight gradient) and before the step ends
  LLMK_TRY(mark(g->ev_j1));
  LLMK_TRY(wait_mark(g->ev_j1));
  // encoder backward (gpt2cuda.cu:413): dwte += scatter, dwpe += sum over batch
  {
    TimedScope ts(g, KC_ENCODER, bt_c * 12.0 + 8.0 * static_cast<double>(T) * C + 4.0 * BT);
    LLMK_TRY(llmk_encoder_backward(G + g->off_wte, G + g->off_wpe, g->dres, g->inputs, B, T, C, Vp, ws, wsb, s));
  }
  // Everything but the embeddings is reduced once the comm stream passes
  // here; the wte/wpe bucket (the encoder backward's scatter completes it)
  // goes last, and llmk_gpt2_update updates every other parameter while it
  // is still being reduced.
  if (g->world > 1) LLMK_CUDA(cudaEventRecord(g->layers_reduced, g->comm_stream));
  LLMK_TRY(allreduce_bucket(g, g->embed_done, g->off_wte, g->off_wpe + g->tsize[llmk::WPE]));
  if (g->world > 1) LLMK_CUDA(cudaEventRecord(g->comm_done, g->comm_stream));
  return LLMK_OK;
}

// AdamW over the flat buffer: one multi-tensor launch (the reference launches
// one AdamW per tensor, gpt2cuda.cu:434-441), gradients averaged over ranks.
// Under data parallelism it runs in two ranges: every parameter but the
// embeddings as soon as their buckets are reduced, then wte / wpe once
// their bucket is — so that update overlaps the embedding all-reduce, the
// one the backward cannot hide. hp: the hyperparameters in device memory
// (the form a captured graph replays), or nullptr to pass them by value.
static int adamw_ranges(llmk_gpt2* g, const float* hp, float lr, float beta1, float beta2, float eps,
                        float weight_decay, int t) {
  const float scale = 1.0f / static_cast<float>(g->world);
  auto range = [&](size_t begin, size_t end) -> int {
    // p, g, m, v read; p, m, v written; plus the bf16 mirror in bf16 mode
    TimedScope ts(g, KC_ADAMW, static_cast<double>(end - begin) * (28.0 + (g->params_bf16 ? 2.0 : 0.0)));
    __nv_bfloat16* pb = g->params_bf16 ? g->params_bf16 + begin : nullptr;
    const long long n = static_cast<long long>(end - begin);
    if (hp)
      return llmk_adamw_device_hparams(g->params + begin, pb, g->grads + begin, g->m + begin, g->v + begin, n, hp,
                                       g->stream);
    return llmk_adamw(g->params + begin, pb, g->grads + begin, g->m + begin, g->v + begin, n, lr, beta1, beta2, eps,
                      weight_decay, t, scale, g->stream);
  };
  if (g->world <= 1) return range(0, g->nparams);
  const size_t emb_end = g->off_wpe + g->tsize[llmk::WPE];  // [wte | wpe] lead the flat buffer
  LLMK_CUDA(cudaStreamWaitEvent(g->stream, g->layers_reduced, 0));
  LLMK_TRY(range(emb_end, g->nparams));
  LLMK_CUDA(cudaStreamWaitEvent(g->stream, g->comm_done, 0));
  return range(0, emb_end);
}

static int update_device_hparams(llmk_gpt2* g) { return adamw_ranges(g, g->hp_dev, 0.f, 0.f, 0.f, 0.f, 0.f, 1); }

int llmk_gpt2_update(llmk_gpt2* g, float lr, float beta1, float beta2, float eps, float weight_decay, int t) {
  if (!g || t < 1) return fail(LLMK_ERR_INVALID_ARG, "gpt2_update");
  LLMK_TRY(adamw_ranges(g, nullptr, lr, beta1, beta2, eps, weight_decay, t));
  ++g->steps;
  return LLMK_OK;
}

int llmk_gpt2_set_train_data(llmk_gpt2* g, const int* host_inputs, const int* host_targets) {
  if (!g || !host_inputs) return fail(LLMK_ERR_INVALID_ARG, "gpt2_set_train_data");
  const size_t BT = static_cast<size_t>(g->B) * g->T;
  // the pinned staging buffers are reused: the previous step's copies out of
  // them must have finished before they are overwritten
  LLMK_CUDA(cudaEventSynchronize(g->h2d_done));
  std::memcpy(g->h_inputs, host_inputs, BT * sizeof(int));
  LLMK_CUDA(cudaMemcpyAsync(g->inputs, g->h_inputs, BT * sizeof(int), cudaMemcpyHostToDevice, g->stream));
  if (host_targets) {
    std::memcpy(g->h_targets, host_targets, BT * sizeof(int));
    LLMK_CUDA(cudaMemcpyAsync(g->targets, g->h_targets, BT * sizeof(int), cudaMemcpyHostToDevice, g->stream));
  }
  LLMK_CUDA(cudaEventRecord(g->h2d_done, g->stream));
  return LLMK_OK;
}

int llmk_gpt2_loss(llmk_gpt2* g, float* host_loss) {
  if (!g || !host_loss) return fail(LLMK_ERR_INVALID_ARG, "gpt2_loss");
  LLMK_CUDA(cudaMemcpyAsync(g->h_loss, g->loss, sizeof(float), cudaMemcpyDeviceToHost, g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  *host_loss = *g->h_loss;
  return LLMK_OK;
}

int llmk_gpt2_device_loss(llmk_gpt2* g, const float** d_loss) {
  if (!g || !d_loss) return fail(LLMK_ERR_INVALID_ARG, "gpt2_device_loss");
  *d_loss = g->loss;
  return LLMK_OK;
}

int llmk_gpt2_step_device(llmk_gpt2* g, const int* d_inputs, const int* d_targets, float lr, float beta1, float beta2,
                          float eps, float weight_decay, int t) {
  if (!g || !d_inputs || !d_targets || t < 1) return fail(LLMK_ERR_INVALID_ARG, "gpt2_step_device");
  if (!g->use_graph || g->timing) {
    LLMK_TRY(llmk_gpt2_forward(g, d_inputs, d_targets));
    LLMK_TRY(llmk_gpt2_backward(g));
    return llmk_gpt2_update(g, lr, beta1, beta2, eps, weight_decay, t);
  }
  // this step's AdamW values, copied from pageable memory (staged before the
  // call returns), ahead of the replay on the same stream
  float hp[8];
  llmk_adamw_hparams(hp, lr, beta1, beta2, eps, weight_decay, t, 1.0f / static_cast<float>(g->world));
  LLMK_CUDA(cudaMemcpyAsync(g->hp_dev, hp, sizeof(hp), cudaMemcpyHostToDevice, g->stream));
  if (!g->graph_exec || d_inputs != g->graph_in || d_targets != g->graph_tg) {
    if (g->graph_exec) {
      cudaGraphExecDestroy(g->graph_exec);
      g->graph_exec = nullptr;
    }
    const unsigned long long n0 = llmk_launch_count();
    LLMK_CUDA(cudaStreamBeginCapture(g->stream, cudaStreamCaptureModeThreadLocal));
    int rc = llmk_gpt2_forward(g, d_inputs, d_targets);
    if (rc == LLMK_OK) rc = llmk_gpt2_backward(g);
    if (rc == LLMK_OK) rc = update_device_hparams(g);
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(g->stream, &graph);  // always leave capture mode
    if (rc != LLMK_OK) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    LLMK_CUDA(ec);
    const cudaError_t ei = cudaGraphInstantiate(&g->graph_exec, graph, 0);
    cudaGraphDestroy(graph);
    LLMK_CUDA(ei);
    g->graph_in = d_inputs;
    g->graph_tg = d_targets;
    // the captured launches run at each replay, not at capture time
    g->graph_launches = llmk_launch_count() - n0;
    llmk::count_launch(0ull - g->graph_launches);
  }
  LLMK_CUDA(cudaGraphLaunch(g->graph_exec, g->stream));
  llmk::count_launch(g->graph_launches);
  ++g->steps;
  return LLMK_OK;
}

int llmk_gpt2_use_graph(llmk_gpt2* g, int enable) {
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_use_graph");
  g->use_graph = enable != 0;
  if (!g->use_graph && g->graph_exec) {
    LLMK_CUDA(cudaStreamSynchronize(g->stream));
    cudaGraphExecDestroy(g->graph_exec);
    g->graph_exec = nullptr;
  }
  return LLMK_OK;
}

int llmk_gpt2_train_step(llmk_gpt2* g, const int* host_inputs, const int* host_targets, float lr, float beta1,
                         float beta2, float eps, float weight_decay, int t, float* host_loss) {
  if (!g || !host_inputs || !host_targets) return fail(LLMK_ERR_INVALID_ARG, "gpt2_train_step");
  LLMK_TRY(ensure_device(g));
  LLMK_TRY(llmk_gpt2_set_train_data(g, host_inputs, host_targets));
  LLMK_TRY(llmk_gpt2_step_device(g, g->inputs, g->targets, lr, beta1, beta2, eps, weight_decay, t));
  if (host_loss) return llmk_gpt2_loss(g, host_loss);
  return LLMK_OK;
}

int llmk_gpt2_stream(llmk_gpt2* g, void** stream) {
  if (!g || !stream) return fail(LLMK_ERR_INVALID_ARG, "gpt2_stream");
  *stream = g->stream;
  return LLMK_OK;
}

int llmk_gpt2_buffers(llmk_gpt2* g, int** d_inputs, int** d_targets) {
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_buffers");
  if (d_inputs) *d_inputs = g->inputs;
  if (d_targets) *d_targets = g->targets;
  return LLMK_OK;
}

/* ----------------------------------------------------- data parallelism */
// Host-only planning helpers (no device needed): the gradient buckets in the
// order llmk_gpt2_backward all-reduces them, and the llm.c <-> layer-major
// parameter permutation.
int llmk_gpt2_dp_buckets(const llmk_gpt2_config* cfg, size_t* ranges, int max_buckets) {
  if (!cfg || cfg->num_layers < 0) return -1;
  llmk_gpt2 tmp;
  tmp.cfg = *cfg;
  layout(&tmp);
  const int L = cfg->num_layers;
  const int n = L + 2;
  if (ranges && max_buckets >= n) {
    int k = 0;
    for (int l = L - 1; l >= 0; --l, ++k) {
      ranges[2 * k] = tmp.lp[l].begin;
      ranges[2 * k + 1] = tmp.lp[l].end;
    }
    ranges[2 * k] = tmp.off_wte;
    ranges[2 * k + 1] = tmp.off_wpe + tmp.tsize[llmk::WPE];
    ++k;
    ranges[2 * k] = tmp.off_lnfw;
    ranges[2 * k + 1] = tmp.off_lnfw + 2 * static_cast<size_t>(cfg->channels);
  }
  return n;
}

int llmk_gpt2_to_layer_major(const llmk_gpt2_config* cfg, const float* src, float* dst, int reverse) {
  if (!cfg || !src || !dst) return fail(LLMK_ERR_INVALID_ARG, "gpt2_to_layer_major");
  llmk_gpt2 tmp;
  tmp.cfg = *cfg;
  layout(&tmp);
  permute_params(&tmp, src, dst, reverse ? 1 : 0);
  return LLMK_OK;
}

int llmk_nccl_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId)) return fail(LLMK_ERR_INVALID_ARG, "nccl_unique_id: need 128 bytes");
  ncclUniqueId id;
  LLMK_TRY(nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId"));
  std::memcpy(out, &id, sizeof(id));
  return LLMK_OK;
}

int llmk_gpt2_enable_dp(llmk_gpt2* g, const void* unique_id, size_t bytes, int rank, int world) {
  if (!g || !unique_id || bytes < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
    return fail(LLMK_ERR_INVALID_ARG, "gpt2_enable_dp: bad arguments");
  LLMK_TRY(ensure_device(g));
  if (world == 1) return LLMK_OK;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  LLMK_TRY(nccl_check(ncclCommInitRank(&g->comm, world, id, rank), "ncclCommInitRank"));
  g->rank = rank;
  g->world = world;
  return LLMK_OK;
}

int llmk_gpt2_broadcast_parameters(llmk_gpt2* g, int root) {
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_broadcast_parameters");
  if (g->world <= 1) return LLMK_OK;
  LLMK_TRY(nccl_check(ncclBroadcast(g->params, g->params, g->nparams, ncclFloat, root, g->comm, g->stream),
                      "ncclBroadcast"));
  if (g->params_bf16)
    LLMK_TRY(llmk_cast(g->params_bf16, LLMK_BF16, g->params, LLMK_F32, static_cast<long long>(g->nparams), g->stream));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  return LLMK_OK;
}

int llmk_gpt2_set_timing(llmk_gpt2* g, int enable) {
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_set_timing");
  g->timing = enable != 0;
  g->marks.clear();
  g->tev_used = 0;
  return LLMK_OK;
}

int llmk_gpt2_timing_report(llmk_gpt2* g, llmk_kernel_stat* out, int max, int* count) {
  if (!g || (!out && max > 0)) return fail(LLMK_ERR_INVALID_ARG, "gpt2_timing_report");
  LLMK_TRY(ensure_device(g));
  LLMK_CUDA(cudaStreamSynchronize(g->stream));
  llmk_kernel_stat acc[KC_COUNT];
  std::memset(acc, 0, sizeof(acc));
  for (int c = 0; c < KC_COUNT; ++c) {
    std::strncpy(acc[c].name, kClassName[c], sizeof(acc[c].name) - 1);
    acc[c].unit = kClassUnit[c];
  }
  for (const auto& m : g->marks) {
    if (m.e1 < 0) continue;
    float ms = 0.f;
    LLMK_CUDA(cudaEventElapsedTime(&ms, g->tev[m.e0], g->tev[m.e1]));
    llmk_kernel_stat& a = acc[m.cls];
    a.calls += 1;
    a.launches += static_cast<long long>(m.launches);
    a.ms += ms;
    a.work += m.work;
  }
  const int n = std::min<int>(max, KC_COUNT);
  for (int c = 0; c < n; ++c) out[c] = acc[c];
  if (count) *count = KC_COUNT;
  return LLMK_OK;
}

// Waits (host side, bounded) for the step's device work and checks the NCCL
// communicator for asynchronous errors; aborts the communicator on error or
// timeout so the other ranks' pending collectives fail instead of hanging.
int llmk_gpt2_synchronize(llmk_gpt2* g, int timeout_ms) {
  if (!g) return fail(LLMK_ERR_INVALID_ARG, "gpt2_synchronize");
  LLMK_TRY(ensure_device(g));
  cudaEvent_t ev;
  LLMK_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaEventRecord(ev, g->stream);
  const auto t0 = std::chrono::steady_clock::now();
  int rc = LLMK_OK;
  while (true) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      rc = llmk::cuda_check(q, "step");
      break;
    }
    if (g->comm) {
      ncclResult_t ar = ncclSuccess;
      ncclCommGetAsyncError(g->comm, &ar);
      if (ar != ncclSuccess && ar != ncclInProgress) {
        ncclCommAbort(g->comm);
        g->comm = nullptr;
        rc = fail(LLMK_ERR_NCCL, std::string("nccl async error: ") + ncclGetErrorString(ar));
        break;
      }
    }
    const auto ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms > 0 && ms > timeout_ms) {
      if (g->comm) {
        ncclCommAbort(g->comm);
        g->comm = nullptr;
      }
      rc = fail(LLMK_ERR_DEVICE_TIMEOUT, "gpt2_synchronize: step did not finish in time");
      break;
    }
  }
  cudaEventDestroy(ev);
  return rc;
}

}  // extern "C"
