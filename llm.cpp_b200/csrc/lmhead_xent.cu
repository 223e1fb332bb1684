// Fused lm_head + softmax (+ cross-entropy) for sm_100a.
//
// The reference computes the lm_head logits with one GEMM, then softmax and
// cross-entropy in separate passes over the BT x Vp logits
// (gpt2/cuda/gpt2cuda.cu:323-325,398; softmax.cu:13-91, cross_entropy.cu:7-32),
// and has a CUTLASS GEMM+softmax (gpt2/cuda/matmul_softmax.cu:9-98) whose
// epilogue emits per-tile partial row maxima and sums that a second kernel
// finishes. Here the tcgen05 GEMM's epilogue (gemm.cu) folds every row's
// values into (max, sum exp(x - max)) per 64-column slot while the tile is in
// registers, so the logits are never read back to find the normaliser: one
// pass per row (this file) combines the slot statistics into
// lse = max + log(sum) and streams the row once, writing either the softmax
// probabilities or the cross-entropy gradient (softmax - onehot) * dscale in
// place, with loss = lse - logit[target]. Against the unfused path this drops
// one full read of the logits and half the exponentials.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "ptx.cuh"
#include "runtime.h"

namespace llmk {
namespace {

constexpr int kRowsPerBlock = 8;  // one warp per row in the streaming pass
constexpr int kGroups = 32;       // slot groups per row in the combine

__device__ __forceinline__ void lse_fold(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else {
    s += s2 * __expf(m2 - m);
  }
}

__device__ __forceinline__ void load8v(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8v(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8v(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8v(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  u.x = *reinterpret_cast<uint32_t*>(&h[0]);
  u.y = *reinterpret_cast<uint32_t*>(&h[1]);
  u.z = *reinterpret_cast<uint32_t*>(&h[2]);
  u.w = *reinterpret_cast<uint32_t*>(&h[3]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Combine: block = 8 rows, 256 threads; thread (row r = t & 7, group
// g = t >> 3) folds slots g, g + 32, ... of its row (8 consecutive rows = 64
// contiguous bytes of a slot plane per load), then the 32 group results of
// each row are folded in group order (deterministic). Writes lse[row] and, in
// cross-entropy mode, losses[row] = lse - x[target] (NaN for a target outside
// [0, V)) before the streaming pass may overwrite the logits.
template <typename T, int kMode>
__global__ void __launch_bounds__(256) rowstats_lse_kernel(float* __restrict__ lse_out, float* __restrict__ losses,
                                                           const T* __restrict__ logits,
                                                           const float2* __restrict__ stats,
                                                           const int* __restrict__ targets, int rows, int V, int ld,
                                                           int nslots) {
  __shared__ float2 part[kGroups][kRowsPerBlock];
  const int t = threadIdx.x;
  const long long row0 = static_cast<long long>(blockIdx.x) * kRowsPerBlock;
  const int nrows = static_cast<int>(rows - row0 < kRowsPerBlock ? rows - row0 : kRowsPerBlock);
  {
    const int r = t & (kRowsPerBlock - 1), g = t >> 3;
    float m = -INFINITY, s = 0.f;
    if (r < nrows) {
      const float2* p = stats + row0 + r;
      int k = g;
      for (; k + 3 * kGroups < nslots; k += 4 * kGroups) {
        const float2 a = p[static_cast<long long>(k) * rows], b = p[static_cast<long long>(k + kGroups) * rows];
        const float2 c = p[static_cast<long long>(k + 2 * kGroups) * rows];
        const float2 d = p[static_cast<long long>(k + 3 * kGroups) * rows];
        lse_fold(m, s, a.x, a.y);
        lse_fold(m, s, b.x, b.y);
        lse_fold(m, s, c.x, c.y);
        lse_fold(m, s, d.x, d.y);
      }
      for (; k < nslots; k += kGroups) {
        const float2 a = p[static_cast<long long>(k) * rows];
        lse_fold(m, s, a.x, a.y);
      }
    }
    part[g][r] = make_float2(m, s);
  }
  __syncthreads();
  if (t < nrows) {
    float m = -INFINITY, s = 0.f;
    for (int g = 0; g < kGroups; ++g) lse_fold(m, s, part[g][t].x, part[g][t].y);
    const float lse = m + logf(s);
    const long long row = row0 + t;
    lse_out[row] = lse;
    if constexpr (kMode == 0) {
      const int tgt = targets[row];
      losses[row] = (tgt >= 0 && tgt < V) ? lse - static_cast<float>(logits[row * ld + tgt]) : NAN;
    }
  }
}

// Stream: a persistent pass over the logits in units of 16 KB row segments
// (unit u = row u / units_per_row, segment u % units_per_row). Warp 0 lane 0
// streams this CTA's units into a ring of shared-memory stages with bulk
// copies (two CTAs per SM, up to 2 * kStages * 16 KB in flight per SM: enough
// to cover HBM latency); the consumer warps turn each stage into output values
// and store them with 16-byte stores. kMode 0: out (which may be the logits
// buffer) = (softmax - onehot) * dscale, 0 on [V, ld); kMode 1: out =
// softmax, 0 on [V, ld). Every wait is bounded (device status on timeout).
constexpr int kStageBytes = 16384;
constexpr int kStages = 6;
constexpr int kStreamCtasPerSm = 2;
constexpr int kConsumerWarps = 16;
constexpr int kStreamThreads = 32 * (kConsumerWarps + 1);
constexpr size_t kStreamSmem = size_t(kStages) * kStageBytes + 2 * kStages * 8 + 16;

template <typename T, int kMode>
__global__ void __launch_bounds__(kStreamThreads, kStreamCtasPerSm)
    rowstats_stream_kernel(T* out, const T* logits, const float* __restrict__ lse, const int* __restrict__ targets,
                           int rows, int V, int ld, float dscale, unsigned int* status) {
  constexpr int CH = kStageBytes / static_cast<int>(sizeof(T));  // elements per unit
  extern __shared__ __align__(128) uint8_t smem_stream[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_stream + size_t(kStages) * kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int upr = (ld + CH - 1) / CH;
  const long long total = static_cast<long long>(rows) * upr;
  if (warp == 0) {
    if (lane == 0) {
      int k = 0;
      for (long long u = blockIdx.x; u < total; u += gridDim.x, ++k) {
        const int st = k % kStages;
        const uint32_t ph = static_cast<uint32_t>(k / kStages) & 1u;
        if (!mbar_wait(empty + st, ph ^ 1u, status, abort_flag, 20)) break;
        const long long row = u / upr;
        const int c0 = static_cast<int>(u - row * upr) * CH;
        const int n = min(CH, ld - c0);
        mbar_arrive_expect_tx(full + st, static_cast<uint32_t>(n * sizeof(T)));
        bulk_load_1d(smem_stream + size_t(st) * kStageBytes, logits + row * ld + c0, static_cast<uint32_t>(n * sizeof(T)),
                     full + st);
      }
      // the CTA exits only after every copy it issued has landed
      for (int j = max(0, k - kStages); j < k; ++j)
        mbar_wait(full + j % kStages, static_cast<uint32_t>(j / kStages) & 1u, status, nullptr, 21);
    }
    return;
  }
  const int ct = threadIdx.x - 32;
  int k = 0;
  for (long long u = blockIdx.x; u < total; u += gridDim.x, ++k) {
    const int st = k % kStages;
    const uint32_t ph = static_cast<uint32_t>(k / kStages) & 1u;
    const bool ok = mbar_wait(full + st, ph, status, abort_flag, 22);
    if (!__all_sync(0xffffffffu, ok)) break;
    const long long row = u / upr;
    const int c0 = static_cast<int>(u - row * upr) * CH;
    const int n = min(CH, ld - c0);
    // p * scale = 2^(x log2e - (lse log2e - log2 scale)): one FMA and one SFU op
    // per element; the one-hot term and the [V, ld) mask only where they fall
    const float scale = kMode == 0 ? dscale : 1.f;
    const float l2 = lse[row] * kLog2e - log2f(scale);
    const int tgt = kMode == 0 ? targets[row] : -1;
    const T* src = reinterpret_cast<const T*>(smem_stream + size_t(st) * kStageBytes);
    T* dst = out + row * ld + c0;
    for (int e = ct * 8; e < n; e += 32 * kConsumerWarps * 8) {
      float v[8];
      load8v(src + e, v);
      const int c = c0 + e;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = ex2_approx(fmaf(v[j], kLog2e, -l2));
      if (c + 8 > V) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c + j >= V) v[j] = 0.f;
      }
      if (kMode == 0 && static_cast<unsigned>(tgt - c) < 8u) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c + j == tgt) v[j] -= scale;
      }
      store8v(dst + e, v);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + st);
  }
}

template <typename T, int kMode>
int rowstats_finish_t(float* losses, void* out, const void* logits, const float2* stats, float* lse,
                      const int* targets, int rows, int V, int ld, float dscale, int backward, cudaStream_t s) {
  const int nslots = (ld + 63) / 64;
  const T* x = static_cast<const T*>(logits);
  rowstats_lse_kernel<T, kMode><<<(rows + kRowsPerBlock - 1) / kRowsPerBlock, 256, 0, s>>>(
      lse, losses, x, stats, targets, rows, V, ld, nslots);
  count_launch();
  if (kMode == 0 && !backward) return LLMK_OK;
  auto kern = rowstats_stream_kernel<T, kMode>;
  static bool attr_done[64] = {};
  int dev = 0;
  LLMK_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !attr_done[dev]) {
    LLMK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kStreamSmem)));
    attr_done[dev] = true;
  }
  const long long units = static_cast<long long>(rows) * ((ld + kStageBytes / static_cast<int>(sizeof(T)) - 1) /
                                                          (kStageBytes / static_cast<int>(sizeof(T))));
  const int grid = static_cast<int>(std::min<long long>(units, kStreamCtasPerSm * num_sms()));
  kern<<<grid, kStreamThreads, kStreamSmem, s>>>(static_cast<T*>(out), x, lse, targets, rows, V, ld, dscale,
                                                 device_status_ptr());
  count_launch();
  return LLMK_OK;
}

}  // namespace

int rowstats_finish(int mode, float* losses, void* out, const void* logits, llmk_dtype dtype, const float2* stats,
                    const int* targets, int rows, int V, int ld, float dscale, int backward, cudaStream_t s) {
  // lse per row sits after the slot planes (rowstats_bytes counts both)
  float* lse = reinterpret_cast<float*>(const_cast<float2*>(stats) + static_cast<size_t>((ld + 63) / 64) * rows);
  if (dtype == LLMK_BF16) {
    if (mode == 0)
      LLMK_TRY((rowstats_finish_t<__nv_bfloat16, 0>(losses, out, logits, stats, lse, targets, rows, V, ld, dscale,
                                                    backward, s)));
    else
      LLMK_TRY((rowstats_finish_t<__nv_bfloat16, 1>(losses, out, logits, stats, lse, targets, rows, V, ld, dscale, 1,
                                                    s)));
  } else {
    if (mode == 0)
      LLMK_TRY((rowstats_finish_t<float, 0>(losses, out, logits, stats, lse, targets, rows, V, ld, dscale, backward, s)));
    else
      LLMK_TRY((rowstats_finish_t<float, 1>(losses, out, logits, stats, lse, targets, rows, V, ld, dscale, 1, s)));
  }
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

}  // namespace llmk

using namespace llmk;

namespace {

int check_lmhead(const void* logits, llmk_dtype dtype, const void* inp, const void* W, int BT, int C, int Vp, int V,
                 llmk_math math, void* workspace, size_t workspace_bytes, const char* what) {
  if (!logits || !inp || !W || BT <= 0 || C <= 0 || V <= 0 || Vp < V)
    return fail(LLMK_ERR_INVALID_ARG, std::string(what) + ": null operand or bad size");
  if (dtype != LLMK_BF16 && dtype != LLMK_F32) return fail(LLMK_ERR_INVALID_ARG, std::string(what) + ": dtype");
  if (math != LLMK_MATH_BF16 && math != LLMK_MATH_TF32) return fail(LLMK_ERR_INVALID_ARG, std::string(what) + ": math");
  if (Vp % 8) return fail(LLMK_ERR_UNSUPPORTED, std::string(what) + ": Vp % 8");
  if (!workspace || !aligned16(workspace) || workspace_bytes < rowstats_bytes(BT, Vp))
    return fail(LLMK_ERR_WORKSPACE, std::string(what) + ": workspace missing or too small");
  return LLMK_OK;
}

}  // namespace

extern "C" {

size_t llmk_matmul_softmax_workspace(int BT, int Vp) {
  if (BT <= 0 || Vp <= 0) return 0;
  return rowstats_bytes(BT, Vp);
}

int llmk_matmul_softmax_forward(void* probs, void* logits, llmk_dtype dtype, const void* inp, const void* W,
                                const float* bias, int BT, int C, int Vp, int V, llmk_math math, void* workspace,
                                size_t workspace_bytes, void* stream) {
  LLMK_TRY(check_lmhead(logits, dtype, inp, W, BT, C, Vp, V, math, workspace, workspace_bytes, "matmul_softmax"));
  if (!probs) return fail(LLMK_ERR_INVALID_ARG, "matmul_softmax: null probs");
  if (!aligned16(probs)) return fail(LLMK_ERR_UNSUPPORTED, "matmul_softmax: probs need 16-byte alignment");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* stats = static_cast<float2*>(workspace);
  LLMK_TRY(gemm_rowstats(logits, dtype, Vp, inp, C, W, C, math, BT, Vp, C, bias, stats, V, s));
  return rowstats_finish(1, nullptr, probs, logits, dtype, stats, nullptr, BT, V, Vp, 1.f, 1, s);
}

int llmk_matmul_crossentropy_forward(float* losses, void* logits, llmk_dtype dtype, const void* inp, const void* W,
                                     const float* bias, const int* targets, int BT, int C, int Vp, int V,
                                     float dscale, int backward, llmk_math math, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  LLMK_TRY(check_lmhead(logits, dtype, inp, W, BT, C, Vp, V, math, workspace, workspace_bytes, "matmul_crossentropy"));
  if (!losses || !targets) return fail(LLMK_ERR_INVALID_ARG, "matmul_crossentropy: null losses / targets");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* stats = static_cast<float2*>(workspace);
  LLMK_TRY(gemm_rowstats(logits, dtype, Vp, inp, C, W, C, math, BT, Vp, C, bias, stats, V, s));
  return rowstats_finish(0, losses, logits, logits, dtype, stats, targets, BT, V, Vp, dscale, backward, s);
}

}  // extern "C"
