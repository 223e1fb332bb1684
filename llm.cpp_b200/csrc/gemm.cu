// tcgen05 GEMM host side: the planner (kernel kind, split-K), the split-K
// reduction and the C entry points (reference gpt2/cuda/matmul.cu:223-449).
// The kernels live in gemm_kernel.cuh, instantiated by gemm_{bf16,tf32}_*.cu.
#include "gemm_kernel.cuh"

namespace llmk {
namespace {

// Applies the epilogue to 8 consecutive columns [gn, gn+8) of row gm, all in
// bounds, and stores them (split-K reduction path).
__device__ __forceinline__ void epi_apply8(const EpiParams& ep, long long gm, int gn, float* v) {
  float t[8];
  if (ep.bias) {
    load8(ep.bias + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += t[j];
  }
  if (ep.residual) {
    load8(ep.residual + gm * ep.ldr + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += t[j];
  }
  if (ep.flags & LLMK_EPI_GELU) {
    if (ep.aux) {
      if (ep.flags & LLMK_EPI_AUX_F32) store8(reinterpret_cast<float*>(ep.aux) + gm * ep.ldaux + gn, v);
      else store8_bf16(ep.aux + gm * ep.ldaux + gn, v);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = gelu_tanh(v[j]);
  } else if (ep.flags & LLMK_EPI_GELU_BWD) {
    if (ep.flags & LLMK_EPI_AUX_F32) load8(reinterpret_cast<const float*>(ep.aux) + gm * ep.ldaux + gn, t);
    else load8_bf16(ep.aux + gm * ep.ldaux + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= gelu_tanh_grad(t[j]);
  }
  if (ep.d_bf16) {
    __nv_bfloat16* dp = static_cast<__nv_bfloat16*>(ep.D) + gm * ep.ldd + gn;
    if (ep.flags & LLMK_EPI_ACCUMULATE) {
      load8_bf16(dp, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += t[j];
    }
    store8_bf16(dp, v);
  } else {
    float* dp = static_cast<float*>(ep.D) + gm * ep.ldd + gn;
    if (ep.flags & LLMK_EPI_ACCUMULATE) {
      load8(dp, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += t[j];
    }
    store8(dp, v);
  }
}

// out = epilogue(sum_s partial[s]) over 8-column groups; grid-stride.
__global__ void gemm_splitk_reduce(EpiParams ep, int M, int N, int splits) {
  const long long groups = static_cast<long long>(M) * (N / 8);
  const long long plane = static_cast<long long>(M) * N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long gm = i / (N / 8);
    const int gn = static_cast<int>(i - gm * (N / 8)) * 8;
    float v[8], t[8];
    load8(ep.partial + gm * N + gn, v);
    for (int s = 1; s < splits; ++s) {
      load8(ep.partial + s * plane + gm * N + gn, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += t[j];
    }
    epi_apply8(ep, gm, gn, v);
  }
}

int dispatch_kind(bool tf32, int kind, int a_trans, int b_trans, const void* A, long long lda, const void* B,
                  long long ldb, int M, int N, int K, const EpiParams& ep, int splits, cudaStream_t s) {
  if (tf32) {
    if (kind == 2) return gemm_dispatch_tf32_pair256(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
    if (kind == 1) return gemm_dispatch_tf32_pair128(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
    return gemm_dispatch_tf32_cta(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
  }
  if (kind == 2) return gemm_dispatch_bf16_pair256(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
  if (kind == 1) return gemm_dispatch_bf16_pair128(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
  return gemm_dispatch_bf16_cta(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
}

}  // namespace

// Chooses the kernel kind (CTA pair with BN 256 or 128 for M >= 256, else a
// single CTA with BN 128) and the split-K factor.
//  - K long (>= 64 K blocks: the weight gradients, M, N = layer widths,
//    K = B*T tokens): 256-wide pair tiles, and split-K by the largest power
//    of two that keeps the work units within one wave of CTA pairs. Measured
//    on B200 for the GPT-2 124M weight gradients this beats 128-wide tiles
//    and deeper splits by 1.5-1.9x.
//  - otherwise the tile width with the fewer waves (128-wide tiles cost about
//    half a 256-wide one plus a fixed overhead), split only when a short tile
//    grid leaves most SMs idle.
static void plan_gemm(int M, int N, int K, int elem, int* kind, int* splits) {
  const int sms = num_sms();
  const int bk = 128 / elem;
  const int num_kb = (K + bk - 1) / bk;
  int tiles, units;
  if (M >= 256) {
    units = sms / 2;
    const int num_m = (M + 255) / 256;
    const int t256 = num_m * ((N + 255) / 256), t128 = num_m * ((N + 127) / 128);
    const long long w256 = (t256 + units - 1) / units, w128 = (t128 + units - 1) / units;
    if (num_kb >= 64) *kind = 2;
    else *kind = (w256 * 256 * 10 <= w128 * 128 * 11) ? 2 : 1;
    tiles = (*kind == 2) ? t256 : t128;
  } else {
    units = sms;
    *kind = 0;
    tiles = ((M + 127) / 128) * ((N + 127) / 128);
  }
  int s = 1;
  while (tiles * s * 2 <= units && num_kb / (s * 2) >= 8) s *= 2;
  // Every split must own at least one K block (an empty split would publish
  // a stale accumulator).
  while (s > 1 && ((num_kb + s - 1) / s) * (s - 1) >= num_kb) s /= 2;
  *splits = s;
}

}  // namespace llmk

using namespace llmk;

static int gemm_impl(void* D, llmk_dtype d_dtype, long long ldd, const void* A, int a_trans, long long lda,
                     const void* B, int b_trans, long long ldb, llmk_math math, int M, int N, int K,
                     const llmk_epilogue* epi, void* workspace, size_t workspace_bytes, void* stream,
                     float2* stats = nullptr, int stats_cols = 0) {
  if (!D || !A || !B) return fail(LLMK_ERR_INVALID_ARG, "gemm: null operand");
  if (M <= 0 || N <= 0 || K <= 0) return fail(LLMK_ERR_INVALID_ARG, "gemm: non-positive size");
  if (math != LLMK_MATH_BF16 && math != LLMK_MATH_TF32) return fail(LLMK_ERR_INVALID_ARG, "gemm: bad math mode");
  const int elem = (math == LLMK_MATH_TF32) ? 4 : 2;
  const int d_elem = (d_dtype == LLMK_BF16) ? 2 : 4;
  if (!aligned16(A) || !aligned16(B) || !aligned16(D) || (lda * elem) % 16 || (ldb * elem) % 16 ||
      (ldd * d_elem) % 16 || N % 8)
    return fail(LLMK_ERR_UNSUPPORTED, "gemm: operands need 16-byte aligned bases/row strides and N % 8 == 0");
  EpiParams ep{};
  ep.D = D;
  ep.ldd = ldd;
  ep.d_bf16 = d_dtype == LLMK_BF16;
  if (epi) {
    ep.bias = epi->bias;
    ep.residual = epi->residual;
    ep.ldr = epi->ldr;
    ep.aux = static_cast<__nv_bfloat16*>(epi->aux);
    ep.ldaux = epi->ldaux;
    ep.flags = epi->flags;
    if ((ep.bias && !aligned16(ep.bias)) || (ep.residual && (!aligned16(ep.residual) || ep.ldr % 4)) ||
        (ep.aux && (!aligned16(ep.aux) || ep.ldaux % ((ep.flags & LLMK_EPI_AUX_F32) ? 4 : 8))))
      return fail(LLMK_ERR_UNSUPPORTED, "gemm: epilogue operands need 16-byte alignment");
    if ((ep.flags & LLMK_EPI_GELU_BWD) && !ep.aux) return fail(LLMK_ERR_INVALID_ARG, "gemm: GELU_BWD needs aux");
  }
  int kind, splits;
  plan_gemm(M, N, K, elem, &kind, &splits);
  const size_t need = static_cast<size_t>(splits) * M * N * sizeof(float);
  if (splits > 1 && (!workspace || workspace_bytes < need || !aligned16(workspace))) splits = 1;
  if (stats) {
    // statistics are taken from whole accumulators: no split-K, and only a
    // bias may come before them
    if (epi && (epi->residual || epi->aux || epi->flags))
      return fail(LLMK_ERR_INVALID_ARG, "gemm: row statistics take a bias-only epilogue");
    splits = 1;
    ep.stats = stats;
    ep.stats_cols = stats_cols;
  }
  if (splits > 1) ep.partial = static_cast<float*>(workspace);
  // the pre-activation store rides the TMA path when it has D's element type
  ep.aux_tma = (ep.flags & LLMK_EPI_GELU) && ep.aux && !ep.partial &&
               ((ep.flags & LLMK_EPI_AUX_F32) != 0) == (ep.d_bf16 == 0) &&
               (ep.ldaux * (ep.d_bf16 ? 2 : 4)) % 16 == 0;
  {
    // the epilogue program (kOp*): specialised drains for the common
    // combinations, the flag-driven one for the rest
    const int f = ep.flags & ~LLMK_EPI_AUX_F32;
    const bool aux_is_d = ((ep.flags & LLMK_EPI_AUX_F32) != 0) == (ep.d_bf16 == 0);
    if (ep.partial || (!ep.bias && !ep.residual && f == 0)) ep.op = kOpNone;
    else if (ep.bias && !ep.residual && f == 0) ep.op = kOpBias;
    else if (ep.bias && ep.residual && f == 0 && !ep.d_bf16) ep.op = kOpBiasRes;
    else if (ep.bias && !ep.residual && f == LLMK_EPI_GELU && ep.aux_tma) ep.op = kOpBiasGelu;
    else if (!ep.bias && !ep.residual && f == LLMK_EPI_GELU_BWD && aux_is_d) ep.op = kOpGeluBwd;
    else ep.op = kOpGeneric;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = dispatch_kind(elem == 4, kind, a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
  if (rc != LLMK_OK || splits == 1) return rc;
  const long long groups = static_cast<long long>(M) * (N / 8);
  const int grid = static_cast<int>(std::min<long long>((groups + 255) / 256, num_sms() * 8LL));
  gemm_splitk_reduce<<<grid, 256, 0, s>>>(ep, M, N, splits);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

namespace llmk {

int gemm_rowstats(void* D, llmk_dtype d_dtype, long long ldd, const void* A, long long lda, const void* B,
                  long long ldb, llmk_math math, int M, int N, int K, const float* bias, float2* stats,
                  int stats_cols, cudaStream_t stream) {
  if (!stats || !aligned16(stats) || stats_cols <= 0 || stats_cols > N)
    return fail(LLMK_ERR_INVALID_ARG, "gemm_rowstats: statistics buffer / column count");
  llmk_epilogue e{};
  e.bias = bias;
  return gemm_impl(D, d_dtype, ldd, A, 0, lda, B, 0, ldb, math, M, N, K, &e, nullptr, 0, stream, stats, stats_cols);
}

}  // namespace llmk

extern "C" {

size_t llmk_gemm_workspace(int M, int N, int K, llmk_math math) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int kind, splits;
  plan_gemm(M, N, K, math == LLMK_MATH_TF32 ? 4 : 2, &kind, &splits);
  return splits > 1 ? static_cast<size_t>(splits) * M * N * sizeof(float) : 0;
}

int llmk_gemm(void* D, llmk_dtype d_dtype, long long ldd, const void* A, int a_trans, long long lda, const void* B,
              int b_trans, long long ldb, llmk_math math, int M, int N, int K, const llmk_epilogue* epi,
              void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_impl(D, d_dtype, ldd, A, a_trans, lda, B, b_trans, ldb, math, M, N, K, epi, workspace,
                   workspace_bytes, stream);
}

}  // extern "C"
