// Reference-facing linear-layer entry points built on llmk_gemm, plus the
// deterministic column-sum used for the bias gradient.
//
// Reference: gpt2cuda::BatchMatmulNTForward / BatchMatmulNTBackward
// (gpt2/cuda/matmul.cu:653-669) and MatrixColSumKernel (matmul.cu:26-187).
// The reference runs the weight gradient as B batched GEMMs writing the same
// output (matmul.cu:430-435); here it is one GEMM with K = B*T.
#include <algorithm>
#include <mutex>
#include <string>

#include "ptx.cuh"
#include "runtime.h"

namespace llmk {
namespace {

constexpr int kColsPerBlock = 256;  // 32 threads x 8 columns
constexpr int kRowLanes = 8;

// Pass 1: partial[chunk][n] = sum of rows in the chunk (fp32 accumulate).
template <bool kBF16>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const void* __restrict__ x, float* __restrict__ partial,
                                                             int M, int N, int rows_per_chunk) {
  __shared__ float red[kRowLanes][kColsPerBlock + 4];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int n0 = blockIdx.x * kColsPerBlock + tx * 8;
  const int r0 = blockIdx.y * rows_per_chunk;
  const int r1 = min(M, r0 + rows_per_chunk);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  auto add_row = [&](int r) {
    if (kBF16) {
      uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + static_cast<long long>(r) * N + n0);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    } else {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + static_cast<long long>(r) * N + n0);
      float4 a = p[0], b = p[1];
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
  };
  if (n0 < N) {
    // four rows per iteration: their loads are independent and in flight together
    int r = r0 + ty;
    for (; r + 3 * kRowLanes < r1; r += 4 * kRowLanes) {
#pragma unroll
      for (int u = 0; u < 4; ++u) add_row(r + u * kRowLanes);
    }
    for (; r < r1; r += kRowLanes) add_row(r);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[ty][tx * 8 + j] = acc[j];
  __syncthreads();
  // 256 threads reduce 256 columns over the 8 row lanes in a fixed order.
  const int t = ty * 32 + tx;
  const int n = blockIdx.x * kColsPerBlock + t;
  float s = 0.f;
#pragma unroll
  for (int y = 0; y < kRowLanes; ++y) s += red[y][t];
  if (n < N) partial[static_cast<long long>(blockIdx.y) * N + n] = s;
}

// Pass 2: out[n] (+)= sum over chunks in a fixed order: block (32 columns x
// 8 chunk lanes), lane y sums chunks y, y+8, ..., then the 8 lane sums are
// added in order.
__global__ void colsum_final_kernel(const float* __restrict__ partial, float* __restrict__ out, int N, int chunks,
                                    int accumulate) {
  __shared__ float red[8][33];
  const int n = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (n < N)
    for (int c = threadIdx.y; c < chunks; c += 8) s += partial[static_cast<long long>(c) * N + n];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || n >= N) return;
  float t = 0.f;
#pragma unroll
  for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
  out[n] = accumulate ? out[n] + t : t;
}

int colsum_chunks(int M, int N) {
  const int col_blocks = (N + kColsPerBlock - 1) / kColsPerBlock;
  // about 8 blocks (64 warps) per SM: enough loads in flight to stream HBM
  int chunks = (8 * num_sms() + col_blocks - 1) / col_blocks;
  chunks = std::max(1, std::min(chunks, (M + 63) / 64));
  return chunks;
}

}  // namespace

// max_chunks > 0 caps the row chunks (and so the partial buffer) below the
// bandwidth-optimal count.
int colsum_launch(float* out, const void* x, bool bf16, int M, int N, int accumulate, float* partial,
                  cudaStream_t s, int max_chunks = 0) {
  const int chunks = max_chunks > 0 ? std::min(colsum_chunks(M, N), max_chunks) : colsum_chunks(M, N);
  const int rows_per_chunk = (M + chunks - 1) / chunks;
  dim3 grid((N + kColsPerBlock - 1) / kColsPerBlock, chunks);
  dim3 block(32, kRowLanes);
  if (bf16) colsum_partial_kernel<true><<<grid, block, 0, s>>>(x, partial, M, N, rows_per_chunk);
  else colsum_partial_kernel<false><<<grid, block, 0, s>>>(x, partial, M, N, rows_per_chunk);
  colsum_final_kernel<<<(N + 31) / 32, dim3(32, 8), 0, s>>>(partial, out, N, chunks, accumulate);
  count_launch(2);
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

size_t colsum_workspace(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return static_cast<size_t>(colsum_chunks(M, N)) * N * sizeof(float);
}

// Scratch of llmk_colsum_noalloc: a fixed device array that every GPU loading
// this library holds until the process exits (1 MiB). Host code must not pass
// `g_colsum_noalloc_scratch` itself to a kernel (on the host it names a
// host-side stand-in); it passes the device address that SymbolCache looks
// up with cudaGetSymbolAddress once per device (and again after a device
// reset gave the device a new context).
constexpr int kColsumNoAllocFloats = 1 << 18;
static __device__ __align__(256) float g_colsum_noalloc_scratch[kColsumNoAllocFloats];
static cudaError_t lookup_colsum_noalloc(void** p) { return cudaGetSymbolAddress(p, g_colsum_noalloc_scratch); }
static SymbolCache g_colsum_noalloc_addr(lookup_colsum_noalloc);

// The column sums read fp32 or bf16; anything else is refused rather than
// reinterpreted.
static int colsum_dtype_ok(llmk_dtype t, const char* what) {
  if (t == LLMK_F32 || t == LLMK_BF16) return LLMK_OK;
  return fail(LLMK_ERR_UNSUPPORTED, std::string(what) + ": x must be fp32 or bf16");
}

}  // namespace llmk

using namespace llmk;

extern "C" {

size_t llmk_colsum_workspace(int M, int N) { return colsum_workspace(M, N); }

int llmk_colsum(float* dbias, const void* x, llmk_dtype x_dtype, int M, int N, int accumulate, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (!dbias || !x || M <= 0 || N <= 0) return fail(LLMK_ERR_INVALID_ARG, "colsum: bad arguments");
  LLMK_TRY(colsum_dtype_ok(x_dtype, "colsum"));
  if (N % 8 || !aligned16(x)) return fail(LLMK_ERR_UNSUPPORTED, "colsum: N % 8 == 0 and 16-byte alignment required");
  if (!workspace || workspace_bytes < colsum_workspace(M, N))
    return fail(LLMK_ERR_WORKSPACE, "colsum: workspace too small");
  return colsum_launch(dbias, x, x_dtype == LLMK_BF16, M, N, accumulate, static_cast<float*>(workspace),
                       static_cast<cudaStream_t>(stream));
}

// Column sum for callers that may not allocate device memory (see llmk.h).
// The first call on a device resolves the device address of the file-scope
// scratch array with that device current; later calls reuse it.
int llmk_colsum_noalloc(float* dbias, const void* x, llmk_dtype x_dtype, int M, int N, int accumulate, void* stream) {
  if (!dbias || !x || M <= 0 || N <= 0) return fail(LLMK_ERR_INVALID_ARG, "colsum_noalloc: bad arguments");
  LLMK_TRY(colsum_dtype_ok(x_dtype, "colsum_noalloc"));
  if (N % 8 || !aligned16(x))
    return fail(LLMK_ERR_UNSUPPORTED, "colsum_noalloc: N % 8 == 0 and 16-byte alignment required");
  // One row chunk needs N partial sums: N up to the array's size is
  // accepted, with as many row chunks (any M) as the array holds.
  if (N > kColsumNoAllocFloats)
    return fail(LLMK_ERR_UNSUPPORTED, "colsum_noalloc: N = " + std::to_string(N) + " exceeds the fixed scratch of " +
                                          std::to_string(kColsumNoAllocFloats) +
                                          " floats (use llmk_colsum with a caller workspace)");
  const int max_chunks = static_cast<int>(std::min<size_t>(colsum_chunks(M, N), kColsumNoAllocFloats / N));
  void* scratch = nullptr;
  LLMK_TRY(g_colsum_noalloc_addr.get(&scratch));
  // Pass 1 overwrites every partial that pass 2 reads, so nothing in the
  // shared scratch has to start at zero.
  return colsum_launch(dbias, x, x_dtype == LLMK_BF16, M, N, accumulate, static_cast<float*>(scratch),
                       static_cast<cudaStream_t>(stream), max_chunks);
}

int llmk_matmul_forward(void* out, llmk_dtype out_dtype, const void* inp, const void* weight, const float* bias,
                        int BT, int C, int OC, llmk_math math, void* stream) {
  llmk_epilogue ep{};
  ep.bias = bias;
  // out[BT,OC] = inp[BT,C] * weight[OC,C]^T: both operands K-major.
  return llmk_gemm(out, out_dtype, OC, inp, 0, C, weight, 0, C, math, BT, OC, C, &ep, nullptr, 0, stream);
}

size_t llmk_matmul_backward_workspace(int BT, int C, int OC, llmk_math math) {
  size_t a = llmk_gemm_workspace(OC, C, BT, math);
  size_t b = colsum_workspace(BT, OC);
  return std::max(a, b);
}

int llmk_matmul_backward(void* dinp, llmk_dtype dinp_dtype, float* dweight, float* dbias, const void* dout,
                         const void* inp, const void* weight, int BT, int C, int OC, llmk_math math, int flags,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!dout || !inp || !weight || !dweight) return fail(LLMK_ERR_INVALID_ARG, "matmul_backward: null operand");
  if (dbias && (!workspace || workspace_bytes < colsum_workspace(BT, OC)))
    return fail(LLMK_ERR_WORKSPACE, "matmul_backward: workspace too small for dbias");
  // dinp[BT,C] = dout[BT,OC] * weight[OC,C]: A K-major, B stored [K=OC][N=C] (N-major).
  if (dinp) {
    llmk_epilogue ep{};
    ep.flags = (flags & LLMK_ACCUM_DINP) ? LLMK_EPI_ACCUMULATE : 0;
    LLMK_TRY(llmk_gemm(dinp, dinp_dtype, C, dout, 0, OC, weight, 1, C, math, BT, C, OC, &ep, nullptr, 0, stream));
  }
  // dweight[OC,C] = dout^T * inp: A stored [K=BT][M=OC], B stored [K=BT][N=C].
  {
    llmk_epilogue ep{};
    ep.flags = (flags & LLMK_ACCUM_DWEIGHT) ? LLMK_EPI_ACCUMULATE : 0;
    LLMK_TRY(llmk_gemm(dweight, LLMK_F32, C, dout, 1, OC, inp, 1, C, math, OC, C, BT, &ep, workspace,
                       workspace_bytes, stream));
  }
  if (dbias) {
    LLMK_TRY(colsum_launch(dbias, dout, math == LLMK_MATH_BF16, BT, OC, (flags & LLMK_ACCUM_DBIAS) ? 1 : 0,
                           static_cast<float*>(workspace), static_cast<cudaStream_t>(stream)));
  }
  return LLMK_OK;
}

}  // extern "C"
