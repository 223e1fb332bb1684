// Host-side runtime shared by every translation unit of libllmk: error
// reporting, the per-device status word, the launch counter and TMA
// tensor-map construction.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "llmk.h"

namespace llmk {

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const std::string& msg);
// Converts a CUDA error into LLMK_ERR_CUDA with context; LLMK_OK on success.
int cuda_check(cudaError_t e, const char* what);

// Device address of the status word of the current device (kernels atomicOr
// LLMK_DEV_TIMEOUT into it). Never null after a successful call.
unsigned int* device_status_ptr();

// Device address of a file-scope __device__ array, looked up with
// cudaGetSymbolAddress once per device and context and cached. A module's
// symbols get new addresses when the device's primary context is destroyed
// (cudaDeviceReset) and created again, so the cache is keyed on the current
// context as well as the device and is refreshed when that context changes.
// `lookup` calls cudaGetSymbolAddress on the symbol in its own translation
// unit (host code only ever sees a host-side stand-in of the array).
class SymbolCache {
 public:
  using Lookup = cudaError_t (*)(void**);
  explicit SymbolCache(Lookup lookup) : lookup_(lookup) {}
  // Device address for the current device; LLMK_OK or LLMK_ERR_*.
  int get(void** out);

 private:
  static constexpr int kDevices = 64;
  Lookup lookup_;
  void* ptr_[kDevices] = {};
  void* ctx_[kDevices] = {};
};

// Number of SMs of the current device (cached per device).
int num_sms();

void count_launch(unsigned long long n = 1);

// 2D/3D tensor maps with 128-byte swizzle. dims/strides are in elements /
// bytes, innermost first. Returns LLMK_OK or LLMK_ERR_*.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                 uint32_t box2, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Row softmax statistics of a logits GEMM (gemm.cu): D[M, N] = A[M, K] *
// B[N, K]^T (+ bias), both operands K-major, and for every row and 64-column
// slot (max, sum exp(x - max)) over the slot's columns below stats_cols,
// written to stats[slot * M + row] (ceil(N / 64) * M float2 values).
int gemm_rowstats(void* D, llmk_dtype d_dtype, long long ldd, const void* A, long long lda, const void* B,
                  long long ldb, llmk_math math, int M, int N, int K, const float* bias, float2* stats,
                  int stats_cols, cudaStream_t stream);
// One pass over logits[rows, ld] given their slot statistics (lmhead_xent.cu):
// mode 0 = cross-entropy (losses; dlogits in place when `backward`), mode 1 =
// softmax probabilities into `out`.
int rowstats_finish(int mode, float* losses, void* out, const void* logits, llmk_dtype dtype, const float2* stats,
                    const int* targets, int rows, int V, int ld, float dscale, int backward, cudaStream_t stream);
// Workspace of the two: the slot planes, then one fp32 logsumexp per row.
inline size_t rowstats_bytes(int rows, int ld) {
  return static_cast<size_t>((ld + 63) / 64) * rows * 8 + (static_cast<size_t>(rows) * 4 + 15) / 16 * 16;
}

}  // namespace llmk

#define LLMK_TRY(expr)            \
  do {                            \
    int _llmk_rc = (expr);        \
    if (_llmk_rc != LLMK_OK) return _llmk_rc; \
  } while (0)

#define LLMK_CUDA(expr) LLMK_TRY(::llmk::cuda_check((expr), #expr))
