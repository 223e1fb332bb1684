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

}  // namespace llmk

#define LLMK_TRY(expr)            \
  do {                            \
    int _llmk_rc = (expr);        \
    if (_llmk_rc != LLMK_OK) return _llmk_rc; \
  } while (0)

#define LLMK_CUDA(expr) LLMK_TRY(::llmk::cuda_check((expr), #expr))
