// Host runtime: error strings, per-device status word, launch counter and
// TMA tensor-map encoding (driver entry point fetched through the runtime, so
// the library does not link libcuda directly).
#include "runtime.h"

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

namespace llmk {

namespace {
thread_local std::string t_last_error;
std::atomic<unsigned long long> g_launches{0};
constexpr int kMaxDevices = 64;
// One status word per device, in device global memory of this module.
__device__ unsigned int g_device_status;
int g_num_sms[kMaxDevices] = {};
std::mutex g_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get = nullptr;
bool g_ctx_get_tried = false;

// The current CUDA context (the device's primary context once the runtime
// has touched it), fetched through the runtime's driver entry point; nullptr
// when it cannot be queried. Caller holds g_mu.
CUcontext current_context_locked() {
  if (!g_ctx_get_tried) {
    g_ctx_get_tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get) g_ctx_get(&ctx);
  return ctx;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

int get_encode(EncodeTiledFn* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(LLMK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = g_encode;
  return LLMK_OK;
}
}  // namespace

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LLMK_OK;
  return fail(LLMK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int SymbolCache::get(void** out) {
  int dev = 0;
  LLMK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LLMK_ERR_UNSUPPORTED, "device index out of range");
  // No device call here: this runs on every kernel launch, also inside stream
  // capture. Before the runtime has made a context current the context reads
  // as null; the lookup below creates it, and the next call refreshes the
  // entry once under the real context.
  std::lock_guard<std::mutex> lk(g_mu);
  const CUcontext ctx = current_context_locked();
  if (!ptr_[dev] || ctx_[dev] != static_cast<void*>(ctx)) {
    void* p = nullptr;
    const cudaError_t e = lookup_(&p);
    if (e != cudaSuccess || p == nullptr)
      return fail(LLMK_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    ptr_[dev] = p;
    ctx_[dev] = ctx;
  }
  *out = ptr_[dev];
  return LLMK_OK;
}

namespace {
cudaError_t lookup_status(void** p) { return cudaGetSymbolAddress(p, g_device_status); }
SymbolCache g_status_cache(lookup_status);
}  // namespace

unsigned int* device_status_ptr() {
  void* p = nullptr;
  if (g_status_cache.get(&p) != LLMK_OK) return nullptr;
  return static_cast<unsigned int*>(p);
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_num_sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 148;
  }
  return g_num_sms[dev];
}

void count_launch(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc;
  LLMK_TRY(get_encode(&enc));
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled(2d) failed (%d): inner=%llu outer=%llu stride=%llu box=%ux%u",
             static_cast<int>(r), (unsigned long long)inner, (unsigned long long)outer,
             (unsigned long long)row_stride_bytes, box_inner, box_outer);
    return fail(LLMK_ERR_UNSUPPORTED, buf);
  }
  return LLMK_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn enc;
  LLMK_TRY(get_encode(&enc));
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled(3d) failed (%d)", static_cast<int>(r));
    return fail(LLMK_ERR_UNSUPPORTED, buf);
  }
  return LLMK_OK;
}

}  // namespace llmk

extern "C" {

const char* llmk_status_string(int s) {
  switch (s) {
    case LLMK_OK: return "ok";
    case LLMK_ERR_INVALID_ARG: return "invalid argument";
    case LLMK_ERR_UNSUPPORTED: return "unsupported";
    case LLMK_ERR_CUDA: return "cuda error";
    case LLMK_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case LLMK_ERR_WORKSPACE: return "workspace missing or too small";
    case LLMK_ERR_NCCL: return "nccl error";
    case LLMK_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

const char* llmk_last_error(void) { return llmk::t_last_error.c_str(); }

const char* llmk_version(void) { return "llmk 0.1 (sm_100a)"; }

unsigned long long llmk_launch_count(void) { return llmk::g_launches.load(); }

int llmk_device_status(unsigned int* out, int reset) {
  if (!out) return llmk::fail(LLMK_ERR_INVALID_ARG, "out is null");
  unsigned int* p = llmk::device_status_ptr();
  if (!p) return llmk::fail(LLMK_ERR_CUDA, "device status word unavailable");
  LLMK_CUDA(cudaDeviceSynchronize());
  LLMK_CUDA(cudaMemcpy(out, p, sizeof(unsigned int), cudaMemcpyDeviceToHost));
  if (reset) LLMK_CUDA(cudaMemset(p, 0, sizeof(unsigned int)));
  return LLMK_OK;
}

}  // extern "C"
