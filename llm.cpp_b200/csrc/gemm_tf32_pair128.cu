// Instantiates the GEMM kernels for fp32 (tf32) operands, a CTA pair per 256 x 128 tile.
#include "gemm_kernel.cuh"

namespace llmk {
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_pair128) {
  return dispatch_major<true, 128, true>(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
}
}  // namespace llmk
