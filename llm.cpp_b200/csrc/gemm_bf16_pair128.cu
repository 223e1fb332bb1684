// Instantiates the GEMM kernels for bf16 operands, a CTA pair per 256 x 128 tile.
#include "gemm_kernel.cuh"

namespace llmk {
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_pair128) {
  return dispatch_major<false, 128, true>(a_trans, b_trans, A, lda, B, ldb, M, N, K, ep, splits, s);
}
}  // namespace llmk
