// shims.cpp -- the reference's C++ entry points (include/attn.h, attn_api.h,
// gemm.h) as thin wrappers over the C ABI.  Status codes become the
// reference's exception types: std::invalid_argument for shape / null /
// stride problems, std::runtime_error for everything else.
#include <new>
#include <stdexcept>
#include <string>

#include "../../include/attn.h"
#include "../../include/attn_api.h"
#include "../../include/attnb.h"
#include "../../include/gemm.h"

namespace {
void rethrow(int rc) {
  if (rc == ATTNB_OK) return;
  const std::string msg = attnb_last_error();
  if (rc == ATTNB_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  if (rc == ATTNB_ERR_OUT_OF_MEMORY) throw std::bad_alloc();
  throw std::runtime_error(msg);
}
attnb_tensor to_c(const attn::TensorF32& t) {
  return attnb_tensor{t.data, t.H, t.T, t.Dh, t.strideH, t.strideT, t.strideDh};
}
}  // namespace

namespace attn {

void attn_step_dense(const TensorF32& Q, const TensorF32& K, const TensorF32& V,
                     MutableTensorF32& O) {
  validate_dense_shapes(Q, K, V, O);
  attnb_tensor q = to_c(Q), k = to_c(K), v = to_c(V);
  q.T = 1;
  q.strideT = 0;
  attnb_mtensor o{O.data, O.H, 1, O.Dh, O.strideH, 0, O.strideDh};
  rethrow(attnb_attn_step_dense(&q, &k, &v, &o));
}

void attn_block_dense(const TensorF32& Q, const TensorF32& K, const TensorF32& V,
                      MutableTensor3F32& O, bool causal) {
  attnb_tensor q = to_c(Q), k = to_c(K), v = to_c(V);
  attnb_mtensor o{O.data, O.H, O.T, O.Dh, O.strideH, O.strideT, O.strideDh};
  rethrow(attnb_attn_block_dense(&q, &k, &v, &o, causal ? 1 : 0, ATTNB_PREC_DEFAULT));
}

void mha_block_dense(const float* x, int T, int D, const float* W_in, const float* b_in,
                     const float* W_out, const float* b_out, int H, bool causal, float* y_out) {
  rethrow(attnb_mha_block_dense(x, T, D, W_in, b_in, W_out, b_out, H, causal ? 1 : 0, y_out,
                                ATTNB_PREC_DEFAULT));
}

}  // namespace attn

namespace gemm {

void sgemm_blocked(const float* A, int M, int K, const float* B, int N, float* C, float alpha,
                   float beta) {
  rethrow(attnb_sgemm(A, M, K, B, N, C, alpha, beta, ATTNB_PREC_DEFAULT));
}

void gemm_blocked_jit(const float* A, int M, int K, const float* B, int N, float* C, float alpha,
                      float beta) {
  rethrow(attnb_gemm_jit(A, M, K, B, N, C, alpha, beta, ATTNB_PREC_DEFAULT));
}

}  // namespace gemm
