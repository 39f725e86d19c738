// gemm.h -- drop-in for the reference's include/gemm.h (lines 11-20): the same
// two SGEMM entry points, now computed on the current CUDA device through the
// C ABI in attnb.h.  Row-major fp32 host buffers, C = alpha*(A@B) + beta*C.
// Errors throw std::invalid_argument / std::runtime_error like the reference.
#pragma once
#include <cstddef>

namespace gemm {

// Replaces gemm::sgemm_blocked (src/gemm.cpp:319-415).
void sgemm_blocked(const float* A, int M, int K, const float* B, int N, float* C,
                   float alpha = 1.0f, float beta = 0.0f);

// Replaces gemm::gemm_blocked_jit (src/jit_gemm.cpp:740-754); same kernel.
void gemm_blocked_jit(const float* A, int M, int K, const float* B, int N, float* C,
                      float alpha = 1.0f, float beta = 0.0f);

}  // namespace gemm
