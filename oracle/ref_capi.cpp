// ref_capi.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI wrapper, written for this project, around the reference's own
// functions so that tests and the bench's reference arm can call them through
// ctypes.  oracle/Makefile compiles it together with the reference sources
// (src/gemm.cpp, src/attn_dense.cpp, src/attn_block.cpp, src/attn_dispatch.cpp)
// where they lie; no reference source is copied.  src/jit_gemm.cpp is not
// built: it needs the un-vendored Xbyak submodule (.gitmodules:7-9).
//
// Each function returns 0 on success, 1 for std::invalid_argument, 2 for any
// other exception, mirroring how the reference signals errors
// (include/attn.h:54-83, src/attn_dispatch.cpp:22,132).
#include <stdexcept>

#include "attn.h"
#include "gemm.h"

#define REF_API extern "C" __attribute__((visibility("default")))

template <class F>
static int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::invalid_argument&) {
    return 1;
  } catch (...) {
    return 2;
  }
}

// gemm::sgemm_blocked, src/gemm.cpp:319
REF_API int ref_sgemm(const float* A, int M, int K, const float* B, int N, float* C,
                      float alpha, float beta) {
  return guarded([&] { gemm::sgemm_blocked(A, M, K, B, N, C, alpha, beta); });
}

// attn::attn_step_dense, src/attn_dense.cpp:21
REF_API int ref_attn_step(const float* Q, long long qsH, long long qsD, const float* K,
                          long long ksH, long long ksT, long long ksD, const float* V,
                          long long vsH, long long vsT, long long vsD, float* O,
                          long long osH, long long osD, int H, int T, int Dh) {
  attn::TensorF32 q{Q, H, 1, Dh, qsH, 0, qsD};
  attn::TensorF32 k{K, H, T, Dh, ksH, ksT, ksD};
  attn::TensorF32 v{V, H, T, Dh, vsH, vsT, vsD};
  attn::MutableTensorF32 o{O, H, Dh, osH, osD};
  return guarded([&] { attn::attn_step_dense(q, k, v, o); });
}

// attn::attn_block_dense, src/attn_block.cpp:104
REF_API int ref_attn_block(const float* Q, long long qsH, long long qsT, long long qsD,
                           const float* K, long long ksH, long long ksT, long long ksD,
                           const float* V, long long vsH, long long vsT, long long vsD,
                           float* O, long long osH, long long osT, long long osD, int H,
                           int L, int T, int Dh, int causal) {
  attn::TensorF32 q{Q, H, L, Dh, qsH, qsT, qsD};
  attn::TensorF32 k{K, H, T, Dh, ksH, ksT, ksD};
  attn::TensorF32 v{V, H, T, Dh, vsH, vsT, vsD};
  attn::MutableTensor3F32 o{O, H, L, Dh, osH, osT, osD};
  return guarded([&] { attn::attn_block_dense(q, k, v, o, causal != 0); });
}

// attn::mha_block_dense, src/attn_dispatch.cpp:17
REF_API int ref_mha_block(const float* x, int T, int D, const float* W_in,
                          const float* b_in, const float* W_out, const float* b_out,
                          int H, int causal, float* y) {
  return guarded(
      [&] { attn::mha_block_dense(x, T, D, W_in, b_in, W_out, b_out, H, causal != 0, y); });
}
