// attn.h -- drop-in for the reference's include/attn.h: the same tensor views
// (lines 10-26), entry points (lines 35-51) and validation helper (lines 54-83),
// now computed on the current CUDA device through the C ABI in attnb.h.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>

namespace attn {

// Non-owning views over fp32 tensors; strides in elements.
struct TensorF32 {
  const float* data = nullptr;
  int H = 0, T = 0, Dh = 0;
  int64_t strideH = 0, strideT = 0, strideDh = 0;
};

struct MutableTensorF32 {
  float* data = nullptr;
  int H = 0, Dh = 0;
  int64_t strideH = 0, strideDh = 0;
};

struct MutableTensor3F32 {
  float* data = nullptr;
  int H = 0, T = 0, Dh = 0;
  int64_t strideH = 0, strideT = 0, strideDh = 0;
};

// Decode step. Q: [H, Dh], K/V: [H, T, Dh] -> O: [H, Dh].
void attn_step_dense(const TensorF32& Q, const TensorF32& K, const TensorF32& V,
                     MutableTensorF32& O);

// Prefill. Q: [H, L, Dh], K/V: [H, T, Dh] -> O: [H, L, Dh]; causal needs L == T.
void attn_block_dense(const TensorF32& Q, const TensorF32& K, const TensorF32& V,
                      MutableTensor3F32& O, bool causal);

void mha_block_dense(const float* x, int T, int D, const float* W_in, const float* b_in,
                     const float* W_out, const float* b_out, int num_heads, bool causal,
                     float* y_out);

// Same checks and messages as the reference helper; throws std::invalid_argument.
inline void validate_dense_shapes(const TensorF32& Q, const TensorF32& K, const TensorF32& V,
                                  const MutableTensorF32& O) {
  if (!Q.data || !K.data || !V.data || !O.data) throw std::invalid_argument("Null data pointer");
  if (Q.H <= 0 || Q.Dh <= 0) throw std::invalid_argument("Q has invalid H/Dh");
  if (K.H != Q.H || V.H != Q.H) throw std::invalid_argument("K/V H must match Q.H");
  if (K.Dh != Q.Dh || V.Dh != Q.Dh) throw std::invalid_argument("K/V Dh must match Q.Dh");
  if (K.T <= 0 || V.T != K.T) throw std::invalid_argument("K/V T must be positive and equal");
  if (O.H != Q.H || O.Dh != Q.Dh) throw std::invalid_argument("O must be [H, Dh] matching Q");
  if (Q.strideH == 0 || Q.strideDh == 0 || K.strideH == 0 || K.strideT == 0 ||
      K.strideDh == 0 || V.strideH == 0 || V.strideT == 0 || V.strideDh == 0 ||
      O.strideH == 0 || O.strideDh == 0)
    throw std::invalid_argument("Zero stride encountered");
}

}  // namespace attn
