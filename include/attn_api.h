// attn_api.h -- drop-in for the reference's include/attn_api.h (lines 4-7).
#pragma once

namespace attn {
// Replaces attn::mha_block_dense (src/attn_dispatch.cpp:17-133); computed on
// the current CUDA device.  Throws std::runtime_error when D % H != 0 or
// D % 16 != 0, like the reference.
void mha_block_dense(const float* x, int T, int D, const float* W_in, const float* b_in,
                     const float* W_out, const float* b_out, int H, bool causal,
                     float* y_out);
}  // namespace attn
