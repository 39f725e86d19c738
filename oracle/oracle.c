/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A float64 CPU restatement of attn-cpu's two hot paths, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker.
 * Nothing in the shipped library links, loads or calls this file.
 *
 * Parity is pinned: tests/test_oracle.py checks every function below against
 * the reference itself (oracle/_ref/libattnref.so, compiled from the
 * reference sources by oracle/Makefile) and against the committed golden
 * vectors in tests/golden/ that the reference produced.
 *
 * Every routine accumulates in double and rounds once to float at the end, so
 * it is at least as accurate as any fp32 ordering the reference or the GPU
 * kernels use.  Strides are in elements, like the reference's TensorF32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

/*
 * C = alpha * A.B + beta * C, row-major, ld = K, N, N.
 * Follows gemm::sgemm_blocked, src/gemm.cpp:319-415:
 *   - M, N or K <= 0 returns without touching C          (gemm.cpp:324)
 *   - alpha == 0: C = 0 if beta == 0 else C *= beta      (gemm.cpp:328-336)
 *   - beta == 0: C is overwritten and never read         (gemm.cpp:338-401)
 *   - beta != 0: C = alpha*acc + beta*C                  (gemm.cpp:404-414)
 * gemm::gemm_blocked_jit (src/jit_gemm.cpp:624-754) computes the same
 * function, so one restatement serves both.
 */
ORACLE_API void oracle_sgemm(const float *A, int M, int K, const float *B, int N,
                             float *C, float alpha, float beta) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  if (alpha == 0.0f) {
    for (int64_t i = 0; i < (int64_t)M * N; ++i)
      C[i] = (beta == 0.0f) ? 0.0f : (beta == 1.0f ? C[i] : C[i] * beta);
    return;
  }
  double *row = (double *)malloc(sizeof(double) * (size_t)N);
  for (int i = 0; i < M; ++i) {
    for (int j = 0; j < N; ++j) row[j] = 0.0;
    const float *a = A + (size_t)i * K;
    for (int k = 0; k < K; ++k) {
      const double aik = a[k];
      const float *b = B + (size_t)k * N;
      for (int j = 0; j < N; ++j) row[j] += aik * (double)b[j];
    }
    float *c = C + (size_t)i * N;
    for (int j = 0; j < N; ++j) {
      double v = (double)alpha * row[j];
      if (beta != 0.0f) v += (double)beta * (double)c[j];
      c[j] = (float)v;
    }
  }
  free(row);
}

/*
 * y[T,N] = x[T,K] . W[N,K]^T + b[N]  (PyTorch Linear convention).
 * Follows the projection step of attn::mha_block_dense: W is transposed and
 * packed into 16x16 tiles (src/attn_dispatch.cpp:45-60, include/pack_16x16.h:9-25),
 * then gemm_row4/row1_packed_16x16 start each accumulator from the bias and
 * add x.Wt (include/gemm_16x16.h:7-60).
 */
ORACLE_API void oracle_linear(const float *x, int T, int K, const float *W, int N,
                              const float *b, float *y) {
  for (int t = 0; t < T; ++t) {
    const float *xr = x + (size_t)t * K;
    for (int n = 0; n < N; ++n) {
      const float *wr = W + (size_t)n * K;
      double acc = b ? (double)b[n] : 0.0;
      for (int k = 0; k < K; ++k) acc += (double)xr[k] * (double)wr[k];
      y[(size_t)t * N + n] = (float)acc;
    }
  }
}

/*
 * One query row against `len` keys: exact two-pass softmax.
 * Pass 1 takes the logits q.k/sqrt(Dh) and their max, pass 2 forms
 * exp(l - max), the denominator and the V mix, then scales by 1/denom.
 * This is the arithmetic of attn::attn_step_dense (src/attn_dense.cpp:34-72)
 * and of each (h,l) row of attn::attn_block_dense (src/attn_block.cpp:143-226).
 * The online (running max/sum) forms in include/online_softmax.h:8-17,
 * include/attn_generic_m1.h:20-32 and include/kernels/attn_dhk16_m4_nocausal.h:149-290
 * compute the same function.
 */
static void attend_row(const float *q, int64_t qsD, const float *Kh, int64_t ksT,
                       int64_t ksD, const float *Vh, int64_t vsT, int64_t vsD,
                       int len, int Dh, float *out, int64_t osD, double *logits,
                       double *acc) {
  const double scale = 1.0 / sqrt((double)Dh);
  double m = -INFINITY;
  for (int t = 0; t < len; ++t) {
    const float *kr = Kh + (int64_t)t * ksT;
    double dot = 0.0;
    for (int d = 0; d < Dh; ++d) dot += (double)q[d * qsD] * (double)kr[d * ksD];
    logits[t] = dot * scale;
    if (logits[t] > m) m = logits[t];
  }
  double denom = 0.0;
  for (int d = 0; d < Dh; ++d) acc[d] = 0.0;
  for (int t = 0; t < len; ++t) {
    const double w = exp(logits[t] - m);
    denom += w;
    const float *vr = Vh + (int64_t)t * vsT;
    for (int d = 0; d < Dh; ++d) acc[d] += w * (double)vr[d * vsD];
  }
  for (int d = 0; d < Dh; ++d) out[d * osD] = (float)(acc[d] / denom);
}

/*
 * Decode step: O[h,:] = softmax(Q[h].K[h]^T / sqrt(Dh)) . V[h].
 * attn::attn_step_dense, src/attn_dense.cpp:21-73 (declared include/attn.h:35-38).
 * Shape checks live in the caller (validate_dense_shapes, include/attn.h:54-83).
 */
ORACLE_API void oracle_attn_step(const float *Q, int64_t qsH, int64_t qsD,
                                 const float *K, int64_t ksH, int64_t ksT, int64_t ksD,
                                 const float *V, int64_t vsH, int64_t vsT, int64_t vsD,
                                 float *O, int64_t osH, int64_t osD, int H, int T,
                                 int Dh) {
  double *logits = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1));
  double *acc = (double *)malloc(sizeof(double) * (size_t)Dh);
  for (int h = 0; h < H; ++h)
    attend_row(Q + (int64_t)h * qsH, qsD, K + (int64_t)h * ksH, ksT, ksD,
               V + (int64_t)h * vsH, vsT, vsD, T, Dh, O + (int64_t)h * osH, osD,
               logits, acc);
  free(logits);
  free(acc);
}

/*
 * Prefill with given Q/K/V: O[h,l,:] over keys t < T (t <= l when causal).
 * attn::attn_block_dense, src/attn_block.cpp:104-241 (include/attn.h:40-44);
 * causal requires L == T (attn_block.cpp:119-120), checked by the caller.
 */
ORACLE_API void oracle_attn_block(const float *Q, int64_t qsH, int64_t qsT, int64_t qsD,
                                  const float *K, int64_t ksH, int64_t ksT, int64_t ksD,
                                  const float *V, int64_t vsH, int64_t vsT, int64_t vsD,
                                  float *O, int64_t osH, int64_t osT, int64_t osD,
                                  int H, int L, int T, int Dh, int causal) {
  double *logits = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1));
  double *acc = (double *)malloc(sizeof(double) * (size_t)Dh);
  for (int h = 0; h < H; ++h)
    for (int l = 0; l < L; ++l) {
      const int len = causal ? (l + 1 < T ? l + 1 : T) : T;
      attend_row(Q + (int64_t)h * qsH + (int64_t)l * qsT, qsD, K + (int64_t)h * ksH,
                 ksT, ksD, V + (int64_t)h * vsH, vsT, vsD, len, Dh,
                 O + (int64_t)h * osH + (int64_t)l * osT, osD, logits, acc);
    }
  free(logits);
  free(acc);
}

/*
 * Full MHA block: y = (softmax(QK^T/sqrt(Dh)) V) W_out^T + b_out with
 * [Q|K|V] = x W_in^T + b_in, heads split column-wise (Dh = D/H).
 * attn::mha_block_dense, src/attn_dispatch.cpp:17-133:
 *   QKV projection (:63-95), scatter to heads (include/layout.h:9-42),
 *   attention dispatch (:98-107; causal rows see keys 0..t, i.e.
 *   valid_len = t+1, include/attn_generic_m1.h:20), output projection (:110-127).
 * The caller checks D % H == 0 (:22) and D % 16 == 0 (:45, :132).
 */
ORACLE_API void oracle_mha_block(const float *x, int T, int D, const float *W_in,
                                 const float *b_in, const float *W_out,
                                 const float *b_out, int H, int causal, float *y) {
  const int Dh = D / H;
  float *qkv = (float *)malloc(sizeof(float) * (size_t)T * 3 * D);
  float *ctx = (float *)malloc(sizeof(float) * (size_t)T * D);
  oracle_linear(x, T, D, W_in, 3 * D, b_in, qkv);
  /* Q[h,t,d] = qkv[t, h*Dh+d], K at +D, V at +2D: strides address the
     projected rows in place, which is what the scatter produces. */
  oracle_attn_block(qkv, Dh, 3 * D, 1, qkv + D, Dh, 3 * D, 1, qkv + 2 * D, Dh, 3 * D, 1,
                    ctx, Dh, D, 1, H, T, T, Dh, causal);
  oracle_linear(ctx, T, D, W_out, D, b_out, y);
  free(qkv);
  free(ctx);
}
